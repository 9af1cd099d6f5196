// Forward-in-time adjoint of the LQR solve (symplectic_iter.py:715-885) on warp-level
// tensor-core MMAs, for the backward of a forward that saved lambda0 (and M = Y1^-1 Y3, or
// the contracted d_p = Y1^-1 Y3 d_u).
//
// Every head of a batch row n shares that row's B and Q, so the T-step adjoint of the row's
// heads is a chain of small matrix products: per step, [h; dh] Q^T, [lambda; dlambda] B and
// [u e^lgB; du e^lgB] B^T, plus the rank-2 updates of grad_B and grad_Q summed over heads.
// One warp owns 8 heads of one row.  The 16 rows of an m16n8k8 MMA are the 8 heads'
// primal vectors (rows 0-7) and their tangents (rows 8-15), so thread (g, t) = (lane / 4,
// lane % 4) holds, for head g, entries {8j + 2t, 8j + 2t + 1} (j < d / 8) of both: all the
// elementwise work of the recursion is thread-local.  The output fragment of one product is
// fed back as the A fragment of the next without moving data: the K order of the constant
// operand is permuted to match (fragment slot t <-> entry 8kk + 2t, slot t + 4 <-> entry
// 8kk + 2t + 1).  Each product runs in 3xTF32 (A_lo B_hi + A_hi B_lo + A_hi B_hi), close to
// the fp32 sums of the reference.  grad_B and grad_Q sum over heads, i.e. contract over the
// MMA's M rows: the vectors go through a small shared staging matrix and a second MMA with
// K = the 16 (head, primal / tangent) rows accumulates them in registers over all steps.
// Per-row partial sums of the warps meet in shared memory in warp order: deterministic.
#pragma once

#include "lqr_kernels.cuh"

namespace ttc {

namespace wmma {

__device__ __forceinline__ void split(float x, uint32_t& hi, uint32_t& lo) {
  hi = __float_as_uint(x) & 0xffffe000u;
  lo = __float_as_uint(x - __uint_as_float(hi));
}

// D (16x8, f32) += A (16x8, tf32, row) * B (8x8, tf32, col).
__device__ __forceinline__ void m16n8k8(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

}  // namespace wmma

template <int D>
struct AdjMma {
  static_assert(D % 16 == 0, "d must be a multiple of 16");
  static constexpr int NT = D / 8;             // n-tiles of an output = k-steps of an input
  static constexpr int MT = D / 16;            // m-tiles of grad_B / grad_Q
  static constexpr int kFrag = NT * NT * 128;  // floats of one constant operand (hi + lo)
  static constexpr int SS = D + 8;             // staging row stride (bank-conflict free)
  static constexpr int kStage = 16 * SS;
  // per row: operands Q^T, B, B^T, Q and a symmetry flag; per warp: 3 staging matrices
  static constexpr int kRow = 4 * kFrag + 4;
  static constexpr int kWarp = 3 * kStage;
  static constexpr int kMaxWarps = 8;
  static int rows_per_cta(int nh) {
    const int wpr = (nh + 7) / 8;
    return wpr >= kMaxWarps ? 1 : kMaxWarps / wpr;
  }
  static int warps(int nh) { return ((nh + 7) / 8) * rows_per_cta(nh); }
  static size_t bytes(int nh) {
    const int w = warps(nh), r = rows_per_cta(nh);
    // the final grad_B / grad_Q exchange reuses the staging area: 2 D^2 floats per warp
    const int per_warp = kWarp > 2 * D * D ? kWarp : 2 * D * D;
    return sizeof(float) * ((size_t)r * kRow + (size_t)w * per_warp);
  }
};

// Constant operand W (K x N = D x D, W[k][n] = get(k, n)) in fragment order: for k-step kk,
// n-tile nj and lane (g, t), the float4 (hi b0, hi b1, lo b0, lo b1) with
// b0 = W[8kk + 2t][8nj + g], b1 = W[8kk + 2t + 1][8nj + g].
template <int D, typename Get>
__device__ __forceinline__ void build_operand(float* dst, Get get, int tid, int nthreads) {
  constexpr int NT = D / 8;
  for (int e = tid; e < NT * NT * 32; e += nthreads) {
    const int lane = e & 31, kn = e >> 5, kk = kn / NT, nj = kn % NT;
    const int g = lane >> 2, t = lane & 3;
    const float w0 = get(8 * kk + 2 * t, 8 * nj + g), w1 = get(8 * kk + 2 * t + 1, 8 * nj + g);
    const float h0 = __uint_as_float(__float_as_uint(w0) & 0xffffe000u);
    const float h1 = __uint_as_float(__float_as_uint(w1) & 0xffffe000u);
    reinterpret_cast<float4*>(dst)[e] = make_float4(h0, h1, w0 - h0, w1 - h1);
  }
}

// out (16 x D, output-fragment order) = in (16 x D, output-fragment order) * W, 3xTF32.
// in[j] = {row g e0, row g e1, row g+8 e0, row g+8 e1} with e0/e1 = entries 8j+2t, 8j+2t+1.
template <int D>
__device__ __forceinline__ void frag_product(const float (&in)[D / 8][4], float (&out)[D / 8][4],
                                             const float4* W, int lane) {
  constexpr int NT = D / 8;
  uint32_t ah[NT][4], al[NT][4];
#pragma unroll
  for (int kk = 0; kk < NT; ++kk) {
    wmma::split(in[kk][0], ah[kk][0], al[kk][0]);  // a0: row g,   slot t     <- entry 8kk+2t
    wmma::split(in[kk][2], ah[kk][1], al[kk][1]);  // a1: row g+8, slot t
    wmma::split(in[kk][1], ah[kk][2], al[kk][2]);  // a2: row g,   slot t + 4 <- entry 8kk+2t+1
    wmma::split(in[kk][3], ah[kk][3], al[kk][3]);  // a3: row g+8, slot t + 4
  }
#pragma unroll
  for (int nj = 0; nj < NT; ++nj) {
    float4 w[NT];
#pragma unroll
    for (int kk = 0; kk < NT; ++kk) w[kk] = W[(kk * NT + nj) * 32 + lane];
    float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kk = 0; kk < NT; ++kk) {
      wmma::m16n8k8(c, al[kk], __float_as_uint(w[kk].x), __float_as_uint(w[kk].y));
      wmma::m16n8k8(c, ah[kk], __float_as_uint(w[kk].z), __float_as_uint(w[kk].w));
    }
#pragma unroll
    for (int kk = 0; kk < NT; ++kk)
      wmma::m16n8k8(c, ah[kk], __float_as_uint(w[kk].x), __float_as_uint(w[kk].y));
#pragma unroll
    for (int r = 0; r < 4; ++r) out[nj][r] = c[r];
  }
}

// Rows g and g + 8 of a 16 x D fragment-order matrix into the staging matrix S (stride SS).
template <int D>
__device__ __forceinline__ void stage_rows(float* S, const float (&v)[D / 8][4], int g, int t) {
  constexpr int SS = AdjMma<D>::SS;
#pragma unroll
  for (int j = 0; j < D / 8; ++j) {
    *reinterpret_cast<float2*>(S + g * SS + 8 * j + 2 * t) = make_float2(v[j][0], v[j][1]);
    *reinterpret_cast<float2*>(S + (g + 8) * SS + 8 * j + 2 * t) = make_float2(v[j][2], v[j][3]);
  }
}

// acc[m][n] += sum_r SX[r][m] * SY[(r + 8) % 16][n]  (K = the 16 staged rows), 3xTF32.
template <int D>
__device__ __forceinline__ void accumulate_outer(float (&acc)[D / 16][D / 8][4], const float* SX,
                                                 const float* SY, int g, int t) {
  constexpr int SS = AdjMma<D>::SS, NT = D / 8, MT = D / 16;
#pragma unroll
  for (int kk = 0; kk < 2; ++kk) {
    uint32_t bh[NT][2], bl[NT][2];
    const float* y0 = SY + ((8 * kk + t + 8) & 15) * SS;
    const float* y1 = SY + ((8 * kk + t + 12) & 15) * SS;
#pragma unroll
    for (int nj = 0; nj < NT; ++nj) {
      wmma::split(y0[8 * nj + g], bh[nj][0], bl[nj][0]);
      wmma::split(y1[8 * nj + g], bh[nj][1], bl[nj][1]);
    }
    const float* x0 = SX + (8 * kk + t) * SS;
    const float* x1 = SX + (8 * kk + t + 4) * SS;
#pragma unroll
    for (int mi = 0; mi < MT; ++mi) {
      uint32_t ah[4], al[4];
      wmma::split(x0[16 * mi + g], ah[0], al[0]);
      wmma::split(x0[16 * mi + g + 8], ah[1], al[1]);
      wmma::split(x1[16 * mi + g], ah[2], al[2]);
      wmma::split(x1[16 * mi + g + 8], ah[3], al[3]);
#pragma unroll
      for (int nj = 0; nj < NT; ++nj) {
        wmma::m16n8k8(acc[mi][nj], al, bh[nj][0], bh[nj][1]);
        wmma::m16n8k8(acc[mi][nj], ah, bl[nj][0], bl[nj][1]);
        wmma::m16n8k8(acc[mi][nj], ah, bh[nj][0], bh[nj][1]);
      }
    }
  }
}

// Backward from the forward's lambda0 and either M (d_p = M d_u per head, fused_lqr.py:
// 185-187) or d_p itself.  Grid: ceil(N / R) CTAs of R rows x ceil(nh / 8) warps.
template <int D, typename TIn, bool FROM_M>
__global__ void __launch_bounds__(256, 2)
lqr_bwd_mma_kernel(const TIn* __restrict__ A_diag, const TIn* __restrict__ Bm,
                   const TIn* __restrict__ Qm, const TIn* __restrict__ Rinv,
                   const TIn* __restrict__ lgA, const TIn* __restrict__ lgB,
                   const TIn* __restrict__ lgQ, const TIn* __restrict__ H0,
                   const float* __restrict__ lam0_in, const float* __restrict__ M_or_dp,
                   const TIn* __restrict__ dU, int64_t N, int nh, int T, int rows_per_cta,
                   TIn* __restrict__ gA_out, TIn* __restrict__ gB_out, TIn* __restrict__ gQ_out,
                   TIn* __restrict__ gR_out, TIn* __restrict__ gQf_out, TIn* __restrict__ glgA_out,
                   TIn* __restrict__ glgB_out, TIn* __restrict__ glgQ_out, TIn* __restrict__ gh0_out,
                   int* __restrict__ status) {
  using C = AdjMma<D>;
  constexpr int NT = C::NT, MT = C::MT;
  extern __shared__ __align__(16) float smem[];
  const int tid = threadIdx.x, nthreads = blockDim.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int wpr = (nh + 7) / 8;
  const int rloc = warp / wpr, hb = warp % wpr;
  const int64_t n0 = (int64_t)blockIdx.x * rows_per_cta;
  const int64_t n = n0 + rloc;
  const bool row_ok = n < N;
  float* rows_s = smem;
  float* warp_s = smem + (size_t)rows_per_cta * C::kRow;
  const int per_warp = C::kWarp > 2 * D * D ? C::kWarp : 2 * D * D;
  float* stg = warp_s + warp * per_warp;

  // The CTA's rows: constant operands Q^T, B, B^T, Q in fragment order, symmetry flag.
  for (int r = 0; r < rows_per_cta; ++r) {
    if (tid == 0) reinterpret_cast<int*>(rows_s + r * C::kRow + 4 * C::kFrag)[0] = 1;
  }
  __syncthreads();
  for (int r = 0; r < rows_per_cta; ++r) {
    const int64_t nr = n0 + r;
    if (nr >= N) break;
    float* base = rows_s + r * C::kRow;
    const TIn* Bn = Bm + nr * (D * D);
    const TIn* Qn = Qm + nr * (D * D);
    build_operand<D>(base, [&](int k, int c) { return ldf(Qn + c * D + k); }, tid, nthreads);
    build_operand<D>(base + C::kFrag, [&](int k, int c) { return ldf(Bn + k * D + c); }, tid, nthreads);
    build_operand<D>(base + 2 * C::kFrag, [&](int k, int c) { return ldf(Bn + c * D + k); }, tid, nthreads);
    build_operand<D>(base + 3 * C::kFrag, [&](int k, int c) { return ldf(Qn + k * D + c); }, tid, nthreads);
    bool asym = false;
    for (int e = tid; e < D * D; e += nthreads) asym |= ldf(Qn + e) != ldf(Qn + (e % D) * D + e / D);
    if (asym) reinterpret_cast<int*>(base + 4 * C::kFrag)[0] = 0;
  }
  __syncthreads();

  const float* rbase = rows_s + (row_ok ? rloc : 0) * C::kRow;
  const float4* Wqt = reinterpret_cast<const float4*>(rbase);
  const float4* Wb = reinterpret_cast<const float4*>(rbase + C::kFrag);
  const float4* Wbt = reinterpret_cast<const float4*>(rbase + 2 * C::kFrag);
  const float4* Wq = reinterpret_cast<const float4*>(rbase + 3 * C::kFrag);
  const bool sym = reinterpret_cast<const int*>(rbase + 4 * C::kFrag)[0] != 0;

  const int h = hb * 8 + g;
  const bool valid = row_ok && h < nh;
  const int64_t p = valid ? n * nh + h : 0;
  // entry of slot (j, s): 8j + 2t + s
  float a[NT][2], lgQ2[NT][2], lgB2[NT][2], rinv[NT][2], rinv2[NT][2], dUi[NT][2];
  float L[NT][4], H[NT][4];
  float lgA2 = valid ? ldf(lgA + p) * kLog2e : 0.f;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int e = 8 * j + 2 * t + s;
      a[j][s] = valid ? ldf(A_diag + p * D + e) : 0.f;
      lgQ2[j][s] = valid ? ldf(lgQ + p * D + e) * kLog2e : 0.f;
      lgB2[j][s] = valid ? ldf(lgB + p * D + e) * kLog2e : 0.f;
      rinv[j][s] = valid ? ldf(Rinv + p * D + e) : 1.f;
      rinv2[j][s] = recip(rinv[j][s] * rinv[j][s]);
      dUi[j][s] = valid ? ldf(dU + p * D + e) : 0.f;
      H[j][s] = valid ? ldf(H0 + p * D + e) : 0.f;
      H[j][2 + s] = 0.f;
      L[j][s] = valid ? lam0_in[p * D + e] : 0.f;
      float dl = 0.f;
      if (valid) {
        if constexpr (FROM_M) {
          const float* mrow = M_or_dp + (p * D + e) * D;
          for (int c = 0; c < D; ++c) dl = fmaf(mrow[c], ldf(dU + p * D + c), dl);
        } else {
          dl = M_or_dp[p * D + e];
        }
      }
      L[j][2 + s] = dl;
    }
  }

  float gA[NT][2], glgQ[NT][2], gR[NT][2], glgB[NT][2], dqp[NT][2], At[NT][2];
  float HD[NT][4];
  float glgA = 0.f;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      gA[j][s] = glgQ[j][s] = gR[j][s] = glgB[j][s] = 0.f;
      dqp[j][s] = 1.0f;
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) HD[j][r] = 0.f;
  }
  float accB[MT][NT][4], accQ[MT][NT][4];
#pragma unroll
  for (int mi = 0; mi < MT; ++mi)
#pragma unroll
    for (int nj = 0; nj < NT; ++nj)
#pragma unroll
      for (int r = 0; r < 4; ++r) accB[mi][nj][r] = accQ[mi][nj][r] = 0.f;

  float* S0 = stg;                 // [lambda; dlambda]
  float* S1 = stg + C::kStage;     // [u e^lgB; du e^lgB]
  float* S2 = stg + 2 * C::kStage; // [h Dq; dh Dq]
  bool bad = false;
  for (int k = 0; k < T; ++k) {
    const float ke = static_cast<float>(k + 1);
    if (k > 0) {
      // lambda -= Q_k h, dlambda -= Q_k dh with Q_k = Dq Q Dq (symplectic_iter.py:766-775)
      // and the log_gamma_Q gradient of step k-1 (:871-877).
      float QH[NT][4], QTH[NT][4];
      frag_product<D>(HD, QH, Wqt, lane);
      if (!sym) {
        frag_product<D>(HD, QTH, Wq, lane);
      }
#pragma unroll
      for (int j = 0; j < NT; ++j) {
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          const float qh = QH[j][s], qdh = QH[j][2 + s];
          const float qth = sym ? qh : QTH[j][s], qtdh = sym ? qdh : QTH[j][2 + s];
          L[j][s] = fmaf(-dqp[j][s], qh, L[j][s]);
          L[j][2 + s] = fmaf(-dqp[j][s], qdh, L[j][2 + s]);
          glgQ[j][s] = fmaf(0.5f * fmaf(H[j][2 + s], qh + qth, H[j][s] * (qdh + qtdh)),
                            static_cast<float>(k) * dqp[j][s], glgQ[j][s]);
        }
      }
    } else if (valid) {
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          bad |= unstable(L[j][2 + s]);
          stf(gh0_out + p * D + 8 * j + 2 * t + s, L[j][2 + s]);  // dh_0 = dlambda_0
        }
    }
    const float eA = exp_scaled(lgA2, ke);
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        At[j][s] = fmaf(a[j][s], eA, 1.0f);
        const float rAt = recip(At[j][s]);
        L[j][s] *= rAt;
        L[j][2 + s] *= rAt;
        const float dA = fmaf(L[j][s], H[j][2 + s], L[j][2 + s] * H[j][s]);
        gA[j][s] = fmaf(dA, eA, gA[j][s]);
        glgA = fmaf(dA * a[j][s], ke * eA, glgA);
      }
    }
    // u = -R_inv (B e^lgB)^T lambda and its tangent (symplectic_iter.py:800-830)
    float UE[NT][4];
    {
      float BL[NT][4];
      frag_product<D>(L, BL, Wb, lane);
#pragma unroll
      for (int j = 0; j < NT; ++j) {
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          const float eB = exp_scaled(lgB2[j][s], ke);
          const float bl = BL[j][s], bdl = BL[j][2 + s];
          const float u = -(bl * eB) * rinv[j][s];
          float du = -(bdl * eB) * rinv[j][s];
          if (k == 0) du = fmaf(dUi[j][s], -rinv[j][s], du);
          glgB[j][s] = fmaf(fmaf(du, bl, u * bdl), ke * eB, glgB[j][s]);
          gR[j][s] = fmaf(-(u * du), rinv2[j][s], gR[j][s]);
          UE[j][s] = u * eB;
          UE[j][2 + s] = du * eB;
        }
      }
    }
    __syncwarp();
    stage_rows<D>(S0, L, g, t);
    stage_rows<D>(S1, UE, g, t);
    // h <- A h + B e^lgB u (symplectic_iter.py:832-850)
    {
      float BU[NT][4];
      frag_product<D>(UE, BU, Wbt, lane);
#pragma unroll
      for (int j = 0; j < NT; ++j) {
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          H[j][s] = fmaf(H[j][s], At[j][s], BU[j][s]);
          H[j][2 + s] = fmaf(H[j][2 + s], At[j][s], BU[j][2 + s]);
          const float dq = exp_scaled(lgQ2[j][s], ke);
          HD[j][s] = H[j][s] * dq;
          HD[j][2 + s] = H[j][2 + s] * dq;
          dqp[j][s] = dq;
        }
      }
    }
    if (k < T - 1) stage_rows<D>(S2, HD, g, t);
    __syncwarp();
    // grad_B += lambda (du e^lgB)^T + dlambda (u e^lgB)^T ;
    // grad_Q += (h Dq)(dh Dq)^T + (dh Dq)(h Dq)^T  (the 1/2 is applied at the end)
    accumulate_outer<D>(accB, S0, S1, g, t);
    if (k < T - 1) accumulate_outer<D>(accQ, S2, S2, g, t);
  }

  // grad_Qf = (h dh^T + dh h^T) / 2 at the final state (symplectic_iter.py:855-857).
  __syncwarp();
  stage_rows<D>(S0, H, g, t);
  __syncwarp();
  for (int e = lane; e < 8 * D * D; e += 32) {
    const int hh = e / (D * D), i = (e / D) % D, jj = e % D;
    const int h2 = hb * 8 + hh;
    if (row_ok && h2 < nh) {
      const float v = 0.5f * fmaf(S0[hh * C::SS + i], S0[(hh + 8) * C::SS + jj],
                                  S0[(hh + 8) * C::SS + i] * S0[hh * C::SS + jj]);
      bad |= unstable(v);
      stf(gQf_out + ((n * nh + h2) * D + i) * D + jj, v);
    }
  }
  // Per-head outputs.
  float glgA_sum = glgA;
  glgA_sum += __shfl_xor_sync(0xffffffffu, glgA_sum, 1);
  glgA_sum += __shfl_xor_sync(0xffffffffu, glgA_sum, 2);
  if (valid) {
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const int e = 8 * j + 2 * t + s;
        bad |= unstable(gA[j][s]) | unstable(glgQ[j][s]) | unstable(gR[j][s]) | unstable(glgB[j][s]);
        stf(gA_out + p * D + e, gA[j][s]);
        stf(glgQ_out + p * D + e, glgQ[j][s]);
        stf(gR_out + p * D + e, gR[j][s]);
        stf(glgB_out + p * D + e, glgB[j][s]);
      }
    }
    if (t == 0) {
      bad |= unstable(glgA_sum);
      stf(glgA_out + p, glgA_sum);
    }
  }
  // grad_B / grad_Q of the row: the warps' partial sums in warp order.
  __syncthreads();
  float* red = stg;  // [D][D] grad_B then [D][D] grad_Q, row-major
#pragma unroll
  for (int mi = 0; mi < MT; ++mi)
#pragma unroll
    for (int nj = 0; nj < NT; ++nj) {
      const int r0 = 16 * mi + g, c0 = 8 * nj + 2 * t;
      red[r0 * D + c0] = accB[mi][nj][0];
      red[r0 * D + c0 + 1] = accB[mi][nj][1];
      red[(r0 + 8) * D + c0] = accB[mi][nj][2];
      red[(r0 + 8) * D + c0 + 1] = accB[mi][nj][3];
      red[D * D + r0 * D + c0] = 0.5f * accQ[mi][nj][0];
      red[D * D + r0 * D + c0 + 1] = 0.5f * accQ[mi][nj][1];
      red[D * D + (r0 + 8) * D + c0] = 0.5f * accQ[mi][nj][2];
      red[D * D + (r0 + 8) * D + c0 + 1] = 0.5f * accQ[mi][nj][3];
    }
  __syncthreads();
  for (int r = 0; r < rows_per_cta; ++r) {
    const int64_t nr = n0 + r;
    if (nr >= N) break;
    for (int e = tid; e < 2 * D * D; e += nthreads) {
      float s = 0.f;
      for (int w = 0; w < wpr; ++w) s += warp_s[(r * wpr + w) * per_warp + e];
      bad |= unstable(s);
      if (e < D * D) {
        stf(gB_out + nr * (D * D) + e, s);
      } else {
        stf(gQ_out + nr * (D * D) + (e - D * D), s);
      }
    }
  }
  if (bad) atomicOr(status, TTC_STATUS_BWD_UNSTABLE);
}

}  // namespace ttc
