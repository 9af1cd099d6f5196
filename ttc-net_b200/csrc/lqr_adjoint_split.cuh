// Forward-in-time adjoint of the LQR solve (symplectic_iter.py:715-885) on warp-level
// tensor-core MMAs for h_dim = 64, the backward of a forward that saved lambda0 and
// M = Y1^-1 Y3.
//
// The formulation is the one of lqr_adjoint_mma.cuh: the 16 rows of an m16n8k8 MMA are the
// primal vectors (rows 0-7) and tangents (rows 8-15) of 8 heads of one batch row, and every
// step is the products [h; dh] Q^T, [lambda; dlambda] B and [u e^lgB; du e^lgB] B^T plus the
// rank-2 updates of grad_B and grad_Q summed over the row's heads.  At d = 64 one warp cannot
// hold a group's state (16 fragment columns of both vectors, the per-entry coefficients and
// their gradients: twice what already fills the 255 registers of a thread at d = 32), so the
// 8 heads of a group belong to a warp pair.  Warp c of the pair owns entries 32c..32c+31
// (n-tiles 4c..4c+3) of every vector and does all the elementwise work on them.  A product
// needs the whole vector as its A operand: both warps stage their halves in the group's
// shared staging matrix, which the grad_B / grad_Q contractions read anyway, meet at a
// pair barrier and load the full 16 x 64 operand from it; each warp then forms its own
// n-tiles of the output over all eight k-steps, in the k order of the one-warp kernels.
// The constant operands (B, B^T, Q^T and Q for a non-symmetric Q) are kept as fp32 pairs in
// fragment order (16 KB each) and split into tf32 hi / lo while loading.  The grad_B /
// grad_Q tiles are dealt out to the row's warps, which meet at one row barrier per step and
// each sum every group's staged vectors in group order: deterministic.
// The kernel is written for any d >= 32; d = 32 builds it only with TTC_ADJ_SPLIT32=1 (there
// the one-warp kernel of lqr_adjoint_mma.cuh is 10 % faster: the operand reloads and pair
// barriers cost more than the doubled occupancy hides).
#pragma once

#include "lqr_adjoint_mma.cuh"

namespace ttc {

template <int D>
struct AdjSplit {
  static_assert(D % 16 == 0 && D >= 32, "d must be a multiple of 16, at least 32");
  static constexpr int NT = D / 8;             // k-steps of a product = n-tiles of a vector
  static constexpr int NH = NT / 2;            // n-tiles a warp of the pair owns
  static constexpr int MT = D / 16;            // m-tiles of grad_B / grad_Q
  // grad_B / grad_Q work units: (matrix, m-tile, part) of NTU n-tiles; at d = 32 each m-tile
  // row is cut in two so that the eight warps of a 32-head row all get one
  static constexpr int kParts = D == 32 ? 2 : 1;
  static constexpr int NTU = NT / kParts;
  static constexpr int kUnits = 2 * MT * kParts;
  // constant operands in fragment order: at d = 32 pre-split tf32 hi / lo (float4 per lane,
  // shared memory is not the limit); at d = 64 fp32 pairs split while loading (16 KB each)
  static constexpr bool kPreSplit = D <= 32;
  static constexpr int kFrag = NT * NT * (kPreSplit ? 128 : 64);
  static constexpr int kMinBlocks = D <= 32 ? 2 : 1;
  static constexpr int SS = AdjMma<D>::SS;     // staging row stride (bank-conflict free)
  static constexpr int kStage = 16 * SS;
  // per group: [lambda; dlambda], [u e^lgB; du e^lgB], [h Dq; dh Dq], double-buffered by step
  // parity, and the two warps' partial log_gamma_A gradients of the 8 heads
  static constexpr int kGroup = 2 * 3 * kStage + 16;
  static constexpr int kRow = 4 * kFrag + 4;   // Q^T, B, B^T, Q, symmetry flag
  static constexpr int kMaxWarps = 8;
  static constexpr int kRowBar = 1;            // named barriers 1.. of the CTA's rows
  static constexpr int kPairBar = 1 + kMaxWarps / 4;  // then those of its pairs
  static constexpr size_t kSmemLimit = 227 * 1024;
  static int groups_per_row(int nh) { return (nh + 7) / 8; }
  static int warps_per_row(int nh) { return 2 * groups_per_row(nh); }
  static size_t bytes_for(int rows, int gpr) {
    return sizeof(float) * ((size_t)rows * kRow + (size_t)rows * gpr * kGroup);
  }
  static int rows_per_cta(int nh) {
    const int wpr = warps_per_row(nh);
    int r = wpr >= kMaxWarps ? 1 : kMaxWarps / wpr;
    while (r > 1 && bytes_for(r, groups_per_row(nh)) > kSmemLimit) --r;
    return r;
  }
  static int warps(int nh) { return warps_per_row(nh) * rows_per_cta(nh); }
  static int units_per_warp(int nh) {
    const int wpr = warps_per_row(nh);
    return (kUnits + wpr - 1) / wpr;
  }
  static size_t bytes(int nh) { return bytes_for(rows_per_cta(nh), groups_per_row(nh)); }
  // More than 8 heads (fewer would leave more than two units of grad tiles per warp), at
  // most kMaxWarps / 2 groups per row.
  static bool fits(int nh) {
    return nh > 8 && warps_per_row(nh) <= kMaxWarps && units_per_warp(nh) <= 2 && bytes(nh) <= kSmemLimit;
  }
};

// Constant operand W (K x N = D x D, W[k][n] = get(k, n)) in fragment order as fp32 pairs:
// for k-step kk, n-tile nj and lane (g, t), (W[8kk + 2t][8nj + g], W[8kk + 2t + 1][8nj + g]).
template <int D, typename Get>
__device__ __forceinline__ void build_operand_pairs(float* dst, Get get, int tid, int nthreads) {
  constexpr int NT = D / 8;
  for (int e = tid; e < NT * NT * 32; e += nthreads) {
    const int lane = e & 31, kn = e >> 5, kk = kn / NT, nj = kn % NT;
    const int g = lane >> 2, t = lane & 3;
    reinterpret_cast<float2*>(dst)[e] = make_float2(get(8 * kk + 2 * t, 8 * nj + g), get(8 * kk + 2 * t + 1, 8 * nj + g));
  }
}

// Warp c's n-tiles of out = S W (S: the 16 x D staged operand, both halves), 3xTF32, k-steps
// in order.  out[jl] is n-tile NH c + jl in output-fragment order.  W: the operand in the
// layout AdjSplit<D>::kPreSplit selects.
template <int D, bool EXACT_W = false>
__device__ __forceinline__ void split_product(const float* S, float (&out)[D / 16][4], const float* W, int c,
                                              int lane, int g, int t) {
  constexpr int NT = D / 8, NH = NT / 2, SS = AdjSplit<D>::SS;
#pragma unroll
  for (int jl = 0; jl < NH; ++jl)
#pragma unroll
    for (int r = 0; r < 4; ++r) out[jl][r] = 0.f;
  const float2* Wc = reinterpret_cast<const float2*>(W) + NH * c * 32 + lane;
  const float4* Wc4 = reinterpret_cast<const float4*>(W) + NH * c * 32 + lane;
#pragma unroll
  for (int kk = 0; kk < NT; ++kk) {
    // a0: row g slot t <- entry 8kk+2t; a1: row g+8 slot t; a2 / a3: slot t+4 <- 8kk+2t+1
    const float2 p0 = *reinterpret_cast<const float2*>(S + g * SS + 8 * kk + 2 * t);
    const float2 p1 = *reinterpret_cast<const float2*>(S + (g + 8) * SS + 8 * kk + 2 * t);
    uint32_t ah[4], al[4];
    wmma::split(p0.x, ah[0], al[0]);
    wmma::split(p1.x, ah[1], al[1]);
    wmma::split(p0.y, ah[2], al[2]);
    wmma::split(p1.y, ah[3], al[3]);
    uint32_t bh0[NH], bl0[NH], bh1[NH], bl1[NH];
#pragma unroll
    for (int jl = 0; jl < NH; ++jl) {
      if constexpr (AdjSplit<D>::kPreSplit) {
        const float4 w = Wc4[(kk * NT + jl) * 32];
        bh0[jl] = __float_as_uint(w.x);
        bh1[jl] = __float_as_uint(w.y);
        bl0[jl] = __float_as_uint(w.z);
        bl1[jl] = __float_as_uint(w.w);
      } else {
        const float2 w = Wc[(kk * NT + jl) * 32];
        wmma::split(w.x, bh0[jl], bl0[jl]);
        wmma::split(w.y, bh1[jl], bl1[jl]);
      }
    }
    // passes over the n-tiles: consecutive MMAs go to independent accumulators
#pragma unroll
    for (int jl = 0; jl < NH; ++jl) wmma::m16n8k8(out[jl], al, bh0[jl], bh1[jl]);
    if constexpr (!EXACT_W) {  // W's residual is zero for bf16 activations (frag_product)
#pragma unroll
      for (int jl = 0; jl < NH; ++jl) wmma::m16n8k8(out[jl], ah, bl0[jl], bl1[jl]);
    }
#pragma unroll
    for (int jl = 0; jl < NH; ++jl) wmma::m16n8k8(out[jl], ah, bh0[jl], bh1[jl]);
  }
}

// Warp c's half (n-tiles NH c ..) of rows g and g + 8 into the staging matrix S.
template <int D>
__device__ __forceinline__ void stage_half(float* S, const float (&v)[D / 16][4], int c, int g, int t) {
  constexpr int NH = D / 16, SS = AdjSplit<D>::SS;
#pragma unroll
  for (int jl = 0; jl < NH; ++jl) {
    const int col = 8 * (NH * c + jl) + 2 * t;
    *reinterpret_cast<float2*>(S + g * SS + col) = make_float2(v[jl][0], v[jl][1]);
    *reinterpret_cast<float2*>(S + (g + 8) * SS + col) = make_float2(v[jl][2], v[jl][3]);
  }
}

// acc[nj][.] += sum_r SX[r][16 mi + m] * SY[(r + 8) % 16][8 (nj0 + nj) + n] over the 16
// staged rows: n-tiles nj0 .. nj0 + NTU - 1 of one m-tile of grad_B / grad_Q, 3xTF32 (the
// sums of accumulate_unit, restricted to the unit's n-tiles).
template <int D, int NTU, bool ONE = false>
__device__ __forceinline__ void accumulate_tiles(float (&acc)[NTU][4], const float* SX, const float* SY, int mi,
                                                 int nj0, int g, int t) {
  constexpr int SS = AdjSplit<D>::SS;
  if constexpr (ONE) {  // single-pass rounded tf32, as accumulate_unit<.., ONE>
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      const float* x0 = SX + (8 * kk + t) * SS + 16 * mi;
      const float* x1 = SX + (8 * kk + t + 4) * SS + 16 * mi;
      const uint32_t a[4] = {wmma::rna(x0[g]), wmma::rna(x0[g + 8]), wmma::rna(x1[g]), wmma::rna(x1[g + 8])};
      const float* y0 = SY + ((8 * kk + t + 8) & 15) * SS + 8 * nj0;
      const float* y1 = SY + ((8 * kk + t + 12) & 15) * SS + 8 * nj0;
#pragma unroll
      for (int nj = 0; nj < NTU; ++nj) wmma::m16n8k8(acc[nj], a, wmma::rna(y0[8 * nj + g]), wmma::rna(y1[8 * nj + g]));
    }
    return;
  }
#pragma unroll
  for (int kk = 0; kk < 2; ++kk) {
    const float* x0 = SX + (8 * kk + t) * SS + 16 * mi;
    const float* x1 = SX + (8 * kk + t + 4) * SS + 16 * mi;
    uint32_t ah[4], al[4];
    wmma::split(x0[g], ah[0], al[0]);
    wmma::split(x0[g + 8], ah[1], al[1]);
    wmma::split(x1[g], ah[2], al[2]);
    wmma::split(x1[g + 8], ah[3], al[3]);
    const float* y0 = SY + ((8 * kk + t + 8) & 15) * SS + 8 * nj0;
    const float* y1 = SY + ((8 * kk + t + 12) & 15) * SS + 8 * nj0;
    uint32_t bh0[NTU], bl0[NTU], bh1[NTU], bl1[NTU];
#pragma unroll
    for (int nj = 0; nj < NTU; ++nj) {
      wmma::split(y0[8 * nj + g], bh0[nj], bl0[nj]);
      wmma::split(y1[8 * nj + g], bh1[nj], bl1[nj]);
    }
#pragma unroll
    for (int nj = 0; nj < NTU; ++nj) wmma::m16n8k8(acc[nj], al, bh0[nj], bh1[nj]);
#pragma unroll
    for (int nj = 0; nj < NTU; ++nj) wmma::m16n8k8(acc[nj], ah, bl0[nj], bl1[nj]);
#pragma unroll
    for (int nj = 0; nj < NTU; ++nj) wmma::m16n8k8(acc[nj], ah, bh0[nj], bh1[nj]);
  }
}

// Backward from the forward's lambda0 and M (d_p = M d_u per head, fused_lqr.py:185-187).
// Grid: ceil(N / R) CTAs of R rows x W = 2 ceil(nh / 8) warps.  Warp w of a row is half
// c = w % 2 of head group w / 2; the pair meets at a named barrier before each product whose
// operand it has just staged, the row's warps at one per step, after which warp w
// accumulates grad_B / grad_Q units w, w + W (UPW at most) over every group's staged vectors
// of that step, in group order.
template <int D, typename TIn, int UPW>
__global__ void __launch_bounds__(256, AdjSplit<D>::kMinBlocks)
lqr_bwd_split_kernel(const TIn* __restrict__ A_diag, const TIn* __restrict__ Bm, const TIn* __restrict__ Qm,
                     const TIn* __restrict__ Rinv, const TIn* __restrict__ lgA, const TIn* __restrict__ lgB,
                     const TIn* __restrict__ lgQ, const TIn* __restrict__ H0, const float* __restrict__ lam0_in,
                     const float* __restrict__ M_in, const TIn* __restrict__ dU, int64_t N, int nh, int T,
                     int rows_per_cta, TIn* __restrict__ gA_out, TIn* __restrict__ gB_out,
                     TIn* __restrict__ gQ_out, TIn* __restrict__ gR_out, TIn* __restrict__ gQf_out,
                     TIn* __restrict__ glgA_out, TIn* __restrict__ glgB_out, TIn* __restrict__ glgQ_out,
                     TIn* __restrict__ gh0_out, int* __restrict__ status) {
  using C = AdjSplit<D>;
  constexpr int NH = C::NH, MT = C::MT, NTU = C::NTU, kP = C::kParts;
  extern __shared__ __align__(128) float smem[];
  const int tid = threadIdx.x, nthreads = blockDim.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int gpr = (nh + 7) / 8, wpr = 2 * gpr;
  const int rloc = warp / wpr, hb = warp % wpr;  // hb: warp index within the row
  const int grp = hb >> 1, c = hb & 1;            // head group, column half
  float* rows_s = smem;
  float* grp_s = smem + (size_t)rows_per_cta * C::kRow;
  float* row_stage = grp_s + (size_t)(rloc * gpr) * C::kGroup;  // group 0 of this row
  float* stg = grp_s + (size_t)(rloc * gpr + grp) * C::kGroup;
  const int pair_bar = C::kPairBar + (warp >> 1);
  auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(pair_bar) : "memory"); };
  auto row_sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(C::kRowBar + rloc), "r"(32 * wpr) : "memory"); };

  bool bad = false;
  const int64_t ngroups = (N + rows_per_cta - 1) / rows_per_cta;
  for (int64_t rg = blockIdx.x; rg < ngroups; rg += gridDim.x) {
    const int64_t n0 = rg * rows_per_cta;
    const int64_t n = n0 + rloc;
    const bool row_ok = n < N;

    // The CTA's rows: constant operands Q^T, B, B^T, Q in fragment order, symmetry flag.
    if (tid < rows_per_cta) reinterpret_cast<int*>(rows_s + tid * C::kRow + 4 * C::kFrag)[0] = 1;
    __syncthreads();
    for (int r = 0; r < rows_per_cta; ++r) {
      const int64_t nr = n0 + r;
      if (nr >= N) break;
      float* base = rows_s + r * C::kRow;
      const TIn* Bn = Bm + nr * (D * D);
      const TIn* Qn = Qm + nr * (D * D);
      auto build = [&](float* dst, auto get) {
        if constexpr (C::kPreSplit) {
          build_operand<D>(dst, get, tid, nthreads);
        } else {
          build_operand_pairs<D>(dst, get, tid, nthreads);
        }
      };
      build(base, [&](int k, int cc) { return ldf(Qn + cc * D + k); });
      build(base + C::kFrag, [&](int k, int cc) { return ldf(Bn + k * D + cc); });
      build(base + 2 * C::kFrag, [&](int k, int cc) { return ldf(Bn + cc * D + k); });
      build(base + 3 * C::kFrag, [&](int k, int cc) { return ldf(Qn + k * D + cc); });
      bool asym = false;
      for (int e = tid; e < D * D; e += nthreads) asym |= ldf(Qn + e) != ldf(Qn + (e % D) * D + e / D);
      if (asym) reinterpret_cast<int*>(base + 4 * C::kFrag)[0] = 0;
    }
    __syncthreads();

    const float* rbase = rows_s + rloc * C::kRow;
    const float* Wqt = rbase;
    const float* Wb = rbase + C::kFrag;
    const float* Wbt = rbase + 2 * C::kFrag;
    const float* Wq = rbase + 3 * C::kFrag;
    const bool sym = reinterpret_cast<const int*>(rbase + 4 * C::kFrag)[0] != 0;

    const int h = grp * 8 + g;
    const bool valid = row_ok && h < nh;
    const int64_t p = valid ? n * nh + h : 0;
    // slot (jl, s) of a thread is entry 8 (NH c + jl) + 2t + s; index 2 + s of a pair array
    // is the tangent
    float a[NH][2], lgQ2[NH][2], lgB2[NH][2], rinv[NH][2];
    float L[NH][4], H[NH][4];
    const float lgA2 = valid ? ldf(lgA + p) * kLog2e : 0.f;
#pragma unroll
    for (int jl = 0; jl < NH; ++jl) {
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const int e = 8 * (NH * c + jl) + 2 * t + s;
        a[jl][s] = valid ? ldf(A_diag + p * D + e) : 0.f;
        lgQ2[jl][s] = valid ? ldf(lgQ + p * D + e) * kLog2e : 0.f;
        lgB2[jl][s] = valid ? ldf(lgB + p * D + e) * kLog2e : 0.f;
        rinv[jl][s] = valid ? ldf(Rinv + p * D + e) : 1.f;
        H[jl][s] = valid ? ldf(H0 + p * D + e) : 0.f;
        H[jl][2 + s] = 0.f;
        L[jl][s] = valid ? lam0_in[p * D + e] : 0.f;
        // d_p = M d_u (fused_lqr.py:185-187): the row of M as 16-byte loads, summed in
        // column order
        float dl = 0.f;
        if (valid) {
          const float4* m4 = reinterpret_cast<const float4*>(M_in + (p * D + e) * D);
#pragma unroll 4
          for (int c4 = 0; c4 < D / 4; ++c4) {
            const float4 mv = m4[c4];
            const float4 dv = ld4(dU + p * D + 4 * c4);
            dl = fmaf(mv.x, dv.x, dl);
            dl = fmaf(mv.y, dv.y, dl);
            dl = fmaf(mv.z, dv.z, dl);
            dl = fmaf(mv.w, dv.w, dl);
          }
        }
        L[jl][2 + s] = dl;
      }
    }

    float gA[NH][2], glgQ[NH][2], gR[NH][2], glgB[NH][2], dqp[NH][2];
    float glgA = 0.f;
#pragma unroll
    for (int jl = 0; jl < NH; ++jl)
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        gA[jl][s] = glgQ[jl][s] = gR[jl][s] = glgB[jl][s] = 0.f;
        dqp[jl][s] = 1.0f;
      }
    float acc[UPW][NTU][4];
#pragma unroll
    for (int q = 0; q < UPW; ++q)
#pragma unroll
      for (int nj = 0; nj < NTU; ++nj)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[q][nj][r] = 0.f;

    // grad_B += lambda (du e^lgB)^T + dlambda (u e^lgB)^T ;
    // grad_Q += (h Dq)(dh Dq)^T + (dh Dq)(h Dq)^T  (the 1/2 is applied at the end)
    // for step ks, from the vectors every group of the row staged for it.
    auto accumulate_step = [&](int ks) {
#pragma unroll
      for (int q = 0; q < UPW; ++q) {
        const int unit = hb + q * wpr;
        if (unit < C::kUnits) {
          const bool isq = unit >= MT * kP;
          if (!isq || ks < T - 1) {
            const int um = isq ? unit - MT * kP : unit;
            const int mi = um / kP, nj0 = (um % kP) * NTU;
            const int off = (ks & 1) * 3 * C::kStage + (isq ? 2 * C::kStage : 0);
            const int offy = (ks & 1) * 3 * C::kStage + (isq ? 2 * C::kStage : C::kStage);
            for (int w = 0; w < gpr; ++w) {
              const float* base = row_stage + (size_t)w * C::kGroup;
              accumulate_tiles<D, NTU, sizeof(TIn) == 2 && TTC_BF16_ONEPASS>(acc[q], base + off, base + offy, mi,
                                                                              nj0, g, t);
            }
          }
        }
      }
    };
    for (int k = 0; k < T; ++k) {
      const float ke = static_cast<float>(k + 1);
      float* S0 = stg + (k & 1) * 3 * C::kStage;  // [lambda; dlambda]
      float* S1 = S0 + C::kStage;                 // [u e^lgB; du e^lgB]
      float* S2 = S0 + 2 * C::kStage;             // [h Dq; dh Dq]
      if (k > 0) {
        // lambda -= Q_k h, dlambda -= Q_k dh with Q_k = Dq Q Dq (symplectic_iter.py:766-775)
        // and the log_gamma_Q gradient of step k-1 (:871-877), from [h Dq; dh Dq] staged by
        // the pair at step k-1 (visible since the row barrier of that step).
        const float* Sp = stg + ((k - 1) & 1) * 3 * C::kStage + 2 * C::kStage;
        float QH[NH][4], QTH[NH][4];
        split_product<D, sizeof(TIn) == 2>(Sp, QH, Wqt, c, lane, g, t);
        if (!sym) split_product<D, sizeof(TIn) == 2>(Sp, QTH, Wq, c, lane, g, t);
#pragma unroll
        for (int jl = 0; jl < NH; ++jl) {
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            const float qh = QH[jl][s], qdh = QH[jl][2 + s];
            const float qth = sym ? qh : QTH[jl][s], qtdh = sym ? qdh : QTH[jl][2 + s];
            L[jl][s] = fmaf(-dqp[jl][s], qh, L[jl][s]);
            L[jl][2 + s] = fmaf(-dqp[jl][s], qdh, L[jl][2 + s]);
            glgQ[jl][s] = fmaf(0.5f * fmaf(H[jl][2 + s], qh + qth, H[jl][s] * (qdh + qtdh)),
                               static_cast<float>(k) * dqp[jl][s], glgQ[jl][s]);
          }
        }
      } else if (valid) {
#pragma unroll
        for (int jl = 0; jl < NH; ++jl)
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            bad |= unstable(L[jl][2 + s]);
            stf(gh0_out + p * D + 8 * (NH * c + jl) + 2 * t + s, L[jl][2 + s]);  // dh_0 = dlambda_0
          }
      }
      const float eA = exp_scaled(lgA2, ke);
      float At[NH][2];
#pragma unroll
      for (int jl = 0; jl < NH; ++jl) {
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          At[jl][s] = fmaf(a[jl][s], eA, 1.0f);
          const float rAt = recip(At[jl][s]);
          L[jl][s] *= rAt;
          L[jl][2 + s] *= rAt;
          const float dA = fmaf(L[jl][s], H[jl][2 + s], L[jl][2 + s] * H[jl][s]);
          gA[jl][s] = fmaf(dA, eA, gA[jl][s]);
          glgA = fmaf(dA * a[jl][s], ke * eA, glgA);
        }
      }
      stage_half<D>(S0, L, c, g, t);
      pair_sync();
      // u = -R_inv (B e^lgB)^T lambda and its tangent (symplectic_iter.py:800-830)
      float UE[NH][4];
      {
        float BL[NH][4];
        split_product<D, sizeof(TIn) == 2>(S0, BL, Wb, c, lane, g, t);
#pragma unroll
        for (int jl = 0; jl < NH; ++jl) {
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            const float eB = exp_scaled(lgB2[jl][s], ke);
            const float bl = BL[jl][s], bdl = BL[jl][2 + s];
            const float u = -(bl * eB) * rinv[jl][s];
            float du = -(bdl * eB) * rinv[jl][s];
            if (k == 0 && valid) du = fmaf(ldf(dU + p * D + 8 * (NH * c + jl) + 2 * t + s), -rinv[jl][s], du);
            glgB[jl][s] = fmaf(fmaf(du, bl, u * bdl), ke * eB, glgB[jl][s]);
            gR[jl][s] = fmaf(-(u * du), recip(rinv[jl][s] * rinv[jl][s]), gR[jl][s]);
            UE[jl][s] = u * eB;
            UE[jl][2 + s] = du * eB;
          }
        }
      }
      stage_half<D>(S1, UE, c, g, t);
      pair_sync();
      // h <- A h + B e^lgB u (symplectic_iter.py:832-850)
      {
        float BU[NH][4];
        split_product<D, sizeof(TIn) == 2>(S1, BU, Wbt, c, lane, g, t);
#pragma unroll
        for (int jl = 0; jl < NH; ++jl) {
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            H[jl][s] = fmaf(H[jl][s], At[jl][s], BU[jl][s]);
            H[jl][2 + s] = fmaf(H[jl][2 + s], At[jl][s], BU[jl][2 + s]);
            dqp[jl][s] = exp_scaled(lgQ2[jl][s], ke);
          }
        }
      }
      if (k < T - 1) {
        float HD[NH][4];
#pragma unroll
        for (int jl = 0; jl < NH; ++jl)
#pragma unroll
          for (int r = 0; r < 4; ++r) HD[jl][r] = H[jl][r] * dqp[jl][r & 1];
        stage_half<D>(S2, HD, c, g, t);
      }
      // Every warp of the row has staged step k (and finished reading step k - 1's buffers).
      row_sync();
      accumulate_step(k);
    }

    // grad_Qf = (h dh^T + dh h^T) / 2 at the final state (symplectic_iter.py:855-857): the
    // pair stages both halves of the final state in the buffer of parity T (last read by the
    // row at step T - 2) and each warp writes the rows i of its half.
    float* S = stg + (T & 1) * 3 * C::kStage;
    stage_half<D>(S, H, c, g, t);
    // log_gamma_A gradient of the head: the two warps' partial sums, added in half order
    float glgA_half = glgA;
    glgA_half += __shfl_xor_sync(0xffffffffu, glgA_half, 1);
    glgA_half += __shfl_xor_sync(0xffffffffu, glgA_half, 2);
    float* ex = stg + 2 * 3 * C::kStage;
    if (t == 0) ex[8 * c + g] = glgA_half;
    pair_sync();
    for (int e = lane; e < 8 * (D / 2) * D; e += 32) {
      const int hh = e / ((D / 2) * D), i = (D / 2) * c + (e / D) % (D / 2), jj = e % D;
      const int h2 = grp * 8 + hh;
      if (row_ok && h2 < nh) {
        const float v = 0.5f * fmaf(S[hh * C::SS + i], S[(hh + 8) * C::SS + jj], S[(hh + 8) * C::SS + i] * S[hh * C::SS + jj]);
        bad |= unstable(v);
        stf(gQf_out + ((n * nh + h2) * D + i) * D + jj, v);
      }
    }
    if (valid) {
#pragma unroll
      for (int jl = 0; jl < NH; ++jl) {
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          const int e = 8 * (NH * c + jl) + 2 * t + s;
          bad |= unstable(gA[jl][s]) | unstable(glgQ[jl][s]) | unstable(gR[jl][s]) | unstable(glgB[jl][s]);
          stf(gA_out + p * D + e, gA[jl][s]);
          stf(glgQ_out + p * D + e, glgQ[jl][s]);
          stf(gR_out + p * D + e, gR[jl][s]);
          stf(glgB_out + p * D + e, glgB[jl][s]);
        }
      }
      if (c == 0 && t == 0) {
        const float v = ex[g] + ex[8 + g];
        bad |= unstable(v);
        stf(glgA_out + p, v);
      }
    }
    if (row_ok) {
      // Each unit holds the sum over all the row's heads.
#pragma unroll
      for (int q = 0; q < UPW; ++q) {
        const int unit = hb + q * wpr;
        if (unit < C::kUnits) {
          const bool isq = unit >= MT * kP;
          const int um = isq ? unit - MT * kP : unit;
          const int mi = um / kP, nj0 = (um % kP) * NTU;
          const float sc = isq ? 0.5f : 1.0f;
          TIn* out = (isq ? gQ_out : gB_out) + n * (D * D);
#pragma unroll
          for (int nj = 0; nj < NTU; ++nj) {
            const int r0 = 16 * mi + g, c0 = 8 * (nj0 + nj) + 2 * t;
            const float v[4] = {sc * acc[q][nj][0], sc * acc[q][nj][1], sc * acc[q][nj][2], sc * acc[q][nj][3]};
            bad |= unstable(v[0]) | unstable(v[1]) | unstable(v[2]) | unstable(v[3]);
            stf(out + r0 * D + c0, v[0]);
            stf(out + r0 * D + c0 + 1, v[1]);
            stf(out + (r0 + 8) * D + c0, v[2]);
            stf(out + (r0 + 8) * D + c0 + 1, v[3]);
          }
        }
      }
    }
    __syncthreads();  // the next row group reuses the shared operands and staging
  }
  if (bad) atomicOr(status, TTC_STATUS_BWD_UNSTABLE);
}

}  // namespace ttc
