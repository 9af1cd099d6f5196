// TTC LQR solve for B200 (sm_100a): the closed-loop trajectory of a solved problem.
//
// From the forward's lambda0 = P h0 (and, with an affine action cost r0 on step 0,
// lambda0 += M r0 where M = Y1^-1 Y3 and Y3 = -Y2 B R^-1 of the sweep's last step -- the
// y3 = Y3 r of the reference's IS_AFFINE sweep, symplectic_iter.py:211-238), the state and
// costate are integrated forward in time with the primal half of the reference's adjoint
// (symplectic_iter.py:766-845):
//     k > 0:  lambda -= Q_k h                          (Q_k = Dq_k Q Dq_k, exponent k)
//     lambda /= A_{k+1}                                 (A_e = 1 + A_diag e^{lgA e})
//     u_k = -R_inv (B_{k+1}^T lambda)   (k = 0: - R_inv r0)
//     h   = A_{k+1} h + B_{k+1} u_k
// which gives the actions of solve_traj_actions(..., r_traj, return_traj=True) and the
// states / costates / total cost of solve_traj_states (lin_solver_lqr.py:13-110,187-203)
// with r_traj zero after step 0.  With an affine cost on every step (r_steps = T, the
// CUDA-core kernel) lambda0 comes from the per-step affine forward, which already holds every
// r_t's offset, and u_k -= R_inv r_k on every step.  Per head and step it writes u_k [du] (activation dtype)
// and, optionally, h_{k+1} [d] and lambda_{k+1} [d] (fp32, as the reference's fp32
// buffers); per head, optionally, lambda0 and the total cost
//     sum_k 0.5 h_{k+1}^T Q_k h_{k+1} + 0.5 u_k^T R u_k + r_k^T u_k      (Q_{T-1} = Q_f).
//
// Grid: one CTA per row n; the row's B and Q sit in padded shared copies and the CTA's
// groups of D threads walk the row's heads, H heads at a time (their step chains interleave
// and share the matrix rows each thread holds), thread i carrying entry i of h and lambda
// (and of u for i < du).  Fixed summation order: results are reproducible run to run.
#pragma once

#include "lqr_adjoint_mma.cuh"
#include "lqr_kernels.cuh"

namespace ttc {

template <int D, int DU, int H>
struct RolloutLayout {
  // per step parity and head: lambda [D], h Dq [D], u e^{lgB} [DU]
  static constexpr int kBuf = 2 * D + DU;
  static constexpr int kGroup = round4(2 * H * kBuf + H * DU + 2);  // + r0 [H][DU], group_sum scratch
  static constexpr int kBp = round4(D * (DU + 1));
  static constexpr int kQp = round4(D * (D + 1));
  static constexpr int kShared = kBp + kQp;
  static size_t bytes(int groups) { return sizeof(float) * (size_t)(kShared + groups * kGroup); }
};

__device__ __forceinline__ bool nonfinite(float v) { return !isfinite(v); }

// Rows of Q and B and the column of B a thread multiplies with every step, held in registers
// (2d + du floats at d = 16, the Q and B rows at d = 32) instead of being re-read from shared
// memory: the step's matrix-vector products then issue only their FMAs and the broadcast
// vector loads.  At d = 64 they stay in shared memory.
#ifndef TTC_ROLL_CACHE16
#define TTC_ROLL_CACHE16 2
#endif
#ifndef TTC_ROLL_CACHE32
#define TTC_ROLL_CACHE32 1
#endif
#ifndef TTC_ROLL_HEADS16
#define TTC_ROLL_HEADS16 1
#endif
#ifndef TTC_ROLL_HEADS32
#define TTC_ROLL_HEADS32 1
#endif
#ifndef TTC_ROLL_THREADS
#define TTC_ROLL_THREADS 128
#endif
template <int D>
__host__ __device__ constexpr int rollout_cache() {
  return D <= 16 ? TTC_ROLL_CACHE16 : (D <= 32 ? TTC_ROLL_CACHE32 : 0);
}

// Heads a group carries at once (interleaved step chains sharing the thread's matrix rows).
// Measured at config-2 and config-3 shapes, one head per group with 128-thread CTAs is the
// fastest: the kernel is bound by instruction issue, not by the latency of a step's chain.
template <int D>
__host__ __device__ constexpr int rollout_heads() {
  return D <= 16 ? TTC_ROLL_HEADS16 : (D <= 32 ? TTC_ROLL_HEADS32 : 1);
}

// Threads per CTA (a multiple of 64, so of D) and the resident CTAs asked of ptxas: the
// register cap is 65536 / (threads * CTAs) = 128 per thread at d <= 32.
constexpr int kRollThreads = TTC_ROLL_THREADS;
template <int D>
__host__ __device__ constexpr int rollout_min_ctas() {
  return D <= 32 ? 65536 / (kRollThreads * 128) : 1;
}

template <int D, int DU, typename TIn, int H>
__global__ void __launch_bounds__(kRollThreads, rollout_min_ctas<D>())
lqr_rollout_kernel(const TIn* __restrict__ A_diag, const TIn* __restrict__ Bm,
                   const TIn* __restrict__ Qm, const TIn* __restrict__ Rinv,
                   const TIn* __restrict__ lgA, const TIn* __restrict__ lgB,
                   const TIn* __restrict__ lgQ, const TIn* __restrict__ H0,
                   const TIn* __restrict__ Qf, const float* __restrict__ lam0_in,
                   const float* __restrict__ M_in, const TIn* __restrict__ R0, int r_steps, int nh, int T,
                   TIn* __restrict__ u_out, float* __restrict__ h_out,
                   float* __restrict__ lam_out, float* __restrict__ lam0_out,
                   float* __restrict__ cost_out, int* __restrict__ status) {
  static_assert(D % 4 == 0 && DU % 4 == 0, "dimensions must be multiples of 4");
  using L = RolloutLayout<D, DU, H>;
  constexpr int kB = L::kBuf;
  extern __shared__ __align__(128) float smem[];
  float* sBp = smem;          // [D][DU+1]
  float* sQp = sBp + L::kBp;  // [D][D+1]
  const int ngroups = blockDim.x / D;
  const Group<D> G(threadIdx.x);
  float* buf = smem + L::kShared + G.g * L::kGroup;  // [2][H][kB]
  float* sr0 = buf + 2 * H * kB;                     // [H][DU]
  float* red = sr0 + H * DU;

  const int64_t n = blockIdx.x;
  const int tid = threadIdx.x;
  for (int e = tid; e < D * DU; e += blockDim.x)
    sBp[(e / DU) * (DU + 1) + (e % DU)] = ldf(Bm + n * (D * DU) + e);
  for (int e = tid; e < D * D; e += blockDim.x)
    sQp[(e / D) * (D + 1) + (e % D)] = ldf(Qm + n * (D * D) + e);
  __syncthreads();

  const int i = G.i;
  constexpr int kC = rollout_cache<D>();
  f2 qrow_r[kC >= 1 ? D / 2 : 1], brow_r[kC >= 1 ? DU / 2 : 1], bcol_r[kC >= 2 ? D / 2 : 1];
  auto ld_qrow = [&](int j2) { return pk2(sQp[i * (D + 1) + 2 * j2], sQp[i * (D + 1) + 2 * j2 + 1]); };
  auto ld_brow = [&](int j2) { return pk2(sBp[i * (DU + 1) + 2 * j2], sBp[i * (DU + 1) + 2 * j2 + 1]); };
  auto ld_bcol = [&](int r2) {
    return i < DU ? pk2(sBp[2 * r2 * (DU + 1) + i], sBp[(2 * r2 + 1) * (DU + 1) + i]) : f2(0);
  };
  if constexpr (kC >= 1) {
#pragma unroll
    for (int j2 = 0; j2 < D / 2; ++j2) qrow_r[j2] = ld_qrow(j2);
#pragma unroll
    for (int j2 = 0; j2 < DU / 2; ++j2) brow_r[j2] = ld_brow(j2);
  }
  if constexpr (kC >= 2) {
#pragma unroll
    for (int r2 = 0; r2 < D / 2; ++r2) bcol_r[r2] = ld_bcol(r2);
  }
  auto qrow = [&](int j2) { if constexpr (kC >= 1) return qrow_r[j2]; else return ld_qrow(j2); };
  auto brow = [&](int j2) { if constexpr (kC >= 1) return brow_r[j2]; else return ld_brow(j2); };
  auto bcol = [&](int r2) { if constexpr (kC >= 2) return bcol_r[r2]; else return ld_bcol(r2); };
  bool bad = false;
  for (int h0 = G.g * H; h0 < nh; h0 += ngroups * H) {
    // Heads h0 .. h0+H-1; a head past nh repeats the last one and writes nothing.
    int64_t p[H];
    bool valid[H];
    float a[H], lgA2[H], lgQ2[H], lgB2[H], rinv[H], rrinv[H], r0i[H], hs[H], lam[H], cost[H],
        dq_prev[H], At[H];
#pragma unroll
    for (int m = 0; m < H; ++m) {
      valid[m] = h0 + m < nh;
      p[m] = n * nh + (valid[m] ? h0 + m : nh - 1);
      a[m] = ldf(A_diag + p[m] * D + i);
      lgA2[m] = ldf(lgA + p[m]) * kLog2e;
      lgQ2[m] = ldf(lgQ + p[m] * D + i) * kLog2e;
      lgB2[m] = rinv[m] = r0i[m] = 0.f;
      if (i < DU) {
        lgB2[m] = ldf(lgB + p[m] * DU + i) * kLog2e;
        rinv[m] = ldf(Rinv + p[m] * DU + i);
        if (R0 != nullptr) r0i[m] = ldf(R0 + p[m] * r_steps * DU + i);
        sr0[m * DU + i] = r0i[m];
      }
      rrinv[m] = i < DU ? recip(rinv[m]) : 0.f;
      hs[m] = ldf(H0 + p[m] * D + i);
      lam[m] = lam0_in[p[m] * D + i];
      cost[m] = 0.f;
      dq_prev[m] = 1.0f;  // exp(lgQ_i k) at the top of step k
    }
    G.sync();  // sr0 visible to the group
    if (R0 != nullptr && M_in != nullptr) {
      // lambda0 += M r0: the affine offset Y1^-1 (Y3 r0).
#pragma unroll
      for (int m = 0; m < H; ++m) {
        const float* mrow = M_in + (p[m] * D + i) * DU;
        float acc = 0.f;
#pragma unroll 4
        for (int j = 0; j < DU; ++j) acc = fmaf(mrow[j], sr0[m * DU + j], acc);
        lam[m] += acc;
      }
    }
#pragma unroll
    for (int m = 0; m < H; ++m)
      if (lam0_out != nullptr && valid[m]) lam0_out[p[m] * D + i] = lam[m];
    for (int k = 0; k < T; ++k) {
      float* cb = buf + (k & 1) * H * kB;
      const float* pb = buf + ((k + 1) & 1) * H * kB;
      const float ke = static_cast<float>(k + 1);
#pragma unroll
      for (int m = 0; m < H; ++m) {
        if (k > 0) {
          // lambda -= Dq Q Dq h: row i of Q against the previous step's Dq h.
          const float4* h4 = reinterpret_cast<const float4*>(pb + m * kB + D);
          f2 s0 = 0, s1 = 0;
#pragma unroll
          for (int j4 = 0; j4 < D / 4; ++j4) {
            const float4 hv = h4[j4];
            s0 = fma2(qrow(2 * j4), lo2(hv), s0);
            s1 = fma2(qrow(2 * j4 + 1), hi2(hv), s1);
          }
          const float qh = dq_prev[m] * (sum2(s0) + sum2(s1));  // (Q_{k-1} h_k)_i
          lam[m] -= qh;
          cost[m] = fmaf(0.5f * hs[m], qh, cost[m]);
        }
        At[m] = fmaf(a[m], exp_scaled(lgA2[m], ke), 1.0f);
        lam[m] *= recip(At[m]);
        cb[m * kB + i] = lam[m];
      }
      G.sync();
      if (i < DU) {
#pragma unroll
        for (int m = 0; m < H; ++m) {
          // u = -R_inv e^{lgB} (B^T lambda): column i of B against lambda.
          const float4* l4 = reinterpret_cast<const float4*>(cb + m * kB);
          f2 s0 = 0, s1 = 0;
#pragma unroll
          for (int r4 = 0; r4 < D / 4; ++r4) {
            const float4 lv = l4[r4];
            s0 = fma2(bcol(2 * r4), lo2(lv), s0);
            s1 = fma2(bcol(2 * r4 + 1), hi2(lv), s1);
          }
          const float eB = exp_scaled(lgB2[m], ke);
          float u = -((sum2(s0) + sum2(s1)) * eB) * rinv[m];
          // the affine cost of step k: r0 on step 0, or row k of r [T][DU]
          float rk = k == 0 ? r0i[m] : 0.f;
          if (k > 0 && k < r_steps && R0 != nullptr) rk = ldf(R0 + (p[m] * r_steps + k) * DU + i);
          u = fmaf(rk, -rinv[m], u);
          cost[m] = fmaf(0.5f * u, u * rrinv[m], cost[m]);
          cost[m] = fmaf(rk, u, cost[m]);
          cb[m * kB + 2 * D + i] = u * eB;
          bad |= nonfinite(u);
          if (valid[m]) stf(u_out + (p[m] * T + k) * DU + i, u);
        }
      }
      G.sync();
#pragma unroll
      for (int m = 0; m < H; ++m) {
        // h = A h + B (e^{lgB} u): row i of B against the scaled action.
        const float4* u4 = reinterpret_cast<const float4*>(cb + m * kB + 2 * D);
        f2 s0 = 0, s1 = 0;
#pragma unroll
        for (int j4 = 0; j4 < DU / 4; ++j4) {
          const float4 uv = u4[j4];
          s0 = fma2(brow(2 * j4), lo2(uv), s0);
          s1 = fma2(brow(2 * j4 + 1), hi2(uv), s1);
        }
        hs[m] = fmaf(hs[m], At[m], sum2(s0) + sum2(s1));
        bad |= nonfinite(hs[m] + lam[m]);
        if (valid[m]) {
          if (h_out != nullptr) h_out[(p[m] * T + k) * D + i] = hs[m];
          if (lam_out != nullptr) lam_out[(p[m] * T + k) * D + i] = lam[m];
        }
        const float dq = exp_scaled(lgQ2[m], ke);
        cb[m * kB + D + i] = hs[m] * dq;
        dq_prev[m] = dq;
      }
      G.sync();
    }
    if (cost_out != nullptr) {
      // Terminal term 0.5 h_T^T Q_f h_T: row i of Q_f against h_T (in the free buffer).
      float* hT = buf + (T & 1) * H * kB;
#pragma unroll
      for (int m = 0; m < H; ++m) hT[m * kB + i] = hs[m];
      G.sync();
#pragma unroll
      for (int m = 0; m < H; ++m) {
        const TIn* qf = Qf + (p[m] * D + i) * D;
        float acc = 0.f;
#pragma unroll 4
        for (int j = 0; j < D; ++j) acc = fmaf(ldf(qf + j), hT[m * kB + j], acc);
        cost[m] = fmaf(0.5f * hs[m], acc, cost[m]);
        const float total = group_sum<D>(G, cost[m], red);
        bad |= nonfinite(total);
        if (i == 0 && valid[m]) cost_out[p[m]] = total;
      }
      G.sync();
    }
  }
  if (bad) atomicOr(status, TTC_STATUS_TRAJ_NONFINITE);
}

// --------------------------------------------------------------------------------------
// The same rollout on warp-level tensor-core MMAs, for d = du in {16, 32}.  All heads of a
// batch row share B and Q, so a step of 16 heads is three small matrix products
// [h Dq] Q^T, [lambda] B and [u e^lgB] B^T: one warp carries 16 heads of a row as the 16
// rows of mma.sync.m16n8k8 (3xTF32, the operand layout and K permutation of the warp-MMA
// adjoint: thread (g, t) = (lane / 4, lane % 4) holds entries {8j + 2t, 8j + 2t + 1} of heads
// g and g + 8), and every elementwise update is thread-local.  Grid: ceil(N / R) CTAs of R
// rows x ceil(nh / 16) warps; the rows' operands are built once per CTA in shared memory.
// --------------------------------------------------------------------------------------
template <int D>
struct RollMma {
  static constexpr int NT = D / 8;
  static constexpr int kFrag = AdjMma<D>::kFrag;
  static constexpr int SS = AdjMma<D>::SS;
  static constexpr int kRow = 3 * kFrag;        // Q^T, B, B^T
  static constexpr int kWarp = 16 * SS;         // final-state staging for the terminal cost
  static constexpr int kMaxWarps = 8;
  __host__ __device__ static int warps_per_row(int nh) { return (nh + 15) / 16; }
  static int rows_per_cta(int nh) {
    const int wpr = warps_per_row(nh);
    return wpr >= kMaxWarps ? 1 : kMaxWarps / wpr;
  }
  static int warps(int nh) { return warps_per_row(nh) * rows_per_cta(nh); }
  static size_t bytes(int nh) {
    return sizeof(float) * ((size_t)rows_per_cta(nh) * kRow + (size_t)warps(nh) * kWarp);
  }
  static bool fits(int nh) { return warps_per_row(nh) <= kMaxWarps && bytes(nh) <= 227 * 1024; }
};

__device__ __forceinline__ void st_pair(float* p, float a, float b) {
  *reinterpret_cast<float2*>(p) = make_float2(a, b);
}
__device__ __forceinline__ void st_pair(__nv_bfloat16* p, float a, float b) {
  *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
}

template <int D, typename TIn>
__global__ void __launch_bounds__(256, D <= 16 ? 2 : 1)
lqr_rollout_mma_kernel(const TIn* __restrict__ A_diag, const TIn* __restrict__ Bm,
                       const TIn* __restrict__ Qm, const TIn* __restrict__ Rinv,
                       const TIn* __restrict__ lgA, const TIn* __restrict__ lgB,
                       const TIn* __restrict__ lgQ, const TIn* __restrict__ H0,
                       const TIn* __restrict__ Qf, const float* __restrict__ lam0_in,
                       const float* __restrict__ M_in, const TIn* __restrict__ R0, int64_t N,
                       int nh, int T, int rows_per_cta, TIn* __restrict__ u_out,
                       float* __restrict__ h_out, float* __restrict__ lam_out,
                       float* __restrict__ lam0_out, float* __restrict__ cost_out,
                       int* __restrict__ status) {
  using C = RollMma<D>;
  constexpr int NT = C::NT, SS = C::SS;
  extern __shared__ __align__(128) float smem[];
  const int tid = threadIdx.x, nthreads = blockDim.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int wpr = C::warps_per_row(nh);
  const int rloc = warp / wpr, hb = warp % wpr;
  float* rows_s = smem;
  float* stg = smem + (size_t)rows_per_cta * C::kRow + (size_t)warp * C::kWarp;
  const int64_t n0 = (int64_t)blockIdx.x * rows_per_cta;
  for (int r = 0; r < rows_per_cta; ++r) {
    const int64_t nr = n0 + r;
    if (nr >= N) break;
    float* base = rows_s + r * C::kRow;
    const TIn* Bn = Bm + nr * (D * D);
    const TIn* Qn = Qm + nr * (D * D);
    build_operand<D>(base, [&](int k, int c) { return ldf(Qn + c * D + k); }, tid, nthreads);
    build_operand<D>(base + C::kFrag, [&](int k, int c) { return ldf(Bn + k * D + c); }, tid, nthreads);
    build_operand<D>(base + 2 * C::kFrag, [&](int k, int c) { return ldf(Bn + c * D + k); }, tid, nthreads);
  }
  __syncthreads();
  const int64_t n = n0 + rloc;
  // Past the last row there is nothing to write and that row's operands were not built: the
  // warp stops here (no CTA-wide barrier follows).
  if (n >= N) return;
  const float* rbase = rows_s + rloc * C::kRow;
  const float4* Wqt = reinterpret_cast<const float4*>(rbase);
  const float4* Wb = reinterpret_cast<const float4*>(rbase + C::kFrag);
  const float4* Wbt = reinterpret_cast<const float4*>(rbase + 2 * C::kFrag);

  // rows q = 0, 1 of this thread: heads g and g + 8 of the warp's 16
  bool valid[2];
  int64_t p[2];
  float lgA2[2], cost[2] = {0.f, 0.f};
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int h = hb * 16 + g + 8 * q;
    valid[q] = h < nh;
    p[q] = valid[q] ? n * nh + h : 0;
    lgA2[q] = valid[q] ? ldf(lgA + p[q]) * kLog2e : 0.f;
  }
  // r0 of the warp's 16 heads into its staging rows (coalesced; read back per entry)
  if (R0 != nullptr) {
    for (int e = lane; e < 16 * D; e += 32) {
      const int hr = e / D, h = hb * 16 + hr;
      stg[hr * SS + e % D] = h < nh ? ldf(R0 + (n * nh + h) * D + e % D) : 0.f;
    }
    __syncwarp();
  }
  // fragment index [j][2q + s] <-> head row q, entry 8j + 2t + s; a head past nh runs on
  // zeros (finite with the row's operands) and writes nothing
  float a[NT][4], lgQ2[NT][4], lgB2[NT][4], rinv[NT][4], dqp[NT][4], H[NT][4], L[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int q = 0; q < 2; ++q)
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const int r = 2 * q + s, e = 8 * j + 2 * t + s;
        const bool v = valid[q];
        const int64_t pe = p[q] * D + e;
        a[j][r] = v ? ldf(A_diag + pe) : 0.f;
        lgQ2[j][r] = v ? ldf(lgQ + pe) * kLog2e : 0.f;
        lgB2[j][r] = v ? ldf(lgB + pe) * kLog2e : 0.f;
        rinv[j][r] = v ? ldf(Rinv + pe) : 1.f;
        H[j][r] = v ? ldf(H0 + pe) : 0.f;
        float lam = v ? lam0_in[pe] : 0.f;
        if (v && R0 != nullptr) {
          // lambda0 += M r0: the affine offset Y1^-1 (Y3 r0)
          const float4* mrow = reinterpret_cast<const float4*>(M_in + pe * D);
          const float* r0 = stg + (g + 8 * q) * SS;
#pragma unroll 4
          for (int c4 = 0; c4 < D / 4; ++c4) {
            const float4 m = mrow[c4];
            lam = fmaf(m.x, r0[4 * c4], lam);
            lam = fmaf(m.y, r0[4 * c4 + 1], lam);
            lam = fmaf(m.z, r0[4 * c4 + 2], lam);
            lam = fmaf(m.w, r0[4 * c4 + 3], lam);
          }
        }
        L[j][r] = lam;
        dqp[j][r] = 1.0f;
      }
  if (lam0_out != nullptr) {
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int q = 0; q < 2; ++q)
        if (valid[q]) st_pair(lam0_out + p[q] * D + 8 * j + 2 * t, L[j][2 * q], L[j][2 * q + 1]);
  }
  bool bad = false;
  for (int k = 0; k < T; ++k) {
    const float ke = static_cast<float>(k + 1);
    if (k > 0) {
      // lambda -= Dq Q Dq h
      float HD[NT][4], QH[NT][4];
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int r = 0; r < 4; ++r) HD[j][r] = H[j][r] * dqp[j][r];
      frag_product<D, sizeof(TIn) == 2>(HD, QH, Wqt, lane);
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const float qh = dqp[j][r] * QH[j][r];  // (Q_{k-1} h_k)_e
          L[j][r] -= qh;
          cost[r >> 1] = fmaf(0.5f * H[j][r], qh, cost[r >> 1]);
        }
    }
    float At[NT][4];
    {
      const float eA[2] = {exp_scaled(lgA2[0], ke), exp_scaled(lgA2[1], ke)};
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          At[j][r] = fmaf(a[j][r], eA[r >> 1], 1.0f);
          L[j][r] *= recip(At[j][r]);
        }
    }
    // u = -R_inv e^lgB (B^T lambda); step 0: - R_inv r0
    float UE[NT][4];
    {
      float BL[NT][4];
      frag_product<D, sizeof(TIn) == 2>(L, BL, Wb, lane);
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        float u[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const float eB = exp_scaled(lgB2[j][r], ke);
          u[r] = -(BL[j][r] * eB) * rinv[j][r];
          if (k == 0 && R0 != nullptr && valid[r >> 1]) {
            const float r0 = stg[(g + 8 * (r >> 1)) * SS + 8 * j + 2 * t + (r & 1)];
            u[r] = fmaf(r0, -rinv[j][r], u[r]);
            cost[r >> 1] = fmaf(r0, u[r], cost[r >> 1]);
          }
          cost[r >> 1] = fmaf(0.5f * u[r], u[r] * recip(rinv[j][r]), cost[r >> 1]);
          bad |= nonfinite(u[r]);
          UE[j][r] = u[r] * eB;
        }
#pragma unroll
        for (int q = 0; q < 2; ++q)
          if (valid[q]) st_pair(u_out + (p[q] * T + k) * D + 8 * j + 2 * t, u[2 * q], u[2 * q + 1]);
      }
    }
    // h = A h + B (e^lgB u)
    {
      float BU[NT][4];
      frag_product<D, sizeof(TIn) == 2>(UE, BU, Wbt, lane);
#pragma unroll
      for (int j = 0; j < NT; ++j) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          H[j][r] = fmaf(H[j][r], At[j][r], BU[j][r]);
          bad |= nonfinite(H[j][r] + L[j][r]);
          dqp[j][r] = exp_scaled(lgQ2[j][r], ke);
        }
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          if (!valid[q]) continue;
          const int64_t o = (p[q] * T + k) * D + 8 * j + 2 * t;
          if (h_out != nullptr) st_pair(h_out + o, H[j][2 * q], H[j][2 * q + 1]);
          if (lam_out != nullptr) st_pair(lam_out + o, L[j][2 * q], L[j][2 * q + 1]);
        }
      }
    }
  }
  if (cost_out != nullptr) {
    // terminal 0.5 h_T^T Q_f h_T: the final states through the warp's staging rows (which
    // held r0 until step 0)
    __syncwarp();
    stage_rows<D>(stg, H, g, t);
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const float* hrow = stg + (g + 8 * q) * SS;
      if (valid[q]) {
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            const int e = 8 * j + 2 * t + s;
            const TIn* qf = Qf + (p[q] * D + e) * D;
            float acc = 0.f;
#pragma unroll 4
            for (int c = 0; c < D; ++c) acc = fmaf(ldf(qf + c), hrow[c], acc);
            cost[q] = fmaf(0.5f * hrow[e], acc, cost[q]);
          }
      }
      float c = cost[q];
      c += __shfl_xor_sync(0xffffffffu, c, 1);
      c += __shfl_xor_sync(0xffffffffu, c, 2);
      bad |= nonfinite(c);
      if (valid[q] && t == 0) cost_out[p[q]] = c;
    }
  }
  if (bad) atomicOr(status, TTC_STATUS_TRAJ_NONFINITE);
}

}  // namespace ttc
