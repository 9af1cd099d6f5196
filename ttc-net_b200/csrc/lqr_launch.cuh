// Kernel launchers, explicitly instantiated per (d, du, dtype) in inst_*.cu so the
// sm_100a build compiles in parallel; the C-ABI in ttc_abi.cu dispatches to them.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>

#include "lqr_adjoint_mma.cuh"
#include "lqr_adjoint_split.cuh"
#include "lqr_rollout.cuh"
#include "lqr_tc.cuh"

namespace ttc {

// Records `msg` as the text returned by ttc_last_error() and returns `code`.
int set_error(int code, const char* msg);

inline int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return TTC_OK;
  char buf[400];
  snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
  return set_error(TTC_ERR_CUDA, buf);
}

// Groups (heads in flight) per CTA: up to kThreads / d threads, at most one per head.
// D > 32 groups use named barriers 1..15, and kThreads / 64 = 4 stays below that.
inline int groups_for(int nh, int d) {
  int g = kThreads / d;
  if (g > nh) g = nh;
  return g < 1 ? 1 : g;
}

// Q_f given as the layer's rank-rQ mixture instead of [N, nh, d, d]: the Q_f argument then
// holds coeff_Qf [N*nh, rQ] and `basis` [rQ, d, d] (activation dtype); the backward writes
// grad_coeff [N*nh, rQ] in place of grad_Q_f and per-warp partial sums of the basis
// gradient (`grad_basis_partial`, slices x [rQ, d, d] fp32).
struct QMix {
  const void* basis = nullptr;
  int rank = 0;
  void* grad_coeff = nullptr;
  float* grad_basis_partial = nullptr;
  // B and Q given as the layer's low-rank mixtures as well (needs the Q_f mixture): the B and
  // Q arguments are then unused.  B = sum_r coeff_B[n][r] B_basis[r] (B_basis [rB, d, du]),
  // Q = sum_r coeff_Q[n][r] basis[r]; the backward writes grad_coeff_B [N, rB],
  // grad_coeff_Q [N, rQ], adds the Q-basis terms to grad_basis_partial and writes the
  // B-basis terms to grad_B_basis_partial (slices x [rB, d, du] fp32), in place of grad_B
  // and grad_Q.
  const void* coeff_B = nullptr;
  const void* B_basis = nullptr;
  int rB = 0;
  const void* coeff_Q = nullptr;
  void* grad_coeff_B = nullptr;
  void* grad_coeff_Q = nullptr;
  float* grad_B_basis_partial = nullptr;
  template <typename TIn>
  LowRank<TIn> lowrank() const {
    LowRank<TIn> lr;
    lr.cB = static_cast<const TIn*>(coeff_B);
    lr.Bb = static_cast<const TIn*>(B_basis);
    lr.rB = rB;
    lr.cQ = static_cast<const TIn*>(coeff_Q);
    lr.gcB = static_cast<TIn*>(grad_coeff_B);
    lr.gcQ = static_cast<TIn*>(grad_coeff_Q);
    lr.gBb = grad_B_basis_partial;
    return lr;
  }
};

template <int D, int DU, typename TIn>
int launch_fwd(const void* A, const void* B, const void* Q, const void* R, const void* Qf,
               const void* lA, const void* lB, const void* lQ, const void* h0, int64_t N, int nh,
               int T, void* u, float* lam0, float* M, int* status, const QMix& mix, int opts,
               cudaStream_t st);

template <int D, int DU, typename TIn>
int launch_bwd(const void* A, const void* B, const void* Q, const void* R, const void* Qf,
               const void* lA, const void* lB, const void* lQ, const void* h0, const float* lam0,
               const float* M, const void* dU, int64_t N, int nh, int T, void* const* g,
               int* status, const QMix& mix, int opts, cudaStream_t st);

// Partial slices (one per CTA) the mixed-Q_f backward writes for (N, nh) on the current
// device; 0 when the mixed path is not available for the shape and rank, -TTC_ERR_CUDA on
// a CUDA error.
template <int D, int DU, typename TIn>
int64_t bwd_mix_slices(int64_t N, int nh, int rQ);

// Forward with an affine action cost on every step (r_traj [N, nh, T, du]): lambda0 of the
// affine problem and u_0, no M.
template <int D, int DU, typename TIn>
int launch_fwd_affine(const void* A, const void* B, const void* Q, const void* R, const void* Qf,
                      const void* lA, const void* lB, const void* lQ, const void* h0, const void* r_traj,
                      int64_t N, int nh, int T, void* u, float* lam0, int* status, int opts, cudaStream_t st);

// Closed-loop trajectory from the forward's lambda0: r_steps = 1, an affine cost r0 on step 0
// (lambda0 += M r0); r_steps = T, one on every step (r [N, nh, T, du], lambda0 from
// launch_fwd_affine, no M).
template <int D, int DU, typename TIn>
int launch_rollout(const void* A, const void* B, const void* Q, const void* R, const void* Qf,
                   const void* lA, const void* lB, const void* lQ, const void* h0,
                   const float* lam0, const float* M, const void* r0, int r_steps, int64_t N, int nh,
                   int T, void* u, float* hs, float* lams, float* lam0_out, float* cost, int* status,
                   cudaStream_t st);

#ifdef TTC_DEFINE_LAUNCHERS
constexpr size_t kMaxSmem = 227 * 1024;

// Largest d whose saved-state backward runs on the warp-MMA adjoint.
#ifndef TTC_ADJ_MMA_MAXD
#define TTC_ADJ_MMA_MAXD 32
#endif

// Tile slots per CTA for the tensor-core forward: one per 128-row tile of a row, at most
// TcLaunch<D>::kMaxSlots (TMEM: 4 x 96 columns at d = 32), fewer if the shared-memory
// layout would not fit.
template <int D, int DU, bool SAVE_M>
int tc_slots(int nh) {
  using CF = TcCfg<D, DU>;
  const int tiles = (nh * D + 127) / 128;
  int s = tiles < TcLaunch<D>::kMaxSlots ? tiles : TcLaunch<D>::kMaxSlots;
  while (s > 1 && TcFwdLayout<D, DU, SAVE_M>::bytes(s) > kMaxSmem) --s;
  (void)sizeof(CF);
  return s;
}

inline uint32_t tmem_cols_for(int cols) {
  uint32_t c = 32;
  while (c < static_cast<uint32_t>(cols)) c <<= 1;
  return c;
}

template <typename Kern>
int set_smem(Kern k, size_t bytes) {
  if (bytes <= 48 * 1024) return TTC_OK;
  return cuda_check(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes),
                    "cudaFuncSetAttribute");
}

// Two CTAs of two slots per SM at d = 32 (TcLaunch NARROW) when both fit the SM's shared
// memory (TTC_FWD_NARROW=0 builds keep one CTA of four slots).
#ifndef TTC_FWD_NARROW
#define TTC_FWD_NARROW 1
#endif
constexpr size_t kSmPerSm = 228 * 1024;  // shared memory of an SM (each CTA also reserves 1 KB)
// Launch epochs of the forward kernels of this translation unit (for their staggering words).
static std::atomic<unsigned> g_fwd_epoch{0};
inline unsigned next_fwd_epoch() {
  unsigned e = ++g_fwd_epoch;
  while (e == 0) e = ++g_fwd_epoch;
  return e;
}

template <int D, int DU, typename TIn, bool SAVE_M, bool AFF = false>
int launch_fwd_tc(const void* A, const void* B, const void* Q, const void* R, const void* Qf,
                  const void* lA, const void* lB, const void* lQ, const void* h0, int64_t N,
                  int nh, int T, void* u, float* lam0, float* M, int* status, const QMix& mix,
                  int opts, cudaStream_t st, const void* r_traj = nullptr) {
  using CF = TcCfg<D, DU>;
  using L = TcFwdLayout<D, DU, SAVE_M>;
  const size_t extra = mix.basis != nullptr ? BasisSmem<D, TIn>::bytes(mix.rank) : 0;
  const int tiles = (nh * D + 127) / 128;
  bool narrow = false;
  int slots = tc_slots<D, DU, SAVE_M>(nh);
  if constexpr (D == 32 && TTC_FWD_NARROW) {
    const int s2 = tiles < 2 ? tiles : 2;
    if (tiles > 1 && 2 * (L::bytes(s2) + extra + 1024) <= kSmPerSm) {
      narrow = true;
      slots = s2;
    }
  }
  while (slots > 1 && L::bytes(slots) + extra > kMaxSmem) --slots;
  if (L::bytes(slots) + extra > kMaxSmem)
    return set_error(TTC_ERR_UNSUPPORTED, "the Q_f basis does not fit in shared memory");
  const uint32_t cols = tmem_cols_for(slots * CF::kSlotCols);
  const size_t smem = L::bytes(slots) + extra;
  auto k = narrow ? ttc::lqr_fwd_tc_kernel<D, DU, TIn, SAVE_M, AFF, true>
                  : ttc::lqr_fwd_tc_kernel<D, DU, TIn, SAVE_M, AFF, false>;
  if (int rc = set_smem(k, smem)) return rc;
  k<<<dim3((unsigned)N), dim3(slots * 128), smem, st>>>(
      (const TIn*)A, (const TIn*)B, (const TIn*)Q, (const TIn*)R, (const TIn*)Qf,
      (const TIn*)mix.basis, mix.rank, (const TIn*)lA, (const TIn*)lB, (const TIn*)lQ, (const TIn*)h0,
      nh, T, opts, cols, (TIn*)u, lam0, M, status, mix.lowrank<TIn>(), (const TIn*)r_traj,
      narrow ? next_fwd_epoch() : 0u);
  return cuda_check(cudaGetLastError(), "lqr_fwd_tc_kernel launch");
}

template <int D, int DU, typename TIn>
int launch_fwd_affine(const void* A, const void* B, const void* Q, const void* R, const void* Qf,
                      const void* lA, const void* lB, const void* lQ, const void* h0, const void* r_traj,
                      int64_t N, int nh, int T, void* u, float* lam0, int* status, int opts, cudaStream_t st) {
  return launch_fwd_tc<D, DU, TIn, false, true>(A, B, Q, R, Qf, lA, lB, lQ, h0, N, nh, T, u, lam0, nullptr,
                                                status, QMix{}, opts, st, r_traj);
}

template <int D, int DU, typename TIn>
int launch_fwd(const void* A, const void* B, const void* Q, const void* R, const void* Qf,
               const void* lA, const void* lB, const void* lQ, const void* h0, int64_t N, int nh,
               int T, void* u, float* lam0, float* M, int* status, const QMix& mix, int opts,
               cudaStream_t st) {
  if (M != nullptr)
    return launch_fwd_tc<D, DU, TIn, true>(A, B, Q, R, Qf, lA, lB, lQ, h0, N, nh, T, u, lam0, M,
                                           status, mix, opts, st);
  return launch_fwd_tc<D, DU, TIn, false>(A, B, Q, R, Qf, lA, lB, lQ, h0, N, nh, T, u, lam0,
                                          nullptr, status, mix, opts, st);
}

// Saved-state backward on the warp-MMA adjoint: R rows x ceil(nh / 8) warps per CTA.
template <int D, typename TIn, bool FROM_M>
auto bwd_mma_kernel_for(int nh) {
  using C = AdjMma<D>;
  constexpr int kU = C::kOwn ? C::kUnits : 1;
  return C::units_per_warp(nh) == kU ? ttc::lqr_bwd_mma_kernel<D, TIn, FROM_M, kU>
                                     : ttc::lqr_bwd_mma_kernel<D, TIn, FROM_M, 2>;
}

// Grid of the warp-MMA backward: one CTA per row group, or, with a mixed Q_f (whose basis
// gradient is accumulated per warp over all the groups a CTA walks), at most one wave of
// resident CTAs.  Returns 0 on a CUDA error (recorded).
template <int D, typename TIn, bool FROM_M>
int64_t bwd_mma_grid(int64_t N, int nh, bool mix) {
  using C = AdjMma<D>;
  const int64_t groups = (N + C::rows_per_cta(nh) - 1) / C::rows_per_cta(nh);
  if (!mix) return groups;
  auto k = bwd_mma_kernel_for<D, TIn, FROM_M>(nh);
  const size_t smem = C::bytes(nh);
  if (set_smem(k, smem)) return 0;
  int dev = 0, sms = 0, per_sm = 0;
  if (cuda_check(cudaGetDevice(&dev), "cudaGetDevice") ||
      cuda_check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "cudaDeviceGetAttribute") ||
      cuda_check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, 32 * C::warps(nh), smem),
                 "cudaOccupancyMaxActiveBlocksPerMultiprocessor"))
    return 0;
  const int64_t wave = (int64_t)sms * (per_sm > 0 ? per_sm : 1);
  return groups < wave ? groups : wave;
}

template <int D, typename TIn, bool FROM_M>
int launch_bwd_mma(const void* A, const void* B, const void* Q, const void* R, const void* lA,
                   const void* lB, const void* lQ, const void* h0, const float* lam0,
                   const float* M_or_dp, const void* dU, int64_t N, int nh, int T, void* const* g,
                   int* status, const QMix& mix, const void* coeff_Qf, cudaStream_t st) {
  using C = AdjMma<D>;
  const int rpc = C::rows_per_cta(nh);
  const size_t smem = C::bytes(nh);
  auto k = bwd_mma_kernel_for<D, TIn, FROM_M>(nh);
  if (int rc = set_smem(k, smem)) return rc;
  const int64_t grid = bwd_mma_grid<D, TIn, FROM_M>(N, nh, mix.basis != nullptr);
  if (grid == 0) return TTC_ERR_CUDA;
  k<<<dim3((unsigned)grid), dim3(32 * C::warps(nh)), smem, st>>>(
      (const TIn*)A, (const TIn*)B, (const TIn*)Q, (const TIn*)R, (const TIn*)lA, (const TIn*)lB,
      (const TIn*)lQ, (const TIn*)h0, lam0, M_or_dp, (const TIn*)dU, N, nh, T, rpc, (TIn*)g[0],
      (TIn*)g[1], (TIn*)g[2], (TIn*)g[3], (TIn*)g[4], (TIn*)g[5], (TIn*)g[6], (TIn*)g[7],
      (TIn*)g[8], (const TIn*)mix.basis, mix.rank, (const TIn*)coeff_Qf, (TIn*)mix.grad_coeff,
      mix.grad_basis_partial, status, mix.lowrank<TIn>());
  return cuda_check(cudaGetLastError(), "lqr_bwd_mma_kernel launch");
}

// Saved-state backward at d = 64 on the warp-MMA adjoint with each 8-head group split over a
// warp pair (TTC_ADJ_SPLIT=0 builds keep the CUDA-core adjoint there).
#ifndef TTC_ADJ_SPLIT
#define TTC_ADJ_SPLIT 1
#endif

template <int D, typename TIn>
int launch_bwd_split(const void* A, const void* B, const void* Q, const void* R, const void* lA,
                     const void* lB, const void* lQ, const void* h0, const float* lam0, const float* M,
                     const void* dU, int64_t N, int nh, int T, void* const* g, int* status, cudaStream_t st) {
  using C = AdjSplit<D>;
  const int rpc = C::rows_per_cta(nh);
  const size_t smem = C::bytes(nh);
  auto k = C::units_per_warp(nh) == 1 ? ttc::lqr_bwd_split_kernel<D, TIn, 1> : ttc::lqr_bwd_split_kernel<D, TIn, 2>;
  if (int rc = set_smem(k, smem)) return rc;
  const int64_t grid = (N + rpc - 1) / rpc;
  k<<<dim3((unsigned)grid), dim3(32 * C::warps(nh)), smem, st>>>(
      (const TIn*)A, (const TIn*)B, (const TIn*)Q, (const TIn*)R, (const TIn*)lA, (const TIn*)lB,
      (const TIn*)lQ, (const TIn*)h0, lam0, M, (const TIn*)dU, N, nh, T, rpc, (TIn*)g[0], (TIn*)g[1],
      (TIn*)g[2], (TIn*)g[3], (TIn*)g[4], (TIn*)g[5], (TIn*)g[6], (TIn*)g[7], (TIn*)g[8], status);
  return cuda_check(cudaGetLastError(), "lqr_bwd_split_kernel launch");
}

template <int D, int DU, typename TIn>
int64_t bwd_mix_slices(int64_t N, int nh, int rQ) {
  if constexpr (D == DU && D <= TTC_ADJ_MMA_MAXD) {
    if (!AdjMma<D>::fits(nh)) return 0;
    // the backward stages each warp's [8][rQ] coefficients in one staging buffer
    if (8 * rQ > 3 * AdjMma<D>::kStage) return 0;
    // the forward keeps the basis in shared memory next to one tile slot at least
    if (TcFwdLayout<D, DU, true>::bytes(1) + BasisSmem<D, TIn>::bytes(rQ) > kMaxSmem) return 0;
    const int64_t grid = bwd_mma_grid<D, TIn, true>(N, nh, true);
    if (grid == 0) return -TTC_ERR_CUDA;
    return grid;
  } else {
    (void)N;
    (void)nh;
    (void)rQ;
    return 0;
  }
}

#ifndef TTC_ADJ_SPLIT32
#define TTC_ADJ_SPLIT32 0
#endif

template <int D, int DU, typename TIn>
int launch_bwd(const void* A, const void* B, const void* Q, const void* R, const void* Qf,
               const void* lA, const void* lB, const void* lQ, const void* h0, const float* lam0,
               const float* M, const void* dU, int64_t N, int nh, int T, void* const* g,
               int* status, const QMix& mix, int opts, cudaStream_t st) {
  if constexpr (TTC_ADJ_SPLIT32 && D == DU && D == 32) {
    if (M != nullptr && mix.basis == nullptr && AdjSplit<D>::fits(nh))
      return launch_bwd_split<D, TIn>(A, B, Q, R, lA, lB, lQ, h0, lam0, M, dU, N, nh, T, g, status, st);
  }
  if constexpr (D == DU && D <= TTC_ADJ_MMA_MAXD) {
    if (M != nullptr && AdjMma<D>::fits(nh))
      return launch_bwd_mma<D, TIn, true>(A, B, Q, R, lA, lB, lQ, h0, lam0, M, dU, N, nh, T, g, status,
                                          mix, Qf, st);
  }
  if constexpr (TTC_ADJ_SPLIT && D == DU && D == 64) {
    if (M != nullptr && mix.basis == nullptr && AdjSplit<D>::fits(nh))
      return launch_bwd_split<D, TIn>(A, B, Q, R, lA, lB, lQ, h0, lam0, M, dU, N, nh, T, g, status, st);
  }
  if (mix.basis != nullptr)
    return set_error(TTC_ERR_UNSUPPORTED,
                     "a mixed Q_f needs the saved-state warp-MMA backward (d = du <= 32, <= 64 heads, M saved)");
  if (M != nullptr) {
    // The forward saved lambda0 and M: adjoint only, on the CUDA cores.
    const int G = groups_for(nh, D);
    auto k = ttc::lqr_bwd_kernel<D, DU, TIn>;
    const size_t smem = ttc::BwdLayout<D, DU>::bytes(G);
    if (int rc = set_smem(k, smem)) return rc;
    k<<<dim3((unsigned)N), dim3(G * D), smem, st>>>(
        (const TIn*)A, (const TIn*)B, (const TIn*)Q, (const TIn*)R, (const TIn*)lA, (const TIn*)lB,
        (const TIn*)lQ, (const TIn*)h0, lam0, M, (const TIn*)dU, nh, T, (TIn*)g[0], (TIn*)g[1],
        (TIn*)g[2], (TIn*)g[3], (TIn*)g[4], (TIn*)g[5], (TIn*)g[6], (TIn*)g[7], (TIn*)g[8], status);
    return cuda_check(cudaGetLastError(), "lqr_bwd_kernel launch");
  }
  // Recompute: the sweep again on the tensor cores, then the adjoint.
  using CF = TcCfg<D, DU>;
  const int tiles = (nh * D + 127) / 128;
  int slots = tiles < TcLaunch<D>::kMaxSlots ? tiles : TcLaunch<D>::kMaxSlots;
  while (slots > 1 && TcBwdLayout<D, DU>::bytes(slots) > kMaxSmem) --slots;
  const uint32_t cols = tmem_cols_for(slots * CF::kSlotCols);
  const size_t smem = TcBwdLayout<D, DU>::bytes(slots);
  auto k = ttc::lqr_bwd_tc_kernel<D, DU, TIn>;
  if (int rc = set_smem(k, smem)) return rc;
  k<<<dim3((unsigned)N), dim3(slots * 128), smem, st>>>(
      (const TIn*)A, (const TIn*)B, (const TIn*)Q, (const TIn*)R, (const TIn*)Qf, (const TIn*)lA,
      (const TIn*)lB, (const TIn*)lQ, (const TIn*)h0, (const TIn*)dU, nh, T, opts, cols, (TIn*)g[0],
      (TIn*)g[1], (TIn*)g[2], (TIn*)g[3], (TIn*)g[4], (TIn*)g[5], (TIn*)g[6], (TIn*)g[7],
      (TIn*)g[8], status);
  return cuda_check(cudaGetLastError(), "lqr_bwd_tc_kernel launch");
}

template <int D, int DU, typename TIn>
int launch_rollout(const void* A, const void* B, const void* Q, const void* R, const void* Qf,
                   const void* lA, const void* lB, const void* lQ, const void* h0,
                   const float* lam0, const float* M, const void* r0, int r_steps, int64_t N, int nh,
                   int T, void* u, float* hs, float* lams, float* lam0_out, float* cost, int* status,
                   cudaStream_t st) {
#ifndef TTC_ROLL_MMA
#define TTC_ROLL_MMA 1
#endif
  if constexpr (TTC_ROLL_MMA && D == DU && D <= 32) {
    // 16 heads per warp on warp-level tensor-core MMAs: 1.25x (d = 16, 16 heads) and 1.9x
    // (d = 32, 32 heads) the CUDA-core rollout; with fewer than 16 heads at d = 16 half of
    // each warp's MMA rows would idle and the CUDA-core kernel is faster.
    using C = RollMma<D>;
    // (an affine cost on every step runs on the CUDA-core rollout)
    if (r_steps == 1 && C::fits(nh) && (D > 16 || nh >= 16)) {
      const int rpc = C::rows_per_cta(nh);
      const size_t smem = C::bytes(nh);
      auto k = ttc::lqr_rollout_mma_kernel<D, TIn>;
      if (int rc = set_smem(k, smem)) return rc;
      const int64_t grid = (N + rpc - 1) / rpc;
      k<<<dim3((unsigned)grid), dim3(32 * C::warps(nh)), smem, st>>>(
          (const TIn*)A, (const TIn*)B, (const TIn*)Q, (const TIn*)R, (const TIn*)lA, (const TIn*)lB,
          (const TIn*)lQ, (const TIn*)h0, (const TIn*)Qf, lam0, M, (const TIn*)r0, N, nh, T, rpc,
          (TIn*)u, hs, lams, lam0_out, cost, status);
      return cuda_check(cudaGetLastError(), "lqr_rollout_mma_kernel launch");
    }
  }
  constexpr int H = rollout_heads<D>();
  // Groups per CTA: enough to cover the row's heads H at a time, at most kRollThreads / D.
  int G = (nh + H - 1) / H;
  if (G > kRollThreads / D) G = kRollThreads / D;
  auto k = ttc::lqr_rollout_kernel<D, DU, TIn, H>;
  const size_t smem = RolloutLayout<D, DU, H>::bytes(G);
  if (int rc = set_smem(k, smem)) return rc;
  k<<<dim3((unsigned)N), dim3(G * D), smem, st>>>(
      (const TIn*)A, (const TIn*)B, (const TIn*)Q, (const TIn*)R, (const TIn*)lA, (const TIn*)lB,
      (const TIn*)lQ, (const TIn*)h0, (const TIn*)Qf, lam0, M, (const TIn*)r0, r_steps, nh, T, (TIn*)u,
      hs, lams, lam0_out, cost, status);
  return cuda_check(cudaGetLastError(), "lqr_rollout_kernel launch");
}

#endif  // TTC_DEFINE_LAUNCHERS

}  // namespace ttc

#define TTC_INSTANTIATE(D, DU, TIn)                                                          \
  template int ttc::launch_fwd<D, DU, TIn>(const void*, const void*, const void*, const void*, \
                                           const void*, const void*, const void*, const void*, \
                                           const void*, int64_t, int, int, void*, float*,      \
                                           float*, int*, const ttc::QMix&, int, cudaStream_t); \
  template int ttc::launch_bwd<D, DU, TIn>(const void*, const void*, const void*, const void*, \
                                           const void*, const void*, const void*, const void*, \
                                           const void*, const float*, const float*,            \
                                           const void*, int64_t, int, int, void* const*, int*, \
                                           const ttc::QMix&, int, cudaStream_t);               \
  template int64_t ttc::bwd_mix_slices<D, DU, TIn>(int64_t, int, int);                      \
  template int ttc::launch_rollout<D, DU, TIn>(const void*, const void*, const void*,         \
                                               const void*, const void*, const void*,         \
                                               const void*, const void*, const void*,         \
                                               const float*, const float*, const void*, int,  \
                                               int64_t, int, int, void*, float*, float*,      \
                                               float*, float*, int*, cudaStream_t);           \
  template int ttc::launch_fwd_affine<D, DU, TIn>(const void*, const void*, const void*,      \
                                                  const void*, const void*, const void*,      \
                                                  const void*, const void*, const void*,      \
                                                  const void*, int64_t, int, int, void*, float*, \
                                                  int*, int, cudaStream_t);
