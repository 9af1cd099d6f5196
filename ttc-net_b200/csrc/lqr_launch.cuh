// Kernel launchers, explicitly instantiated per (d, du, dtype) in inst_*.cu so the
// sm_100a build compiles in parallel; the C-ABI in ttc_abi.cu dispatches to them.
#pragma once

#include <cuda_runtime.h>

#include <cstdio>

#include "lqr_adjoint_mma.cuh"
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

template <int D, int DU, typename TIn>
int launch_fwd(const void* A, const void* B, const void* Q, const void* R, const void* Qf,
               const void* lA, const void* lB, const void* lQ, const void* h0, int64_t N, int nh,
               int T, void* u, float* lam0, float* M, int* status, cudaStream_t st);

template <int D, int DU, typename TIn>
int launch_bwd(const void* A, const void* B, const void* Q, const void* R, const void* Qf,
               const void* lA, const void* lB, const void* lQ, const void* h0, const float* lam0,
               const float* M, const void* dU, int64_t N, int nh, int T, void* const* g,
               int* status, cudaStream_t st);

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

template <int D, int DU, typename TIn, bool SAVE_M>
int launch_fwd_tc(const void* A, const void* B, const void* Q, const void* R, const void* Qf,
                  const void* lA, const void* lB, const void* lQ, const void* h0, int64_t N,
                  int nh, int T, void* u, float* lam0, float* M, int* status, cudaStream_t st) {
  using CF = TcCfg<D, DU>;
  const int slots = tc_slots<D, DU, SAVE_M>(nh);
  const uint32_t cols = tmem_cols_for(slots * CF::kSlotCols);
  const size_t smem = TcFwdLayout<D, DU, SAVE_M>::bytes(slots);
  auto k = ttc::lqr_fwd_tc_kernel<D, DU, TIn, SAVE_M>;
  if (int rc = set_smem(k, smem)) return rc;
  k<<<dim3((unsigned)N), dim3(slots * 128), smem, st>>>(
      (const TIn*)A, (const TIn*)B, (const TIn*)Q, (const TIn*)R, (const TIn*)Qf, (const TIn*)lA,
      (const TIn*)lB, (const TIn*)lQ, (const TIn*)h0, nh, T, cols, (TIn*)u, lam0, M, status);
  return cuda_check(cudaGetLastError(), "lqr_fwd_tc_kernel launch");
}

template <int D, int DU, typename TIn>
int launch_fwd(const void* A, const void* B, const void* Q, const void* R, const void* Qf,
               const void* lA, const void* lB, const void* lQ, const void* h0, int64_t N, int nh,
               int T, void* u, float* lam0, float* M, int* status, cudaStream_t st) {
  if (M != nullptr)
    return launch_fwd_tc<D, DU, TIn, true>(A, B, Q, R, Qf, lA, lB, lQ, h0, N, nh, T, u, lam0, M,
                                           status, st);
  return launch_fwd_tc<D, DU, TIn, false>(A, B, Q, R, Qf, lA, lB, lQ, h0, N, nh, T, u, lam0,
                                          nullptr, status, st);
}

// Saved-state backward on the warp-MMA adjoint: R rows x ceil(nh / 8) warps per CTA.
template <int D, typename TIn, bool FROM_M>
int launch_bwd_mma(const void* A, const void* B, const void* Q, const void* R, const void* lA,
                   const void* lB, const void* lQ, const void* h0, const float* lam0,
                   const float* M_or_dp, const void* dU, int64_t N, int nh, int T, void* const* g,
                   int* status, cudaStream_t st) {
  using C = AdjMma<D>;
  const int rpc = C::rows_per_cta(nh);
  const size_t smem = C::bytes(nh);
  constexpr int kU = C::kOwn ? C::kUnits : 1;
  auto k = C::units_per_warp(nh) == kU ? ttc::lqr_bwd_mma_kernel<D, TIn, FROM_M, kU>
                                       : ttc::lqr_bwd_mma_kernel<D, TIn, FROM_M, 2>;
  if (int rc = set_smem(k, smem)) return rc;
  const int64_t grid = (N + rpc - 1) / rpc;
  k<<<dim3((unsigned)grid), dim3(32 * C::warps(nh)), smem, st>>>(
      (const TIn*)A, (const TIn*)B, (const TIn*)Q, (const TIn*)R, (const TIn*)lA, (const TIn*)lB,
      (const TIn*)lQ, (const TIn*)h0, lam0, M_or_dp, (const TIn*)dU, N, nh, T, rpc, (TIn*)g[0],
      (TIn*)g[1], (TIn*)g[2], (TIn*)g[3], (TIn*)g[4], (TIn*)g[5], (TIn*)g[6], (TIn*)g[7],
      (TIn*)g[8], status);
  return cuda_check(cudaGetLastError(), "lqr_bwd_mma_kernel launch");
}

template <int D, int DU, typename TIn>
int launch_bwd(const void* A, const void* B, const void* Q, const void* R, const void* Qf,
               const void* lA, const void* lB, const void* lQ, const void* h0, const float* lam0,
               const float* M, const void* dU, int64_t N, int nh, int T, void* const* g,
               int* status, cudaStream_t st) {
  if constexpr (D == DU && D <= TTC_ADJ_MMA_MAXD) {
    if (M != nullptr && AdjMma<D>::fits(nh))
      return launch_bwd_mma<D, TIn, true>(A, B, Q, R, lA, lB, lQ, h0, lam0, M, dU, N, nh, T, g, status, st);
  }
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
      (const TIn*)lB, (const TIn*)lQ, (const TIn*)h0, (const TIn*)dU, nh, T, cols, (TIn*)g[0],
      (TIn*)g[1], (TIn*)g[2], (TIn*)g[3], (TIn*)g[4], (TIn*)g[5], (TIn*)g[6], (TIn*)g[7],
      (TIn*)g[8], status);
  return cuda_check(cudaGetLastError(), "lqr_bwd_tc_kernel launch");
}

#endif  // TTC_DEFINE_LAUNCHERS

}  // namespace ttc

#define TTC_INSTANTIATE(D, DU, TIn)                                                          \
  template int ttc::launch_fwd<D, DU, TIn>(const void*, const void*, const void*, const void*, \
                                           const void*, const void*, const void*, const void*, \
                                           const void*, int64_t, int, int, void*, float*,      \
                                           float*, int*, cudaStream_t);                        \
  template int ttc::launch_bwd<D, DU, TIn>(const void*, const void*, const void*, const void*, \
                                           const void*, const void*, const void*, const void*, \
                                           const void*, const float*, const float*,            \
                                           const void*, int64_t, int, int, void* const*, int*, \
                                           cudaStream_t);
