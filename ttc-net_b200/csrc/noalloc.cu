// ttc_lqr_bwd_mix_noalloc: the mixed-Q_f backward (ttc_lqr_bwd_mix) for callers that cannot
// allocate device memory.
//
// ttc_lqr_bwd_mix needs a scratch buffer from its caller: one fp32 [rQ, d, d] slice of partial
// basis-gradient sums per CTA of its persistent grid, which the caller then sums and
// symmetrises.  Some hosts cannot provide it: a runtime that owns all device memory through
// its own pool and forbids plug-ins from calling cudaMalloc, or a latency-bound loop where a
// cudaMalloc / cudaFree (both may synchronise the device) is not acceptable.  This variant
// keeps the slices in a fixed array in the library's own device memory (kScratchFloats floats,
// 16 MiB, held by every GPU that loads the library until the process exits), caps its grid
// so that the slices fit, and reduces them itself into the caller's grad_basis output.
//
// The array is shared by every call on a device and keeps the last call's contents; each CTA
// zeroes its own slice before accumulating, so nothing carries over.  Calls whose kernels
// overlap on the GPU (other streams, other host threads) race on the array: serialise them.
// The first call on a device looks up the array's device address (cudaGetSymbolAddress), so
// make that first call before any stream capture.  Under CUDA's lazy module loading (the
// default since CUDA 12.2) that lookup is also when the driver loads this module and reserves
// the 16 MiB on the device: a host whose pool already holds all device memory should make the
// first call while 16 MiB are still free, or set CUDA_MODULE_LOADING=EAGER so that the array
// is reserved when the context is created.  An empty batch (N = 0) writes a zero grad_basis.
#define TTC_DEFINE_LAUNCHERS
#include <cstdio>
#include <mutex>

#include "lqr_launch.cuh"
#include "ttc_b200.h"

namespace {

constexpr size_t kScratchFloats = size_t(4) << 20;  // 16 MiB
static __device__ __align__(256) float g_basis_scratch[kScratchFloats];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_scratch[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once per device).
int scratch_address(float** out) {
  int dev = 0;
  if (int rc = ttc::cuda_check(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev < 0 || dev >= kMaxDevices) return ttc::set_error(TTC_ERR_UNSUPPORTED, "device index beyond 63");
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch[dev] == nullptr) {
    void* p = nullptr;
    if (int rc = ttc::cuda_check(cudaGetSymbolAddress(&p, g_basis_scratch), "cudaGetSymbolAddress"))
      return rc;
    g_scratch[dev] = static_cast<float*>(p);
  }
  *out = g_scratch[dev];
  return TTC_OK;
}

// grad_basis[r][i][j] = (S[r][i][j] + S[r][j][i]) / 2 with S the sum of the slices, summed in
// slice order (deterministic).
__global__ void basis_reduce_kernel(const float* __restrict__ partial, int64_t slices, int rQ, int D,
                                    float* __restrict__ out) {
  const int64_t per = (int64_t)rQ * D * D;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < per; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / (D * D);
    const int i = static_cast<int>((e / D) % D), j = static_cast<int>(e % D);
    const int64_t et = r * D * D + (int64_t)j * D + i;
    float s = 0.f;
    for (int64_t k = 0; k < slices; ++k) s += partial[k * per + e] + partial[k * per + et];
    out[e] = 0.5f * s;
  }
}

template <int D, typename TIn>
int launch_noalloc(const void* A, const void* B, const void* Q, const void* R, const void* cQf,
                   const void* basis, int rQ, const void* lA, const void* lB, const void* lQ,
                   const void* h0, const float* lam0, const float* M, const void* dU, int64_t N,
                   int nh, int T, void* const* g, void* gcQf, float* grad_basis, int* status,
                   cudaStream_t st) {
  using C = ttc::AdjMma<D>;
  const int64_t wave = ttc::bwd_mix_slices<D, D, TIn>(N, nh, rQ);
  if (wave < 0) return static_cast<int>(-wave);
  if (wave == 0) return ttc::set_error(TTC_ERR_UNSUPPORTED, "no mixed-Q_f backward for this shape");
  const int64_t per = (int64_t)rQ * D * D;
  const int64_t cap = static_cast<int64_t>(kScratchFloats) / per;
  if (cap < 1) {
    char buf[200];
    snprintf(buf, sizeof(buf), "rank %d x %d x %d basis slice exceeds the %zu-float scratch array", rQ, D, D,
             kScratchFloats);
    return ttc::set_error(TTC_ERR_INVALID, buf);
  }
  const int64_t grid = wave < cap ? wave : cap;
  float* scratch = nullptr;
  if (int rc = scratch_address(&scratch)) return rc;
  auto k = ttc::bwd_mma_kernel_for<D, TIn, true>(nh);
  const size_t smem = C::bytes(nh);
  if (int rc = ttc::set_smem(k, smem)) return rc;
  k<<<dim3((unsigned)grid), dim3(32 * C::warps(nh)), smem, st>>>(
      (const TIn*)A, (const TIn*)B, (const TIn*)Q, (const TIn*)R, (const TIn*)lA, (const TIn*)lB,
      (const TIn*)lQ, (const TIn*)h0, lam0, M, (const TIn*)dU, N, nh, T, C::rows_per_cta(nh),
      (TIn*)g[0], (TIn*)g[1], (TIn*)g[2], (TIn*)g[3], nullptr, (TIn*)g[5], (TIn*)g[6], (TIn*)g[7],
      (TIn*)g[8], (const TIn*)basis, rQ, (const TIn*)cQf, (TIn*)gcQf, scratch, status, ttc::LowRank<TIn>{});
  if (int rc = ttc::cuda_check(cudaGetLastError(), "lqr_bwd_mma_kernel launch")) return rc;
  const int64_t blocks = (per + 255) / 256;
  basis_reduce_kernel<<<dim3((unsigned)(blocks < 1024 ? blocks : 1024)), dim3(256), 0, st>>>(scratch, grid, rQ, D,
                                                                                           grad_basis);
  return ttc::cuda_check(cudaGetLastError(), "basis_reduce_kernel launch");
}

}  // namespace

extern "C" int ttc_lqr_bwd_mix_noalloc(const void* A_diag, const void* B, const void* Q, const void* R_inv,
                                       const void* coeff_Qf, const void* Q_basis, int rQ,
                                       const void* log_gamma_A, const void* log_gamma_B,
                                       const void* log_gamma_Q, const void* h0, const float* lam0,
                                       const float* M, const void* d_u, int64_t N, int nh, int d, int du,
                                       int T, int dtype, void* grad_A, void* grad_B, void* grad_Q,
                                       void* grad_R_inv, void* grad_coeff_Qf, float* grad_basis,
                                       void* grad_lgA, void* grad_lgB, void* grad_lgQ, void* grad_h0,
                                       int* status, void* stream) {
  if (N < 0 || N > 0x7fffffffLL) return ttc::set_error(TTC_ERR_INVALID, "N (rows) must be in [0, 2^31)");
  if (nh < 1) return ttc::set_error(TTC_ERR_INVALID, "num_heads must be >= 1");
  if (T < 1) return ttc::set_error(TTC_ERR_INVALID, "T must be >= 1");
  if (rQ < 1) return ttc::set_error(TTC_ERR_INVALID, "rank of the Q_f mixture must be >= 1");
  if (dtype != TTC_DTYPE_F32 && dtype != TTC_DTYPE_BF16)
    return ttc::set_error(TTC_ERR_INVALID, "unknown dtype code (0 = float32, 1 = bfloat16)");
  if (!(d == du && (d == 16 || d == 32))) {
    char buf[128];
    snprintf(buf, sizeof(buf), "no mixed-Q_f backward for h_dim=%d u_dim=%d (needs h_dim = u_dim in {16, 32})", d, du);
    return ttc::set_error(TTC_ERR_UNSUPPORTED, buf);
  }
  if (N == 0) {
    // An empty batch has a zero basis gradient (the allocating path's caller sums no slices).
    // A memset allocates nothing.
    if (grad_basis == nullptr) return TTC_OK;
    return ttc::cuda_check(cudaMemsetAsync(grad_basis, 0, sizeof(float) * (size_t)rQ * d * d,
                                           static_cast<cudaStream_t>(stream)),
                           "cudaMemsetAsync(grad_basis)");
  }
  void* g[9] = {grad_A, grad_B, grad_Q, grad_R_inv, nullptr, grad_lgA, grad_lgB, grad_lgQ, grad_h0};
  if (!A_diag || !B || !Q || !R_inv || !coeff_Qf || !Q_basis || !log_gamma_A || !log_gamma_B ||
      !log_gamma_Q || !h0 || !lam0 || !M || !d_u || !grad_A || !grad_B || !grad_Q || !grad_R_inv ||
      !grad_coeff_Qf || !grad_basis || !grad_lgA || !grad_lgB || !grad_lgQ || !grad_h0 || !status)
    return ttc::set_error(TTC_ERR_INVALID, "null pointer argument");
  if ((reinterpret_cast<uintptr_t>(M) | reinterpret_cast<uintptr_t>(d_u)) & 15u)
    return ttc::set_error(TTC_ERR_INVALID, "M and d_u must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define TTC_NA(DD, TT)                                                                                 \
  return launch_noalloc<DD, TT>(A_diag, B, Q, R_inv, coeff_Qf, Q_basis, rQ, log_gamma_A, log_gamma_B,     \
                                log_gamma_Q, h0, lam0, M, d_u, N, nh, T, g, grad_coeff_Qf, grad_basis, \
                                status, st)
  if (dtype == TTC_DTYPE_F32) {
    if (d == 16) TTC_NA(16, float);
    TTC_NA(32, float);
  }
  if (d == 16) TTC_NA(16, __nv_bfloat16);
  TTC_NA(32, __nv_bfloat16);
#undef TTC_NA
}
