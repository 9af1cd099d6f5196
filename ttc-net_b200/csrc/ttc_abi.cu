// C-ABI entry points of include/ttc_b200.h: argument checks, kernel selection, launch.
#include <cstdio>
#include <mutex>

#include "lqr_launch.cuh"
#include "ttc_b200.h"

// ======================================================================================
// C-ABI
// ======================================================================================
namespace {

std::mutex g_err_mu;
char g_err[512] = "";

int fail(int code, const char* msg) { return ttc::set_error(code, msg); }

// (h_dim, u_dim) pairs with kernels: u_dim <= h_dim, both multiples of 16 (the MMA N of a
// 128-row tcgen05 tile), h_dim in {16, 32, 64}.
bool supported(int d, int du) {
  return (d == 16 || d == 32 || d == 64) && (du == 16 || du == 32 || du == 64) && du <= d;
}

// Expands X(D, DU, TIn) for the supported pair (d, du); callers checked supported() first.
#define TTC_FOR_DIMS(X, TT)             \
  do {                                  \
    if (d == 16) X(16, 16, TT);         \
    if (d == 32 && du == 32) X(32, 32, TT); \
    if (d == 32) X(32, 16, TT);         \
    if (d == 64 && du == 64) X(64, 64, TT); \
    if (d == 64 && du == 32) X(64, 32, TT); \
    X(64, 16, TT);                      \
  } while (0)

bool misaligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; }

int check_flags(int flags) {
  if (flags & ~TTC_FLAG_INV_GUARD) return fail(TTC_ERR_INVALID, "unknown flag bits");
  return TTC_OK;
}

int check_common(int64_t N, int nh, int d, int du, int T, int dtype) {
  if (N < 0 || N > 0x7fffffffLL) return fail(TTC_ERR_INVALID, "N (rows) must be in [0, 2^31)");
  if (nh < 1) return fail(TTC_ERR_INVALID, "num_heads must be >= 1");
  if (T < 1) return fail(TTC_ERR_INVALID, "T must be >= 1");
  if (dtype != TTC_DTYPE_F32 && dtype != TTC_DTYPE_BF16)
    return fail(TTC_ERR_INVALID, "unknown dtype code (0 = float32, 1 = bfloat16)");
  if (!supported(d, du)) {
    char buf[128];
    snprintf(buf, sizeof(buf), "no kernel for h_dim=%d u_dim=%d", d, du);
    return fail(TTC_ERR_UNSUPPORTED, buf);
  }
  return TTC_OK;
}

}  // namespace

int ttc::set_error(int code, const char* msg) {
  std::lock_guard<std::mutex> lk(g_err_mu);
  snprintf(g_err, sizeof(g_err), "%s", msg);
  return code;
}

extern "C" {

int ttc_abi_version(void) { return TTC_ABI_VERSION; }

int ttc_supported(int d, int du) { return supported(d, du) ? 1 : 0; }

const char* ttc_last_error(void) { return g_err; }

int ttc_lqr_fwd(const void* A_diag, const void* B, const void* Q, const void* R_inv,
                const void* Q_f, const void* log_gamma_A, const void* log_gamma_B,
                const void* log_gamma_Q, const void* h0, int64_t N, int nh, int d, int du,
                int T, int dtype, int flags, void* u, float* lam0, float* M, int* status, void* stream) {
  if (int rc = check_common(N, nh, d, du, T, dtype)) return rc;
  if (int rc = check_flags(flags)) return rc;
  if (N == 0) return TTC_OK;
  if (!A_diag || !B || !Q || !R_inv || !Q_f || !log_gamma_A || !log_gamma_B || !log_gamma_Q ||
      !h0 || !u || !status)
    return fail(TTC_ERR_INVALID, "null pointer argument");
  if (misaligned16(M)) return fail(TTC_ERR_INVALID, "M must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define TTC_FWD(DD, DDU, TT)                                                                 \
  return ttc::launch_fwd<DD, DDU, TT>(A_diag, B, Q, R_inv, Q_f, log_gamma_A, log_gamma_B,        \
                                 log_gamma_Q, h0, N, nh, T, u, lam0, M, status, ttc::QMix{}, flags, st)
  if (dtype == TTC_DTYPE_F32) TTC_FOR_DIMS(TTC_FWD, float);
  TTC_FOR_DIMS(TTC_FWD, __nv_bfloat16);
#undef TTC_FWD
}

int ttc_lqr_bwd(const void* A_diag, const void* B, const void* Q, const void* R_inv,
                const void* Q_f, const void* log_gamma_A, const void* log_gamma_B,
                const void* log_gamma_Q, const void* h0, const float* lam0, const float* M,
                const void* d_u, int64_t N, int nh, int d, int du, int T, int dtype, int flags,
                void* grad_A, void* grad_B, void* grad_Q, void* grad_R_inv, void* grad_Q_f,
                void* grad_lgA, void* grad_lgB, void* grad_lgQ, void* grad_h0, int* status,
                void* stream) {
  if (int rc = check_common(N, nh, d, du, T, dtype)) return rc;
  if (int rc = check_flags(flags)) return rc;
  if (N == 0) return TTC_OK;
  if (!A_diag || !B || !Q || !R_inv || !log_gamma_A || !log_gamma_B || !log_gamma_Q || !h0 ||
      !d_u || !status)
    return fail(TTC_ERR_INVALID, "null pointer argument");
  if (M == nullptr && Q_f == nullptr)
    return fail(TTC_ERR_INVALID, "Q_f is required when M is NULL (sweep recompute)");
  if (M != nullptr && lam0 == nullptr)
    return fail(TTC_ERR_INVALID, "lam0 is required together with M");
  if (misaligned16(M) || misaligned16(d_u)) return fail(TTC_ERR_INVALID, "M and d_u must be 16-byte aligned");
  void* g[9] = {grad_A, grad_B, grad_Q, grad_R_inv, grad_Q_f, grad_lgA, grad_lgB, grad_lgQ, grad_h0};
  for (void* p : g)
    if (!p) return fail(TTC_ERR_INVALID, "null gradient pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define TTC_BWD(DD, DDU, TT)                                                                  \
  return ttc::launch_bwd<DD, DDU, TT>(A_diag, B, Q, R_inv, Q_f, log_gamma_A, log_gamma_B,         \
                                 log_gamma_Q, h0, lam0, M, d_u, N, nh, T, g, status, ttc::QMix{}, flags, st)
  if (dtype == TTC_DTYPE_F32) TTC_FOR_DIMS(TTC_BWD, float);
  TTC_FOR_DIMS(TTC_BWD, __nv_bfloat16);
#undef TTC_BWD
}

int ttc_lqr_rollout(const void* A_diag, const void* B, const void* Q, const void* R_inv,
                    const void* Q_f, const void* log_gamma_A, const void* log_gamma_B,
                    const void* log_gamma_Q, const void* h0, const float* lam0, const float* M,
                    const void* r0, int r_steps, int64_t N, int nh, int d, int du, int T, int dtype,
                    void* u_traj, float* h_traj, float* lam_traj, float* lam0_out, float* cost,
                    int* status, void* stream) {
  if (int rc = check_common(N, nh, d, du, T, dtype)) return rc;
  if (r_steps != 1 && r_steps != T) return fail(TTC_ERR_INVALID, "r_steps must be 1 or T");
  if (N == 0) return TTC_OK;
  if (!A_diag || !B || !Q || !R_inv || !log_gamma_A || !log_gamma_B || !log_gamma_Q || !h0 ||
      !lam0 || !u_traj || !status)
    return fail(TTC_ERR_INVALID, "null pointer argument");
  // (T = 1: both forms coincide; without M, lam0 is taken to hold r0's offset already)
  if (r_steps == 1 && T > 1 && r0 != nullptr && M == nullptr)
    return fail(TTC_ERR_INVALID, "an affine term r0 on step 0 needs the forward's M");
  if (r_steps > 1 && M != nullptr)
    return fail(TTC_ERR_INVALID, "an affine term on every step takes lam0 from ttc_lqr_fwd_affine, not M");
  if (cost != nullptr && Q_f == nullptr)
    return fail(TTC_ERR_INVALID, "the total cost needs Q_f");
  if (N * nh * (int64_t)T > 0x7fffffffLL)
    return fail(TTC_ERR_INVALID, "N * num_heads * T must be below 2^31");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define TTC_ROLL(DD, DDU, TT)                                                                 \
  return ttc::launch_rollout<DD, DDU, TT>(A_diag, B, Q, R_inv, Q_f, log_gamma_A, log_gamma_B,     \
                                     log_gamma_Q, h0, lam0, M, r0, r_steps, N, nh, T, u_traj, h_traj, \
                                     lam_traj, lam0_out, cost, status, st)
  if (dtype == TTC_DTYPE_F32) TTC_FOR_DIMS(TTC_ROLL, float);
  TTC_FOR_DIMS(TTC_ROLL, __nv_bfloat16);
#undef TTC_ROLL
}

int ttc_lqr_fwd_affine(const void* A_diag, const void* B, const void* Q, const void* R_inv,
                       const void* Q_f, const void* log_gamma_A, const void* log_gamma_B,
                       const void* log_gamma_Q, const void* h0, const void* r_traj, int64_t N, int nh,
                       int d, int du, int T, int dtype, int flags, void* u, float* lam0, int* status,
                       void* stream) {
  if (int rc = check_common(N, nh, d, du, T, dtype)) return rc;
  if (int rc = check_flags(flags)) return rc;
  if (N == 0) return TTC_OK;
  if (!A_diag || !B || !Q || !R_inv || !Q_f || !log_gamma_A || !log_gamma_B || !log_gamma_Q ||
      !h0 || !r_traj || !u || !lam0 || !status)
    return fail(TTC_ERR_INVALID, "null pointer argument");
  if (N * nh * (int64_t)T > 0x7fffffffLL)
    return fail(TTC_ERR_INVALID, "N * num_heads * T must be below 2^31");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define TTC_FWDA(DD, DDU, TT)                                                                  \
  return ttc::launch_fwd_affine<DD, DDU, TT>(A_diag, B, Q, R_inv, Q_f, log_gamma_A, log_gamma_B,   \
                                        log_gamma_Q, h0, r_traj, N, nh, T, u, lam0, status, flags, st)
  if (dtype == TTC_DTYPE_F32) TTC_FOR_DIMS(TTC_FWDA, float);
  TTC_FOR_DIMS(TTC_FWDA, __nv_bfloat16);
#undef TTC_FWDA
}

int ttc_lqr_fwd_mix(const void* A_diag, const void* B, const void* Q, const void* R_inv,
                    const void* coeff_Qf, const void* Q_basis, int rQ, const void* log_gamma_A,
                    const void* log_gamma_B, const void* log_gamma_Q, const void* h0, int64_t N, int nh,
                    int d, int du, int T, int dtype, int flags, void* u, float* lam0, float* M, int* status,
                    void* stream) {
  if (int rc = check_common(N, nh, d, du, T, dtype)) return rc;
  if (int rc = check_flags(flags)) return rc;
  if (rQ < 1) return fail(TTC_ERR_INVALID, "rank of the Q_f mixture must be >= 1");
  if (N == 0) return TTC_OK;
  if (!A_diag || !B || !Q || !R_inv || !coeff_Qf || !Q_basis || !log_gamma_A || !log_gamma_B ||
      !log_gamma_Q || !h0 || !u || !status)
    return fail(TTC_ERR_INVALID, "null pointer argument");
  if (misaligned16(Q_basis) || misaligned16(M))
    return fail(TTC_ERR_INVALID, "Q_basis and M must be 16-byte aligned");
  ttc::QMix mix;
  mix.basis = Q_basis;
  mix.rank = rQ;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define TTC_FWD(DD, DDU, TT)                                                                 \
  return ttc::launch_fwd<DD, DDU, TT>(A_diag, B, Q, R_inv, coeff_Qf, log_gamma_A, log_gamma_B,   \
                                 log_gamma_Q, h0, N, nh, T, u, lam0, M, status, mix, flags, st)
  if (dtype == TTC_DTYPE_F32) TTC_FOR_DIMS(TTC_FWD, float);
  TTC_FOR_DIMS(TTC_FWD, __nv_bfloat16);
#undef TTC_FWD
}

int64_t ttc_lqr_bwd_mix_slices(int64_t N, int nh, int d, int du, int rQ, int dtype) {
  if (int rc = check_common(N, nh, d, du, 1, dtype)) return -rc;
  if (N == 0 || rQ < 1) return 0;
#define TTC_SL(DD, DDU, TT) return ttc::bwd_mix_slices<DD, DDU, TT>(N, nh, rQ)
  if (dtype == TTC_DTYPE_F32) TTC_FOR_DIMS(TTC_SL, float);
  TTC_FOR_DIMS(TTC_SL, __nv_bfloat16);
#undef TTC_SL
}

int ttc_lqr_bwd_mix(const void* A_diag, const void* B, const void* Q, const void* R_inv,
                    const void* coeff_Qf, const void* Q_basis, int rQ, const void* log_gamma_A,
                    const void* log_gamma_B, const void* log_gamma_Q, const void* h0, const float* lam0,
                    const float* M, const void* d_u, int64_t N, int nh, int d, int du, int T, int dtype,
                    void* grad_A, void* grad_B, void* grad_Q, void* grad_R_inv, void* grad_coeff_Qf,
                    float* grad_basis_partial, int64_t slices, void* grad_lgA, void* grad_lgB,
                    void* grad_lgQ, void* grad_h0, int* status, void* stream) {
  if (int rc = check_common(N, nh, d, du, T, dtype)) return rc;
  if (rQ < 1) return fail(TTC_ERR_INVALID, "rank of the Q_f mixture must be >= 1");
  if (N == 0) return TTC_OK;
  if (!A_diag || !B || !Q || !R_inv || !coeff_Qf || !Q_basis || !log_gamma_A || !log_gamma_B ||
      !log_gamma_Q || !h0 || !d_u || !status || !lam0 || !M || !grad_basis_partial)
    return fail(TTC_ERR_INVALID, "null pointer argument (the mixed-Q_f backward needs lam0 and M)");
  if (misaligned16(M) || misaligned16(d_u)) return fail(TTC_ERR_INVALID, "M and d_u must be 16-byte aligned");
  void* g[9] = {grad_A, grad_B, grad_Q, grad_R_inv, nullptr, grad_lgA, grad_lgB, grad_lgQ, grad_h0};
  for (int i = 0; i < 9; ++i)
    if (i != 4 && !g[i]) return fail(TTC_ERR_INVALID, "null gradient pointer");
  if (!grad_coeff_Qf) return fail(TTC_ERR_INVALID, "null gradient pointer");
  const int64_t need = ttc_lqr_bwd_mix_slices(N, nh, d, du, rQ, dtype);
  if (need < 0) return static_cast<int>(-need);
  if (need == 0) return fail(TTC_ERR_UNSUPPORTED, "no mixed-Q_f backward for this shape");
  if (slices != need) {
    char buf[160];
    snprintf(buf, sizeof(buf), "grad_basis_partial has %lld slices, this launch needs %lld",
             (long long)slices, (long long)need);
    return fail(TTC_ERR_INVALID, buf);
  }
  ttc::QMix mix;
  mix.basis = Q_basis;
  mix.rank = rQ;
  mix.grad_coeff = grad_coeff_Qf;
  mix.grad_basis_partial = grad_basis_partial;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define TTC_BWD(DD, DDU, TT)                                                                  \
  return ttc::launch_bwd<DD, DDU, TT>(A_diag, B, Q, R_inv, coeff_Qf, log_gamma_A, log_gamma_B,    \
                                 log_gamma_Q, h0, lam0, M, d_u, N, nh, T, g, status, mix, 0, st)
  if (dtype == TTC_DTYPE_F32) TTC_FOR_DIMS(TTC_BWD, float);
  TTC_FOR_DIMS(TTC_BWD, __nv_bfloat16);
#undef TTC_BWD
}

int ttc_lqr_fwd_lowrank(const void* A_diag, const void* coeff_B, const void* B_basis, int rB,
                        const void* coeff_Q, const void* R_inv, const void* coeff_Qf, const void* Q_basis,
                        int rQ, const void* log_gamma_A, const void* log_gamma_B, const void* log_gamma_Q,
                        const void* h0, int64_t N, int nh, int d, int du, int T, int dtype, int flags,
                        void* u, float* lam0, float* M, int* status, void* stream) {
  if (int rc = check_common(N, nh, d, du, T, dtype)) return rc;
  if (int rc = check_flags(flags)) return rc;
  if (rQ < 1 || rB < 1) return fail(TTC_ERR_INVALID, "ranks of the B and Q mixtures must be >= 1");
  if (N == 0) return TTC_OK;
  if (!A_diag || !coeff_B || !B_basis || !coeff_Q || !R_inv || !coeff_Qf || !Q_basis || !log_gamma_A ||
      !log_gamma_B || !log_gamma_Q || !h0 || !u || !status)
    return fail(TTC_ERR_INVALID, "null pointer argument");
  if (misaligned16(B_basis) || misaligned16(Q_basis) || misaligned16(M))
    return fail(TTC_ERR_INVALID, "B_basis, Q_basis and M must be 16-byte aligned");
  ttc::QMix mix;
  mix.basis = Q_basis;
  mix.rank = rQ;
  mix.coeff_B = coeff_B;
  mix.B_basis = B_basis;
  mix.rB = rB;
  mix.coeff_Q = coeff_Q;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define TTC_FWD(DD, DDU, TT)                                                                   \
  return ttc::launch_fwd<DD, DDU, TT>(A_diag, nullptr, nullptr, R_inv, coeff_Qf, log_gamma_A, log_gamma_B, \
                                      log_gamma_Q, h0, N, nh, T, u, lam0, M, status, mix, flags, st)
  if (dtype == TTC_DTYPE_F32) TTC_FOR_DIMS(TTC_FWD, float);
  TTC_FOR_DIMS(TTC_FWD, __nv_bfloat16);
#undef TTC_FWD
}

int ttc_lqr_bwd_lowrank(const void* A_diag, const void* coeff_B, const void* B_basis, int rB,
                        const void* coeff_Q, const void* R_inv, const void* coeff_Qf, const void* Q_basis,
                        int rQ, const void* log_gamma_A, const void* log_gamma_B, const void* log_gamma_Q,
                        const void* h0, const float* lam0, const float* M, const void* d_u, int64_t N,
                        int nh, int d, int du, int T, int dtype, void* grad_A, void* grad_coeff_B,
                        float* grad_B_basis_partial, void* grad_coeff_Q, void* grad_R_inv,
                        void* grad_coeff_Qf, float* grad_basis_partial, int64_t slices, void* grad_lgA,
                        void* grad_lgB, void* grad_lgQ, void* grad_h0, int* status, void* stream) {
  if (int rc = check_common(N, nh, d, du, T, dtype)) return rc;
  if (rQ < 1 || rB < 1) return fail(TTC_ERR_INVALID, "ranks of the B and Q mixtures must be >= 1");
  if (N == 0) return TTC_OK;
  if (!A_diag || !coeff_B || !B_basis || !coeff_Q || !R_inv || !coeff_Qf || !Q_basis || !log_gamma_A ||
      !log_gamma_B || !log_gamma_Q || !h0 || !d_u || !status || !lam0 || !M || !grad_basis_partial ||
      !grad_B_basis_partial)
    return fail(TTC_ERR_INVALID, "null pointer argument (the low-rank backward needs lam0 and M)");
  if (misaligned16(B_basis) || misaligned16(Q_basis) || misaligned16(grad_basis_partial) ||
      misaligned16(grad_B_basis_partial) || misaligned16(M) || misaligned16(d_u))
    return fail(TTC_ERR_INVALID, "the bases, the partial buffers, M and d_u must be 16-byte aligned");
  void* g[9] = {grad_A, nullptr, nullptr, grad_R_inv, nullptr, grad_lgA, grad_lgB, grad_lgQ, grad_h0};
  for (int i = 0; i < 9; ++i)
    if ((i == 0 || i == 3 || i > 4) && !g[i]) return fail(TTC_ERR_INVALID, "null gradient pointer");
  if (!grad_coeff_Qf || !grad_coeff_B || !grad_coeff_Q) return fail(TTC_ERR_INVALID, "null gradient pointer");
  const int64_t need = ttc_lqr_bwd_mix_slices(N, nh, d, du, rQ, dtype);
  if (need < 0) return static_cast<int>(-need);
  if (need == 0) return fail(TTC_ERR_UNSUPPORTED, "no low-rank backward for this shape");
  if (slices != need) {
    char buf[160];
    snprintf(buf, sizeof(buf), "the basis partials have %lld slices, this launch needs %lld",
             (long long)slices, (long long)need);
    return fail(TTC_ERR_INVALID, buf);
  }
  ttc::QMix mix;
  mix.basis = Q_basis;
  mix.rank = rQ;
  mix.grad_coeff = grad_coeff_Qf;
  mix.grad_basis_partial = grad_basis_partial;
  mix.coeff_B = coeff_B;
  mix.B_basis = B_basis;
  mix.rB = rB;
  mix.coeff_Q = coeff_Q;
  mix.grad_coeff_B = grad_coeff_B;
  mix.grad_coeff_Q = grad_coeff_Q;
  mix.grad_B_basis_partial = grad_B_basis_partial;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define TTC_BWD(DD, DDU, TT)                                                                    \
  return ttc::launch_bwd<DD, DDU, TT>(A_diag, nullptr, nullptr, R_inv, coeff_Qf, log_gamma_A, log_gamma_B, \
                                      log_gamma_Q, h0, lam0, M, d_u, N, nh, T, g, status, mix, 0, st)
  if (dtype == TTC_DTYPE_F32) TTC_FOR_DIMS(TTC_BWD, float);
  TTC_FOR_DIMS(TTC_BWD, __nv_bfloat16);
#undef TTC_BWD
}

}  // extern "C"
