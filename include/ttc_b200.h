/*
 * ttc_b200.h -- C-ABI of the B200 (sm_100a) LQR solve behind TTC-Net's TTCLayer.
 *
 * The reference (VITA-Group/TTC-Net) is Python + Triton; its solver boundary is
 * the Python callable registered in LQR_SOLVER_IMPL_MAP (ttc/layers/ttc_layer.py:18-22,
 * called at :137) and, one level down, the host functions of its "fused" solver
 * that launch three Triton kernels.  The entry points below replace those host
 * functions one for one; the Python package ttc_b200 binds them with ctypes and
 * registers the result as solver_impl="cuda".
 *
 * Conventions for every entry point
 *   - All pointers are device pointers (cudaMalloc / torch CUDA storage) unless a
 *     comment says otherwise; every tensor is dense, row-major, contiguous.
 *   - Sizes: N rows, nh heads per row, state dim d, action dim du, horizon T >= 1.
 *     "Activation dtype" tensors are float32 (TTC_DTYPE_F32) or bfloat16
 *     (TTC_DTYPE_BF16); solver state and the saved tensors are always float32.
 *   - Work is enqueued on `stream` (a cudaStream_t, NULL = legacy default stream);
 *     nothing blocks the host.  Instability is reported through `status`, a device
 *     int the kernels OR bits into (TTC_STATUS_*); the caller zeroes it before the
 *     call and reads it afterwards.
 *   - Return value: TTC_OK, or a TTC_ERR_* code for argument errors and launch
 *     failures (ttc_last_error() gives the message).  Calls are thread-safe apart
 *     from the shared last-error text.
 */
#ifndef TTC_B200_H_
#define TTC_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TTC_ABI_VERSION 7

#define TTC_DTYPE_F32 0
#define TTC_DTYPE_BF16 1

#define TTC_OK 0
#define TTC_ERR_INVALID 1      /* null pointer, bad size or dtype */
#define TTC_ERR_UNSUPPORTED 2  /* (d, du) pair without a compiled kernel */
#define TTC_ERR_CUDA 3         /* CUDA launch / attribute error */

/* Status bits -- the reference's RuntimeError checks, same trigger (NaN, Inf or |x| >= 1e6). */
#define TTC_STATUS_FWD_UNSTABLE 1 /* Y1/Y2 after the sweep      (ttc/solvers/fused_lqr.py:99-101)  */
#define TTC_STATUS_LU_UNSTABLE 2  /* pivots / P = Y1^-1 Y2       (ttc/solvers/fused_lqr.py:108-110) */
#define TTC_STATUS_BWD_UNSTABLE 4 /* any of the nine gradients    (ttc/solvers/fused_lqr.py:243-246) */
#define TTC_STATUS_U_NAN 8        /* NaN in u                     (ttc/layers/ttc_layer.py:139-140)  */
#define TTC_STATUS_MMA_TIMEOUT 16 /* a tensor-core MMA did not complete within the kernel's poll limit */
#define TTC_STATUS_TRAJ_NONFINITE 32 /* NaN or Inf in a trajectory written by ttc_lqr_rollout */
#define TTC_STATUS_COPY_TIMEOUT 64 /* a bulk copy into shared memory did not complete within the kernel's wait limit */

/* Option bits (`flags` argument). */
#define TTC_FLAG_INV_GUARD 1 /* Y1 + 1e-6 I after the sweep, before the solve: the reference's
                                inv_guard (fused_lqr.py:26-27,95-96; symplectic_iter.py:302-305) */

/* ABI version of the loaded library (== TTC_ABI_VERSION it was built with). */
int ttc_abi_version(void);

/* 1 if kernels for state dim d and action dim du are compiled in, else 0: d in {16, 32, 64},
 * du in {16, 32, 64} with du <= d (du is the N of a 128-row tcgen05 MMA: a multiple of 16). */
int ttc_supported(int d, int du);

/* Message of the last TTC_ERR_* returned by this library ("" if none). */
const char* ttc_last_error(void);

/*
 * Forward LQR solve.  Replaces fused_lqr_layer_fwd (ttc/solvers/fused_lqr.py:18-146):
 * the symplectic sweep (Triton lqr_symplectic_rev_iter, symplectic_iter.py:48-356),
 * the LU solve P = Y1^-1 Y2 (fused_lqr.py:103-105) and the first-step decode
 * (lqr_symplectic_dec_first_step, symplectic_iter.py:373-539), in one kernel.
 *
 * Inputs (activation dtype): A_diag [N,nh,d], B [N,d,du], Q [N,d,d], R_inv [N,nh,du],
 *   Q_f [N,nh,d,d], log_gamma_A [N,nh], log_gamma_B [N,nh,du], log_gamma_Q [N,nh,d],
 *   h0 [N,nh,d]  -- the solver signature of ttc_layer.py:137.
 * flags: TTC_FLAG_* bits (TTC_FLAG_INV_GUARD); the backward takes the same flags (they
 *   matter to it only when it recomputes the sweep).
 * Outputs: u [N,nh,du] (activation dtype);
 *   lam0 [N,nh,d] float32 = P h0 (may be NULL);
 *   M [N,nh,d,du] float32 = Y1^-1 Y3, what the backward needs to form
 *     d_p = Y1^-1 (Y3 du) (fused_lqr.py:185-187) without the LU factors (may be NULL:
 *     the backward then recomputes the sweep).
 */
int ttc_lqr_fwd(const void* A_diag, const void* B, const void* Q, const void* R_inv,
                const void* Q_f, const void* log_gamma_A, const void* log_gamma_B,
                const void* log_gamma_Q, const void* h0, int64_t N, int nh, int d, int du,
                int T, int dtype, int flags, void* u, float* lam0, float* M, int* status,
                void* stream);

/*
 * Backward LQR solve.  Replaces fused_lqr_layer_bwd (ttc/solvers/fused_lqr.py:148-253):
 * d_p = Y1^-1 (Y3 d_u) and the forward-in-time adjoint integration (Triton
 * lqr_symplectic_fwd_iter_diff, symplectic_iter.py:553-885).  Gradients over the
 * heads of a row (grad_B, grad_Q) are reduced inside one CTA in a fixed order, so
 * results are deterministic (the reference uses gpu-scope atomics).
 *
 * Inputs: the nine forward inputs (Q_f is read only when M == NULL), d_u [N,nh,du]
 *   (activation dtype), and the forward's lam0 and M.  With M == NULL the kernel
 *   recomputes the sweep and ignores lam0 (both may be NULL).  With M != NULL, lam0
 *   must be given.
 * Outputs (activation dtype): grad_A [N,nh,d], grad_B [N,d,du], grad_Q [N,d,d],
 *   grad_R_inv [N,nh,du], grad_Q_f [N,nh,d,d], grad_lgA [N,nh], grad_lgB [N,nh,du],
 *   grad_lgQ [N,nh,d], grad_h0 [N,nh,d].  Q and Q_f gradients use the symmetrised
 *   convention of the reference's fused and kkt backward ((h dh^T + dh h^T)/2).
 */
int ttc_lqr_bwd(const void* A_diag, const void* B, const void* Q, const void* R_inv,
                const void* Q_f, const void* log_gamma_A, const void* log_gamma_B,
                const void* log_gamma_Q, const void* h0, const float* lam0, const float* M,
                const void* d_u, int64_t N, int nh, int d, int du, int T, int dtype, int flags,
                void* grad_A, void* grad_B, void* grad_Q, void* grad_R_inv, void* grad_Q_f,
                void* grad_lgA, void* grad_lgB, void* grad_lgQ, void* grad_h0, int* status,
                void* stream);

/*
 * Closed-loop trajectory of a solved problem, with an optional affine action cost.
 * Replaces solve_traj_actions(..., r_traj, return_traj=True) and solve_traj_states
 * (ttc/solvers/lin_solver_lqr.py:13-110,113-212), integrated forward in time as the primal
 * half of the reference's adjoint (symplectic_iter.py:766-845).
 *
 * Inputs: the forward's nine inputs (activation dtype; Q_f is read only for the cost and
 *   may be NULL without it), the forward's lam0 (float32), and the affine term r0
 *   (activation dtype; NULL = none) with r_steps:
 *   r_steps = 1: r0 [N,nh,du] on step 0 only -- the form the reference's kkt backward solves
 *     (ttc/solvers/torch_lqr.py:41-47) and the affine term of its symplectic sweep
 *     (IS_AFFINE, y3 = Y3 r; symplectic_iter.py:211-238,336-345).  lam0 and M from
 *     ttc_lqr_fwd; lambda0 = lam0 + M r0 and u_0 gets the extra -R_inv r0 (M may be NULL
 *     without r0).
 *   r_steps = T: r0 [N,nh,T,du], a cost r_t^T u_t on every step t (the reference's r_traj,
 *     lin_solver_lqr.py:143-145).  lam0 from ttc_lqr_fwd_affine on the same r0, M must be
 *     NULL; u_t gets the extra -R_inv r_t on every step.
 * Outputs: u_traj [N,nh,T,du] (activation dtype; u_t, t = 0..T-1); float32, each may be
 *   NULL: h_traj [N,nh,T,d] (h_{t+1}), lam_traj [N,nh,T,d] (lambda_{t+1}, the costates of
 *   solve_traj_states), lam0_out [N,nh,d] (lambda0), cost [N,nh] (the total cost
 *   sum_t 0.5 h_{t+1}^T Q_t h_{t+1} + 0.5 u_t^T R_t u_t + r_t^T u_t, Q_{T-1} = Q_f).
 * status: TTC_STATUS_TRAJ_NONFINITE if any value written is NaN or Inf.
 */
int ttc_lqr_rollout(const void* A_diag, const void* B, const void* Q, const void* R_inv,
                    const void* Q_f, const void* log_gamma_A, const void* log_gamma_B,
                    const void* log_gamma_Q, const void* h0, const float* lam0, const float* M,
                    const void* r0, int r_steps, int64_t N, int nh, int d, int du, int T, int dtype,
                    void* u_traj, float* h_traj, float* lam_traj, float* lam0_out, float* cost,
                    int* status, void* stream);

/*
 * The forward of a problem with an affine action cost on every step, r_traj [N,nh,T,du]
 * (activation dtype; the reference's solve_traj_actions(..., r_traj),
 * ttc/solvers/lin_solver_lqr.py:113-212).  The sweep carries one more value per state row,
 * the offset c of Y1 lambda = Y2 h + c, and lambda0 solves Y1 lambda0 = Y2 h0 + c; with
 * r_traj zero after step 0 this is the IS_AFFINE y3 = Y3 r0 of symplectic_iter.py:211-243.
 * Outputs: u [N,nh,du] = u_0 (activation dtype, with the -R_inv r_0 term), lam0 [N,nh,d]
 * (float32, for ttc_lqr_rollout with r_steps = T).  No M.  Flags and status as ttc_lqr_fwd.
 */
int ttc_lqr_fwd_affine(const void* A_diag, const void* B, const void* Q, const void* R_inv,
                       const void* Q_f, const void* log_gamma_A, const void* log_gamma_B,
                       const void* log_gamma_Q, const void* h0, const void* r_traj, int64_t N, int nh,
                       int d, int du, int T, int dtype, int flags, void* u, float* lam0, int* status,
                       void* stream);

/* ttc_lqr_fwd with Q_f given as the layer's rank-rQ mixture (ttc_layer.py:119-123,
 * Q_f[n,h] = sum_r coeff_Qf[n,h,r] Q_basis[r]) instead of the [N,nh,d,d] tensor:
 * coeff_Qf [N,nh,rQ], Q_basis [rQ,d,d], both in the activation dtype; each kernel mixes the
 * rows of Q_f it needs.  Q_basis must be 16-byte aligned.  Everything else as ttc_lqr_fwd. */
int ttc_lqr_fwd_mix(const void* A_diag, const void* B, const void* Q, const void* R_inv,
                    const void* coeff_Qf, const void* Q_basis, int rQ, const void* log_gamma_A,
                    const void* log_gamma_B, const void* log_gamma_Q, const void* h0, int64_t N, int nh,
                    int d, int du, int T, int dtype, int flags, void* u, float* lam0, float* M,
                    int* status, void* stream);

/* Number of grad_basis_partial slices ttc_lqr_bwd_mix writes for this shape on the current
 * device (it runs one wave of CTAs, each summing into its own slice); 0 if the mixed path is
 * not available for the shape and rank (it needs d = du <= 32, at most 64 heads, a forward
 * that saved M, and the rQ x d x d basis in the forward's shared memory), or minus an error
 * code. */
int64_t ttc_lqr_bwd_mix_slices(int64_t N, int nh, int d, int du, int rQ, int dtype);

/* Backward of ttc_lqr_fwd_mix (saved lam0 and M required).  In place of grad_Q_f it writes
 * grad_coeff_Qf [N,nh,rQ] (activation dtype) = <gQf, Q_basis[r]> per head, and
 * grad_basis_partial [slices,rQ,d,d] (fp32; slices from ttc_lqr_bwd_mix_slices, every slice
 * written): S = sum over slices of sum_heads coeff_Qf[r] h_T dh_T^T, so that the basis
 * gradient is (S + S^T) / 2, the symmetrised convention of grad_Q_f.  Other outputs as
 * ttc_lqr_bwd. */
int ttc_lqr_bwd_mix(const void* A_diag, const void* B, const void* Q, const void* R_inv,
                    const void* coeff_Qf, const void* Q_basis, int rQ, const void* log_gamma_A,
                    const void* log_gamma_B, const void* log_gamma_Q, const void* h0, const float* lam0,
                    const float* M, const void* d_u, int64_t N, int nh, int d, int du, int T, int dtype,
                    void* grad_A, void* grad_B, void* grad_Q, void* grad_R_inv, void* grad_coeff_Qf,
                    float* grad_basis_partial, int64_t slices, void* grad_lgA, void* grad_lgB,
                    void* grad_lgQ, void* grad_h0, int* status, void* stream);

/*
 * ttc_lqr_bwd_mix without device allocations.  No counterpart in the reference: this entry
 * point exists for callers that cannot allocate device memory -- a host runtime that owns all
 * device memory through its own pool and forbids plug-ins from calling cudaMalloc, or a
 * latency-bound loop where a cudaMalloc / cudaFree (which may synchronise the device) is not
 * acceptable.  Instead of the caller's grad_basis_partial buffer it uses a fixed scratch array
 * inside the library (16 MiB of device memory per GPU, held until process exit; under CUDA's
 * lazy module loading, the default since CUDA 12.2, it is reserved by the first call on each
 * device, CUDA_MODULE_LOADING=EAGER reserves it when the context is created) and runs at most as many CTAs as there are [rQ, d, d] fp32 slices in it (a rank-rQ
 * slice larger than the array is rejected with TTC_ERR_INVALID).  It writes the finished basis
 * gradient grad_basis [rQ, d, d] (fp32) = (S + S^T) / 2, S the sum of the slices; all other
 * arguments and outputs as ttc_lqr_bwd_mix (d = du in {16, 32}).  Allocates nothing and calls
 * no allocating library routine.  The array is shared by all calls and keeps the last call's
 * contents (each call zeroes the slices it uses); calls that overlap on the GPU race on it and
 * must be serialised.  The first call on a device looks up the array's device address; make
 * it before any stream capture.  N = 0 writes zeros to grad_basis (when it is not null).
 */
int ttc_lqr_bwd_mix_noalloc(const void* A_diag, const void* B, const void* Q, const void* R_inv,
                            const void* coeff_Qf, const void* Q_basis, int rQ,
                            const void* log_gamma_A, const void* log_gamma_B, const void* log_gamma_Q,
                            const void* h0, const float* lam0, const float* M, const void* d_u,
                            int64_t N, int nh, int d, int du, int T, int dtype, void* grad_A,
                            void* grad_B, void* grad_Q, void* grad_R_inv, void* grad_coeff_Qf,
                            float* grad_basis, void* grad_lgA, void* grad_lgB, void* grad_lgQ,
                            void* grad_h0, int* status, void* stream);

/*
 * The layer's whole low-rank solve: ttc_lqr_fwd_mix with B and Q given as the layer's
 * low-rank mixtures too (ttc/layers/ttc_layer.py:115-123, the einsums of coeff_B with Bs and of
 * coeff_Q with Qs), so that no [N,d,du] B or [N,d,d] Q tensor exists either:
 *   B[n] = sum_r coeff_B[n,r] B_basis[r],  Q[n] = sum_r coeff_Q[n,r] Q_basis[r],
 * coeff_B [N,rB], B_basis [rB,d,du], coeff_Q [N,rQ] in the activation dtype; Q_basis [rQ,d,d]
 * is the basis of the Q_f mixture as well (the layer's Qs, or Qs Qs^T / sqrt(d) for its
 * cholesky reparametrisation).  Each sum runs in fp32 in rank order and is rounded to the
 * activation dtype, as the einsum it replaces.  B_basis and Q_basis must be 16-byte aligned
 * (TTC_ERR_INVALID otherwise).  Everything else as ttc_lqr_fwd_mix.
 */
int ttc_lqr_fwd_lowrank(const void* A_diag, const void* coeff_B, const void* B_basis, int rB,
                        const void* coeff_Q, const void* R_inv, const void* coeff_Qf, const void* Q_basis,
                        int rQ, const void* log_gamma_A, const void* log_gamma_B, const void* log_gamma_Q,
                        const void* h0, int64_t N, int nh, int d, int du, int T, int dtype, int flags,
                        void* u, float* lam0, float* M, int* status, void* stream);

/*
 * Backward of ttc_lqr_fwd_lowrank (saved lam0 and M required; d = du in {16, 32}).  In place of
 * grad_B, grad_Q and grad_Q_f it writes, in the activation dtype, grad_coeff_B [N,rB] =
 * <grad_B[n], B_basis[r]>, grad_coeff_Q [N,rQ] = <grad_Q[n], Q_basis[r]> and grad_coeff_Qf
 * [N,nh,rQ] (as ttc_lqr_bwd_mix), and per-CTA fp32 partial sums of the basis gradients:
 * grad_B_basis_partial [slices,rB,d,du] (the B-basis gradient is their sum) and
 * grad_basis_partial [slices,rQ,d,d] (the Q-basis gradient is (S + S^T) / 2 with S their sum:
 * the Q_f terms of ttc_lqr_bwd_mix plus sum_n coeff_Q[n,r] grad_Q[n]).  slices from
 * ttc_lqr_bwd_mix_slices; every slice is written.  The bases and both partial buffers must be
 * 16-byte aligned.  Other outputs as ttc_lqr_bwd.
 */
int ttc_lqr_bwd_lowrank(const void* A_diag, const void* coeff_B, const void* B_basis, int rB,
                        const void* coeff_Q, const void* R_inv, const void* coeff_Qf, const void* Q_basis,
                        int rQ, const void* log_gamma_A, const void* log_gamma_B, const void* log_gamma_Q,
                        const void* h0, const float* lam0, const float* M, const void* d_u, int64_t N,
                        int nh, int d, int du, int T, int dtype, void* grad_A, void* grad_coeff_B,
                        float* grad_B_basis_partial, void* grad_coeff_Q, void* grad_R_inv,
                        void* grad_coeff_Qf, float* grad_basis_partial, int64_t slices, void* grad_lgA,
                        void* grad_lgB, void* grad_lgQ, void* grad_h0, int* status, void* stream);

/* Layer epilogue (replaces the fla l2norm of u, ttc/layers/ttc_layer.py:142-143): for each
 * of `rows` rows of n <= 64 values (activation dtype, contiguous),
 *   y = x rsqrt(sum x^2 + 1e-6)   (fp32, rounded to the activation dtype; fla/modules/l2norm.py:42)
 * and its backward  dx = rs g - x rs^3 sum(g x)  with rs = rsqrt(sum x^2 + 1e-6) recomputed from x. */
int ttc_rownorm_fwd(const void* x, int64_t rows, int n, int dtype, void* y, void* stream);
int ttc_rownorm_bwd(const void* x, const void* g, int64_t rows, int n, int dtype, void* dx, void* stream);

/* Elementwise layer prologue (replaces the PyTorch ops of ttc/layers/ttc_layer.py:106-133
 * between in_proj and the low-rank einsums; the einsums stay with the caller).
 * Z [N, W] row-major in the activation dtype, W = nh*(4d + 2du + 1) + rB + rQ: per row nh
 * head slices [h0 d | A_diag d | R_inv du | coeff_Qf d | lgA 1 | lgB du | lgQ d], then
 * coeff_B (rB) and coeff_Q (rQ).  Outputs (activation dtype, contiguous):
 *   A_diag = l2norm(.) [N,nh,d], R_inv = clamp(l2norm(softplus(.)), 1e-6) [N,nh,du],
 *   coeff_Qf = l2norm(softplus(.)) [N,nh,d], lgA = -softplus(.) [N,nh], lgB [N,nh,du],
 *   lgQ [N,nh,d], h0 [N,nh,d], coeff_B = l2norm(.) [N,rB], coeff_Q = l2norm(softplus(.)) [N,rQ]
 * with l2norm(x) = x * rsqrt(sum(x^2) + 1e-6) in fp32 and torch's softplus (threshold 20).
 * d, du, rB, rQ <= 64.  With a status word (device int, may be NULL) and 16-byte aligned rows
 * (Z and W * sizeof(dtype) multiples of 16 bytes) the rows are staged in shared memory by
 * bulk copies (cp.async.bulk, two rows in flight per CTA); a copy that does not complete
 * within about a second sets TTC_STATUS_COPY_TIMEOUT.  Otherwise the warps read Z directly. */
int ttc_prologue_fwd(const void* Z, int64_t N, int nh, int d, int du, int rB, int rQ, int dtype,
                     void* A_diag, void* R_inv, void* coeff_Qf, void* lgA, void* lgB, void* lgQ,
                     void* h0, void* coeff_B, void* coeff_Q, int* status, void* stream);

/* Backward of ttc_prologue_fwd: dZ [N, W] from the gradients of its nine outputs (same
 * shapes and dtype; any of them may be NULL, read as zero).  Z is the forward's input. */
int ttc_prologue_bwd(const void* Z, int64_t N, int nh, int d, int du, int rB, int rQ, int dtype,
                     const void* g_A_diag, const void* g_R_inv, const void* g_coeff_Qf,
                     const void* g_lgA, const void* g_lgB, const void* g_lgQ, const void* g_h0,
                     const void* g_coeff_B, const void* g_coeff_Q, void* dZ, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TTC_B200_H_ */
