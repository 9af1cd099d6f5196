// Elementwise prologue of TTCLayer.forward (ttc/layers/ttc_layer.py:104-135) and its
// backward, one kernel each way.  The in_proj output Z [N, W] of a batch row is
//   nh head slices [h0 d | A_diag d | R_inv du | coeff_Qf d | lg_A 1 | lg_B du | lg_Q d]
//   then coeff_B (rB) and coeff_Q (rQ),
// W = nh (4d + 2du + 1) + rB + rQ.  Forward:
//   A_diag = l2norm(A), R_inv = clamp(l2norm(softplus(R)), min=1e-6), coeff_Qf =
//   l2norm(softplus(cQf)), lg_* = -softplus(lg_*), h0 = h0, coeff_B = l2norm(cB),
//   coeff_Q = l2norm(softplus(cQ)),
// with l2norm(x) = x rsqrt(sum x^2 + 1e-6) in fp32 (fla/modules/l2norm.py:42) and
// softplus(x) = x > 20 ? x : log1p(exp(x)) (torch's default threshold).  Results are rounded
// to the activation dtype where the reference's PyTorch ops round them (after each op), and
// the backward applies the chain rule of the same ops with the same roundings of the
// intermediate gradients.  One warp per (row, head) slice plus one warp per row for the
// coefficients; every sum is a fixed shuffle tree, so results are run-to-run identical.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>

#include "lqr_common.cuh"
#include "ttc_b200.h"

namespace ttc {
int set_error(int code, const char* msg);
}

namespace {

using ttc::ldf;
using ttc::stf;

constexpr float kEps = 1e-6f;
constexpr float kRinvMin = 1e-6f;
constexpr int kPer = 2;  // elements per lane: vectors up to 64 long

template <typename T>
__device__ __forceinline__ float round_t(float x) {
  if constexpr (sizeof(T) == 2) {
    return __bfloat162float(__float2bfloat16_rn(x));
  } else {
    return x;
  }
}

__device__ __forceinline__ float softplus(float x) { return x > 20.0f ? x : log1pf(expf(x)); }
// d softplus / dx = e^x / (e^x + 1) (1 above the threshold), as torch's softplus backward.
__device__ __forceinline__ float softplus_grad(float x, float g) {
  if (x > 20.0f) return g;
  const float z = expf(x);
  return g * z / (z + 1.0f);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// A vector of n <= 64 values spread over the warp: lane l holds elements l and l + 32.
struct Vec {
  float v[kPer];
  bool on[kPer];
};

template <typename T>
__device__ __forceinline__ Vec load_vec(const T* p, int n, int lane) {
  Vec x;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int e = lane + 32 * k;
    x.on[k] = e < n;
    x.v[k] = x.on[k] ? ldf(p + e) : 0.f;
  }
  return x;
}

template <typename T>
__device__ __forceinline__ void store_vec(T* p, const Vec& x) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < kPer; ++k)
    if (x.on[k]) stf(p + lane + 32 * k, x.v[k]);
}

__device__ __forceinline__ float sum_sq(const Vec& x) {
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < kPer; ++k) s = fmaf(x.v[k], x.v[k], s);
  return warp_sum(s);
}

// y = round_T(x rsqrt(sum x^2 + eps)); returns rs.
template <typename T>
__device__ __forceinline__ float l2norm_fwd(const Vec& x, Vec& y) {
  const float rs = rsqrtf(sum_sq(x) + kEps);
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    y.on[k] = x.on[k];
    y.v[k] = round_t<T>(x.v[k] * rs);
  }
  return rs;
}

// dx = round_T(rs g - x rs^3 sum(g x)) for y = x rs(x) (autograd of the fp32 formula).
template <typename T>
__device__ __forceinline__ void l2norm_bwd(const Vec& x, float rs, const Vec& g, Vec& dx) {
  float dot = 0.f;
#pragma unroll
  for (int k = 0; k < kPer; ++k) dot = fmaf(g.v[k], x.v[k], dot);
  dot = warp_sum(dot);
  const float c = dot * rs * rs * rs;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    dx.on[k] = x.on[k];
    dx.v[k] = round_t<T>(fmaf(rs, g.v[k], -c * x.v[k]));
  }
}

template <typename T>
__device__ __forceinline__ Vec softplus_vec(const Vec& x) {
  Vec y;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    y.on[k] = x.on[k];
    y.v[k] = x.on[k] ? round_t<T>(softplus(x.v[k])) : 0.f;
  }
  return y;
}

template <typename T>
__device__ __forceinline__ Vec grad_or_zero(const T* p, int n, int lane) {
  if (p == nullptr) {
    Vec z;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      z.v[k] = 0.f;
      z.on[k] = lane + 32 * k < n;
    }
    return z;
  }
  return load_vec(p, n, lane);
}

struct Dims {
  int nh, d, du, rB, rQ, Hs, W;
  int oA, oR, oQf, oGA, oGB, oGQ;  // offsets inside a head slice (h0 at 0)
  __host__ __device__ Dims(int nh_, int d_, int du_, int rB_, int rQ_)
      : nh(nh_), d(d_), du(du_), rB(rB_), rQ(rQ_) {
    oA = d;
    oR = 2 * d;
    oQf = 2 * d + du;
    oGA = 3 * d + du;
    oGB = oGA + 1;
    oGQ = oGB + du;
    Hs = 4 * d + 2 * du + 1;
    W = nh * Hs + rB + rQ;
  }
};

template <typename T>
__global__ void __launch_bounds__(256) prologue_fwd_kernel(
    const T* __restrict__ Z, int64_t N, Dims D, T* __restrict__ A_out, T* __restrict__ R_out,
    T* __restrict__ cQf_out, T* __restrict__ lgA_out, T* __restrict__ lgB_out,
    T* __restrict__ lgQ_out, T* __restrict__ h0_out, T* __restrict__ cB_out,
    T* __restrict__ cQ_out) {
  const int lane = threadIdx.x & 31;
  const int64_t slots = N * (D.nh + 1);
  const int64_t stride = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < slots; w += stride) {
    const int64_t n = w / (D.nh + 1);
    const int h = static_cast<int>(w % (D.nh + 1));
    const T* zr = Z + n * D.W;
    if (h == D.nh) {  // per-row mixture coefficients
      Vec cb = load_vec(zr + D.nh * D.Hs, D.rB, lane), y;
      l2norm_fwd<T>(cb, y);
      store_vec(cB_out + n * D.rB, y);
      Vec cq = softplus_vec<T>(load_vec(zr + D.nh * D.Hs + D.rB, D.rQ, lane));
      l2norm_fwd<T>(cq, y);
      store_vec(cQ_out + n * D.rQ, y);
      continue;
    }
    const T* z = zr + (int64_t)h * D.Hs;
    const int64_t p = n * D.nh + h;
    Vec y;
    store_vec(h0_out + p * D.d, load_vec(z, D.d, lane));
    l2norm_fwd<T>(load_vec(z + D.oA, D.d, lane), y);
    store_vec(A_out + p * D.d, y);
    l2norm_fwd<T>(softplus_vec<T>(load_vec(z + D.oR, D.du, lane)), y);
#pragma unroll
    for (int k = 0; k < kPer; ++k) y.v[k] = round_t<T>(fmaxf(y.v[k], kRinvMin));
    store_vec(R_out + p * D.du, y);
    l2norm_fwd<T>(softplus_vec<T>(load_vec(z + D.oQf, D.d, lane)), y);
    store_vec(cQf_out + p * D.d, y);
    if (lane == 0) stf(lgA_out + p, -round_t<T>(softplus(ldf(z + D.oGA))));
    Vec g = softplus_vec<T>(load_vec(z + D.oGB, D.du, lane));
#pragma unroll
    for (int k = 0; k < kPer; ++k) g.v[k] = -g.v[k];
    store_vec(lgB_out + p * D.du, g);
    g = softplus_vec<T>(load_vec(z + D.oGQ, D.d, lane));
#pragma unroll
    for (int k = 0; k < kPer; ++k) g.v[k] = -g.v[k];
    store_vec(lgQ_out + p * D.d, g);
  }
}

// d/dz of l2norm(softplus(z)) (optionally clamped from below after the l2norm) for the
// incoming gradient g of the result.
template <typename T, bool CLAMP>
__device__ __forceinline__ Vec softplus_l2norm_bwd(const Vec& z, const Vec& g) {
  const Vec sp = softplus_vec<T>(z);
  Vec y, gy = g, dsp, dz;
  const float rs = l2norm_fwd<T>(sp, y);
  if constexpr (CLAMP) {
    const float lo = round_t<T>(kRinvMin);
#pragma unroll
    for (int k = 0; k < kPer; ++k) gy.v[k] = y.v[k] >= lo ? g.v[k] : 0.f;
  }
  l2norm_bwd<T>(sp, rs, gy, dsp);
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    dz.on[k] = z.on[k];
    dz.v[k] = z.on[k] ? round_t<T>(softplus_grad(z.v[k], dsp.v[k])) : 0.f;
  }
  return dz;
}

// d/dz of -softplus(z): the negated gradient through softplus.
template <typename T>
__device__ __forceinline__ Vec neg_softplus_bwd(const Vec& z, const Vec& g) {
  Vec dz;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    dz.on[k] = z.on[k];
    dz.v[k] = z.on[k] ? round_t<T>(softplus_grad(z.v[k], -g.v[k])) : 0.f;
  }
  return dz;
}

template <typename T>
__global__ void __launch_bounds__(256) prologue_bwd_kernel(
    const T* __restrict__ Z, int64_t N, Dims D, const T* __restrict__ gA, const T* __restrict__ gR,
    const T* __restrict__ gcQf, const T* __restrict__ glgA, const T* __restrict__ glgB,
    const T* __restrict__ glgQ, const T* __restrict__ gh0, const T* __restrict__ gcB,
    const T* __restrict__ gcQ, T* __restrict__ dZ) {
  const int lane = threadIdx.x & 31;
  const int64_t slots = N * (D.nh + 1);
  const int64_t stride = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < slots; w += stride) {
    const int64_t n = w / (D.nh + 1);
    const int h = static_cast<int>(w % (D.nh + 1));
    const T* zr = Z + n * D.W;
    T* dr = dZ + n * D.W;
    if (h == D.nh) {
      const T* zb = zr + D.nh * D.Hs;
      Vec cb = load_vec(zb, D.rB, lane), y, dcb;
      const float rs = l2norm_fwd<T>(cb, y);
      l2norm_bwd<T>(cb, rs, grad_or_zero(gcB ? gcB + n * D.rB : nullptr, D.rB, lane), dcb);
      store_vec(dr + D.nh * D.Hs, dcb);
      const Vec cq = load_vec(zb + D.rB, D.rQ, lane);
      store_vec(dr + D.nh * D.Hs + D.rB,
                softplus_l2norm_bwd<T, false>(cq, grad_or_zero(gcQ ? gcQ + n * D.rQ : nullptr, D.rQ, lane)));
      continue;
    }
    const T* z = zr + (int64_t)h * D.Hs;
    T* dz = dr + (int64_t)h * D.Hs;
    const int64_t p = n * D.nh + h;
    store_vec(dz, grad_or_zero(gh0 ? gh0 + p * D.d : nullptr, D.d, lane));
    {
      Vec a = load_vec(z + D.oA, D.d, lane), y, da;
      const float rs = l2norm_fwd<T>(a, y);
      l2norm_bwd<T>(a, rs, grad_or_zero(gA ? gA + p * D.d : nullptr, D.d, lane), da);
      store_vec(dz + D.oA, da);
    }
    store_vec(dz + D.oR, softplus_l2norm_bwd<T, true>(load_vec(z + D.oR, D.du, lane),
                                                        grad_or_zero(gR ? gR + p * D.du : nullptr, D.du, lane)));
    store_vec(dz + D.oQf, softplus_l2norm_bwd<T, false>(load_vec(z + D.oQf, D.d, lane),
                                                          grad_or_zero(gcQf ? gcQf + p * D.d : nullptr, D.d, lane)));
    if (lane == 0) {
      const float g = glgA ? ldf(glgA + p) : 0.f;
      stf(dz + D.oGA, round_t<T>(softplus_grad(ldf(z + D.oGA), -g)));
    }
    store_vec(dz + D.oGB, neg_softplus_bwd<T>(load_vec(z + D.oGB, D.du, lane),
                                               grad_or_zero(glgB ? glgB + p * D.du : nullptr, D.du, lane)));
    store_vec(dz + D.oGQ, neg_softplus_bwd<T>(load_vec(z + D.oGQ, D.d, lane),
                                               grad_or_zero(glgQ ? glgQ + p * D.d : nullptr, D.d, lane)));
  }
}

int check_dims(int64_t N, int nh, int d, int du, int rB, int rQ, int dtype) {
  if (N < 0 || nh < 1 || d < 1 || du < 1 || rB < 1 || rQ < 1)
    return ttc::set_error(TTC_ERR_INVALID, "prologue: sizes must be positive");
  if (d > 32 * kPer || du > 32 * kPer || rB > 32 * kPer || rQ > 32 * kPer)
    return ttc::set_error(TTC_ERR_UNSUPPORTED, "prologue: h_dim, u_dim and ranks must be <= 64");
  if (dtype != TTC_DTYPE_F32 && dtype != TTC_DTYPE_BF16)
    return ttc::set_error(TTC_ERR_INVALID, "prologue: dtype must be TTC_DTYPE_F32 or TTC_DTYPE_BF16");
  return TTC_OK;
}

unsigned grid_for(int64_t N, int nh) {
  const int64_t warps = N * (nh + 1);
  int64_t blocks = (warps + 7) / 8;
  const int64_t cap = 148 * 32;  // grid-stride beyond 32 CTAs per SM
  return static_cast<unsigned>(blocks < cap ? blocks : cap);
}

int launched(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return TTC_OK;
  char buf[256];
  snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
  return ttc::set_error(TTC_ERR_CUDA, buf);
}

}  // namespace

extern "C" int ttc_prologue_fwd(const void* Z, int64_t N, int nh, int d, int du, int rB, int rQ, int dtype,
                                void* A_diag, void* R_inv, void* coeff_Qf, void* lgA, void* lgB, void* lgQ,
                                void* h0, void* coeff_B, void* coeff_Q, void* stream) {
  if (int rc = check_dims(N, nh, d, du, rB, rQ, dtype)) return rc;
  if (N == 0) return TTC_OK;
  if (!Z || !A_diag || !R_inv || !coeff_Qf || !lgA || !lgB || !lgQ || !h0 || !coeff_B || !coeff_Q)
    return ttc::set_error(TTC_ERR_INVALID, "prologue_fwd: null pointer");
  const Dims D(nh, d, du, rB, rQ);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = grid_for(N, nh);
  if (dtype == TTC_DTYPE_F32) {
    using T = float;
    prologue_fwd_kernel<T><<<grid, 256, 0, st>>>((const T*)Z, N, D, (T*)A_diag, (T*)R_inv, (T*)coeff_Qf,
                                                 (T*)lgA, (T*)lgB, (T*)lgQ, (T*)h0, (T*)coeff_B, (T*)coeff_Q);
  } else {
    using T = __nv_bfloat16;
    prologue_fwd_kernel<T><<<grid, 256, 0, st>>>((const T*)Z, N, D, (T*)A_diag, (T*)R_inv, (T*)coeff_Qf,
                                                 (T*)lgA, (T*)lgB, (T*)lgQ, (T*)h0, (T*)coeff_B, (T*)coeff_Q);
  }
  return launched("prologue_fwd_kernel launch");
}

extern "C" int ttc_prologue_bwd(const void* Z, int64_t N, int nh, int d, int du, int rB, int rQ, int dtype,
                                const void* g_A_diag, const void* g_R_inv, const void* g_coeff_Qf,
                                const void* g_lgA, const void* g_lgB, const void* g_lgQ, const void* g_h0,
                                const void* g_coeff_B, const void* g_coeff_Q, void* dZ, void* stream) {
  if (int rc = check_dims(N, nh, d, du, rB, rQ, dtype)) return rc;
  if (N == 0) return TTC_OK;
  if (!Z || !dZ) return ttc::set_error(TTC_ERR_INVALID, "prologue_bwd: null pointer");
  const Dims D(nh, d, du, rB, rQ);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = grid_for(N, nh);
  if (dtype == TTC_DTYPE_F32) {
    using T = float;
    prologue_bwd_kernel<T><<<grid, 256, 0, st>>>(
        (const T*)Z, N, D, (const T*)g_A_diag, (const T*)g_R_inv, (const T*)g_coeff_Qf, (const T*)g_lgA,
        (const T*)g_lgB, (const T*)g_lgQ, (const T*)g_h0, (const T*)g_coeff_B, (const T*)g_coeff_Q, (T*)dZ);
  } else {
    using T = __nv_bfloat16;
    prologue_bwd_kernel<T><<<grid, 256, 0, st>>>(
        (const T*)Z, N, D, (const T*)g_A_diag, (const T*)g_R_inv, (const T*)g_coeff_Qf, (const T*)g_lgA,
        (const T*)g_lgB, (const T*)g_lgQ, (const T*)g_h0, (const T*)g_coeff_B, (const T*)g_coeff_Q, (T*)dZ);
  }
  return launched("prologue_bwd_kernel launch");
}
