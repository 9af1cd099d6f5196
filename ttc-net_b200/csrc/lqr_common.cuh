// Shared device helpers for the TTC LQR kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ttc {

// Renormalisation threshold of the symplectic sweep (ttc/solvers/fused_lqr.py:94,
// symplectic_iter.py:286-300) and the instability bound of the reference's checks
// (fused_lqr.py:99-110,243-246).
constexpr float kNormThreshold = 1e3f;
constexpr float kUnstable = 1e6f;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float ldf(const float* p) { return *p; }
__device__ __forceinline__ float ldf(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void stf(float* p, float v) { *p = v; }
__device__ __forceinline__ void stf(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

// Rounds to the activation dtype (identity for float).
template <typename T>
__device__ __forceinline__ float round_to(float x) {
  if constexpr (sizeof(T) == 2) {
    return __bfloat162float(__float2bfloat16_rn(x));
  } else {
    return x;
  }
}

// The layer's low-rank parametrisation of B and Q (ttc_layer.py:115-123): per batch row n
// B[n] = sum_r coeff_B[n][r] B_basis[r] and Q[n] = sum_r coeff_Q[n][r] Q_basis[r], formed
// by the solver kernels instead of being read as [N, d, du] / [N, d, d] tensors.  Q_basis is
// the basis of the Q_f mixture too.  Backward outputs: grad_coeff_B [N, rB] and
// grad_coeff_Q [N, rQ] = <grad_B[n], B_basis[r]>, <grad_Q[n], Q_basis[r]>, and per-CTA
// partial sums of sum_n coeff[n][r] grad[n] (the basis gradients; Q's go into the Q_f
// mixture's partial slices).  cB == nullptr: B and Q are read as tensors.
template <typename TIn>
struct LowRank {
  const TIn* cB = nullptr;
  const TIn* Bb = nullptr;
  int rB = 0;
  const TIn* cQ = nullptr;
  TIn* gcB = nullptr;
  TIn* gcQ = nullptr;
  float* gBb = nullptr;  // [gridDim.x][rB][d][du]
};

// Four consecutive values as floats (16-byte aligned for float, 8-byte for bf16).
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ld4(const __nv_bfloat16* p) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u), __uint_as_float(v.y << 16),
                     __uint_as_float(v.y & 0xffff0000u));
}

// Element e of the mixture sum_r c[r] basis[r][e] (each basis matrix `len` elements),
// summed in rank order in fp32 and rounded to the activation dtype like the einsum it
// replaces.
template <typename TIn>
__device__ __forceinline__ float mix_elem(const TIn* __restrict__ c, const TIn* __restrict__ basis, int rank,
                                          int len, int e) {
  float s = 0.f;
  // unrolled so that the loads of eight ranks are in flight together (the sum stays in rank
  // order); the bases are L2-resident, so this is latency, not bandwidth
#pragma unroll 8
  for (int r = 0; r < rank; ++r) s = fmaf(ldf(c + r), ldf(basis + (int64_t)r * len + e), s);
  return round_to<TIn>(s);
}

// Four consecutive elements e..e+3 of the mixture (e a multiple of 4), as mix_elem.
template <typename TIn>
__device__ __forceinline__ float4 mix4(const TIn* __restrict__ c, const TIn* __restrict__ basis, int rank, int len,
                                       int e) {
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
  for (int r = 0; r < rank; ++r) {
    const float cr = ldf(c + r);
    const float4 b = ld4(basis + (int64_t)r * len + e);
    s.x = fmaf(cr, b.x, s.x);
    s.y = fmaf(cr, b.y, s.y);
    s.z = fmaf(cr, b.z, s.z);
    s.w = fmaf(cr, b.w, s.w);
  }
  return make_float4(round_to<TIn>(s.x), round_to<TIn>(s.y), round_to<TIn>(s.z), round_to<TIn>(s.w));
}

// mix4 of two mixtures at once (B and Q of a row): their loads interleave in one rank loop.
template <typename TIn>
__device__ __forceinline__ void mix4_pair(const TIn* __restrict__ c1, const TIn* __restrict__ b1, int rank1,
                                          const TIn* __restrict__ c2, const TIn* __restrict__ b2, int rank2,
                                          int len, int e, float4& o1, float4& o2) {
  float4 s1 = make_float4(0.f, 0.f, 0.f, 0.f), s2 = s1;
  const int rank = rank1 > rank2 ? rank1 : rank2;
#pragma unroll 8
  for (int r = 0; r < rank; ++r) {
    if (r < rank1) {
      const float cr = ldf(c1 + r);
      const float4 b = ld4(b1 + (int64_t)r * len + e);
      s1.x = fmaf(cr, b.x, s1.x);
      s1.y = fmaf(cr, b.y, s1.y);
      s1.z = fmaf(cr, b.z, s1.z);
      s1.w = fmaf(cr, b.w, s1.w);
    }
    if (r < rank2) {
      const float cr = ldf(c2 + r);
      const float4 b = ld4(b2 + (int64_t)r * len + e);
      s2.x = fmaf(cr, b.x, s2.x);
      s2.y = fmaf(cr, b.y, s2.y);
      s2.z = fmaf(cr, b.z, s2.z);
      s2.w = fmaf(cr, b.w, s2.w);
    }
  }
  o1 = make_float4(round_to<TIn>(s1.x), round_to<TIn>(s1.y), round_to<TIn>(s1.z), round_to<TIn>(s1.w));
  o2 = make_float4(round_to<TIn>(s2.x), round_to<TIn>(s2.y), round_to<TIn>(s2.z), round_to<TIn>(s2.w));
}

// True for NaN, +-Inf and |v| >= 1e6: the reference's isnan | isinf | abs >= 1e6.
__device__ __forceinline__ bool unstable(float v) { return !(fabsf(v) < kUnstable); }

// 1/x without the IEEE-division slow-path call (whose register save/restore spills every
// live value of the unrolled state): the hardware approximation from __fdividef refined by
// one Newton-Raphson step r <- r + r (1 - x r), within about 1 ulp for normal x.
__device__ __forceinline__ float recip(float x) {
  const float r = __fdividef(1.0f, x);
  return fmaf(r, fmaf(-x, r, 1.0f), r);
}

// Paired fp32 arithmetic (PTX `fma/add/mul.rn.f32x2`, sm_100a): one instruction performs
// two independent fp32 operations, each rounded exactly like its scalar counterpart, so a
// kernel written with pairs gives bitwise the results of the scalar code in the same order
// while issuing half the instructions.  A pair lives in one 64-bit register (x = low half).
using f2 = unsigned long long;
__device__ __forceinline__ f2 pk2(float x, float y) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(x), "f"(y));
  return r;
}
__device__ __forceinline__ f2 dup2(float x) { return pk2(x, x); }
__device__ __forceinline__ void up2(f2 v, float& x, float& y) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(x), "=f"(y) : "l"(v));
}
__device__ __forceinline__ float sum2(f2 v) {
  float x, y;
  up2(v, x, y);
  return x + y;
}
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
  f2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b) {
  f2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
  f2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2 sub2(f2 a, f2 b) {
  f2 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// The two halves of a float4 (broadcast shared-memory reads come as float4).
__device__ __forceinline__ f2 lo2(const float4& v) { return pk2(v.x, v.y); }
__device__ __forceinline__ f2 hi2(const float4& v) { return pk2(v.z, v.w); }

// exp(lg * t) as exp2(lg * log2(e) * t); lg2 is lg pre-multiplied by log2(e).
__device__ __forceinline__ float exp_scaled(float lg2, float t) { return exp2f(lg2 * t); }

// A group of D threads owns one LQR problem (one head of one row); thread i of the
// group holds row i of the d x d state.  D = 16 packs two groups in a warp; D = 64
// spans two warps and synchronises with a named barrier (0 is __syncthreads).
template <int D>
struct Group {
  int g;          // group index in the CTA
  int i;          // row owned by this thread
  unsigned mask;  // lanes of this group inside its warp
  __device__ __forceinline__ explicit Group(int tid) : g(tid / D), i(tid % D) {
    if constexpr (D < 32) {
      mask = ((1u << D) - 1u) << (((tid & 31) / D) * D);
    } else {
      mask = 0xffffffffu;
    }
  }
  // D > 32: named barrier 8 + g (the tensor-core kernels use ids 1..4 for their tile
  // slots; a CTA has at most 8 such groups).
  __device__ __forceinline__ void sync() const {
    if constexpr (D <= 32) {
      __syncwarp(mask);
    } else {
      asm volatile("bar.sync %0, %1;" ::"r"(g + 8), "r"(D) : "memory");
    }
  }
};

// Max over the lanes of a warp-sized row block (min(D, 32) rows).  Deterministic.
template <int D>
__device__ __forceinline__ float rowblock_max(const Group<D>& G, float v) {
  constexpr int W = D < 32 ? D : 32;
#pragma unroll
  for (int o = W / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(G.mask, v, o, W));
  return v;
}

// Sum over the D threads of a group, same fixed order on every call.  For D = 64
// the two warp partials meet in `red` (2 floats of group scratch).
template <int D>
__device__ __forceinline__ float group_sum(const Group<D>& G, float v, float* red) {
  constexpr int W = D < 32 ? D : 32;
#pragma unroll
  for (int o = W / 2; o > 0; o >>= 1) v += __shfl_xor_sync(G.mask, v, o, W);
  if constexpr (D > 32) {
    if ((G.i & 31) == 0) red[G.i >> 5] = v;
    G.sync();
    v = red[0] + red[1];
    G.sync();
  }
  return v;
}

}  // namespace ttc
