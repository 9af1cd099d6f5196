// Pieces of the symplectic Riccati sweep shared by the kernels: the per-step vector layout
// and the in-group Gauss-Jordan solve of Y1 X = RHS.
//
// One group of D threads owns one LQR problem (row n, head h); thread i holds row i of
// that problem's d x d state.
#pragma once

#include "lqr_common.cuh"

namespace ttc {

// Per-step vectors of one head, laid out in group shared memory:
//   [0,D) A_tau   [D,2D) 1/A_tau   [2D,3D) Dq = exp(lgQ tq)
//   [3D,3D+DU) exp(2 lgB tau) R_inv   [3D+DU,3D+2DU) exp(lgB tau) R_inv
template <int D, int DU>
struct SweepVec {
  static constexpr int kAt = 0, kIA = D, kDq = 2 * D, kS2 = 3 * D, kEBR = 3 * D + DU;
  static constexpr int kSize = 3 * D + 2 * DU;
};

// The pivot row of Gauss-Jordan step k: the largest |y| among the rows not yet used, lowest
// index on ties; NaN counts as 0 (so every thread gets exactly one pivot column whatever the
// data).  A whole-warp group (D = 32) reduces one 32-bit key with redux.sync: |y|'s bits with
// the low five replaced by 31 - row (rows whose |y| agree to 2^-18 relative count as tied, so
// the lowest index wins), plus 32 so that a candidate never ties with a used row (key 0);
// 1.8 % faster forward at d = 32, T = 128.  Narrower groups reduce (|y|, row) pairs with
// shuffles (at d = 16 two whole-warp reductions, one per 16-thread group, were 0.6 % slower
// at T = 64).
template <int D>
__device__ __forceinline__ int pivot_row(const Group<D>& G, float y, bool done) {
  const int i = G.i;
  if constexpr (D == 32) {
    const uint32_t mag = __float_as_uint(fmaxf(fabsf(y), 0.0f));
    const uint32_t key = done ? 0u : (((mag & ~31u) + 32u) | static_cast<uint32_t>(31 - i));
    return 31 - static_cast<int>(__reduce_max_sync(0xffffffffu, key) & 31u);
  } else {
    float bv = done ? -1.0f : fmaxf(fabsf(y), 0.0f);
    int bi = i;
#pragma unroll
    for (int o = D / 2; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(G.mask, bv, o, D);
      const int oi = __shfl_xor_sync(G.mask, bi, o, D);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    return bi;
  }
}

// Gauss-Jordan with partial pivoting in registers (D <= 32, one group = D lanes of a
// warp): thread i holds row i of Y1 in y1 and of NR right-hand sides in rhs; the pivot
// row is broadcast by warp shuffles.  Pivot rows are never swapped: each step picks the
// pivot row of the current column (pivot_row) and eliminates that column from every other
// row.  On return rhs holds piv * (row pc
// of Y1^-1 RHS); returns pc and writes piv.
template <int D, int NR>
__device__ __forceinline__ int gauss_jordan_regs(const Group<D>& G, float (&y1)[D], float (&rhs)[NR],
                                                 float& piv) {
  static_assert(D <= 32, "register Gauss-Jordan needs the group inside one warp");
  const int i = G.i;
  bool done = false;
  int pc = 0;
  piv = 1.0f;
#pragma unroll
  for (int k = 0; k < D; ++k) {
    const int bi = pivot_row<D>(G, y1[k], done);
    const float pk = __shfl_sync(G.mask, y1[k], bi, D);
    const bool me = (i == bi);
    const float f = me ? 0.0f : y1[k] * recip(pk);
    if (me) {
      done = true;
      pc = k;
      piv = y1[k];
    } else {
      y1[k] = 0.0f;
    }
#pragma unroll
    for (int c = k + 1; c < D; ++c) y1[c] = fmaf(-f, __shfl_sync(G.mask, y1[c], bi, D), y1[c]);
#pragma unroll
    for (int c = 0; c < NR; ++c) rhs[c] = fmaf(-f, __shfl_sync(G.mask, rhs[c], bi, D), rhs[c]);
  }
  return pc;
}

// gauss_jordan_regs with the pivot row published in group shared memory instead of by warp
// shuffles (D <= 32): the pivot thread writes its row of Y1 and of the right-hand sides
// (16-byte stores), every thread of the group reads it back as 16-byte broadcasts.  Same
// pivots, same arithmetic in the same order: bitwise the results of gauss_jordan_regs with a
// quarter of the instructions for the row transfer.  pbuf: 2 * (D + NR) floats, 16-byte
// aligned, double-buffered by step parity.
template <int D, int NR>
__device__ __forceinline__ int gauss_jordan_smem(const Group<D>& G, float (&y1)[D], float (&rhs)[NR],
                                                 float& piv, float* pbuf) {
  static_assert(D <= 32 && D % 4 == 0 && NR % 4 == 0, "shared-row Gauss-Jordan: one warp, quads");
  constexpr int kRow = D + NR;
  const int i = G.i;
  bool done = false;
  int pc = 0;
  piv = 1.0f;
#pragma unroll
  for (int k = 0; k < D; ++k) {
    const int bi = pivot_row<D>(G, y1[k], done);
    const bool me = (i == bi);
    float4* pr = reinterpret_cast<float4*>(pbuf + (k & 1) * kRow);
    if (me) {
#pragma unroll
      for (int c4 = k / 4; c4 < D / 4; ++c4)
        pr[c4] = make_float4(y1[4 * c4], y1[4 * c4 + 1], y1[4 * c4 + 2], y1[4 * c4 + 3]);
#pragma unroll
      for (int c4 = 0; c4 < NR / 4; ++c4)
        pr[D / 4 + c4] = make_float4(rhs[4 * c4], rhs[4 * c4 + 1], rhs[4 * c4 + 2], rhs[4 * c4 + 3]);
    }
    __syncwarp(G.mask);
    const float4 pk4 = pr[k / 4];
    const float pk = (k & 3) == 0 ? pk4.x : ((k & 3) == 1 ? pk4.y : ((k & 3) == 2 ? pk4.z : pk4.w));
    const float f = me ? 0.0f : y1[k] * recip(pk);
    if (me) {
      done = true;
      pc = k;
      piv = y1[k];
    } else {
      y1[k] = 0.0f;
    }
#pragma unroll
    for (int c4 = (k + 1) / 4; c4 < D / 4; ++c4) {
      const float4 v = pr[c4];
      if (4 * c4 > k) y1[4 * c4] = fmaf(-f, v.x, y1[4 * c4]);
      if (4 * c4 + 1 > k) y1[4 * c4 + 1] = fmaf(-f, v.y, y1[4 * c4 + 1]);
      if (4 * c4 + 2 > k) y1[4 * c4 + 2] = fmaf(-f, v.z, y1[4 * c4 + 2]);
      if (4 * c4 + 3 > k) y1[4 * c4 + 3] = fmaf(-f, v.w, y1[4 * c4 + 3]);
    }
#pragma unroll
    for (int c4 = 0; c4 < NR / 4; ++c4) {
      const float4 v = pr[D / 4 + c4];
      rhs[4 * c4] = fmaf(-f, v.x, rhs[4 * c4]);
      rhs[4 * c4 + 1] = fmaf(-f, v.y, rhs[4 * c4 + 1]);
      rhs[4 * c4 + 2] = fmaf(-f, v.z, rhs[4 * c4 + 2]);
      rhs[4 * c4 + 3] = fmaf(-f, v.w, rhs[4 * c4 + 3]);
    }
  }
  __syncwarp(G.mask);
  return pc;
}

// The same elimination for a group spanning several warps (D = 64): the pivot search
// combines the warps' shuffle results through shared memory and the pivot row is published
// in a double-buffered shared row.  pbuf holds GjBcast<D, NR>::kSize floats.
template <int D, int NR>
struct GjBcast {
  static constexpr int kRow = D + NR;
  static constexpr int kSize = 2 * kRow + 4 * (D / 32);
};

template <int D, int NR>
__device__ __forceinline__ int gauss_jordan_bcast(const Group<D>& G, float (&y1)[D], float (&rhs)[NR],
                                                  float& piv, float* pbuf) {
  constexpr int kWarps = D / 32;
  const int i = G.i, w = i >> 5;
  float* cbuf = pbuf + 2 * GjBcast<D, NR>::kRow;
  bool done = false;
  int pc = 0;
  piv = 1.0f;
#pragma unroll
  for (int k = 0; k < D; ++k) {
    float bv = done ? -1.0f : fmaxf(fabsf(y1[k]), 0.0f);
    int bi = i;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    float* cb = cbuf + (k & 1) * 2 * kWarps;
    if ((i & 31) == 0) {
      cb[2 * w] = bv;
      cb[2 * w + 1] = __int_as_float(bi);
    }
    G.sync();
    bv = cb[0];
    bi = __float_as_int(cb[1]);
#pragma unroll
    for (int ww = 1; ww < kWarps; ++ww) {
      const float ov = cb[2 * ww];
      const int oi = __float_as_int(cb[2 * ww + 1]);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    const bool me = (i == bi);
    float* pr = pbuf + (k & 1) * GjBcast<D, NR>::kRow;
    if (me) {
#pragma unroll
      for (int c = k; c < D; ++c) pr[c] = y1[c];
#pragma unroll
      for (int c = 0; c < NR; ++c) pr[D + c] = rhs[c];
      done = true;
      pc = k;
      piv = y1[k];
    }
    G.sync();
    if (!me) {
      const float f = y1[k] * recip(pr[k]);
      y1[k] = 0.0f;
#pragma unroll
      for (int c = k + 1; c < D; ++c) y1[c] = fmaf(-f, pr[c], y1[c]);
#pragma unroll
      for (int c = 0; c < NR; ++c) rhs[c] = fmaf(-f, pr[D + c], rhs[c]);
    }
  }
  G.sync();
  return pc;
}

// Shared floats the group's pivot-row buffer needs (GjRow<D, NR>::kSize, 16-byte aligned):
// the shared-row elimination for D > 32, or for D <= 32 with quads of right-hand sides.
template <int D, int NR>
struct GjRow {
  static constexpr bool kShared = D > 32 || NR % 4 == 0;
  static constexpr int kSize = D > 32 ? GjBcast<D, NR>::kSize : (kShared ? 2 * (D + NR) : 0);
};

// Gauss-Jordan for any supported D; pbuf (GjRow<D, NR>::kSize floats of group shared memory)
// carries the pivot row when the group spans several warps, or when the right-hand sides come
// in quads (16-byte transfers instead of one shuffle per value; bitwise the same results).
template <int D, int NR>
__device__ __forceinline__ int gauss_jordan_group(const Group<D>& G, float (&y1)[D], float (&rhs)[NR],
                                                  float& piv, float* pbuf) {
  if constexpr (D > 32) {
    return gauss_jordan_bcast<D, NR>(G, y1, rhs, piv, pbuf);
  } else if constexpr (NR % 4 == 0) {
    return gauss_jordan_smem<D, NR>(G, y1, rhs, piv, pbuf);
  } else {
    return gauss_jordan_regs<D, NR>(G, y1, rhs, piv);
  }
}

}  // namespace ttc
