// Forward-in-time adjoint of the LQR solve (symplectic_iter.py:715-885) on warp-level
// tensor-core MMAs, for the backward of a forward that saved lambda0 (and M = Y1^-1 Y3, or
// the contracted d_p = Y1^-1 Y3 d_u).
//
// Every head of a batch row n shares that row's B and Q, so the T-step adjoint of the row's
// heads is a chain of small matrix products: per step, [h; dh] Q^T, [lambda; dlambda] B and
// [u e^lgB; du e^lgB] B^T, plus the rank-2 updates of grad_B and grad_Q summed over heads.
// One warp owns 8 heads of one row.  The 16 rows of an m16n8k8 MMA are the 8 heads'
// primal vectors (rows 0-7) and their tangents (rows 8-15), so thread (g, t) = (lane / 4,
// lane % 4) holds, for head g, entries {8j + 2t, 8j + 2t + 1} (j < d / 8) of both: all the
// elementwise work of the recursion is thread-local.  The output fragment of one product is
// fed back as the A fragment of the next without moving data: the K order of the constant
// operand is permuted to match (fragment slot t <-> entry 8kk + 2t, slot t + 4 <-> entry
// 8kk + 2t + 1).  Each product runs in 3xTF32 (A_lo B_hi + A_hi B_lo + A_hi B_hi), close to
// the fp32 sums of the reference.  grad_B and grad_Q sum over heads, i.e. contract over the
// MMA's M rows: the vectors go through a small shared staging matrix and a second MMA with
// K = the 16 (head, primal / tangent) rows accumulates them in registers over all steps;
// the output tiles are shared out among the row's warps, each summing every warp's staged
// vectors in warp order: deterministic.
#pragma once

#include "lqr_kernels.cuh"

namespace ttc {

namespace wmma {

__device__ __forceinline__ void split(float x, uint32_t& hi, uint32_t& lo) {
  hi = __float_as_uint(x) & 0xffffe000u;
  lo = __float_as_uint(x - __uint_as_float(hi));
}

// x rounded to tf32 (nearest, ties away from zero): the operand of a single-pass tf32 MMA.
__device__ __forceinline__ uint32_t rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// D (16x8, f32) += A (16x8, tf32, row) * B (8x8, tf32, col).
__device__ __forceinline__ void m16n8k8(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

}  // namespace wmma

// bf16 activations: the grad_B / grad_Q contractions over heads in single-pass rounded tf32
// (TTC_BF16_ONEPASS=0 builds keep them in 3xTF32).
#ifndef TTC_BF16_ONEPASS
#define TTC_BF16_ONEPASS 1
#endif

template <int D>
struct AdjMma {
  static_assert(D % 16 == 0, "d must be a multiple of 16");
  static constexpr int NT = D / 8;             // n-tiles of an output = k-steps of an input
  static constexpr int MT = D / 16;            // m-tiles of grad_B / grad_Q
  static constexpr int kUnits = 2 * MT;        // (grad_B | grad_Q, m-tile) units of NT tiles
  static constexpr int kFrag = NT * NT * 128;  // floats of one constant operand (hi + lo)
  static constexpr int SS = D + 8;             // staging row stride (bank-conflict free)
  static constexpr int kStage = 16 * SS;
  // per row: operands Q^T, B, B^T, Q and a symmetry flag; per warp: 3 staging matrices,
  // double-buffered by step parity
  static constexpr int kRow = 4 * kFrag + 4;
  static constexpr int kWarp = 2 * 3 * kStage;
  static constexpr int kMaxWarps = 8;
  // OWN (d = 16): every warp accumulates all units from its own heads and the row's warps
  // add their partial sums at the end.  Shared (d >= 32, where all units would not fit in
  // registers): the units are dealt out to the row's warps, which meet at a named barrier
  // every step and sum all the row's staged vectors.
  static constexpr bool kOwn = D <= 16;
  static constexpr size_t kSmemLimit = 227 * 1024;
  static int warps_per_row(int nh) { return (nh + 7) / 8; }
  static size_t bytes_for(int rows, int wpr) {
    return sizeof(float) * ((size_t)rows * kRow + (size_t)rows * wpr * kWarp);
  }
  static int rows_per_cta(int nh) {
    const int wpr = warps_per_row(nh);
    int r = wpr >= kMaxWarps ? 1 : kMaxWarps / wpr;
    while (r > 1 && bytes_for(r, wpr) > kSmemLimit) --r;
    return r;
  }
  static int warps(int nh) { return warps_per_row(nh) * rows_per_cta(nh); }
  // grad_B / grad_Q units each warp of a row accumulates
  static int units_per_warp(int nh) {
    if (kOwn) return kUnits;
    const int wpr = warps_per_row(nh);
    return (kUnits + wpr - 1) / wpr;
  }
  static size_t bytes(int nh) { return bytes_for(rows_per_cta(nh), warps_per_row(nh)); }
  static bool fits(int nh) {
    return warps_per_row(nh) <= kMaxWarps && bytes(nh) <= kSmemLimit && units_per_warp(nh) <= 2;
  }
};

// Constant operand W (K x N = D x D, W[k][n] = get(k, n)) in fragment order: for k-step kk,
// n-tile nj and lane (g, t), the float4 (hi b0, hi b1, lo b0, lo b1) with
// b0 = W[8kk + 2t][8nj + g], b1 = W[8kk + 2t + 1][8nj + g].
template <int D, typename Get>
__device__ __forceinline__ void build_operand(float* dst, Get get, int tid, int nthreads) {
  constexpr int NT = D / 8;
  for (int e = tid; e < NT * NT * 32; e += nthreads) {
    const int lane = e & 31, kn = e >> 5, kk = kn / NT, nj = kn % NT;
    const int g = lane >> 2, t = lane & 3;
    const float w0 = get(8 * kk + 2 * t, 8 * nj + g), w1 = get(8 * kk + 2 * t + 1, 8 * nj + g);
    const float h0 = __uint_as_float(__float_as_uint(w0) & 0xffffe000u);
    const float h1 = __uint_as_float(__float_as_uint(w1) & 0xffffe000u);
    reinterpret_cast<float4*>(dst)[e] = make_float4(h0, h1, w0 - h0, w1 - h1);
  }
}

// out (16 x D, output-fragment order) = in (16 x D, output-fragment order) * W, 3xTF32.
// in[j] = {row g e0, row g e1, row g+8 e0, row g+8 e1} with e0/e1 = entries 8j+2t, 8j+2t+1.
// k-steps outer, n-tiles inner: one A fragment live at a time and NT independent chains.
// EXACT_W: W is exactly representable in tf32 (bf16 activations: B and Q are bf16 values), so
// its residual is zero and the in_hi * W_lo terms, exact zeros, are not issued.
template <int D, bool EXACT_W = false>
__device__ __forceinline__ void frag_product(const float (&in)[D / 8][4], float (&out)[D / 8][4],
                                             const float4* W, int lane) {
  constexpr int NT = D / 8;
#pragma unroll
  for (int nj = 0; nj < NT; ++nj)
#pragma unroll
    for (int r = 0; r < 4; ++r) out[nj][r] = 0.f;
#pragma unroll
  for (int kk = 0; kk < NT; ++kk) {
    uint32_t ah[4], al[4];
    wmma::split(in[kk][0], ah[0], al[0]);  // a0: row g,   slot t     <- entry 8kk+2t
    wmma::split(in[kk][2], ah[1], al[1]);  // a1: row g+8, slot t
    wmma::split(in[kk][1], ah[2], al[2]);  // a2: row g,   slot t + 4 <- entry 8kk+2t+1
    wmma::split(in[kk][3], ah[3], al[3]);  // a3: row g+8, slot t + 4
    if constexpr (D >= 32) {
      // the three terms of each n-tile issued in passes over the n-tiles, so consecutive MMAs
      // go to independent accumulators (2.4 % faster backward at d = 32; at d = 16, with two
      // n-tiles, the extra live registers cost more than the interleave gains)
      float4 w[NT];
#pragma unroll
      for (int nj = 0; nj < NT; ++nj) w[nj] = W[(kk * NT + nj) * 32 + lane];
#pragma unroll
      for (int nj = 0; nj < NT; ++nj) wmma::m16n8k8(out[nj], al, __float_as_uint(w[nj].x), __float_as_uint(w[nj].y));
      if constexpr (!EXACT_W) {
#pragma unroll
        for (int nj = 0; nj < NT; ++nj) wmma::m16n8k8(out[nj], ah, __float_as_uint(w[nj].z), __float_as_uint(w[nj].w));
      }
#pragma unroll
      for (int nj = 0; nj < NT; ++nj) wmma::m16n8k8(out[nj], ah, __float_as_uint(w[nj].x), __float_as_uint(w[nj].y));
    } else {
#pragma unroll
      for (int nj = 0; nj < NT; ++nj) {
        const float4 w = W[(kk * NT + nj) * 32 + lane];
        wmma::m16n8k8(out[nj], al, __float_as_uint(w.x), __float_as_uint(w.y));
        if constexpr (!EXACT_W) wmma::m16n8k8(out[nj], ah, __float_as_uint(w.z), __float_as_uint(w.w));
        wmma::m16n8k8(out[nj], ah, __float_as_uint(w.x), __float_as_uint(w.y));
      }
    }
  }
}

// Rows g and g + 8 of a 16 x D fragment-order matrix into the staging matrix S (stride SS).
template <int D>
__device__ __forceinline__ void stage_rows(float* S, const float (&v)[D / 8][4], int g, int t) {
  constexpr int SS = AdjMma<D>::SS;
#pragma unroll
  for (int j = 0; j < D / 8; ++j) {
    *reinterpret_cast<float2*>(S + g * SS + 8 * j + 2 * t) = make_float2(v[j][0], v[j][1]);
    *reinterpret_cast<float2*>(S + (g + 8) * SS + 8 * j + 2 * t) = make_float2(v[j][2], v[j][3]);
  }
}

// acc[n-tile][.] += sum_r SX[r][16 mi + m] * SY[(r + 8) % 16][n]  over the 16 staged rows
// (K) for one m-tile of the output, 3xTF32.  KK = 1 takes the first 8 rows only (the primal
// rows against the tangent rows): for a symmetric pair X = Y = [v; dv] that is
// S = sum v dv^T, whose S + S^T is the full sum at half the MMAs.
// ONE: single-pass tf32 with both operands rounded to nearest (relative error ~2^-11 per
// product, unbiased), for bf16 activations, where these sums only reach outputs rounded to
// bf16 (2^-9): grad_B, grad_Q and, in the layer's low-rank solve, the coefficient and basis
// gradients formed from them.  The recursion's own products stay 3xTF32.
template <int D, int KK = 2, bool ONE = false>
__device__ __forceinline__ void accumulate_unit(float (&acc)[D / 8][4], const float* SX, const float* SY,
                                                int mi, int g, int t) {
  constexpr int SS = AdjMma<D>::SS, NT = D / 8;
  if constexpr (ONE) {
#pragma unroll
    for (int kk = 0; kk < KK; ++kk) {
      const float* x0 = SX + (8 * kk + t) * SS + 16 * mi;
      const float* x1 = SX + (8 * kk + t + 4) * SS + 16 * mi;
      const uint32_t a[4] = {wmma::rna(x0[g]), wmma::rna(x0[g + 8]), wmma::rna(x1[g]), wmma::rna(x1[g + 8])};
      const float* y0 = SY + ((8 * kk + t + 8) & 15) * SS;
      const float* y1 = SY + ((8 * kk + t + 12) & 15) * SS;
#pragma unroll
      for (int nj = 0; nj < NT; ++nj) wmma::m16n8k8(acc[nj], a, wmma::rna(y0[8 * nj + g]), wmma::rna(y1[8 * nj + g]));
    }
    return;
  }
#pragma unroll
  for (int kk = 0; kk < KK; ++kk) {
    const float* x0 = SX + (8 * kk + t) * SS + 16 * mi;
    const float* x1 = SX + (8 * kk + t + 4) * SS + 16 * mi;
    uint32_t ah[4], al[4];
    wmma::split(x0[g], ah[0], al[0]);
    wmma::split(x0[g + 8], ah[1], al[1]);
    wmma::split(x1[g], ah[2], al[2]);
    wmma::split(x1[g + 8], ah[3], al[3]);
    const float* y0 = SY + ((8 * kk + t + 8) & 15) * SS;
    const float* y1 = SY + ((8 * kk + t + 12) & 15) * SS;
    if constexpr (D >= 32) {
      uint32_t bh0[NT], bl0[NT], bh1[NT], bl1[NT];
#pragma unroll
      for (int nj = 0; nj < NT; ++nj) {
        wmma::split(y0[8 * nj + g], bh0[nj], bl0[nj]);
        wmma::split(y1[8 * nj + g], bh1[nj], bl1[nj]);
      }
      // passes over the n-tiles: consecutive MMAs go to independent accumulators
#pragma unroll
      for (int nj = 0; nj < NT; ++nj) wmma::m16n8k8(acc[nj], al, bh0[nj], bh1[nj]);
#pragma unroll
      for (int nj = 0; nj < NT; ++nj) wmma::m16n8k8(acc[nj], ah, bl0[nj], bl1[nj]);
#pragma unroll
      for (int nj = 0; nj < NT; ++nj) wmma::m16n8k8(acc[nj], ah, bh0[nj], bh1[nj]);
    } else {
#pragma unroll
      for (int nj = 0; nj < NT; ++nj) {
        uint32_t bh0, bl0, bh1, bl1;
        wmma::split(y0[8 * nj + g], bh0, bl0);
        wmma::split(y1[8 * nj + g], bh1, bl1);
        wmma::m16n8k8(acc[nj], al, bh0, bh1);
        wmma::m16n8k8(acc[nj], ah, bl0, bl1);
        wmma::m16n8k8(acc[nj], ah, bh0, bh1);
      }
    }
  }
}

// The layer's Q_f mixture on the backward side (Q_f = sum_r coeff_Qf[r] basis[r],
// ttc_layer.py:119-123) for all heads of a CTA's row group, from every warp's final state
// (h, dh) staged at `stage_off` of its staging area (rows 0-7 h, rows 8-15 dh of its 8 heads,
// output-fragment positions) and its heads' coeff_Qf at `coeff_off` ([8][rQ], zero for
// padding heads).  The Q_f gradient of a head is the rank-2
// gQf = (h dh^T + dh h^T) / 2 (symplectic_iter.py:855-857), so
//   grad_coeff_Qf[r] = <gQf, basis[r]> = ((h basis[r]) . dh + (dh basis[r]) . h) / 2,
//   slice[r] += sum_heads coeff_Qf[r] h dh^T   (the caller forms (S + S^T) / 2 from the sum
//   of all CTAs' slices).
// Basis index r belongs to warp r mod W, which loads basis[r] in fragment order once, runs
// over the staged warps in order and read-modify-writes slice[r] once: deterministic.
template <int D, typename TIn>
__device__ __forceinline__ bool qmix_cta(const float* warp_s, int stage_off, int coeff_off, int nwarps, int wpr,
                                         int64_t n0,
                                         int64_t N, int nh, const TIn* __restrict__ basis, int rQ,
                                         const TIn* __restrict__ coeff, TIn* __restrict__ gcoeff,
                                         float* __restrict__ slice, int warp, int g, int t) {
  constexpr int SS = AdjMma<D>::SS, NT = D / 8, MT = D / 16, kWarp = AdjMma<D>::kWarp;
  // bf16 activations: single-pass tf32 with round-to-nearest operands (relative error ~2^-11
  // per product, unbiased, below the bf16 rounding of the einsum backward it replaces);
  // float: 3xTF32
  constexpr bool kOne = sizeof(TIn) == 2;
  bool bad = false;
  for (int r = warp; r < rQ; r += nwarps) {
    // basis[r] as the constant operand: W[k][n] = basis[r][k][n], K rows permuted as the
    // other products (slot t <-> entry 8kk + 2t, slot t + 4 <-> 8kk + 2t + 1).
    uint32_t wh[NT][NT][2], wl[NT][NT][2];
    const TIn* Wr = basis + (int64_t)r * D * D;
#pragma unroll
    for (int kk = 0; kk < NT; ++kk)
#pragma unroll
      for (int nj = 0; nj < NT; ++nj) {
        const float w0 = ldf(Wr + (8 * kk + 2 * t) * D + 8 * nj + g);
        const float w1 = ldf(Wr + (8 * kk + 2 * t + 1) * D + 8 * nj + g);
        if constexpr (kOne) {
          wh[kk][nj][0] = wmma::rna(w0);
          wh[kk][nj][1] = wmma::rna(w1);
        } else {
          wmma::split(w0, wh[kk][nj][0], wl[kk][nj][0]);
          wmma::split(w1, wh[kk][nj][1], wl[kk][nj][1]);
        }
      }
    float acc[MT][NT][4];
#pragma unroll
    for (int mi = 0; mi < MT; ++mi)
#pragma unroll
      for (int nj = 0; nj < NT; ++nj)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[mi][nj][e] = 0.f;
    for (int sw = 0; sw < nwarps; ++sw) {
      const float* S = warp_s + (size_t)sw * kWarp + stage_off;
      const int64_t ns = n0 + sw / wpr;
      const int hb = sw % wpr;
      const bool rowv = ns < N;
      // A row past N (the last row group of a partial batch) ran the recursion on zero vectors
      // against operands that were never built: shared memory that may hold any bit pattern,
      // NaN included.  Its staged vectors can then be NaN and its zero coefficients would not
      // cancel them (0 * NaN), so it contributes nothing here.  Uniform over the warp.
      if (!rowv) continue;
      const int64_t prow = ns * nh;
      // grad_coeff_Qf of the staged warp's heads: [h; dh] basis[r]
      float Hs[NT][4], P[NT][4];
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const float2 a = *reinterpret_cast<const float2*>(S + g * SS + 8 * j + 2 * t);
        const float2 b = *reinterpret_cast<const float2*>(S + (g + 8) * SS + 8 * j + 2 * t);
        Hs[j][0] = a.x;
        Hs[j][1] = a.y;
        Hs[j][2] = b.x;
        Hs[j][3] = b.y;
#pragma unroll
        for (int e = 0; e < 4; ++e) P[j][e] = 0.f;
      }
#pragma unroll
      for (int kk = 0; kk < NT; ++kk) {
        uint32_t ah[4], al[4];
        if constexpr (kOne) {
          ah[0] = wmma::rna(Hs[kk][0]);
          ah[1] = wmma::rna(Hs[kk][2]);
          ah[2] = wmma::rna(Hs[kk][1]);
          ah[3] = wmma::rna(Hs[kk][3]);
#pragma unroll
          for (int nj = 0; nj < NT; ++nj) wmma::m16n8k8(P[nj], ah, wh[kk][nj][0], wh[kk][nj][1]);
        } else {
          wmma::split(Hs[kk][0], ah[0], al[0]);
          wmma::split(Hs[kk][2], ah[1], al[1]);
          wmma::split(Hs[kk][1], ah[2], al[2]);
          wmma::split(Hs[kk][3], ah[3], al[3]);
#pragma unroll
          for (int nj = 0; nj < NT; ++nj) {
            wmma::m16n8k8(P[nj], al, wh[kk][nj][0], wh[kk][nj][1]);
            wmma::m16n8k8(P[nj], ah, wl[kk][nj][0], wl[kk][nj][1]);
            wmma::m16n8k8(P[nj], ah, wh[kk][nj][0], wh[kk][nj][1]);
          }
        }
      }
      float sdot = 0.f;
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) sdot = fmaf(P[j][e], Hs[j][2 + e], fmaf(P[j][2 + e], Hs[j][e], sdot));
      sdot += __shfl_xor_sync(0xffffffffu, sdot, 1);
      sdot += __shfl_xor_sync(0xffffffffu, sdot, 2);
      sdot *= 0.5f;
      const int hg = hb * 8 + g;
      if (rowv && hg < nh && t == 0) {
        bad |= unstable(sdot);
        stf(gcoeff + (prow + hg) * rQ + r, sdot);
      }
      // slice[r] += sum over the staged heads of coeff[r] h dh^T (MMA with K = the 8 heads):
      // A[i][k] = h_k[i], B[k][j] = coeff_k[r] dh_k[j].
      // coeff[r] of the heads in k-slots t and t + 4, staged by warp sw as [8][rQ]
      const float* Cs = warp_s + (size_t)sw * kWarp + coeff_off;
      const float c0 = Cs[t * rQ + r], c1 = Cs[(t + 4) * rQ + r];
      uint32_t xh[MT][4], xl[MT][4];
#pragma unroll
      for (int mi = 0; mi < MT; ++mi) {
        const float x0 = S[t * SS + 16 * mi + g], x1 = S[t * SS + 16 * mi + g + 8];
        const float x2 = S[(t + 4) * SS + 16 * mi + g], x3 = S[(t + 4) * SS + 16 * mi + g + 8];
        if constexpr (kOne) {
          xh[mi][0] = wmma::rna(x0);
          xh[mi][1] = wmma::rna(x1);
          xh[mi][2] = wmma::rna(x2);
          xh[mi][3] = wmma::rna(x3);
        } else {
          wmma::split(x0, xh[mi][0], xl[mi][0]);
          wmma::split(x1, xh[mi][1], xl[mi][1]);
          wmma::split(x2, xh[mi][2], xl[mi][2]);
          wmma::split(x3, xh[mi][3], xl[mi][3]);
        }
      }
#pragma unroll
      for (int nj = 0; nj < NT; ++nj) {
        const float y0 = c0 * S[(8 + t) * SS + 8 * nj + g], y1 = c1 * S[(12 + t) * SS + 8 * nj + g];
        if constexpr (kOne) {
          const uint32_t b0 = wmma::rna(y0), b1 = wmma::rna(y1);
#pragma unroll
          for (int mi = 0; mi < MT; ++mi) wmma::m16n8k8(acc[mi][nj], xh[mi], b0, b1);
        } else {
          uint32_t bh0, bl0, bh1, bl1;
          wmma::split(y0, bh0, bl0);
          wmma::split(y1, bh1, bl1);
#pragma unroll
          for (int mi = 0; mi < MT; ++mi) {
            wmma::m16n8k8(acc[mi][nj], xl[mi], bh0, bh1);
            wmma::m16n8k8(acc[mi][nj], xh[mi], bl0, bl1);
            wmma::m16n8k8(acc[mi][nj], xh[mi], bh0, bh1);
          }
        }
      }
    }
    float* sr = slice + (int64_t)r * D * D;
#pragma unroll
    for (int mi = 0; mi < MT; ++mi)
#pragma unroll
      for (int nj = 0; nj < NT; ++nj) {
        float2* q0 = reinterpret_cast<float2*>(sr + (16 * mi + g) * D + 8 * nj + 2 * t);
        float2* q1 = reinterpret_cast<float2*>(sr + (16 * mi + g + 8) * D + 8 * nj + 2 * t);
        float2 v0 = *q0, v1 = *q1;
        v0.x += acc[mi][nj][0];
        v0.y += acc[mi][nj][1];
        v1.x += acc[mi][nj][2];
        v1.y += acc[mi][nj][3];
        *q0 = v0;
        *q1 = v1;
      }
  }
  return bad;
}

// Backward from the forward's lambda0 and either M (d_p = M d_u per head, fused_lqr.py:
// 185-187) or d_p itself.  Grid: ceil(N / R) CTAs of R rows x W = ceil(nh / 8) warps; the W
// warps of a row meet at one named barrier per step (id 1 + row), after which warp w
// accumulates grad_B / grad_Q units w, w + W, ... (UPW at most) over all W warps' staged
// vectors of that step, in warp order.
template <int D, typename TIn, bool FROM_M, int UPW>
__global__ void __launch_bounds__(256, D <= 16 ? 2 : 1)
lqr_bwd_mma_kernel(const TIn* __restrict__ A_diag, const TIn* __restrict__ Bm,
                   const TIn* __restrict__ Qm, const TIn* __restrict__ Rinv,
                   const TIn* __restrict__ lgA, const TIn* __restrict__ lgB,
                   const TIn* __restrict__ lgQ, const TIn* __restrict__ H0,
                   const float* __restrict__ lam0_in, const float* __restrict__ M_or_dp,
                   const TIn* __restrict__ dU, int64_t N, int nh, int T, int rows_per_cta,
                   TIn* __restrict__ gA_out, TIn* __restrict__ gB_out, TIn* __restrict__ gQ_out,
                   TIn* __restrict__ gR_out, TIn* __restrict__ gQf_out, TIn* __restrict__ glgA_out,
                   TIn* __restrict__ glgB_out, TIn* __restrict__ glgQ_out, TIn* __restrict__ gh0_out,
                   const TIn* __restrict__ Qbasis, int rQ, const TIn* __restrict__ cQf,
                   TIn* __restrict__ gcQf_out, float* __restrict__ gQb_partial,
                   int* __restrict__ status, LowRank<TIn> lr) {
  using C = AdjMma<D>;
  constexpr int NT = C::NT, MT = C::MT;
  // grad_B / grad_Q contractions in single-pass rounded tf32 for bf16 activations
  constexpr bool kOneContract = sizeof(TIn) == 2 && TTC_BF16_ONEPASS;
  // bf16 activations: B and Q (inputs, or mixtures rounded to bf16) are tf32-exact
  constexpr bool kExactW = sizeof(TIn) == 2;
  extern __shared__ __align__(128) float smem[];
  const int tid = threadIdx.x, nthreads = blockDim.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int wpr = (nh + 7) / 8;
  const int rloc = warp / wpr, hb = warp % wpr;
  float* rows_s = smem;
  float* warp_s = smem + (size_t)rows_per_cta * C::kRow;
  float* row_stage = warp_s + (size_t)(rloc * wpr) * C::kWarp;  // warp 0 of this row
  float* stg = warp_s + (size_t)warp * C::kWarp;
  // Q_f given as a mixture (Qbasis != NULL): this CTA's own [rQ][D][D] partial of the basis
  // gradient, accumulated over every row group the CTA walks.
  float* slice = nullptr;
  if (Qbasis != nullptr) {
    slice = gQb_partial + (int64_t)blockIdx.x * rQ * D * D;
    for (int e = tid; e < rQ * D * D; e += nthreads) slice[e] = 0.f;
  }
  // Low-rank B / Q (which needs the mixed Q_f above): the CTA's partial of the B-basis
  // gradient, and each row's B and Q formed from its coefficients.
  const bool lowrank = lr.cB != nullptr && Qbasis != nullptr;
  float* bslice = nullptr;
  if (lowrank) {
    bslice = lr.gBb + (int64_t)blockIdx.x * lr.rB * D * D;
    for (int e = tid; e < lr.rB * D * D; e += nthreads) bslice[e] = 0.f;
  }
  bool bad = false;
  const int64_t ngroups = (N + rows_per_cta - 1) / rows_per_cta;
  for (int64_t grp = blockIdx.x; grp < ngroups; grp += gridDim.x) {
    const int64_t n0 = grp * rows_per_cta;
    const int64_t n = n0 + rloc;
    const bool row_ok = n < N;

    // The CTA's rows: constant operands Q^T, B, B^T, Q in fragment order, symmetry flag.
    if (tid < rows_per_cta) reinterpret_cast<int*>(rows_s + tid * C::kRow + 4 * C::kFrag)[0] = 1;
    __syncthreads();
    if (lowrank) {
      // B and Q of every row of the group, mixed into the (still unused) staging area first:
      // row r's [B | Q] at warp_s + 2 r d^2 (a row's own warps' staging holds more than 2 d^2)
      static_assert(2 * D * D <= C::kWarp, "mixing area");
      const int nrows = static_cast<int>(N - n0 < rows_per_cta ? N - n0 : rows_per_cta);
      for (int idx = tid; idx < nrows * (D * D / 4); idx += nthreads) {
        const int r = idx / (D * D / 4), e4 = idx % (D * D / 4);
        float4 vb, vq;
        mix4_pair<TIn>(lr.cB + (n0 + r) * lr.rB, lr.Bb, lr.rB, lr.cQ + (n0 + r) * rQ, Qbasis, rQ, D * D, 4 * e4, vb,
                       vq);
        *reinterpret_cast<float4*>(warp_s + 2 * r * D * D + 4 * e4) = vb;
        *reinterpret_cast<float4*>(warp_s + (2 * r + 1) * D * D + 4 * e4) = vq;
      }
      __syncthreads();
    }
    for (int r = 0; r < rows_per_cta; ++r) {
      const int64_t nr = n0 + r;
      if (nr >= N) break;
      float* base = rows_s + r * C::kRow;
      if (lowrank) {
        const float* tB = warp_s + 2 * r * D * D;
        const float* tQ = tB + D * D;
        build_operand<D>(base, [&](int k, int c) { return tQ[c * D + k]; }, tid, nthreads);
        build_operand<D>(base + C::kFrag, [&](int k, int c) { return tB[k * D + c]; }, tid, nthreads);
        build_operand<D>(base + 2 * C::kFrag, [&](int k, int c) { return tB[c * D + k]; }, tid, nthreads);
        build_operand<D>(base + 3 * C::kFrag, [&](int k, int c) { return tQ[k * D + c]; }, tid, nthreads);
        bool asym = false;
        for (int e = tid; e < D * D; e += nthreads) asym |= tQ[e] != tQ[(e % D) * D + e / D];
        if (asym) reinterpret_cast<int*>(base + 4 * C::kFrag)[0] = 0;
        continue;
      }
      const TIn* Bn = Bm + nr * (D * D);
      const TIn* Qn = Qm + nr * (D * D);
      build_operand<D>(base, [&](int k, int c) { return ldf(Qn + c * D + k); }, tid, nthreads);
      build_operand<D>(base + C::kFrag, [&](int k, int c) { return ldf(Bn + k * D + c); }, tid, nthreads);
      build_operand<D>(base + 2 * C::kFrag, [&](int k, int c) { return ldf(Bn + c * D + k); }, tid, nthreads);
      build_operand<D>(base + 3 * C::kFrag, [&](int k, int c) { return ldf(Qn + k * D + c); }, tid, nthreads);
      bool asym = false;
      for (int e = tid; e < D * D; e += nthreads) asym |= ldf(Qn + e) != ldf(Qn + (e % D) * D + e / D);
      if (asym) reinterpret_cast<int*>(base + 4 * C::kFrag)[0] = 0;
    }
    __syncthreads();

    const float* rbase = rows_s + rloc * C::kRow;
    const float4* Wqt = reinterpret_cast<const float4*>(rbase);
    const float4* Wb = reinterpret_cast<const float4*>(rbase + C::kFrag);
    const float4* Wbt = reinterpret_cast<const float4*>(rbase + 2 * C::kFrag);
    const float4* Wq = reinterpret_cast<const float4*>(rbase + 3 * C::kFrag);
    const bool sym = reinterpret_cast<const int*>(rbase + 4 * C::kFrag)[0] != 0;

    const int h = hb * 8 + g;
    const bool valid = row_ok && h < nh;
    const int64_t p = valid ? n * nh + h : 0;
    // slot (j, s) of a thread is entry 8j + 2t + s; index 2 + s of a pair array is the tangent
    float a[NT][2], lgQ2[NT][2], lgB2[NT][2], rinv[NT][2];
    float L[NT][4], H[NT][4];
    const float lgA2 = valid ? ldf(lgA + p) * kLog2e : 0.f;
    // d_p = M d_u (fused_lqr.py:185-187): the head's d_u once, the rows of M as 16-byte loads,
    // each row's sum in column order
    float du_row[FROM_M ? D : 1];
    if constexpr (FROM_M) {
#pragma unroll
      for (int c4 = 0; c4 < D / 4; ++c4) {
        const float4 v = valid ? ld4(dU + p * D + 4 * c4) : make_float4(0.f, 0.f, 0.f, 0.f);
        du_row[4 * c4] = v.x;
        du_row[4 * c4 + 1] = v.y;
        du_row[4 * c4 + 2] = v.z;
        du_row[4 * c4 + 3] = v.w;
      }
    }
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const int e = 8 * j + 2 * t + s;
        a[j][s] = valid ? ldf(A_diag + p * D + e) : 0.f;
        lgQ2[j][s] = valid ? ldf(lgQ + p * D + e) * kLog2e : 0.f;
        lgB2[j][s] = valid ? ldf(lgB + p * D + e) * kLog2e : 0.f;
        rinv[j][s] = valid ? ldf(Rinv + p * D + e) : 1.f;
        H[j][s] = valid ? ldf(H0 + p * D + e) : 0.f;
        H[j][2 + s] = 0.f;
        L[j][s] = valid ? lam0_in[p * D + e] : 0.f;
        float dl = 0.f;
        if (valid) {
          if constexpr (FROM_M) {
            const float4* m4 = reinterpret_cast<const float4*>(M_or_dp + (p * D + e) * D);
#pragma unroll
            for (int c4 = 0; c4 < D / 4; ++c4) {
              const float4 mv = m4[c4];
              dl = fmaf(mv.x, du_row[4 * c4], dl);
              dl = fmaf(mv.y, du_row[4 * c4 + 1], dl);
              dl = fmaf(mv.z, du_row[4 * c4 + 2], dl);
              dl = fmaf(mv.w, du_row[4 * c4 + 3], dl);
            }
          } else {
            dl = M_or_dp[p * D + e];
          }
        }
        L[j][2 + s] = dl;
      }
    }

    float gA[NT][2], glgQ[NT][2], gR[NT][2], glgB[NT][2], dqp[NT][2];
    float glgA = 0.f;
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        gA[j][s] = glgQ[j][s] = gR[j][s] = glgB[j][s] = 0.f;
        dqp[j][s] = 1.0f;
      }
    float acc[UPW][NT][4];
#pragma unroll
    for (int q = 0; q < UPW; ++q)
#pragma unroll
      for (int nj = 0; nj < NT; ++nj)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[q][nj][r] = 0.f;

    // grad_B += lambda (du e^lgB)^T + dlambda (u e^lgB)^T ;
    // grad_Q += (h Dq)(dh Dq)^T + (dh Dq)(h Dq)^T  (the 1/2 is applied at the end; at
    // d = 16 only the first term is accumulated and the transpose added at the end)
    // for step ks, from the vectors every warp of the row staged for it.
    auto accumulate_step = [&](int ks) {
#pragma unroll
      for (int q = 0; q < UPW; ++q) {
        const int unit = C::kOwn ? q : hb + q * wpr;
        if (unit < C::kUnits) {
          const bool isq = unit >= MT;
          if (!isq || ks < T - 1) {
            const int mi = isq ? unit - MT : unit;
            const int off = (ks & 1) * 3 * C::kStage + (isq ? 2 * C::kStage : 0);
            const int offy = (ks & 1) * 3 * C::kStage + (isq ? 2 * C::kStage : C::kStage);
            if constexpr (C::kOwn) {
              // grad_Q as S = sum (h Dq)(dh Dq)^T, symmetrised at the end
              if (isq) {
                accumulate_unit<D, 1, kOneContract>(acc[q], stg + off, stg + offy, mi, g, t);
              } else {
                accumulate_unit<D, 2, kOneContract>(acc[q], stg + off, stg + offy, mi, g, t);
              }
            } else {
              for (int w = 0; w < wpr; ++w) {
                const float* base = row_stage + (size_t)w * C::kWarp;
                accumulate_unit<D, 2, kOneContract>(acc[q], base + off, base + offy, mi, g, t);
              }
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
        // and the log_gamma_Q gradient of step k-1 (:871-877).
        float HD[NT][4], QH[NT][4], QTH[NT][4];
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
          for (int r = 0; r < 4; ++r) HD[j][r] = H[j][r] * dqp[j][r & 1];
        frag_product<D, kExactW>(HD, QH, Wqt, lane);
        if (!sym) frag_product<D, kExactW>(HD, QTH, Wq, lane);
#pragma unroll
        for (int j = 0; j < NT; ++j) {
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            const float qh = QH[j][s], qdh = QH[j][2 + s];
            const float qth = sym ? qh : QTH[j][s], qtdh = sym ? qdh : QTH[j][2 + s];
            L[j][s] = fmaf(-dqp[j][s], qh, L[j][s]);
            L[j][2 + s] = fmaf(-dqp[j][s], qdh, L[j][2 + s]);
            glgQ[j][s] = fmaf(0.5f * fmaf(H[j][2 + s], qh + qth, H[j][s] * (qdh + qtdh)),
                              static_cast<float>(k) * dqp[j][s], glgQ[j][s]);
          }
        }
      } else if (valid) {
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            bad |= unstable(L[j][2 + s]);
            stf(gh0_out + p * D + 8 * j + 2 * t + s, L[j][2 + s]);  // dh_0 = dlambda_0
          }
      }
      const float eA = exp_scaled(lgA2, ke);
      float At[NT][2];
#pragma unroll
      for (int j = 0; j < NT; ++j) {
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          At[j][s] = fmaf(a[j][s], eA, 1.0f);
          const float rAt = recip(At[j][s]);
          L[j][s] *= rAt;
          L[j][2 + s] *= rAt;
          const float dA = fmaf(L[j][s], H[j][2 + s], L[j][2 + s] * H[j][s]);
          gA[j][s] = fmaf(dA, eA, gA[j][s]);
          glgA = fmaf(dA * a[j][s], ke * eA, glgA);
        }
      }
      stage_rows<D>(S0, L, g, t);
      // u = -R_inv (B e^lgB)^T lambda and its tangent (symplectic_iter.py:800-830)
      float UE[NT][4];
      {
        float BL[NT][4];
        frag_product<D, kExactW>(L, BL, Wb, lane);
#pragma unroll
        for (int j = 0; j < NT; ++j) {
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            const float eB = exp_scaled(lgB2[j][s], ke);
            const float bl = BL[j][s], bdl = BL[j][2 + s];
            const float u = -(bl * eB) * rinv[j][s];
            float du = -(bdl * eB) * rinv[j][s];
            if (k == 0 && valid) du = fmaf(ldf(dU + p * D + 8 * j + 2 * t + s), -rinv[j][s], du);
            glgB[j][s] = fmaf(fmaf(du, bl, u * bdl), ke * eB, glgB[j][s]);
            gR[j][s] = fmaf(-(u * du), recip(rinv[j][s] * rinv[j][s]), gR[j][s]);
            UE[j][s] = u * eB;
            UE[j][2 + s] = du * eB;
          }
        }
      }
      stage_rows<D>(S1, UE, g, t);
      // h <- A h + B e^lgB u (symplectic_iter.py:832-850)
      {
        float BU[NT][4];
        frag_product<D, kExactW>(UE, BU, Wbt, lane);
#pragma unroll
        for (int j = 0; j < NT; ++j) {
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            H[j][s] = fmaf(H[j][s], At[j][s], BU[j][s]);
            H[j][2 + s] = fmaf(H[j][2 + s], At[j][s], BU[j][2 + s]);
            dqp[j][s] = exp_scaled(lgQ2[j][s], ke);
          }
        }
      }
      if (k < T - 1) {
        float HD[NT][4];
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
          for (int r = 0; r < 4; ++r) HD[j][r] = H[j][r] * dqp[j][r & 1];
        stage_rows<D>(S2, HD, g, t);
      }
      // Every warp of the row has staged step k (and finished reading step k - 1's buffer).
      if (!C::kOwn && wpr > 1) {
        asm volatile("bar.sync %0, %1;" ::"r"(1 + rloc), "r"(32 * wpr) : "memory");
      } else {
        __syncwarp();
      }
      accumulate_step(k);
    }

    // grad_Qf = (h dh^T + dh h^T) / 2 at the final state (symplectic_iter.py:855-857), from
    // the staging buffer of step T (unused by the row's other warps); for a mixed Q_f its
    // contractions with the basis instead.
    if (Qbasis != nullptr) {
      // final state into this step's staging buffer (the row's other warps last read it at
      // step T - 2); after a CTA barrier, the heads' coeff_Qf into the other buffer
      __syncwarp();
      stage_rows<D>(stg + (T & 1) * 3 * C::kStage, H, g, t);
      __syncthreads();
      {
        float* Cs = stg + ((T + 1) & 1) * 3 * C::kStage;
        for (int e = lane; e < 8 * rQ; e += 32) {
          const int hk = hb * 8 + e / rQ;
          Cs[e] = (row_ok && hk < nh) ? ldf(cQf + (n * nh + hk) * rQ + e % rQ) : 0.f;
        }
      }
      __syncthreads();
      bad |= qmix_cta<D, TIn>(warp_s, (T & 1) * 3 * C::kStage, ((T + 1) & 1) * 3 * C::kStage, blockDim.x >> 5,
                              wpr, n0, N, nh, Qbasis, rQ, cQf, gcQf_out, slice, warp, g, t);
    } else {
      float* S = stg + (T & 1) * 3 * C::kStage;
      stage_rows<D>(S, H, g, t);
      __syncwarp();
      for (int e = lane; e < 8 * D * D; e += 32) {
        const int hh = e / (D * D), i = (e / D) % D, jj = e % D;
        const int h2 = hb * 8 + hh;
        if (row_ok && h2 < nh) {
          const float v = 0.5f * fmaf(S[hh * C::SS + i], S[(hh + 8) * C::SS + jj],
                                      S[(hh + 8) * C::SS + i] * S[hh * C::SS + jj]);
          bad |= unstable(v);
          stf(gQf_out + ((n * nh + h2) * D + i) * D + jj, v);
        }
      }
    }
    // Per-head outputs.
    float glgA_sum = glgA;
    glgA_sum += __shfl_xor_sync(0xffffffffu, glgA_sum, 1);
    glgA_sum += __shfl_xor_sync(0xffffffffu, glgA_sum, 2);
    if (valid) {
#pragma unroll
      for (int j = 0; j < NT; ++j) {
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          const int e = 8 * j + 2 * t + s;
          bad |= unstable(gA[j][s]) | unstable(glgQ[j][s]) | unstable(gR[j][s]) | unstable(glgB[j][s]);
          stf(gA_out + p * D + e, gA[j][s]);
          stf(glgQ_out + p * D + e, glgQ[j][s]);
          stf(gR_out + p * D + e, gR[j][s]);
          stf(glgB_out + p * D + e, glgB[j][s]);
        }
      }
      if (t == 0) {
        bad |= unstable(glgA_sum);
        stf(glgA_out + p, glgA_sum);
      }
    }
    if constexpr (C::kOwn) {
      // The row's warps add their partial sums in warp order (staging area reused).
      static_assert(!C::kOwn || 2 * D * D <= C::kWarp, "reduction area");
      __syncthreads();
#pragma unroll
      for (int q = 0; q < UPW; ++q) {
        const bool isq = q >= MT;
        const int mi = isq ? q - MT : q;
        float* red = stg + (isq ? D * D : 0);
#pragma unroll
        for (int nj = 0; nj < NT; ++nj) {
          const int r0 = 16 * mi + g, c0 = 8 * nj + 2 * t;
          *reinterpret_cast<float2*>(red + r0 * D + c0) = make_float2(acc[q][nj][0], acc[q][nj][1]);
          *reinterpret_cast<float2*>(red + (r0 + 8) * D + c0) = make_float2(acc[q][nj][2], acc[q][nj][3]);
        }
      }
      __syncthreads();
      for (int r = 0; r < rows_per_cta; ++r) {
        const int64_t nr = n0 + r;
        if (nr >= N) break;
        for (int e = tid; e < 2 * D * D; e += nthreads) {
          float v = 0.f;
          if (e < D * D) {
            for (int w = 0; w < wpr; ++w) v += warp_s[(size_t)(r * wpr + w) * C::kWarp + e];
          } else {
            // grad_Q = (S + S^T) / 2 over the warps' partial S
            const int ij = e - D * D, ji = D * D + (ij % D) * D + ij / D;
            for (int w = 0; w < wpr; ++w) {
              const float* ws = warp_s + (size_t)(r * wpr + w) * C::kWarp;
              v += ws[e] + ws[ji];
            }
            v *= 0.5f;
          }
          bad |= unstable(v);
          if (lowrank) {
            rows_s[r * C::kRow + e] = v;  // the row's [grad_B | grad_Q] for the contractions
          } else {
            stf((e < D * D ? gB_out : gQ_out) + nr * (D * D) + (e % (D * D)), v);
          }
        }
      }
    } else if (row_ok) {
      // Each unit holds the sum over all the row's heads.
#pragma unroll
      for (int q = 0; q < UPW; ++q) {
        const int unit = hb + q * wpr;
        if (unit < C::kUnits) {
          const bool isq = unit >= MT;
          const int mi = isq ? unit - MT : unit;
          const float sc = isq ? 0.5f : 1.0f;
          TIn* out = (isq ? gQ_out : gB_out) + n * (D * D);
          // low-rank: into the row's [grad_B | grad_Q] buffer (the operands are no longer read:
          // every warp passed the barrier before the Q_f contractions)
          float* buf = rows_s + rloc * C::kRow + (isq ? D * D : 0);
#pragma unroll
          for (int nj = 0; nj < NT; ++nj) {
            const int r0 = 16 * mi + g, c0 = 8 * nj + 2 * t;
            const float v[4] = {sc * acc[q][nj][0], sc * acc[q][nj][1], sc * acc[q][nj][2], sc * acc[q][nj][3]};
            bad |= unstable(v[0]) | unstable(v[1]) | unstable(v[2]) | unstable(v[3]);
            if (lowrank) {
              buf[r0 * D + c0] = v[0];
              buf[r0 * D + c0 + 1] = v[1];
              buf[(r0 + 8) * D + c0] = v[2];
              buf[(r0 + 8) * D + c0 + 1] = v[3];
            } else {
              stf(out + r0 * D + c0, v[0]);
              stf(out + r0 * D + c0 + 1, v[1]);
              stf(out + (r0 + 8) * D + c0, v[2]);
              stf(out + (r0 + 8) * D + c0 + 1, v[3]);
            }
          }
        }
      }
    }
    if (lowrank) {
      // grad_coeff_B / grad_coeff_Q of the group's rows and their terms of the basis
      // gradients.  Each basis index is handled by one warp (a CTA barrier separates this
      // from the Q_f contractions, which update the same Q slices), which reads its basis
      // matrix and read-modify-writes its slice once for all the group's rows, four
      // consecutive entries per lane and access (the slices are L2-resident), rows added in
      // order: deterministic.
      __syncthreads();
      const int nw = nthreads >> 5;
      const int nrows = static_cast<int>(N - n0 < rows_per_cta ? N - n0 : rows_per_cta);
      constexpr int kQuads = D * D / 128;  // float4 quads of a d x d matrix per lane
      for (int k = warp; k < lr.rB + rQ; k += nw) {
        const bool isb = k < lr.rB;
        const int rr = isb ? k : k - lr.rB;
        const int rank = isb ? lr.rB : rQ;
        const TIn* cf = (isb ? lr.cB : lr.cQ) + n0 * rank + rr;
        const TIn* bas = (isb ? lr.Bb : Qbasis) + (int64_t)rr * D * D;
        float* sl = (isb ? bslice : slice) + (int64_t)rr * D * D;
        const int goff = isb ? 0 : D * D;
        // all of the lane's basis and slice quads in flight at once (one L2 round trip)
        float4 b[kQuads], a[kQuads];
#pragma unroll
        for (int q = 0; q < kQuads; ++q) {
          b[q] = ld4(bas + 4 * (lane + 32 * q));
          a[q] = *reinterpret_cast<const float4*>(sl + 4 * (lane + 32 * q));
        }
#pragma unroll
        for (int r = 0; r < C::kMaxWarps; ++r) {
          if (r < nrows) {
            const float c = ldf(cf + (int64_t)r * rank);
            float dot = 0.f;
#pragma unroll
            for (int q = 0; q < kQuads; ++q) {
              const float4 gv = *reinterpret_cast<const float4*>(rows_s + r * C::kRow + goff + 4 * (lane + 32 * q));
              dot = fmaf(gv.x, b[q].x, fmaf(gv.y, b[q].y, fmaf(gv.z, b[q].z, fmaf(gv.w, b[q].w, dot))));
              a[q].x = fmaf(c, gv.x, a[q].x);
              a[q].y = fmaf(c, gv.y, a[q].y);
              a[q].z = fmaf(c, gv.z, a[q].z);
              a[q].w = fmaf(c, gv.w, a[q].w);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            if (lane == 0) {
              bad |= unstable(dot);
              stf((isb ? lr.gcB : lr.gcQ) + (n0 + r) * rank + rr, dot);
            }
          }
        }
#pragma unroll
        for (int q = 0; q < kQuads; ++q) *reinterpret_cast<float4*>(sl + 4 * (lane + 32 * q)) = a[q];
      }
    }
    __syncthreads();  // the next row group reuses the shared operands and staging
  }
  if (bad) atomicOr(status, TTC_STATUS_BWD_UNSTABLE);
}

}  // namespace ttc
