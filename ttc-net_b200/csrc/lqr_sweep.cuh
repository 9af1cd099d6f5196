// Symplectic Riccati sweep and in-CTA Gauss-Jordan solve, FP32 on the CUDA cores.
//
// One group of D threads owns one LQR problem (row n, head h); thread i keeps row i
// of Y1 and Y2 (and at the end of Y3) in registers.  B [D,DU] and Q [D,D] are shared
// by every head of a row (ttc/layers/ttc_layer.py:117-120) and sit in shared memory;
// each thread streams them with 128-bit broadcast loads, so one load feeds 4 FMAs.
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

// Streams the R rows (C4 float4 each) of a shared-memory matrix to f(r, row) with a
// one-row prefetch.  __syncwarp(mask) is a scheduling fence for ptxas: without it the
// fully unrolled loads of a whole step are issued up front and spill ~D*(DU+2D) registers.
template <int R, int C4, typename F>
__device__ __forceinline__ void stream_rows(const float4* M, unsigned mask, F&& f) {
  float4 cur[C4], nxt[C4];
#pragma unroll
  for (int c = 0; c < C4; ++c) cur[c] = M[c];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (r + 1 < R) {
#pragma unroll
      for (int c = 0; c < C4; ++c) nxt[c] = M[(r + 1) * C4 + c];
    }
    __syncwarp(mask);
    f(r, cur);
    if (r + 1 < R) {
#pragma unroll
      for (int c = 0; c < C4; ++c) cur[c] = nxt[c];
    }
  }
}

// One step of the sweep (symplectic_iter.py:226-264) for the thread's state row.
//   t    = Y2 B                         ( x diag(exp(lgB tau)) R_inv folded into S2/EBR)
//   Y1   = (Y1 + (t * S2) B^T) / A_tau
//   Y2   = Y2 * A_tau + ((Y1 * Dq) Q) * Dq        (not on the last step)
//   Y3   = -t * EBR                                (last step only)
template <int D, int DU, bool LAST>
__device__ __forceinline__ void sweep_step(float (&y1)[D], float (&y2)[D], float (&y3)[DU],
                                           const float* sB, const float* sQ, const float* v,
                                           unsigned mask) {
  using V = SweepVec<D, DU>;
  const float4* B4 = reinterpret_cast<const float4*>(sB);
  const float4* Q4 = reinterpret_cast<const float4*>(sQ);
  const float4* V4 = reinterpret_cast<const float4*>(v);
  float t[DU];
#pragma unroll
  for (int j = 0; j < DU; ++j) t[j] = 0.f;
  stream_rows<D, DU / 4>(B4, mask, [&](int k, const float4 (&b)[DU / 4]) {
#pragma unroll
    for (int j4 = 0; j4 < DU / 4; ++j4) {
      t[4 * j4 + 0] = fmaf(y2[k], b[j4].x, t[4 * j4 + 0]);
      t[4 * j4 + 1] = fmaf(y2[k], b[j4].y, t[4 * j4 + 1]);
      t[4 * j4 + 2] = fmaf(y2[k], b[j4].z, t[4 * j4 + 2]);
      t[4 * j4 + 3] = fmaf(y2[k], b[j4].w, t[4 * j4 + 3]);
    }
  });
  if constexpr (LAST) {
#pragma unroll
    for (int j4 = 0; j4 < DU / 4; ++j4) {
      const float4 e = V4[V::kEBR / 4 + j4];
      y3[4 * j4 + 0] = -t[4 * j4 + 0] * e.x;
      y3[4 * j4 + 1] = -t[4 * j4 + 1] * e.y;
      y3[4 * j4 + 2] = -t[4 * j4 + 2] * e.z;
      y3[4 * j4 + 3] = -t[4 * j4 + 3] * e.w;
    }
  }
#pragma unroll
  for (int j4 = 0; j4 < DU / 4; ++j4) {
    const float4 s = V4[V::kS2 / 4 + j4];
    t[4 * j4 + 0] *= s.x;
    t[4 * j4 + 1] *= s.y;
    t[4 * j4 + 2] *= s.z;
    t[4 * j4 + 3] *= s.w;
  }
  stream_rows<D, DU / 4>(B4, mask, [&](int k, const float4 (&b)[DU / 4]) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
    for (int j4 = 0; j4 < DU / 4; ++j4) {
      a0 = fmaf(t[4 * j4 + 0], b[j4].x, a0);
      a1 = fmaf(t[4 * j4 + 1], b[j4].y, a1);
      a2 = fmaf(t[4 * j4 + 2], b[j4].z, a2);
      a3 = fmaf(t[4 * j4 + 3], b[j4].w, a3);
    }
    y1[k] += (a0 + a1) + (a2 + a3);
  });
#pragma unroll
  for (int k4 = 0; k4 < D / 4; ++k4) {
    const float4 ia = V4[V::kIA / 4 + k4];
    y1[4 * k4 + 0] *= ia.x;
    y1[4 * k4 + 1] *= ia.y;
    y1[4 * k4 + 2] *= ia.z;
    y1[4 * k4 + 3] *= ia.w;
  }
  if constexpr (!LAST) {
    float z[D];
#pragma unroll
    for (int k = 0; k < D; ++k) z[k] = 0.f;
    stream_rows<D, D / 4>(Q4, mask, [&](int m, const float4 (&q)[D / 4]) {
      const float w = y1[m] * v[V::kDq + m];
#pragma unroll
      for (int k4 = 0; k4 < D / 4; ++k4) {
        z[4 * k4 + 0] = fmaf(w, q[k4].x, z[4 * k4 + 0]);
        z[4 * k4 + 1] = fmaf(w, q[k4].y, z[4 * k4 + 1]);
        z[4 * k4 + 2] = fmaf(w, q[k4].z, z[4 * k4 + 2]);
        z[4 * k4 + 3] = fmaf(w, q[k4].w, z[4 * k4 + 3]);
      }
    });
#pragma unroll
    for (int k4 = 0; k4 < D / 4; ++k4) {
      const float4 at = V4[V::kAt / 4 + k4];
      const float4 dq = V4[V::kDq / 4 + k4];
      y2[4 * k4 + 0] = fmaf(y2[4 * k4 + 0], at.x, z[4 * k4 + 0] * dq.x);
      y2[4 * k4 + 1] = fmaf(y2[4 * k4 + 1], at.y, z[4 * k4 + 1] * dq.y);
      y2[4 * k4 + 2] = fmaf(y2[4 * k4 + 2], at.z, z[4 * k4 + 2] * dq.z);
      y2[4 * k4 + 3] = fmaf(y2[4 * k4 + 3], at.w, z[4 * k4 + 3] * dq.w);
    }
  } else {
#pragma unroll
    for (int k4 = 0; k4 < D / 4; ++k4) {
      const float4 at = V4[V::kAt / 4 + k4];
      y2[4 * k4 + 0] *= at.x;
      y2[4 * k4 + 1] *= at.y;
      y2[4 * k4 + 2] *= at.z;
      y2[4 * k4 + 3] *= at.w;
    }
  }
}

// NORMALIZE_TYPE=2 of the reference (symplectic_iter.py:286-300): divide the row block
// by its largest row abs-sum of Y1 or Y2 when that exceeds 1e3.  The row block is the
// group's warp (min(D,32) rows) -- the reference's BY-row tile with BY = min(D, 32).
// Any row scaling leaves P = Y1^-1 Y2 and Y1^-1 Y3 unchanged.
template <int D, int DU, bool LAST>
__device__ __forceinline__ void renormalize(const Group<D>& G, float (&y1)[D], float (&y2)[D],
                                            float (&y3)[DU]) {
  float r1 = 0.f, r2 = 0.f;
#pragma unroll
  for (int k = 0; k < D; ++k) {
    r1 += fabsf(y1[k]);
    r2 += fabsf(y2[k]);
  }
  const float m = rowblock_max<D>(G, fmaxf(r1, r2));
  if (m > kNormThreshold) {
    // Any common factor is exact for P and Y1^-1 Y3; 1/m need not be correctly rounded.
    const float r = recip(m);
#pragma unroll
    for (int k = 0; k < D; ++k) {
      y1[k] *= r;
      y2[k] *= r;
    }
    if constexpr (LAST) {
#pragma unroll
      for (int j = 0; j < DU; ++j) y3[j] *= r;
    }
  }
}

// Horizon-T sweep from (Y1, Y2) = (I, Q_f) for one head.  `vec` is 2 x SweepVec::kSize
// floats of group shared memory (double-buffered by step parity: one group barrier per
// step).  Per-thread inputs: a = A_diag[i], lgA2 = log_gamma_A*log2(e),
// lgQ2 = log_gamma_Q[i]*log2(e), and for i < DU lgB2 = log_gamma_B[i]*log2(e), rinv = R_inv[i].
template <int D, int DU>
__device__ __forceinline__ void sweep(const Group<D>& G, float (&y1)[D], float (&y2)[D],
                                      float (&y3)[DU], const float* sB,
                                      const float* sQ, float* vec, float a,
                                      float lgA2, float lgQ2, float lgB2, float rinv, int T) {
  using V = SweepVec<D, DU>;
  const int i = G.i;
  for (int s = 0; s < T; ++s) {
    float* v = vec + (s & 1) * V::kSize;
    const float tau = static_cast<float>(T - s);
    const float at = fmaf(a, exp_scaled(lgA2, tau), 1.0f);
    v[V::kAt + i] = at;
    v[V::kIA + i] = recip(at);
    v[V::kDq + i] = exp_scaled(lgQ2, static_cast<float>(T - 1 - s));
    if (i < DU) {
      const float eb = exp_scaled(lgB2, tau);
      v[V::kS2 + i] = eb * eb * rinv;
      v[V::kEBR + i] = eb * rinv;
    }
    G.sync();
    if (s + 1 < T) {
      sweep_step<D, DU, false>(y1, y2, y3, sB, sQ, v, G.mask);
      renormalize<D, DU, false>(G, y1, y2, y3);
    } else {
      sweep_step<D, DU, true>(y1, y2, y3, sB, sQ, v, G.mask);
      renormalize<D, DU, true>(G, y1, y2, y3);
    }
  }
}

// Gauss-Jordan elimination with partial pivoting over the D threads of a group.
// `rows` is (D + NR) x D floats of group shared memory, column c of thread i at
// rows[c*D + i]: the thread's row of Y1 in columns [0,D) and of the right-hand sides in
// [D, D+NR).  Pivot rows are never swapped: each step picks the largest |entry| in the
// current column among the rows not yet used (first index on ties) and eliminates that
// column from every other row.  On return the thread's row holds piv * (row `pc` of
// Y1^-1 RHS) in [D, D+NR); the function returns pc and writes piv.  A NaN candidate
// counts as 0, so every thread gets exactly one pivot column and all indices stay in
// [0, D) whatever the data.
template <int D, int NR>
__device__ __forceinline__ int gauss_jordan(const Group<D>& G, float* rows, float* cand,
                                            float& piv) {
  const int i = G.i;
  bool done = false;
  int pc = 0;
  piv = 1.0f;
  for (int k = 0; k < D; ++k) {
    float* cd = cand + (k & 1) * D;
    cd[i] = done ? -1.0f : fmaxf(fabsf(rows[k * D + i]), 0.0f);
    G.sync();
    int p = 0;
    float best = cd[0];
    for (int r = 1; r < D; ++r) {
      const float c = cd[r];
      if (c > best) {
        best = c;
        p = r;
      }
    }
    if (i == p) {
      done = true;
      pc = k;
      piv = rows[k * D + i];
    } else {
      const float f = rows[k * D + i] * recip(rows[k * D + p]);
      rows[k * D + i] = 0.0f;
      for (int c = k + 1; c < D + NR; ++c) rows[c * D + i] = fmaf(-f, rows[c * D + p], rows[c * D + i]);
    }
  }
  G.sync();
  return pc;
}

}  // namespace ttc
