// TTC LQR solve for B200 (sm_100a): the forward's per-head scratch layout, the
// forward-in-time adjoint shared by both backward kernels, and the backward kernel for a
// forward that saved M = Y1^-1 Y3.  The tensor-core sweep kernels are in lqr_tc.cuh.
//
// Grid: one CTA per row n of the batch.  The CTA holds that row's B and Q (shared by
// all heads) in shared memory; its G groups of D threads walk the row's heads
// h = g, g + G, ... .  Every reduction is done in a fixed order inside the CTA, so
// results are bitwise reproducible from run to run.
#pragma once

#include "lqr_sweep.cuh"
#include "ttc_b200.h"

namespace ttc {

constexpr int kThreads = 256;

__host__ __device__ constexpr int round4(int x) { return (x + 3) & ~3; }

// --------------------------------------------------------------------------------------
// Forward
// --------------------------------------------------------------------------------------
// --------------------------------------------------------------------------------------
// Backward
// --------------------------------------------------------------------------------------
// Adjoint vectors of one head in group shared memory, double-buffered by step parity:
// lam, dlam, hD, dhD, h, dh (D each), uE, duE (DU each).
template <int D, int DU>
struct AdjLayout {
  static constexpr int kBuf = 6 * D + 2 * DU;
  static constexpr int kSize = 2 * kBuf;
};

// Forward-in-time adjoint of one head (symplectic_iter.py:715-885) for the group's D
// threads, from (h, dh, lambda, dlambda) = (h0, 0, lambda0, d_p).  Thread i carries entry i
// of the state vectors (and entry i < DU of the action vectors); B and Q come from the
// padded shared copies sBp [D][DU+1] and sQp [D][D+1] (bank-conflict free along rows and
// columns).  Writes the head's gradients of A_diag, R_inv, Q_f, log-gammas and h0 (when
// `valid`), and returns the head's grad_B row i (transposed into gB, pre-scaled by
// exp(lgB t)) and grad_Q row i (gQ) for the caller's reduction over heads.  Returns true if
// any written gradient is NaN, Inf or >= 1e6.
template <int D, int DU, typename TIn, bool kCache>
__device__ __forceinline__ bool adjoint_head(
    const Group<D>& G, bool valid, int64_t p, int T, float a, float lgA2, float lgQ2, float lgB2,
    float rinv, float dUi, float h0i, float lam, float dlam, const float* sBp, const float* sQp,
    bool sym, float* adj, float* red, float (&gB)[DU], float (&gQ)[D], TIn* gA_out, TIn* gR_out,
    TIn* gQf_out, TIn* glgA_out, TIn* glgB_out, TIn* glgQ_out, TIn* gh0_out) {
  static_assert(D % 4 == 0 && DU % 4 == 0, "dimensions must be multiples of 4");
  constexpr int kAdjB = AdjLayout<D, DU>::kBuf;
  // The matrix-vector products and the rank-2 gradient updates run on fp32 pairs (two
  // columns per instruction) in the summation order of four interleaved partial sums.
  // kCache: the thread's row of Q, row of B and column of B (constant for the head) are
  // held in registers (2d + du of them) instead of being re-read from shared memory every
  // step; the caller decides whether its register budget allows it.
  const int i = G.i;
  f2 qrow_r[kCache ? D / 2 : 1], brow_r[kCache ? DU / 2 : 1], bcol_r[kCache ? D / 2 : 1];
  auto ld_qrow = [&](int j2) { return pk2(sQp[i * (D + 1) + 2 * j2], sQp[i * (D + 1) + 2 * j2 + 1]); };
  auto ld_brow = [&](int j2) { return pk2(sBp[i * (DU + 1) + 2 * j2], sBp[i * (DU + 1) + 2 * j2 + 1]); };
  auto ld_bcol = [&](int r2) {
    return i < DU ? pk2(sBp[2 * r2 * (DU + 1) + i], sBp[(2 * r2 + 1) * (DU + 1) + i]) : f2(0);
  };
  if constexpr (kCache) {
#pragma unroll
    for (int j2 = 0; j2 < D / 2; ++j2) qrow_r[j2] = ld_qrow(j2);
#pragma unroll
    for (int j2 = 0; j2 < DU / 2; ++j2) brow_r[j2] = ld_brow(j2);
#pragma unroll
    for (int r2 = 0; r2 < D / 2; ++r2) bcol_r[r2] = ld_bcol(r2);
  }
  auto qrow = [&](int j2) { if constexpr (kCache) return qrow_r[j2]; else return ld_qrow(j2); };
  auto brow = [&](int j2) { if constexpr (kCache) return brow_r[j2]; else return ld_brow(j2); };
  auto bcol = [&](int r2) { if constexpr (kCache) return bcol_r[r2]; else return ld_bcol(r2); };
  auto qcol = [&](int r2) { return pk2(sQp[2 * r2 * (D + 1) + i], sQp[(2 * r2 + 1) * (D + 1) + i]); };
  float hs = h0i, dh = 0.f;
  float gA = 0.f, glgA = 0.f, glgQ = 0.f, gR = 0.f, glgB = 0.f, gh0 = 0.f;
  f2 gB2[DU / 2], gQ2[D / 2];
#pragma unroll
  for (int j2 = 0; j2 < DU / 2; ++j2) gB2[j2] = 0;
#pragma unroll
  for (int k2 = 0; k2 < D / 2; ++k2) gQ2[k2] = 0;
  float dq_prev = 1.0f;  // exp(lgQ * k) at the top of step k
  bool bad = false;
  for (int k = 0; k < T; ++k) {
    float* cb = adj + (k & 1) * kAdjB;
    const float* pb = adj + ((k + 1) & 1) * kAdjB;
    float* c_lam = cb;
    float* c_dlam = cb + D;
    float* c_hD = cb + 2 * D;
    float* c_dhD = cb + 3 * D;
    float* c_h = cb + 4 * D;
    float* c_dh = cb + 5 * D;
    float* c_uE = cb + 6 * D;
    float* c_duE = cb + 6 * D + DU;
    const float ke = static_cast<float>(k + 1);
    if (k > 0) {
      // lambda -= Q_k h, dlambda -= Q_k dh with Q_k = Dq Q Dq (symplectic_iter.py:766-775);
      // the same products give the log_gamma_Q gradient of step k-1 (:871-877).
      const float4* h4 = reinterpret_cast<const float4*>(pb + 2 * D);
      const float4* dh4 = reinterpret_cast<const float4*>(pb + 3 * D);
      f2 ph0 = 0, ph1 = 0, pd0 = 0, pd1 = 0, pth0 = 0, pth1 = 0, ptd0 = 0, ptd1 = 0;
#pragma unroll
      for (int j4 = 0; j4 < D / 4; ++j4) {
        const float4 hv = h4[j4], dv = dh4[j4];  // broadcast 128-bit reads
        const f2 qa = qrow(2 * j4), qb = qrow(2 * j4 + 1);
        ph0 = fma2(qa, lo2(hv), ph0);
        ph1 = fma2(qb, hi2(hv), ph1);
        pd0 = fma2(qa, lo2(dv), pd0);
        pd1 = fma2(qb, hi2(dv), pd1);
        if (!sym) {
          const f2 ta = qcol(2 * j4), tb = qcol(2 * j4 + 1);
          pth0 = fma2(ta, lo2(hv), pth0);
          pth1 = fma2(tb, hi2(hv), pth1);
          ptd0 = fma2(ta, lo2(dv), ptd0);
          ptd1 = fma2(tb, hi2(dv), ptd1);
        }
      }
      const float qh = sum2(ph0) + sum2(ph1);
      const float qdh = sum2(pd0) + sum2(pd1);
      const float qth = sym ? qh : sum2(pth0) + sum2(pth1);
      const float qtdh = sym ? qdh : sum2(ptd0) + sum2(ptd1);
      lam = fmaf(-dq_prev, qh, lam);
      dlam = fmaf(-dq_prev, qdh, dlam);
      glgQ = fmaf(0.5f * fmaf(dh, qh + qth, hs * (qdh + qtdh)), static_cast<float>(k) * dq_prev, glgQ);
    } else {
      gh0 = dlam;
    }
    const float eA = exp_scaled(lgA2, ke);
    const float At = fmaf(a, eA, 1.0f);
    const float rAt = recip(At);
    lam *= rAt;
    dlam *= rAt;
    const float dA = fmaf(lam, dh, dlam * hs);
    gA = fmaf(dA, eA, gA);
    glgA = fmaf(dA * a, ke * eA, glgA);
    c_lam[i] = lam;
    c_dlam[i] = dlam;
    G.sync();
    if (i < DU) {
      const float4* l4 = reinterpret_cast<const float4*>(c_lam);
      const float4* dl4 = reinterpret_cast<const float4*>(c_dlam);
      f2 pl0 = 0, pl1 = 0, pdl0 = 0, pdl1 = 0;
#pragma unroll
      for (int r4 = 0; r4 < D / 4; ++r4) {
        const float4 lv = l4[r4], dv = dl4[r4];
        const f2 ba = bcol(2 * r4), bb = bcol(2 * r4 + 1);
        pl0 = fma2(ba, lo2(lv), pl0);
        pl1 = fma2(bb, hi2(lv), pl1);
        pdl0 = fma2(ba, lo2(dv), pdl0);
        pdl1 = fma2(bb, hi2(dv), pdl1);
      }
      const float bl = sum2(pl0) + sum2(pl1);
      const float bdl = sum2(pdl0) + sum2(pdl1);
      const float eB = exp_scaled(lgB2, ke);
      const float u = -(bl * eB) * rinv;
      float du = -(bdl * eB) * rinv;
      if (k == 0) du = fmaf(dUi, -rinv, du);
      glgB = fmaf(fmaf(du, bl, u * bdl), ke * eB, glgB);
      gR = fmaf(-(u * du), recip(rinv * rinv), gR);
      c_uE[i] = u * eB;
      c_duE[i] = du * eB;
    }
    G.sync();
    const float4* ue4 = reinterpret_cast<const float4*>(c_uE);
    const float4* due4 = reinterpret_cast<const float4*>(c_duE);
    const f2 lam2 = dup2(lam), dlam2 = dup2(dlam);
    f2 pu0 = 0, pu1 = 0, pdu0 = 0, pdu1 = 0;
#pragma unroll
    for (int j4 = 0; j4 < DU / 4; ++j4) {
      const float4 uv = ue4[j4], dv = due4[j4];
      const f2 ba = brow(2 * j4), bb = brow(2 * j4 + 1);
      pu0 = fma2(ba, lo2(uv), pu0);
      pu1 = fma2(bb, hi2(uv), pu1);
      pdu0 = fma2(ba, lo2(dv), pdu0);
      pdu1 = fma2(bb, hi2(dv), pdu1);
      gB2[2 * j4] = fma2(lam2, lo2(dv), fma2(dlam2, lo2(uv), gB2[2 * j4]));
      gB2[2 * j4 + 1] = fma2(lam2, hi2(dv), fma2(dlam2, hi2(uv), gB2[2 * j4 + 1]));
    }
    const float bu = sum2(pu0) + sum2(pu1);
    const float bdu = sum2(pdu0) + sum2(pdu1);
    hs = fmaf(hs, At, bu);
    dh = fmaf(dh, At, bdu);
    const float dq = exp_scaled(lgQ2, ke);
    const float hD = hs * dq, dhD = dh * dq;
    c_hD[i] = hD;
    c_dhD[i] = dhD;
    c_h[i] = hs;
    c_dh[i] = dh;
    G.sync();
    if (k == T - 1) {
      // grad_Qf = (h dh^T + dh h^T) / 2 at the final state (symplectic_iter.py:855-857).
      if (valid) {
        TIn* qrow_out = gQf_out + (p * D + i) * D;
        for (int j = 0; j < D; ++j) {
          const float v = 0.5f * fmaf(hs, c_dh[j], dh * c_h[j]);
          bad |= unstable(v);
          stf(qrow_out + j, v);
        }
      }
    } else {
      const float4* hD4 = reinterpret_cast<const float4*>(c_hD);
      const float4* dhD4 = reinterpret_cast<const float4*>(c_dhD);
      const f2 hD2 = dup2(hD), dhD2 = dup2(dhD);
      // (h dh^T + dh h^T) scaled by Dq on both sides; the 1/2 is applied once at the end.
#pragma unroll
      for (int j4 = 0; j4 < D / 4; ++j4) {
        const float4 hv = hD4[j4], dv = dhD4[j4];
        gQ2[2 * j4] = fma2(hD2, lo2(dv), fma2(dhD2, lo2(hv), gQ2[2 * j4]));
        gQ2[2 * j4 + 1] = fma2(hD2, hi2(dv), fma2(dhD2, hi2(hv), gQ2[2 * j4 + 1]));
      }
    }
    dq_prev = dq;
  }
#pragma unroll
  for (int j2 = 0; j2 < DU / 2; ++j2) up2(gB2[j2], gB[2 * j2], gB[2 * j2 + 1]);
#pragma unroll
  for (int k2 = 0; k2 < D / 2; ++k2) up2(mul2(gQ2[k2], dup2(0.5f)), gQ[2 * k2], gQ[2 * k2 + 1]);
  const float glgA_sum = group_sum<D>(G, glgA, red);
  if (valid) {
    bad |= unstable(gA) | unstable(glgQ) | unstable(gh0);
    stf(gA_out + p * D + i, gA);
    stf(glgQ_out + p * D + i, glgQ);
    stf(gh0_out + p * D + i, gh0);
    if (i < DU) {
      bad |= unstable(gR) | unstable(glgB);
      stf(gR_out + p * DU + i, gR);
      stf(glgB_out + p * DU + i, glgB);
    }
    if (i == 0) {
      bad |= unstable(glgA_sum);
      stf(glgA_out + p, glgA_sum);
    }
  }
  G.sync();  // adjoint buffers are reused by the next head
  return bad;
}

// Backward with the forward's saved lambda0 and M = Y1^-1 Y3 (d_p = M du,
// fused_lqr.py:185-187).  One CTA per row; the CTA's groups walk the row's heads and the
// per-group grad_B / grad_Q accumulators are summed in group order at the end.
template <int D, int DU>
struct BwdLayout {
  static constexpr int kAcc = D * DU + D * D;
  static constexpr int kGroup = round4(AdjLayout<D, DU>::kSize + kAcc + 4 * D + 4);
  static constexpr int kBp = round4(D * (DU + 1));
  static constexpr int kQp = round4(D * (D + 1));
  static constexpr int kShared = kBp + kQp;
  static size_t bytes(int groups) { return sizeof(float) * (size_t)(kShared + groups * kGroup); }
};

// Resident CTAs per SM asked of ptxas for the saved-state backward (registers per thread
// <= 65536 / (256 * n)).
#ifndef TTC_BWD_MINB16
#define TTC_BWD_MINB16 2
#endif
#ifndef TTC_BWD_MINB32
#define TTC_BWD_MINB32 2
#endif
template <int D>
constexpr int bwd_min_ctas() { return D <= 16 ? TTC_BWD_MINB16 : (D <= 32 ? TTC_BWD_MINB32 : 1); }

template <int D, int DU, typename TIn>
__global__ void __launch_bounds__(kThreads, bwd_min_ctas<D>())
lqr_bwd_kernel(const TIn* __restrict__ A_diag, const TIn* __restrict__ Bm,
               const TIn* __restrict__ Qm, const TIn* __restrict__ Rinv,
               const TIn* __restrict__ lgA, const TIn* __restrict__ lgB,
               const TIn* __restrict__ lgQ, const TIn* __restrict__ H0,
               const float* __restrict__ lam0_in, const float* __restrict__ M_in,
               const TIn* __restrict__ dU, int nh, int T, TIn* __restrict__ gA_out,
               TIn* __restrict__ gB_out, TIn* __restrict__ gQ_out, TIn* __restrict__ gR_out,
               TIn* __restrict__ gQf_out, TIn* __restrict__ glgA_out, TIn* __restrict__ glgB_out,
               TIn* __restrict__ glgQ_out, TIn* __restrict__ gh0_out, int* __restrict__ status) {
  using L = BwdLayout<D, DU>;
  extern __shared__ __align__(128) float smem[];
  float* sBp = smem;            // [D][DU+1]
  float* sQp = sBp + L::kBp;    // [D][D+1]
  const int ngroups = blockDim.x / D;
  const Group<D> G(threadIdx.x);
  float* gs = smem + L::kShared + G.g * L::kGroup;
  float* adj = gs;
  float* accB = adj + AdjLayout<D, DU>::kSize;  // [DU][D] (transposed: thread i owns column i)
  float* accQ = accB + D * DU;                  // [D][D]
  float* sdu = accQ + D * D;
  float* red = sdu + D;

  const int64_t n = blockIdx.x;
  const int tid = threadIdx.x;
  bool sym_local = true;
  for (int e = tid; e < D * DU; e += blockDim.x)
    sBp[(e / DU) * (DU + 1) + (e % DU)] = ldf(Bm + n * (D * DU) + e);
  for (int e = tid; e < D * D; e += blockDim.x) {
    const float q = ldf(Qm + n * (D * D) + e);
    sQp[(e / D) * (D + 1) + (e % D)] = q;
    sym_local &= (q == ldf(Qm + n * (D * D) + (e % D) * D + (e / D)));
  }
  for (int e = G.i; e < L::kAcc; e += D) accB[e] = 0.0f;  // accB and accQ are contiguous
  const bool sym = __syncthreads_and(sym_local);

  const int i = G.i;
  int flags = 0;
  for (int h = G.g; h < nh; h += ngroups) {
    const int64_t p = n * nh + h;
    const float a = ldf(A_diag + p * D + i);
    const float lgA2 = ldf(lgA + p) * kLog2e;
    const float lgQ2 = ldf(lgQ + p * D + i) * kLog2e;
    float lgB2 = 0.f, rinv = 0.f, dUi = 0.f;
    if (i < DU) {
      lgB2 = ldf(lgB + p * DU + i) * kLog2e;
      rinv = ldf(Rinv + p * DU + i);
      dUi = ldf(dU + p * DU + i);
      sdu[i] = dUi;
    }
    const float h0i = ldf(H0 + p * D + i);
    G.sync();  // sdu visible to the group
    const float lam = lam0_in[p * D + i];
    const float* mrow = M_in + (p * D + i) * DU;
    float dlam = 0.f;
    for (int j = 0; j < DU; ++j) dlam = fmaf(mrow[j], sdu[j], dlam);
    float gB[DU], gQ[D];
    const bool bad = adjoint_head<D, DU, TIn, (D <= 16)>(G, true, p, T, a, lgA2, lgQ2, lgB2, rinv, dUi, h0i,
                                              lam, dlam, sBp, sQp, sym, adj, red, gB, gQ, gA_out,
                                              gR_out, gQf_out, glgA_out, glgB_out, glgQ_out, gh0_out);
#pragma unroll
    for (int j = 0; j < DU; ++j) accB[j * D + i] += gB[j];
#pragma unroll
    for (int k = 0; k < D; ++k) accQ[k * D + i] += gQ[k];
    if (bad) flags |= TTC_STATUS_BWD_UNSTABLE;
  }
  __syncthreads();
  // grad_B / grad_Q of the row: sum of the groups' accumulators in group order.
  const float* acc0 = smem + L::kShared + AdjLayout<D, DU>::kSize;
  bool bad = false;
  for (int e = tid; e < D * DU; e += blockDim.x) {
    const int r = e / DU, c = e % DU;
    float s = 0.f;
    for (int g = 0; g < ngroups; ++g) s += acc0[g * L::kGroup + c * D + r];
    bad |= unstable(s);
    stf(gB_out + n * (D * DU) + e, s);
  }
  for (int e = tid; e < D * D; e += blockDim.x) {
    const int r = e / D, c = e % D;
    float s = 0.f;
    for (int g = 0; g < ngroups; ++g) s += acc0[g * L::kGroup + D * DU + c * D + r];
    bad |= unstable(s);
    stf(gQ_out + n * (D * D) + e, s);
  }
  if (bad) flags |= TTC_STATUS_BWD_UNSTABLE;
  if (flags) atomicOr(status, flags);
}

}  // namespace ttc

