// TTC LQR solve for B200 (sm_100a): forward (sweep + solve + first-step decode) and
// backward (forward-in-time adjoint) kernels.
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
template <int D, int DU, bool SAVE_M>
struct FwdLayout {
  static constexpr int kNR = SAVE_M ? D + DU : D;        // right-hand sides: Y2 [| Y3]
  static constexpr int kVec = 2 * SweepVec<D, DU>::kSize;
  static constexpr int kRows = (D + kNR) * D;
  static constexpr int kGroup = round4(kVec + kRows + 2 * D + 3 * D);  // + cand, h0, a, lam1
  static constexpr int kShared = D * DU + D * D;
  static size_t bytes(int groups) { return sizeof(float) * (size_t)(kShared + groups * kGroup); }
};

template <int D, int DU, typename TIn, bool SAVE_M>
__global__ void __launch_bounds__(kThreads)
lqr_fwd_kernel(const TIn* __restrict__ A_diag, const TIn* __restrict__ Bm,
               const TIn* __restrict__ Qm, const TIn* __restrict__ Rinv,
               const TIn* __restrict__ Qf, const TIn* __restrict__ lgA,
               const TIn* __restrict__ lgB, const TIn* __restrict__ lgQ,
               const TIn* __restrict__ H0, int nh, int T, TIn* __restrict__ u_out,
               float* __restrict__ lam0_out, float* __restrict__ M_out, int* __restrict__ status) {
  using L = FwdLayout<D, DU, SAVE_M>;
  extern __shared__ __align__(16) float smem[];
  float* sB = smem;
  float* sQ = sB + D * DU;
  const int ngroups = blockDim.x / D;
  const Group<D> G(threadIdx.x);
  float* gs = smem + L::kShared + G.g * L::kGroup;
  float* vec = gs;
  float* rows = vec + L::kVec;
  float* cand = rows + L::kRows;
  float* sh0 = cand + 2 * D;
  float* sa = sh0 + D;
  float* slam = sa + D;

  const int64_t n = blockIdx.x;
  for (int e = threadIdx.x; e < D * DU; e += blockDim.x) sB[e] = ldf(Bm + n * (D * DU) + e);
  for (int e = threadIdx.x; e < D * D; e += blockDim.x) sQ[e] = ldf(Qm + n * (D * D) + e);
  __syncthreads();

  const int i = G.i;
  int flags = 0;
  for (int h = G.g; h < nh; h += ngroups) {
    const int64_t p = n * nh + h;
    const float a = ldf(A_diag + p * D + i);
    const float lgA2 = ldf(lgA + p) * kLog2e;
    const float lgQ2 = ldf(lgQ + p * D + i) * kLog2e;
    float lgB2 = 0.f, rinv = 0.f;
    if (i < DU) {
      lgB2 = ldf(lgB + p * DU + i) * kLog2e;
      rinv = ldf(Rinv + p * DU + i);
    }
    sh0[i] = ldf(H0 + p * D + i);
    sa[i] = a;

    float y1[D], y2[D], y3[DU];
    const TIn* qf = Qf + (p * D + i) * D;
#pragma unroll
    for (int k = 0; k < D; ++k) {
      y1[k] = (k == i) ? 1.0f : 0.0f;
      y2[k] = ldf(qf + k);
    }
    sweep<D, DU>(G, y1, y2, y3, sB, sQ, vec, a, lgA2, lgQ2, lgB2, rinv, T);

    bool bad = false;
#pragma unroll
    for (int k = 0; k < D; ++k) {
      bad |= unstable(y1[k]) | unstable(y2[k]);
      rows[k * D + i] = y1[k];
      rows[(D + k) * D + i] = y2[k];
    }
    if constexpr (SAVE_M) {
#pragma unroll
      for (int j = 0; j < DU; ++j) rows[(2 * D + j) * D + i] = y3[j];
    }
    if (bad) flags |= TTC_STATUS_FWD_UNSTABLE;

    float piv;
    const int pc = gauss_jordan<D, L::kNR>(G, rows, cand, piv);
    // Row pc of P = Y1^-1 Y2, then lambda0[pc] = (P h0)[pc] (symplectic_iter.py:437).
    bool lbad = unstable(piv);
    const float rpiv = recip(piv);
    float lam0 = 0.f;
    for (int c = 0; c < D; ++c) {
      const float x = rows[(D + c) * D + i] * rpiv;
      lbad |= unstable(x);
      lam0 = fmaf(x, sh0[c], lam0);
    }
    if (lbad) flags |= TTC_STATUS_LU_UNSTABLE;
    if (lam0_out != nullptr) lam0_out[p * D + pc] = lam0;
    if constexpr (SAVE_M) {
      float* mrow = M_out + (p * D + pc) * DU;
      for (int j = 0; j < DU; ++j) mrow[j] = rows[(2 * D + j) * D + i] * rpiv;
    }
    // lambda1 = lambda0 / (1 + A_diag e^lgA)   (symplectic_iter.py:472-477)
    slam[pc] = lam0 * recip(fmaf(sa[pc], exp_scaled(lgA2, 1.0f), 1.0f));
    G.sync();
    if (i < DU) {
      // u = -R_inv * (B diag(e^lgB))^T lambda1   (symplectic_iter.py:488-517)
      float acc = 0.f;
#pragma unroll 8
      for (int k = 0; k < D; ++k) acc = fmaf(sB[k * DU + i], slam[k], acc);
      const float u = -(acc * exp_scaled(lgB2, 1.0f)) * rinv;
      if (isnan(u)) flags |= TTC_STATUS_U_NAN;
      stf(u_out + p * DU + i, u);
    }
    G.sync();
  }
  if (flags) atomicOr(status, flags);
}

// --------------------------------------------------------------------------------------
// Backward
// --------------------------------------------------------------------------------------
template <int D, int DU, bool RECOMPUTE>
struct BwdLayout {
  static constexpr int kNR = D + 1;  // right-hand sides: Y2 | Y3 du
  static constexpr int kVec = RECOMPUTE ? 2 * SweepVec<D, DU>::kSize : 0;
  static constexpr int kRows = RECOMPUTE ? (D + kNR) * D : 0;
  static constexpr int kCand = RECOMPUTE ? 2 * D : 0;
  // adjoint vectors, double-buffered: lam, dlam, hD, dhD, h, dh (D each), uE, duE (DU each)
  static constexpr int kAdjB = 6 * D + 2 * DU;
  static constexpr int kAcc = D * DU + D * D;
  static constexpr int kGroup = round4(kVec + kRows + kCand + 2 * kAdjB + kAcc + 4 * D + 4);
  static constexpr int kBp = round4(D * (DU + 1));
  static constexpr int kQp = round4(D * (D + 1));
  static constexpr int kShared = D * DU + D * D + kBp + kQp;
  static size_t bytes(int groups) { return sizeof(float) * (size_t)(kShared + groups * kGroup); }
};

template <int D, int DU, typename TIn, bool RECOMPUTE>
__global__ void __launch_bounds__(kThreads)
lqr_bwd_kernel(const TIn* __restrict__ A_diag, const TIn* __restrict__ Bm,
               const TIn* __restrict__ Qm, const TIn* __restrict__ Rinv,
               const TIn* __restrict__ Qf, const TIn* __restrict__ lgA,
               const TIn* __restrict__ lgB, const TIn* __restrict__ lgQ,
               const TIn* __restrict__ H0, const float* __restrict__ lam0_in,
               const float* __restrict__ M_in, const TIn* __restrict__ dU, int nh, int T,
               TIn* __restrict__ gA_out, TIn* __restrict__ gB_out, TIn* __restrict__ gQ_out,
               TIn* __restrict__ gR_out, TIn* __restrict__ gQf_out, TIn* __restrict__ glgA_out,
               TIn* __restrict__ glgB_out, TIn* __restrict__ glgQ_out,
               TIn* __restrict__ gh0_out, int* __restrict__ status) {
  using L = BwdLayout<D, DU, RECOMPUTE>;
  extern __shared__ __align__(16) float smem[];
  float* sB = smem;                 // [D][DU]   (sweep, 128-bit broadcast rows)
  float* sQ = sB + D * DU;          // [D][D]
  float* sBp = sQ + D * D;          // [D][DU+1] (adjoint, conflict-free rows and columns)
  float* sQp = sBp + L::kBp;        // [D][D+1]
  const int ngroups = blockDim.x / D;
  const Group<D> G(threadIdx.x);
  float* gs = smem + L::kShared + G.g * L::kGroup;
  float* vec = gs;
  float* rows = vec + L::kVec;
  float* cand = rows + L::kRows;
  float* adj = cand + L::kCand;
  float* accB = adj + 2 * L::kAdjB;  // [DU][D] (transposed: thread i owns column i)
  float* accQ = accB + D * DU;       // [D][D]
  float* sh0 = accQ + D * D;
  float* sdu = sh0 + D;
  float* sx = sdu + D;               // lambda0 / d_p hand-over after the solve
  float* sdp = sx + D;
  float* red = sdp + D;

  const int64_t n = blockIdx.x;
  const int tid = threadIdx.x;
  bool sym_local = true;
  for (int e = tid; e < D * DU; e += blockDim.x) {
    const float b = ldf(Bm + n * (D * DU) + e);
    sB[e] = b;
    sBp[(e / DU) * (DU + 1) + (e % DU)] = b;
  }
  for (int e = tid; e < D * D; e += blockDim.x) {
    const float q = ldf(Qm + n * (D * D) + e);
    sQ[e] = q;
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
    sh0[i] = h0i;

    float lam, dlam;
    if constexpr (RECOMPUTE) {
      // Re-run the forward sweep; solve Y1 [P | d_p] = [Y2 | Y3 du] (fused_lqr.py:104-105,185-187).
      float y1[D], y2[D], y3[DU];
      const TIn* qf = Qf + (p * D + i) * D;
#pragma unroll
      for (int k = 0; k < D; ++k) {
        y1[k] = (k == i) ? 1.0f : 0.0f;
        y2[k] = ldf(qf + k);
      }
      sweep<D, DU>(G, y1, y2, y3, sB, sQ, vec, a, lgA2, lgQ2, lgB2, rinv, T);
      float y3du = 0.f;
#pragma unroll
      for (int j = 0; j < DU; ++j) y3du = fmaf(y3[j], sdu[j], y3du);
#pragma unroll
      for (int k = 0; k < D; ++k) {
        rows[k * D + i] = y1[k];
        rows[(D + k) * D + i] = y2[k];
      }
      rows[2 * D * D + i] = y3du;
      float piv;
      const int pc = gauss_jordan<D, L::kNR>(G, rows, cand, piv);
      const float rpiv = recip(piv);
      float lam0 = 0.f;
      for (int c = 0; c < D; ++c) lam0 = fmaf(rows[(D + c) * D + i] * rpiv, sh0[c], lam0);
      sx[pc] = lam0;
      sdp[pc] = rows[2 * D * D + i] * rpiv;
      G.sync();
      lam = sx[i];
      dlam = sdp[i];
    } else {
      G.sync();  // sdu visible to the group
      lam = lam0_in[p * D + i];
      const float* mrow = M_in + (p * D + i) * DU;
      dlam = 0.f;
      for (int j = 0; j < DU; ++j) dlam = fmaf(mrow[j], sdu[j], dlam);
    }

    // Forward-in-time adjoint (symplectic_iter.py:715-885).
    float hs = h0i, dh = 0.f;
    float gA = 0.f, glgA = 0.f, glgQ = 0.f, gR = 0.f, glgB = 0.f, gh0 = 0.f;
    float gB[DU], gQ[D];
#pragma unroll
    for (int j = 0; j < DU; ++j) gB[j] = 0.f;
#pragma unroll
    for (int k = 0; k < D; ++k) gQ[k] = 0.f;
    float dq_prev = 1.0f;  // exp(lgQ * k) at the top of step k
    bool bad = false;
    for (int k = 0; k < T; ++k) {
      float* cb = adj + (k & 1) * L::kAdjB;
      const float* pb = adj + ((k + 1) & 1) * L::kAdjB;
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
        const float* p_hD = pb + 2 * D;
        const float* p_dhD = pb + 3 * D;
        float qh = 0.f, qdh = 0.f, qth = 0.f, qtdh = 0.f;
        if (sym) {
#pragma unroll 8
          for (int j = 0; j < D; ++j) {
            const float q = sQp[i * (D + 1) + j];
            qh = fmaf(q, p_hD[j], qh);
            qdh = fmaf(q, p_dhD[j], qdh);
          }
          qth = qh;
          qtdh = qdh;
        } else {
#pragma unroll 8
          for (int j = 0; j < D; ++j) {
            const float q = sQp[i * (D + 1) + j];
            const float qt = sQp[j * (D + 1) + i];
            qh = fmaf(q, p_hD[j], qh);
            qdh = fmaf(q, p_dhD[j], qdh);
            qth = fmaf(qt, p_hD[j], qth);
            qtdh = fmaf(qt, p_dhD[j], qtdh);
          }
        }
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
        float bl = 0.f, bdl = 0.f;
#pragma unroll 8
        for (int r = 0; r < D; ++r) {
          const float b = sBp[r * (DU + 1) + i];
          bl = fmaf(b, c_lam[r], bl);
          bdl = fmaf(b, c_dlam[r], bdl);
        }
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
      float bu = 0.f, bdu = 0.f;
#pragma unroll
      for (int j = 0; j < DU; ++j) {
        const float b = sBp[i * (DU + 1) + j];
        const float ue = c_uE[j], due = c_duE[j];
        bu = fmaf(b, ue, bu);
        bdu = fmaf(b, due, bdu);
        gB[j] = fmaf(lam, due, fmaf(dlam, ue, gB[j]));
      }
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
        TIn* qrow = gQf_out + (p * D + i) * D;
        for (int j = 0; j < D; ++j) {
          const float v = 0.5f * fmaf(hs, c_dh[j], dh * c_h[j]);
          bad |= unstable(v);
          stf(qrow + j, v);
        }
      } else {
#pragma unroll
        for (int j = 0; j < D; ++j) gQ[j] = fmaf(0.5f, fmaf(hD, c_dhD[j], dhD * c_hD[j]), gQ[j]);
      }
      dq_prev = dq;
    }
    const float glgA_sum = group_sum<D>(G, glgA, red);
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
#pragma unroll
    for (int j = 0; j < DU; ++j) accB[j * D + i] += gB[j];
#pragma unroll
    for (int k = 0; k < D; ++k) accQ[k * D + i] += gQ[k];
    if (bad) flags |= TTC_STATUS_BWD_UNSTABLE;
    G.sync();
  }
  __syncthreads();
  // grad_B / grad_Q of the row: sum of the groups' accumulators in group order.
  const int stride = L::kGroup;
  float* acc0 = smem + L::kShared + (L::kVec + L::kRows + L::kCand + 2 * L::kAdjB);
  bool bad = false;
  for (int e = tid; e < D * DU; e += blockDim.x) {
    const int r = e / DU, c = e % DU;
    float s = 0.f;
    for (int g = 0; g < ngroups; ++g) s += acc0[g * stride + c * D + r];
    bad |= unstable(s);
    stf(gB_out + n * (D * DU) + e, s);
  }
  for (int e = tid; e < D * D; e += blockDim.x) {
    const int r = e / D, c = e % D;
    float s = 0.f;
    for (int g = 0; g < ngroups; ++g) s += acc0[g * stride + D * DU + c * D + r];
    bad |= unstable(s);
    stf(gQ_out + n * (D * D) + e, s);
  }
  if (bad) flags |= TTC_STATUS_BWD_UNSTABLE;
  if (flags) atomicOr(status, flags);
}

}  // namespace ttc

