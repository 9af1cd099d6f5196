// Forward LQR solve with the symplectic sweep on the 5th-generation tensor cores.
//
// A tile is 128 state rows = 128 TMEM lanes = 128 / d heads of one batch row n; thread t
// of the tile's four warps owns TMEM lane t, i.e. row (t % d) of head (t / d), and keeps
// that row of Y1 and Y2 in registers exactly as the CUDA-core sweep does.  Each of the
// three products of a step (symplectic_iter.py:231,233,256) is one chain of
// tcgen05.mma kind::tf32 in 3xTF32 form (A_lo*B_hi + A_hi*B_lo + A_hi*B_hi, the
// reference's tf32x3): the scaled state row goes to TMEM as A (hi = the fp32 value, lo
// = its tf32 residual), the row's B, B^T and Q (shared by all heads) sit in shared memory
// as hi/lo K-major operands, the product lands in TMEM and comes back with tcgen05.ld for
// the per-head diagonal scalings.  A CTA runs several tiles ("slots") of the same row
// so that one slot's MMAs overlap the others' elementwise work.
#pragma once

#include <type_traits>

#include "lqr_kernels.cuh"
#include "tc_primitives.cuh"

namespace ttc {

constexpr uint32_t kMaxPolls = 1u << 24;  // bounded mbarrier polls before TTC_STATUS_MMA_TIMEOUT
// At d = 16 (six tiles per SM) sleeping in try_wait instead of polling frees issue slots for
// the other tiles' CUDA-core work (2.4 % on config 2; the hint's value, 50 ns to 5 us, does
// not matter), and 1.5 % at d = 64; at d = 32 (four tiles per SM, the whole TMEM) the
// wake-up costs 1.2 % more than it saves.
#ifndef TTC_WAIT_HINT16
#define TTC_WAIT_HINT16 1000u
#endif
#ifndef TTC_WAIT_HINT32
#define TTC_WAIT_HINT32 0u
#endif
#ifndef TTC_WAIT_HINT64
#define TTC_WAIT_HINT64 1000u
#endif
template <int D>
constexpr uint32_t kWaitHintNs = D <= 16 ? TTC_WAIT_HINT16 : (D <= 32 ? TTC_WAIT_HINT32 : TTC_WAIT_HINT64);

template <int D, int DU>
struct TcCfg {
  static constexpr int kHeadsPerTile = 128 / D;
  static constexpr int kMax = D > DU ? D : DU;
  // TMEM columns of a slot: A_hi | A_lo | accumulator, 32-column aligned.
  static constexpr int kSlotCols = (3 * kMax + 31) / 32 * 32;
  // Operands (hi block then lo block, canonical K-major):
  //   O1: N = DU, K = D,  (j, k) = B[k][j]   for  t  = Y2 B
  //   O2: N = D,  K = DU, (k, j) = B[k][j]   for  dY1 = c B^T
  //   O3: N = D,  K = D,  (k, j) = Q[j][k]   for  z  = w Q
  static constexpr int kO1 = 0;
  static constexpr int kO2 = kO1 + 2 * DU * D;
  static constexpr int kO3 = kO2 + 2 * D * DU;
  static constexpr int kOps = kO3 + 2 * D * D;
  static constexpr int kHeader = 32;  // floats: mbarriers (8 x 8 B), TMEM base, flags
};

// Launch shape: at d = 16 a thread needs ~80 registers, so 256-thread CTAs with three
// resident per SM (6 tiles in flight) beat 512-thread CTAs at 128 registers (measured
// 14 % on config 2); at d = 32 the 128-register budget of 4 tiles per SM is needed: one
// 512-thread CTA of four slots, or (NARROW) two 256-thread CTAs of two slots.  The two CTAs
// of an SM drift apart, so one CTA's per-tile tail (Gauss-Jordan, M, u, the next tile's loads,
// all without MMAs) overlaps the other's sweep: 1.9 % faster at T = 128 and 3 % at T = 32
// (materialised Q_f, 8 192 rows), two tiles alone keeping 77 % of the four-tile throughput.
// NARROW needs both CTAs' shared memory on the SM, hence the layer's Q_f basis staged in its
// own bf16.  At d = 64 a thread holds two 64-wide state rows plus a product row (~220
// registers): 256-thread CTAs, one per SM.
template <int D, bool NARROW = false>
struct TcLaunch {
  static constexpr bool kNarrow = NARROW && D == 32;
  static constexpr int kMaxThreads = (D == 32 && !kNarrow) ? 512 : 256;
  static constexpr int kMinBlocks = D <= 16 ? 3 : (kNarrow ? 2 : 1);
  static constexpr int kMaxSlots = kMaxThreads / 128;
};

template <int D, int DU, bool SAVE_M>
struct TcFwdLayout {
  using C = TcCfg<D, DU>;
  // per head: sweep vectors (double-buffered), h0, lambda1 hand-over, spare, and the
  // pivot-row buffer of the cross-warp Gauss-Jordan (d = 64 only)
  static constexpr int kPb = GjRow<D, D>::kSize;
  static constexpr int kGroup = round4(2 * SweepVec<D, DU>::kSize + 3 * D + kPb);
  static size_t bytes(int slots) {
    return sizeof(float) * (size_t)(C::kOps + C::kHeader + slots * C::kHeadsPerTile * kGroup);
  }
  // A mixed Q_f keeps its rank-rQ basis in shared memory behind the groups (BasisSmem).
  __host__ __device__ static int basis_offset(int slots) { return C::kOps + C::kHeader + slots * C::kHeadsPerTile * kGroup; }
};

// The layer's rank-rQ Q_f basis [rQ, D, D] in shared memory, read one row per thread with
// 16-byte loads (the D threads of a head read rows 0..D-1 of one basis matrix at once).
// float: rows padded to D + 4 floats, conflict-free.  bf16: the activation dtype as is (half
// the bytes, so that two d = 32 CTAs fit on an SM), rows of D / 8 16-byte chunks with chunk
// c of row i stored at c ^ swz(i), which spreads any 8 consecutive rows' same chunk over the
// eight 16-byte bank groups.
template <int D, typename TIn>
struct BasisSmem {
  static constexpr bool kHalf = sizeof(TIn) == 2;
  static constexpr int kChunks = D / 8;  // 16-byte chunks of a bf16 row
  static size_t bytes(int rQ) {
    return kHalf ? (size_t)rQ * D * D * 2 : sizeof(float) * (size_t)rQ * D * (D + 4);
  }
  __host__ __device__ static constexpr int swz(int i) { return ((i * kChunks) >> 3) & (kChunks - 1); }
};

// OR of `pred` over the `count` threads of named barrier `id` (also a barrier).
__device__ __forceinline__ bool slot_sync_or(int id, int count, bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.or.pred po, %2, %3, pi;\n\tselp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(out)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return out != 0;
}

// Issues  acc (+)= A * Op^T  for A[128 x K] at TMEM column a_hi / a_lo and the N x K
// operand whose K-step-0 descriptors are dh / dl, in 3xTF32 (small terms first).  Each
// further K step of 8 is 2*N*16 bytes further on: a constant added to the descriptor's
// start-address field.  Called by one elected lane of a warp-uniform branch, so the
// descriptors stay in uniform registers.
// ACC_IN: the accumulator already holds a value to add to (the first MMA accumulates).
// OP_LO = false: the operand is exactly representable in tf32 (its residual block is zero,
// as for bf16 activations, whose B and Q are bf16 values), so the A_hi * Op_lo terms, which
// would add exact zeros, are not issued: 8 MMAs per K = 32 product instead of 12.
template <int N, int K, bool ACC_IN = false, bool OP_LO = true>
__device__ __forceinline__ void issue_3xtf32(uint32_t acc, uint32_t a_hi, uint32_t a_lo,
                                             uint64_t dh, uint64_t dl) {
  constexpr uint32_t idesc = tc::idesc_tf32(N);
  constexpr uint64_t step = (2 * N * 16) >> 4;
#pragma unroll
  for (int kk = 0; kk < K / 8; ++kk) {
    tc::mma_tf32_ts(acc, a_lo + kk * 8, dh + kk * step, idesc, (kk > 0 || ACC_IN) ? 1 : 0);
    if constexpr (OP_LO) tc::mma_tf32_ts(acc, a_hi + kk * 8, dl + kk * step, idesc, 1);
  }
#pragma unroll
  for (int kk = 0; kk < K / 8; ++kk) tc::mma_tf32_ts(acc, a_hi + kk * 8, dh + kk * step, idesc, 1);
}

// Tile context: TMEM addresses and the slot's barrier / mbarrier.
struct TileCtx {
  uint32_t my_hi, my_lo, my_acc;     // this thread's lane, per region
  uint32_t t_hi, t_lo, t_acc;        // lane 0 of the tile (MMA operands)
  uint64_t* mbar;
  uint32_t parity;
  uint32_t wait_hint_ns;             // mbar_wait's suspend hint (0: plain polls)
  int bar_id;
  bool mma_warp;                     // warp 0 of the tile: one elected lane issues the MMAs
  bool timed_out;
};

// One product: A (this thread's row `a`, C columns) to TMEM, the MMA chain, result back
// into `out`.  A timeout is agreed on slot-wide: a thread whose own wait expired marks the
// context and carries on; the next slot barrier ORs the marks and every thread of the slot
// returns false from the same call.
struct NoOverlap {
  __device__ __forceinline__ void operator()() const {}
};

// With `acc_init` (this thread's row, N columns) the accumulator starts from it, so `out`
// returns acc_init + A * Op^T: the tensor core does the addition.
// PAIRS: the tf32 residuals of A are formed two at a time (one paired subtraction per two
// columns; bitwise the same values): 2.8 % faster at d = 16, 0.5 % at d = 32, 1.6 % slower
// at d = 64 (register pressure).
// OP_LO: issue the A_hi * Op_lo terms (false when the operand is tf32-exact: issue_3xtf32).
template <int C, int N, int K, bool PAIRS = false, bool OP_LO = true, typename Overlap = NoOverlap>
__device__ __forceinline__ bool tile_product(TileCtx& X, const float (&a)[C], float (&out)[N],
                                             uint64_t dh, uint64_t dl, Overlap&& overlap = Overlap(),
                                             const float (*acc_init)[N] = nullptr) {
  static_assert(C == K && C % 8 == 0, "A width must equal K (a multiple of 8)");
  tc::tmem_st<C>(X.my_hi, a);
  if (acc_init != nullptr) tc::tmem_st<N>(X.my_acc, *acc_init);
#pragma unroll
  for (int k = 0; k < C; k += 8) {
    if constexpr (PAIRS) {
      float r[8];
#pragma unroll
      for (int q = 0; q < 8; q += 2) tc::tf32_residual2(a[k + q], a[k + q + 1], r[q], r[q + 1]);
      tc::tmem_st8(X.my_lo + k, r[0], r[1], r[2], r[3], r[4], r[5], r[6], r[7]);
    } else {
      tc::tmem_st8(X.my_lo + k, tc::tf32_residual(a[k]), tc::tf32_residual(a[k + 1]),
                   tc::tf32_residual(a[k + 2]), tc::tf32_residual(a[k + 3]),
                   tc::tf32_residual(a[k + 4]), tc::tf32_residual(a[k + 5]),
                   tc::tf32_residual(a[k + 6]), tc::tf32_residual(a[k + 7]));
    }
  }
  tc::tmem_wait_st();
  tc::fence_before_sync();
  if (slot_sync_or(X.bar_id, 128, X.timed_out)) {
    X.timed_out = true;
    return false;
  }
  tc::fence_after_sync();
  if (X.mma_warp) {
    if (tc::elect_one()) {
      if (acc_init != nullptr) {
        issue_3xtf32<N, K, true, OP_LO>(X.t_acc, X.t_hi, X.t_lo, dh, dl);
      } else {
        issue_3xtf32<N, K, false, OP_LO>(X.t_acc, X.t_hi, X.t_lo, dh, dl);
      }
      tc::mma_commit(X.mbar);
    }
    __syncwarp();
  }
  overlap();  // independent work while the tensor core runs
  const bool ok = tc::mbar_wait(X.mbar, X.parity, kMaxPolls, X.wait_hint_ns);
  X.parity ^= 1u;
  if (!ok) {
    X.timed_out = true;
#pragma unroll
    for (int j = 0; j < N; ++j) out[j] = 0.f;
    return true;
  }
  tc::fence_after_sync();
  tc::tmem_ld<N>(X.my_acc, out);
  return true;
}

// NORMALIZE_TYPE=2 of the reference (symplectic_iter.py:286-300): divide the row block by
// its largest row abs-sum of Y1 or Y2 when that exceeds 1e3.  The row block is the group's
// warp (min(d, 32) rows), the reference's BY-row tile with BY = min(d, 32); any row scaling
// leaves P = Y1^-1 Y2 and Y1^-1 Y3 unchanged, so 1/m need not be correctly rounded.
// Returns the factor applied.
template <int D>
__device__ __forceinline__ float renormalize_rows(const Group<D>& G, float (&y1)[D], float (&y2)[D]) {
  float p1[4] = {0.f, 0.f, 0.f, 0.f}, p2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int k = 0; k < D; ++k) {
    p1[k & 3] += fabsf(y1[k]);
    p2[k & 3] += fabsf(y2[k]);
  }
  const float r1 = (p1[0] + p1[1]) + (p1[2] + p1[3]);
  const float r2 = (p2[0] + p2[1]) + (p2[2] + p2[3]);
  const float m = rowblock_max<D>(G, fmaxf(r1, r2));
  if (m > kNormThreshold) {
    const float r = recip(m);
#pragma unroll
    for (int k = 0; k < D; ++k) {
      y1[k] *= r;
      y2[k] *= r;
    }
    return r;
  }
  return 1.0f;
}

// Where the sweep's last step puts this thread's row of Y3 = -Y2BR (symplectic_iter.py:
// 241-243): put(j, value) per column, then scale(r) if the last renormalisation divided
// the row block by 1/r.
// kEveryStep: put(j, -(Y2 B)_ij e^{lgB tau} R_inv_j) on every step instead (stage(t, i) having
// published step t's vector for it), and scale(r) at every renormalisation.
struct Y3Discard {  // the caller does not need Y3
  static constexpr bool kEveryStep = false;
  __device__ __forceinline__ void stage(int, int) {}
  __device__ __forceinline__ void put(int, float) {}
  __device__ __forceinline__ void scale(float) {}
};
template <int DU>
struct Y3DotDu {  // contracted with the upstream gradient: acc = (Y3 d_u)_i (fused_lqr.py:185)
  static constexpr bool kEveryStep = false;
  const float* du;
  float acc;
  __device__ __forceinline__ void stage(int, int) {}
  __device__ __forceinline__ void put(int j, float v) { acc = fmaf(v, du[j], acc); }
  __device__ __forceinline__ void scale(float r) { acc *= r; }
};
// An affine action cost r_t^T u_t on every step t (r_traj of solve_traj_actions,
// lin_solver_lqr.py:143-145).  A row i of the sweep is the constraint
// Y1_i . lambda = Y2_i . h + c_i between the costate and the state at the current time;
// eliminating u_t = -R_t^-1 (B_t^T lambda_{t+1} + r_t) from h_{t+1} = A_t h_t + B_t u_t
// transforms Y1, Y2 as the sweep does and adds -(Y2 B_t R_t^-1 r_t)_i to c_i, so that at the
// end Y1 lambda0 = Y2 h0 + c.  The step-0 term alone is the reference's IS_AFFINE y3 = Y3 r0
// (symplectic_iter.py:211-243).  acc holds c_i; rs is the head's du floats of group shared
// memory holding the current step's r (written one step ahead, during the step's last
// product, after every thread of the head has read the previous one).
template <typename TIn, int DU>
struct Y3AffineSteps {
  static constexpr bool kEveryStep = true;
  const TIn* r;  // this head's r_traj [T][DU]; nullptr for a padding head
  float* rs;
  float acc;
  __device__ __forceinline__ void stage(int t, int i) {
    if (i < DU) rs[i] = r != nullptr ? ldf(r + (int64_t)t * DU + i) : 0.f;
  }
  __device__ __forceinline__ void put(int j, float v) { acc = fmaf(v, rs[j], acc); }
  __device__ __forceinline__ void scale(float f) { acc *= f; }
};

// The sweep of symplectic_iter.py:226-300 for this thread's row: (Y1, Y2) from (I, Q_f),
// the three products of each step on the tensor cores, the per-head diagonal scalings and
// the NORMALIZE_TYPE=2 renormalisation (per warp row block, see renormalize_rows) on the
// CUDA cores, and Y3 handed to `y3` on the last step.  Returns false, on every thread of the
// slot alike, after an MMA timeout.
struct NoMark {
  __device__ __forceinline__ void operator()(int) const {}
};
// OP_LO = false: B and Q are tf32-exact (bf16 activations), see issue_3xtf32.
template <int D, int DU, bool OP_LO, typename Y3, typename Mark = NoMark>
__device__ __forceinline__ bool tc_sweep(const Group<D>& G, TileCtx& X, float (&y1)[D],
                                         float (&y2)[D], Y3& y3, const float* ops, float* vec,
                                         float a, float lgA2, float lgQ2, float lgB2, float rinv,
                                         int T, bool every_step, Mark&& mark = Mark()) {
  using V = SweepVec<D, DU>;
  using CF = TcCfg<D, DU>;
  constexpr bool kPairs = D <= 32;
  // K-step-0 descriptors of the three operands (hi and lo blocks).
  const uint32_t o1 = tc::smem_u32(ops + CF::kO1), o2 = tc::smem_u32(ops + CF::kO2),
                 o3 = tc::smem_u32(ops + CF::kO3);
  const uint64_t o1h = tc::smem_desc(o1, DU * 16, 128), o1l = tc::smem_desc(o1 + DU * D * 4, DU * 16, 128);
  const uint64_t o2h = tc::smem_desc(o2, D * 16, 128), o2l = tc::smem_desc(o2 + D * DU * 4, D * 16, 128);
  const uint64_t o3h = tc::smem_desc(o3, D * 16, 128), o3l = tc::smem_desc(o3 + D * D * 4, D * 16, 128);
  const int i = G.i;
  // Per-step column vectors of step s go to vec[(s & 1)]; step s+1's are written while
  // step s's last product runs (they do not depend on the state).  The barrier at the
  // start of the next product orders them before any read.
  auto step_vectors = [&](int s) {
    float* w = vec + (s & 1) * V::kSize;
    const float tau = static_cast<float>(T - s);
    const float at = fmaf(a, exp_scaled(lgA2, tau), 1.0f);
    w[V::kAt + i] = at;
    w[V::kIA + i] = recip(at);
    w[V::kDq + i] = exp_scaled(lgQ2, static_cast<float>(T - 1 - s));
    if (i < DU) {
      const float eb = exp_scaled(lgB2, tau);
      w[V::kS2 + i] = eb * eb * rinv;
      w[V::kEBR + i] = eb * rinv;
    }
    y3.stage(T - 1 - s, i);  // the affine cost of time step T - 1 - s (sweep step s: tau)
  };
  step_vectors(0);
  for (int s = 0; s < T; ++s) {
    mark(s);
    const float* v = vec + (s & 1) * V::kSize;
    const bool last = (s == T - 1);
    const float4* v4 = reinterpret_cast<const float4*>(v);  // 16-byte aligned sections
    // t = Y2 B ; Y3 = -t EBR on the last step ; c = t * S2.  The diagonal scalings below
    // run on fp32 pairs (bitwise the scalar results; 1-3 % faster).
    float t[DU];
    if (!tile_product<D, DU, D, kPairs, OP_LO>(X, y2, t, o1h, o1l)) return false;
    if (Y3::kEveryStep || last) {
#pragma unroll
      for (int j4 = 0; j4 < DU / 4; ++j4) {
        const float4 e = v4[V::kEBR / 4 + j4];
        y3.put(4 * j4 + 0, -t[4 * j4 + 0] * e.x);
        y3.put(4 * j4 + 1, -t[4 * j4 + 1] * e.y);
        y3.put(4 * j4 + 2, -t[4 * j4 + 2] * e.z);
        y3.put(4 * j4 + 3, -t[4 * j4 + 3] * e.w);
      }
    }
#pragma unroll
    for (int j4 = 0; j4 < DU / 4; ++j4) {
      const float4 e = v4[V::kS2 / 4 + j4];
      up2(mul2(pk2(t[4 * j4 + 0], t[4 * j4 + 1]), lo2(e)), t[4 * j4 + 0], t[4 * j4 + 1]);
      up2(mul2(pk2(t[4 * j4 + 2], t[4 * j4 + 3]), hi2(e)), t[4 * j4 + 2], t[4 * j4 + 3]);
    }
    // Y1 = (Y1 + c B^T) / A.  At d = 16 the sum is formed in the accumulator, started from
    // Y1 (one TMEM store instead of d adds: 1 % faster); at d >= 32 the wider store costs more
    // than it saves.
    float u[D];
    constexpr bool kAccY1 = D <= 16;
    if (!tile_product<DU, D, DU, kPairs, OP_LO>(X, t, u, o2h, o2l, NoOverlap(), kAccY1 ? &y1 : nullptr)) return false;
#pragma unroll
    for (int k4 = 0; k4 < D / 4; ++k4) {
      const float4 ia = v4[V::kIA / 4 + k4];
      f2 s0 = pk2(u[4 * k4 + 0], u[4 * k4 + 1]), s1 = pk2(u[4 * k4 + 2], u[4 * k4 + 3]);
      if constexpr (!kAccY1) {
        s0 = add2(pk2(y1[4 * k4 + 0], y1[4 * k4 + 1]), s0);
        s1 = add2(pk2(y1[4 * k4 + 2], y1[4 * k4 + 3]), s1);
      }
      up2(mul2(s0, lo2(ia)), y1[4 * k4 + 0], y1[4 * k4 + 1]);
      up2(mul2(s1, hi2(ia)), y1[4 * k4 + 2], y1[4 * k4 + 3]);
    }
    if (!last) {
      // Y2 = Y2 A + ((Y1 Dq) Q) Dq
#pragma unroll
      for (int k4 = 0; k4 < D / 4; ++k4) {
        const float4 dq = v4[V::kDq / 4 + k4];
        up2(mul2(pk2(y1[4 * k4 + 0], y1[4 * k4 + 1]), lo2(dq)), u[4 * k4 + 0], u[4 * k4 + 1]);
        up2(mul2(pk2(y1[4 * k4 + 2], y1[4 * k4 + 3]), hi2(dq)), u[4 * k4 + 2], u[4 * k4 + 3]);
      }
      if (!tile_product<D, D, D, kPairs, OP_LO>(X, u, u, o3h, o3l, [&] { step_vectors(s + 1); })) return false;
#pragma unroll
      for (int k4 = 0; k4 < D / 4; ++k4) {
        const float4 at = v4[V::kAt / 4 + k4];
        const float4 dq = v4[V::kDq / 4 + k4];
        up2(fma2(pk2(y2[4 * k4 + 0], y2[4 * k4 + 1]), lo2(at), mul2(pk2(u[4 * k4 + 0], u[4 * k4 + 1]), lo2(dq))),
            y2[4 * k4 + 0], y2[4 * k4 + 1]);
        up2(fma2(pk2(y2[4 * k4 + 2], y2[4 * k4 + 3]), hi2(at), mul2(pk2(u[4 * k4 + 2], u[4 * k4 + 3]), hi2(dq))),
            y2[4 * k4 + 2], y2[4 * k4 + 3]);
      }
      // The row-block renormalisation is checked every fourth step and on the last one.  A
      // common row scaling of [Y1 | Y2] (and Y3) leaves P = Y1^-1 Y2 and Y1^-1 Y3 exactly
      // unchanged, so the schedule only bounds the magnitudes (at most four steps of growth
      // past the 1e3 threshold before the scaling: fp32 overflows only at a growth above 1e8
      // per step) and changes results at rounding level; checking every second step instead
      // costs 2.4 % (d = 16) to 5 % (d = 64) of the forward.  With an inverse guard (a fixed
      // ridge added to the final, scaled Y1) the scale matters: every step then, as the
      // reference.
      if ((s & 3) == 3 || every_step) {
        const float r = renormalize_rows<D>(G, y1, y2);
        if constexpr (Y3::kEveryStep) {
          if (r != 1.0f) y3.scale(r);
        }
      }
    } else {
#pragma unroll
      for (int k4 = 0; k4 < D / 4; ++k4) {
        const float4 at = v4[V::kAt / 4 + k4];
        y2[4 * k4 + 0] *= at.x;
        y2[4 * k4 + 1] *= at.y;
        y2[4 * k4 + 2] *= at.z;
        y2[4 * k4 + 3] *= at.w;
      }
      const float r = renormalize_rows<D>(G, y1, y2);
      if (r != 1.0f) y3.scale(r);
    }
  }
  return true;
}

// TTC_FLAG_INV_GUARD: Y1 + 1e-6 I after the sweep, before the solve (INV_GUARD,
// symplectic_iter.py:302-305); this thread holds row i of Y1.
template <int D>
__device__ __forceinline__ void add_inv_guard(float (&y1)[D], int i, int opts) {
  if (opts & TTC_FLAG_INV_GUARD) {
#pragma unroll
    for (int k = 0; k < D; ++k)
      if (k == i) y1[k] += 1e-6f;
  }
}

// This thread's row i of the terminal cost Q_f of problem p: read from Q_f [N*nh, D, D], or,
// when `basis_s` is given, mixed from the rank-rQ basis as the layer does
// (Q_f = sum_r coeff_Qf[r] basis[r], ttc_layer.py:119-123): `qf` is then coeff_Qf [N*nh, rQ],
// basis_s the basis in shared memory (BasisSmem), and the sum is rounded to the activation
// dtype like the einsum it replaces.
template <int D, typename TIn>
__device__ __forceinline__ void load_qf_row(float (&y2)[D], bool valid, const TIn* __restrict__ qf,
                                            const void* basis_s, int rQ, int64_t p, int i) {
  if (!valid) {
#pragma unroll
    for (int k = 0; k < D; ++k) y2[k] = 0.0f;
    return;
  }
  if (basis_s == nullptr) {
    const TIn* row = qf + (p * D + i) * D;
#pragma unroll
    for (int k = 0; k < D; ++k) y2[k] = ldf(row + k);
    return;
  }
#pragma unroll
  for (int k = 0; k < D; ++k) y2[k] = 0.0f;
  const TIn* c = qf + p * rQ;
  using BS = BasisSmem<D, TIn>;
  auto add_rank = [&](int r, float cr) {
    if constexpr (BS::kHalf) {
      const uint4* row = reinterpret_cast<const uint4*>(basis_s) + (r * D + i) * BS::kChunks;
      const int sw = BS::swz(i);
#pragma unroll
      for (int c = 0; c < BS::kChunks; ++c) {
        const uint4 q = row[c ^ sw];
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          y2[8 * c + 2 * h] = fmaf(cr, __uint_as_float(w[h] << 16), y2[8 * c + 2 * h]);
          y2[8 * c + 2 * h + 1] = fmaf(cr, __uint_as_float(w[h] & 0xffff0000u), y2[8 * c + 2 * h + 1]);
        }
      }
    } else {
      const float4* row = reinterpret_cast<const float4*>(basis_s) + (r * D + i) * (D / 4 + 1);
#pragma unroll
      for (int k4 = 0; k4 < D / 4; ++k4) {
        const float4 b = row[k4];
        y2[4 * k4] = fmaf(cr, b.x, y2[4 * k4]);
        y2[4 * k4 + 1] = fmaf(cr, b.y, y2[4 * k4 + 1]);
        y2[4 * k4 + 2] = fmaf(cr, b.z, y2[4 * k4 + 2]);
        y2[4 * k4 + 3] = fmaf(cr, b.w, y2[4 * k4 + 3]);
      }
    }
  };
  if ((rQ & 3) == 0 && (reinterpret_cast<uintptr_t>(c) & (4 * sizeof(TIn) - 1)) == 0) {
    // the head's coefficients four at a time (the ranks still added in order)
#pragma unroll 2
    for (int r4 = 0; r4 < rQ / 4; ++r4) {
      const float4 cc = ld4(c + 4 * r4);
      add_rank(4 * r4, cc.x);
      add_rank(4 * r4 + 1, cc.y);
      add_rank(4 * r4 + 2, cc.z);
      add_rank(4 * r4 + 3, cc.w);
    }
  } else {
    for (int r = 0; r < rQ; ++r) add_rank(r, ldf(c + r));
  }
  if constexpr (sizeof(TIn) == 2) {
#pragma unroll
    for (int k = 0; k < D; ++k) y2[k] = __bfloat162float(__float2bfloat16_rn(y2[k]));
  }
}

// Cooperative copy of a rank-rQ basis [rQ, D, D] (activation dtype, 16-byte aligned) into
// shared memory in the BasisSmem layout, 16 bytes per load and store.
template <int D, typename TIn>
__device__ __forceinline__ void stage_basis(void* basis_s, const TIn* __restrict__ basis, int rQ, int tid,
                                            int nthreads) {
  using BS = BasisSmem<D, TIn>;
  if constexpr (BS::kHalf) {
    const uint4* src = reinterpret_cast<const uint4*>(basis);
    uint4* dst = reinterpret_cast<uint4*>(basis_s);
#pragma unroll 4
    for (int e8 = tid; e8 < rQ * D * D / 8; e8 += nthreads) {
      const int row = e8 / BS::kChunks, c = e8 % BS::kChunks;
      dst[row * BS::kChunks + (c ^ BS::swz(row % D))] = src[e8];
    }
  } else {
    float* dst = static_cast<float*>(basis_s);
#pragma unroll 4
    for (int e4 = tid; e4 < rQ * D * D / 4; e4 += nthreads) {
      const int e = 4 * e4;
      *reinterpret_cast<float4*>(dst + (e / D) * (D + 4) + e % D) = ld4(basis + e);
    }
  }
}

// Staggering of the P co-resident CTAs of an SM (P = TcLaunch::kMinBlocks; used for the two
// CTAs of d = 32 NARROW: 0.6 % on top of their natural drift; at d = 16, three CTAs of one
// tile each, it cost 5 %).  They run the same per-tile sequence, a sweep on the tensor cores
// then a tail without MMAs, and started together they would stay in step, their tails
// coinciding.
// So the a-th CTA to arrive on an SM in a launch (a = 2..P) waits until the first one has
// swept (a - 1) / P of its first tile; CTAs that replace them later inherit the offsets.
// Arrivals are counted per SM in a word tagged with the launch's epoch (no reset between
// launches), and the first CTA posts its progress (epoch, marks passed) in another; the wait
// is bounded (2 ms) and only ever on a CTA resident on the same SM.  Each translation unit
// has its own words.
#ifndef TTC_FWD_STAGGER
#define TTC_FWD_STAGGER 1
#endif
constexpr int kStaggerSMs = 1024;
static __device__ unsigned long long g_tc_arrivals[kStaggerSMs];
static __device__ unsigned long long g_tc_progress[kStaggerSMs];

__device__ __forceinline__ unsigned smid() {
  unsigned r;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(r));
  return r;
}

// This CTA's arrival number on SM `sm` in launch `epoch` (1, 2, ...; 0 if undecided).
__device__ __forceinline__ unsigned stagger_arrival(unsigned sm, unsigned epoch) {
  unsigned long long* w = &g_tc_arrivals[sm % kStaggerSMs];
  unsigned long long old = atomicAdd(w, 0ull);
  for (int it = 0; it < 64; ++it) {
    const unsigned long long nv =
        (old >> 32) == epoch ? old + 1ull : ((static_cast<unsigned long long>(epoch) << 32) | 1ull);
    const unsigned long long seen = atomicCAS(w, old, nv);
    if (seen == old) return static_cast<unsigned>(nv & 0xffffffffull);
    old = seen;
  }
  return 0;
}

// AFF: an affine action cost on every step, r_traj [N, nh, T, DU] (Y3AffineSteps): lambda0
// solves Y1 lambda0 = Y2 h0 + c (one right-hand side), u includes -R_inv r_0, no M.
template <int D, int DU, typename TIn, bool SAVE_M, bool AFF = false, bool NARROW = false>
__global__ void __launch_bounds__(TcLaunch<D, NARROW>::kMaxThreads, TcLaunch<D, NARROW>::kMinBlocks)
lqr_fwd_tc_kernel(const TIn* __restrict__ A_diag, const TIn* __restrict__ Bm,
                  const TIn* __restrict__ Qm, const TIn* __restrict__ Rinv,
                  const TIn* __restrict__ Qf, const TIn* __restrict__ Qbasis, int rQ,
                  const TIn* __restrict__ lgA,
                  const TIn* __restrict__ lgB, const TIn* __restrict__ lgQ,
                  const TIn* __restrict__ H0, int nh, int T, int opts, uint32_t tmem_cols,
                  TIn* __restrict__ u_out, float* __restrict__ lam0_out, float* __restrict__ M_out,
                  int* __restrict__ status, LowRank<TIn> lr, const TIn* __restrict__ r_traj = nullptr,
                  unsigned epoch = 0) {
  static_assert(!(AFF && SAVE_M), "the per-step affine forward saves no M");
  constexpr int kParts = TcLaunch<D, NARROW>::kMinBlocks;
  constexpr bool kStagger = TcLaunch<D, NARROW>::kNarrow && TTC_FWD_STAGGER;
  using CF = TcCfg<D, DU>;
  using L = TcFwdLayout<D, DU, SAVE_M>;
  using V = SweepVec<D, DU>;
  extern __shared__ __align__(128) float smem[];
  float* ops = smem;
  uint64_t* mbars = reinterpret_cast<uint64_t*>(smem + CF::kOps);
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(smem + CF::kOps + 16);
  float* groups = smem + CF::kOps + CF::kHeader;
  void* basis_s = Qbasis != nullptr ? smem + L::basis_offset(blockDim.x / 128) : nullptr;

  const int tid = threadIdx.x;
  const int nslots = blockDim.x / 128;
  const int slot = tid / 128;
  const int lane = tid % 128;
  const Group<D> G(tid);
  const int64_t n = blockIdx.x;

  // The row's operands, split into tf32 hi and residual.  With the layer's low-rank
  // parametrisation B and Q are mixed here from the row's coefficients and the bases.
  const TIn* cBn = lr.cB != nullptr ? lr.cB + n * lr.rB : nullptr;
  const TIn* cQn = lr.cB != nullptr ? lr.cQ + n * rQ : nullptr;
  for (int e = tid; e < D * DU; e += blockDim.x) {
    const int k = e / DU, j = e % DU;
    const float b = cBn != nullptr ? mix_elem<TIn>(cBn, lr.Bb, lr.rB, D * DU, e) : ldf(Bm + n * (D * DU) + e);
    const float hi = tc::tf32_trunc(b), lo = b - hi;
    ops[CF::kO1 + tc::canon(j, k, DU)] = hi;
    ops[CF::kO1 + D * DU + tc::canon(j, k, DU)] = lo;
    ops[CF::kO2 + tc::canon(k, j, D)] = hi;
    ops[CF::kO2 + D * DU + tc::canon(k, j, D)] = lo;
  }
  for (int e = tid; e < D * D; e += blockDim.x) {
    const int j = e / D, k = e % D;
    const float q = cQn != nullptr ? mix_elem<TIn>(cQn, Qbasis, rQ, D * D, e) : ldf(Qm + n * (D * D) + e);
    const float hi = tc::tf32_trunc(q);
    ops[CF::kO3 + tc::canon(k, j, D)] = hi;
    ops[CF::kO3 + D * D + tc::canon(k, j, D)] = q - hi;
  }
  if (tid == 0) {
    for (int s = 0; s < nslots; ++s) tc::mbar_init(&mbars[s], 1);
    tc::mbar_init_fence();
  }
  if (basis_s != nullptr) stage_basis<D, TIn>(basis_s, Qbasis, rQ, tid, blockDim.x);
  if (tid < 32) tc::tmem_alloc(tmem_base_s, tmem_cols);
  tc::fence_smem_to_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  // the a-th CTA of the launch on this SM starts (a - 1) / kParts into the first one's first tile
  unsigned stag_sm = 0, stag_arrival = 0;
  if constexpr (kStagger) {
    if (epoch != 0 && tid == 0) {
      stag_sm = smid() % kStaggerSMs;
      stag_arrival = stagger_arrival(stag_sm, epoch);
      if (stag_arrival >= 2 && stag_arrival <= static_cast<unsigned>(kParts)) {
        const uint64_t t0 = tc::global_ns();
        while (tc::global_ns() - t0 < 2000000ull) {
          const unsigned long long w = atomicAdd(&g_tc_progress[stag_sm], 0ull);
          if ((w >> 32) == epoch && (w & 0xffffffffull) + 1 >= stag_arrival) break;
          __nanosleep(500);
        }
      }
    }
    __syncthreads();
  }

  const uint32_t tbase = *tmem_base_s;
  TileCtx X;
  {
    const uint32_t col = tbase + slot * CF::kSlotCols;
    const uint32_t lane_off = static_cast<uint32_t>(32 * (lane / 32)) << 16;
    X.t_hi = col;
    X.t_lo = col + CF::kMax;
    X.t_acc = col + 2 * CF::kMax;
    X.my_hi = X.t_hi + lane_off;
    X.my_lo = X.t_lo + lane_off;
    X.my_acc = X.t_acc + lane_off;
    X.mbar = &mbars[slot];
    X.parity = 0;
    X.wait_hint_ns = kWaitHintNs<D>;
    X.bar_id = 1 + slot;
    X.mma_warp = (lane < 32);
    X.timed_out = false;
  }
  float* gs = groups + G.g * L::kGroup;
  float* vec = gs;
  float* sh0 = vec + 2 * V::kSize;
  float* slam = sh0 + D;
  float* pbuf = sh0 + 3 * D;

  const int i = G.i;
  const int tiles = (nh * D + 127) / 128;
  int flags = 0;
  for (int tile = slot; tile < tiles; tile += nslots) {
    const int h = tile * CF::kHeadsPerTile + lane / D;
    const bool valid = h < nh;
    const int64_t p = n * nh + h;
    float a = 0.f, lgA2 = 0.f, lgQ2 = 0.f, lgB2 = 0.f, rinv = 1.f, h0 = 0.f;
    if (valid) {
      a = ldf(A_diag + p * D + i);
      lgA2 = ldf(lgA + p) * kLog2e;
      lgQ2 = ldf(lgQ + p * D + i) * kLog2e;
      h0 = ldf(H0 + p * D + i);
      if (i < DU) {
        lgB2 = ldf(lgB + p * DU + i) * kLog2e;
        rinv = ldf(Rinv + p * DU + i);
      }
    }
    sh0[i] = h0;
    float y1[D], y2[D];
#pragma unroll
    for (int k = 0; k < D; ++k) y1[k] = (k == i) ? 1.0f : 0.0f;
    load_qf_row<D, TIn>(y2, valid, Qf, basis_s, rQ, p, i);
    using Y3T = std::conditional_t<AFF, Y3AffineSteps<TIn, DU>, Y3Discard>;
    Y3T y3;  // without AFF, M is formed from P below instead of from Y3
    if constexpr (AFF) y3 = Y3T{valid ? r_traj + p * T * DU : nullptr, sh0 + 2 * D, 0.f};
    const bool marker = kStagger && stag_arrival == 1 && tile == 0 && tid == 0;
    const bool swept = tc_sweep<D, DU, (sizeof(TIn) != 2)>(G, X, y1, y2, y3, ops, vec, a, lgA2, lgQ2, lgB2, rinv, T,
                                       (opts & TTC_FLAG_INV_GUARD) != 0, [&](int s) {
                                         if (marker) {
#pragma unroll
                                           for (int m = 1; m < kParts; ++m)
                                             if (s == m * T / kParts)
                                               atomicExch(&g_tc_progress[stag_sm],
                                                          (static_cast<unsigned long long>(epoch) << 32) | m);
                                         }
                                       });
    // Uniform over the slot: a late timeout on the last product surfaces here too.
    if (slot_sync_or(X.bar_id, 128, X.timed_out || !swept)) {
      flags |= TTC_STATUS_MMA_TIMEOUT;
      break;
    }
    add_inv_guard<D>(y1, i, opts);
    bool bad = false;
#pragma unroll
    for (int k = 0; k < D; ++k) bad |= unstable(y1[k]) | unstable(y2[k]);
    if (bad && valid) flags |= TTC_STATUS_FWD_UNSTABLE;
    float piv, lam0 = 0.f;
    int pc;
    bool lbad;
    if constexpr (AFF) {
      // Y1 lambda0 = Y2 h0 + c: one right-hand side
      float rhs[1] = {y3.acc};
#pragma unroll
      for (int c = 0; c < D; ++c) rhs[0] = fmaf(y2[c], sh0[c], rhs[0]);
      pc = gauss_jordan_group<D, 1>(G, y1, rhs, piv, pbuf);
      lbad = unstable(piv);
      lam0 = rhs[0] * recip(piv);
      lbad |= unstable(lam0);
    } else {
      // P = Y1^-1 Y2 (fused_lqr.py:104-105): this thread ends up with row pc of P in y2.
      pc = gauss_jordan_group<D, D>(G, y1, y2, piv, pbuf);
      lbad = unstable(piv);
      const float rpiv = recip(piv);
#pragma unroll
      for (int c = 0; c < D; ++c) {
        y2[c] *= rpiv;
        lbad |= unstable(y2[c]);
        lam0 = fmaf(y2[c], sh0[c], lam0);  // lambda0 = P h0 (symplectic_iter.py:437)
      }
    }
    if (lbad && valid) flags |= TTC_STATUS_LU_UNSTABLE;
    if (valid && lam0_out != nullptr) lam0_out[p * D + pc] = lam0;
    // The last sweep step had tau = 1: its vectors hold 1/A_1 and exp(lgB) R_inv.
    const float* v1 = vec + ((T - 1) & 1) * V::kSize;
    slam[pc] = lam0 * v1[V::kIA + pc];  // lambda1 = lambda0 / A_1 (:472-477)
    if constexpr (SAVE_M) {
      // M = Y1^-1 Y3 with Y3 = -Y2_{T-1} B_1 R_inv and Y2 = Y2_{T-1} A_1 on the last step,
      // so M = -(P A_1^-1) B diag(exp(lgB) R_inv): one more tensor-core product.
      using CF2 = TcCfg<D, DU>;
      const uint32_t o1 = tc::smem_u32(ops + CF2::kO1);
      float w[D], m[DU];
#pragma unroll
      for (int k = 0; k < D; ++k) w[k] = y2[k] * v1[V::kIA + k];
      if (!tile_product<D, DU, D, false, (sizeof(TIn) != 2)>(X, w, m, tc::smem_desc(o1, DU * 16, 128),
                                  tc::smem_desc(o1 + DU * D * 4, DU * 16, 128)) ||
          slot_sync_or(X.bar_id, 128, X.timed_out)) {
        flags |= TTC_STATUS_MMA_TIMEOUT;
        break;
      }
      if (valid) {
        float4* mrow = reinterpret_cast<float4*>(M_out + (p * D + pc) * DU);
#pragma unroll
        for (int j4 = 0; j4 < DU / 4; ++j4)
          mrow[j4] = make_float4(-m[4 * j4] * v1[V::kEBR + 4 * j4], -m[4 * j4 + 1] * v1[V::kEBR + 4 * j4 + 1],
                                 -m[4 * j4 + 2] * v1[V::kEBR + 4 * j4 + 2], -m[4 * j4 + 3] * v1[V::kEBR + 4 * j4 + 3]);
      }
    }
    G.sync();
    if (valid && i < DU) {
      // u = -R_inv * (B diag(e^lgB))^T lambda1   (symplectic_iter.py:488-517)
      float acc = 0.f;
      for (int k = 0; k < D; ++k) {
        const int idx = tc::canon(k, i, D);  // B[k][i] from the hi/lo operand O2
        acc = fmaf(ops[CF::kO2 + idx] + ops[CF::kO2 + D * DU + idx], slam[k], acc);
      }
      float u = -(acc * exp_scaled(lgB2, 1.0f)) * rinv;
      if constexpr (AFF) u = fmaf(ldf(r_traj + p * T * DU + i), -rinv, u);  // u_0 -= R_inv r_0
      if (isnan(u)) flags |= TTC_STATUS_U_NAN;
      stf(u_out + p * DU + i, u);
    }
    G.sync();
  }
  if (flags) atomicOr(status, flags);
  tc::fence_before_sync();
  __syncthreads();
  if (tid < 32) tc::tmem_dealloc(tbase, tmem_cols);
}

// --------------------------------------------------------------------------------------
// Backward with the sweep recomputed on the tensor cores (no saved state beyond the
// forward's inputs): per tile, the sweep of the forward, then Y1 [lambda0 | d_p] =
// [Y2 h0 | Y3 d_u] in registers (fused_lqr.py:104-105,185-187), then the forward-in-time
// adjoint per head on the CUDA cores.  grad_B / grad_Q of the row are summed over the
// heads of a slot in head order and over slots in slot order: deterministic.
// --------------------------------------------------------------------------------------
template <int D, int DU>
struct TcBwdLayout {
  using CF = TcCfg<D, DU>;
  static constexpr int kPb = GjRow<D, 2>::kSize;
  static constexpr int kGroup =
      round4(2 * SweepVec<D, DU>::kSize + AdjLayout<D, DU>::kSize + 4 * D + 4 + kPb);
  static constexpr int kAcc = D * DU + D * D;  // per slot
  static constexpr int kBp = round4(D * (DU + 1));
  static constexpr int kQp = round4(D * (D + 1));
  static constexpr int kFixed = CF::kOps + CF::kHeader + kBp + kQp;
  static constexpr int kSlot = kAcc + CF::kHeadsPerTile * kGroup;
  static size_t bytes(int slots) { return sizeof(float) * (size_t)(kFixed + slots * kSlot); }
};

template <int D, int DU, typename TIn>
__global__ void __launch_bounds__(TcLaunch<D>::kMaxThreads, TcLaunch<D>::kMinBlocks)
lqr_bwd_tc_kernel(const TIn* __restrict__ A_diag, const TIn* __restrict__ Bm,
                  const TIn* __restrict__ Qm, const TIn* __restrict__ Rinv,
                  const TIn* __restrict__ Qf, const TIn* __restrict__ lgA,
                  const TIn* __restrict__ lgB, const TIn* __restrict__ lgQ,
                  const TIn* __restrict__ H0, const TIn* __restrict__ dU, int nh, int T, int opts,
                  uint32_t tmem_cols, TIn* __restrict__ gA_out, TIn* __restrict__ gB_out,
                  TIn* __restrict__ gQ_out, TIn* __restrict__ gR_out, TIn* __restrict__ gQf_out,
                  TIn* __restrict__ glgA_out, TIn* __restrict__ glgB_out,
                  TIn* __restrict__ glgQ_out, TIn* __restrict__ gh0_out, int* __restrict__ status) {
  using CF = TcCfg<D, DU>;
  using L = TcBwdLayout<D, DU>;
  extern __shared__ __align__(128) float smem[];
  float* ops = smem;
  uint64_t* mbars = reinterpret_cast<uint64_t*>(smem + CF::kOps);
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(smem + CF::kOps + 16);
  float* sBp = smem + CF::kOps + CF::kHeader;  // [D][DU+1]
  float* sQp = sBp + L::kBp;                   // [D][D+1]
  float* slots_base = smem + L::kFixed;

  const int tid = threadIdx.x;
  const int nslots = blockDim.x / 128;
  const int slot = tid / 128;
  const int lane = tid % 128;
  const Group<D> G(tid);
  const int64_t n = blockIdx.x;

  float* accB = slots_base + slot * L::kSlot;  // [DU][D] transposed, per slot
  float* accQ = accB + D * DU;                 // [D][D]
  float* gs = accB + L::kAcc + (lane / D) * L::kGroup;
  float* vec = gs;
  float* adj = vec + 2 * SweepVec<D, DU>::kSize;
  float* sh0 = adj + AdjLayout<D, DU>::kSize;
  float* sdu = sh0 + D;
  float* sx = sdu + D;
  float* sdp = sx + D;
  float* red = sdp + D;
  float* pbuf = red + 4;

  bool sym_local = true;
  for (int e = tid; e < D * DU; e += blockDim.x) {
    const int k = e / DU, j = e % DU;
    const float b = ldf(Bm + n * (D * DU) + e);
    const float hi = tc::tf32_trunc(b), lo = b - hi;
    ops[CF::kO1 + tc::canon(j, k, DU)] = hi;
    ops[CF::kO1 + D * DU + tc::canon(j, k, DU)] = lo;
    ops[CF::kO2 + tc::canon(k, j, D)] = hi;
    ops[CF::kO2 + D * DU + tc::canon(k, j, D)] = lo;
    sBp[k * (DU + 1) + j] = b;
  }
  for (int e = tid; e < D * D; e += blockDim.x) {
    const int j = e / D, k = e % D;
    const float q = ldf(Qm + n * (D * D) + e);
    const float hi = tc::tf32_trunc(q);
    ops[CF::kO3 + tc::canon(k, j, D)] = hi;
    ops[CF::kO3 + D * D + tc::canon(k, j, D)] = q - hi;
    sQp[j * (D + 1) + k] = q;
    sym_local &= (q == ldf(Qm + n * (D * D) + k * D + j));
  }
  for (int e = lane; e < L::kAcc; e += 128) accB[e] = 0.0f;  // accB and accQ are contiguous
  if (tid == 0) {
    for (int s = 0; s < nslots; ++s) tc::mbar_init(&mbars[s], 1);
    tc::mbar_init_fence();
  }
  if (tid < 32) tc::tmem_alloc(tmem_base_s, tmem_cols);
  tc::fence_smem_to_async();
  tc::fence_before_sync();
  const bool sym = __syncthreads_and(sym_local);
  tc::fence_after_sync();

  const uint32_t tbase = *tmem_base_s;
  TileCtx X;
  {
    const uint32_t col = tbase + slot * CF::kSlotCols;
    const uint32_t lane_off = static_cast<uint32_t>(32 * (lane / 32)) << 16;
    X.t_hi = col;
    X.t_lo = col + CF::kMax;
    X.t_acc = col + 2 * CF::kMax;
    X.my_hi = X.t_hi + lane_off;
    X.my_lo = X.t_lo + lane_off;
    X.my_acc = X.t_acc + lane_off;
    X.mbar = &mbars[slot];
    X.parity = 0;
    X.wait_hint_ns = kWaitHintNs<D>;
    X.bar_id = 1 + slot;
    X.mma_warp = (lane < 32);
    X.timed_out = false;
  }

  const int i = G.i;
  const int hg = lane / D;  // head within the tile
  const int tiles = (nh * D + 127) / 128;
  int flags = 0;
  for (int tile = slot; tile < tiles; tile += nslots) {
    const int h = tile * CF::kHeadsPerTile + hg;
    const bool valid = h < nh;
    const int64_t p = n * nh + h;
    float a = 0.f, lgA2 = 0.f, lgQ2 = 0.f, lgB2 = 0.f, rinv = 1.f, h0i = 0.f, dUi = 0.f;
    if (valid) {
      a = ldf(A_diag + p * D + i);
      lgA2 = ldf(lgA + p) * kLog2e;
      lgQ2 = ldf(lgQ + p * D + i) * kLog2e;
      h0i = ldf(H0 + p * D + i);
      if (i < DU) {
        lgB2 = ldf(lgB + p * DU + i) * kLog2e;
        rinv = ldf(Rinv + p * DU + i);
        dUi = ldf(dU + p * DU + i);
      }
    }
    sh0[i] = h0i;
    if (i < DU) sdu[i] = dUi;
    float y1[D], y2[D];
    const TIn* qf = Qf + (p * D + i) * D;
#pragma unroll
    for (int k = 0; k < D; ++k) {
      y1[k] = (k == i) ? 1.0f : 0.0f;
      y2[k] = valid ? ldf(qf + k) : 0.0f;
    }
    // sh0 / sdu are read after the sweep's first slot barrier: visible by then.
    Y3DotDu<DU> y3{sdu, 0.0f};
    const bool swept = tc_sweep<D, DU, (sizeof(TIn) != 2)>(G, X, y1, y2, y3, ops, vec, a, lgA2, lgQ2, lgB2, rinv, T,
                                              (opts & TTC_FLAG_INV_GUARD) != 0);
    if (slot_sync_or(X.bar_id, 128, X.timed_out || !swept)) {
      flags |= TTC_STATUS_MMA_TIMEOUT;
      break;
    }
    add_inv_guard<D>(y1, i, opts);
    float rhs[2] = {0.0f, y3.acc};
#pragma unroll
    for (int j = 0; j < D; ++j) rhs[0] = fmaf(y2[j], sh0[j], rhs[0]);
    float piv;
    const int pc = gauss_jordan_group<D, 2>(G, y1, rhs, piv, pbuf);
    const float rp = recip(piv);
    sx[pc] = rhs[0] * rp;   // lambda0 = P h0        (symplectic_iter.py:437)
    sdp[pc] = rhs[1] * rp;  // d_p = Y1^-1 (Y3 d_u)  (fused_lqr.py:185-187)
    G.sync();
    const float lam = sx[i], dlam = sdp[i];
    float gB[DU], gQ[D];
    const bool bad = adjoint_head<D, DU, TIn, false>(G, valid, p, T, a, lgA2, lgQ2, lgB2, rinv, dUi, h0i,
                                              lam, dlam, sBp, sQp, sym, adj, red, gB, gQ, gA_out,
                                              gR_out, gQf_out, glgA_out, glgB_out, glgQ_out,
                                              gh0_out);
    if (bad && valid) flags |= TTC_STATUS_BWD_UNSTABLE;
    // The slot's heads add into the slot accumulator one after the other.
    for (int g = 0; g < CF::kHeadsPerTile; ++g) {
      if (g == hg && valid) {
#pragma unroll
        for (int j = 0; j < DU; ++j) accB[j * D + i] += gB[j];
#pragma unroll
        for (int k = 0; k < D; ++k) accQ[k * D + i] += gQ[k];
      }
      tc::named_sync(X.bar_id, 128);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  // grad_B / grad_Q of the row: the slots' accumulators in slot order.
  bool bad = false;
  for (int e = tid; e < D * DU; e += blockDim.x) {
    const int r = e / DU, c = e % DU;
    float s = 0.f;
    for (int sl = 0; sl < nslots; ++sl) s += slots_base[sl * L::kSlot + c * D + r];
    bad |= unstable(s);
    stf(gB_out + n * (D * DU) + e, s);
  }
  for (int e = tid; e < D * D; e += blockDim.x) {
    const int r = e / D, c = e % D;
    float s = 0.f;
    for (int sl = 0; sl < nslots; ++sl) s += slots_base[sl * L::kSlot + D * DU + c * D + r];
    bad |= unstable(s);
    stf(gQ_out + n * (D * D) + e, s);
  }
  if (bad) flags |= TTC_STATUS_BWD_UNSTABLE;
  if (flags) atomicOr(status, flags);
  if (tid < 32) tc::tmem_dealloc(tbase, tmem_cols);
}

}  // namespace ttc
