// sm_100a tensor-core primitives (tcgen05, TMEM, mbarrier) used by the LQR sweep.
//
// Operand conventions (PTX ISA, tcgen05.mma kind::tf32, cta_group::1):
//   D[M x N] (+)= A[M x K] * B[N x K]^T,  M = 128 TMEM lanes, K = 8 per instruction.
//   A lives in TMEM (K consecutive 32-bit columns per lane), B in shared memory in the
//   canonical K-major layout without swizzle: 8-row x 16-byte core matrices, the two
//   16-byte K chunks of one instruction LBO bytes apart, consecutive 8-row groups SBO
//   bytes apart.  tf32 operands are read from 32-bit containers with the low 13 mantissa
//   bits ignored, so fp32 values can be handed over unconverted.
#pragma once

#include <stdint.h>

namespace ttc {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// x - (x with the low 13 mantissa bits cleared): the part a tf32 operand drops.  With
// hi = x (read as tf32 by the MMA) and lo = tf32_residual(x), hi + lo == x exactly.
__device__ __forceinline__ float tf32_residual(float x) {
  return x - __uint_as_float(__float_as_uint(x) & 0xffffe000u);
}
// Two residuals with one paired subtraction: (x, y) - ((x, y) & mask).
__device__ __forceinline__ void tf32_residual2(float x, float y, float& rx, float& ry) {
  asm("{\n\t.reg .b64 p, m;\n\tmov.b64 p, {%2, %3};\n\t"
      "and.b64 m, p, 0xffffe000ffffe000;\n\tsub.rn.f32x2 p, p, m;\n\t"
      "mov.b64 {%0, %1}, p;\n\t}"
      : "=f"(rx), "=f"(ry)
      : "f"(x), "f"(y));
}
__device__ __forceinline__ float tf32_trunc(float x) {
  return __uint_as_float(__float_as_uint(x) & 0xffffe000u);
}

// Shared-memory matrix descriptor: start, leading (K) and stride (MN) byte offsets,
// version 1 (sm_100), no swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((addr >> 4) & 0x3fffu) |
         (static_cast<uint64_t>((lbo >> 4) & 0x3fffu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3fffu) << 32) | (static_cast<uint64_t>(1) << 46);
}

// Instruction descriptor: D f32, A and B tf32, both K-major, M = 128, N.
__host__ __device__ constexpr uint32_t idesc_tf32(int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(128 >> 4) << 24);
}

// Canonical K-major, no-swizzle float index of element (n, k) of an N x K operand.
__host__ __device__ constexpr int canon(int n, int k, int N) { return ((k >> 2) * N + n) * 4 + (k & 3); }

__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, q;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(mbar))
               : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Generic-proxy shared-memory writes -> visible to the tensor core's (async proxy) reads.
__device__ __forceinline__ void fence_smem_to_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* mbar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(mbar)), "r"(count));
}
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Polls phase `parity` of `mbar` at most `max_polls` times; false if it never completed.
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits for phase `parity` of the mbarrier; false if it did not complete in time.
// hint_ns == 0: at most max_polls polls of try_wait.  hint_ns > 0: try_wait with that
// suspend-time hint, so the thread sleeps until the phase completes (or the hint elapses)
// instead of re-issuing polls that take issue slots from the other warps on the SM; bounded
// by one second of %globaltimer.
__device__ __forceinline__ bool mbar_wait(uint64_t* mbar, uint32_t parity, uint32_t max_polls,
                                          uint32_t hint_ns = 0) {
  uint32_t done = 0;
  if (hint_ns > 0) {
    const uint64_t t0 = global_ns();
    while (true) {
      asm volatile(
          "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
          "selp.u32 %0, 1, 0, p;\n\t}"
          : "=r"(done)
          : "r"(smem_u32(mbar)), "r"(parity), "r"(hint_ns)
          : "memory");
      if (done) return true;
      if (global_ns() - t0 > 1000000000ull) return false;
    }
  }
  for (uint32_t it = 0; it < max_polls; ++it) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(mbar)), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// TMEM allocation by one whole warp; the base address is written to *dst (shared).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols)
               : "memory");
}

// 32 lanes x C 32-bit columns between registers and TMEM (warp w of 4 owns lanes 32w..).
template <int C>
__device__ __forceinline__ void tmem_st(uint32_t taddr, const float (&v)[C]);
template <>
__device__ __forceinline__ void tmem_st<16>(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]),
      "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15])
      : "memory");
}
template <>
__device__ __forceinline__ void tmem_st<32>(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]),
      "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]),
      "f"(v[17]), "f"(v[18]), "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]),
      "f"(v[25]), "f"(v[26]), "f"(v[27]), "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
}

template <>
__device__ __forceinline__ void tmem_st<64>(uint32_t taddr, const float (&v)[64]) {
  tmem_st<32>(taddr, *reinterpret_cast<const float(*)[32]>(&v[0]));
  tmem_st<32>(taddr + 32, *reinterpret_cast<const float(*)[32]>(&v[32]));
}

// 8 consecutive columns.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, float v0, float v1, float v2, float v3,
                                         float v4, float v5, float v6, float v7) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
               "f"(v0), "f"(v1), "f"(v2), "f"(v3), "f"(v4), "f"(v5), "f"(v6), "f"(v7)
               : "memory");
}

template <int C>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float (&v)[C]);
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
template <>
__device__ __forceinline__ void tmem_ld<32>(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
template <>
__device__ __forceinline__ void tmem_ld<64>(uint32_t taddr, float (&v)[64]) {
  tmem_ld<32>(taddr, *reinterpret_cast<float(*)[32]>(&v[0]));
  tmem_ld<32>(taddr + 32, *reinterpret_cast<float(*)[32]>(&v[32]));
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// True on exactly one lane of the (converged) warp.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 r;\n\telect.sync r|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// Named barrier over `count` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

}  // namespace tc
}  // namespace ttc
