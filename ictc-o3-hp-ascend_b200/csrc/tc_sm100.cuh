// Blackwell (sm_100a) tensor-core toolkit: tcgen05 MMA with TMEM accumulators,
// shared-memory matrix descriptors, mbarrier waits with a time limit, and the
// 3xTF32 operand split used for FP32-accurate products on the tensor cores.
//
// Operand tiles are K-major with the 128-byte swizzle: a tile of `rows` rows is
// stored as K-atoms of [rows][128 B] (32 fp32 values of K per row), atoms back
// to back, every atom 1024-byte aligned.  Inside an atom the 16-byte chunk c of
// row r sits at chunk position c ^ (r % 8).  One tf32 MMA consumes K = 8 (32 B
// of a row); its descriptor starts 32 B further into the atom per K step.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace ictc {
namespace tc {

constexpr uint32_t kAtomBytes = 128;       // one row of one K-atom
constexpr uint32_t kAtomK = 32;            // fp32 values of K per atom row

__host__ __device__ __forceinline__ uint32_t sw128_offset(uint32_t rows, uint32_t r, uint32_t k) {
  const uint32_t atom = k / kAtomK, kk = k % kAtomK;
  return atom * rows * kAtomBytes + r * kAtomBytes + ((((kk >> 2) ^ (r & 7u)) << 4)) + ((kk & 3u) << 2);
}

// Byte offset of the 16-byte chunk `chunk` (0..7) of row r inside one atom.
__host__ __device__ __forceinline__ uint32_t sw128_chunk(uint32_t r, uint32_t chunk) {
  return r * kAtomBytes + (((chunk ^ (r & 7u)) & 7u) << 4);
}

// Round to the nearest TF32 value, ties away from zero (the 3xTF32 "big" part).
__host__ __device__ __forceinline__ uint32_t tf32_round_bits(uint32_t bits) {
  return (bits + 0x1000u) & 0xFFFFE000u;
}

// Instruction descriptor of tcgen05.mma kind::tf32: D fp32, A and B tf32, both K-major.
__host__ __device__ constexpr uint32_t idesc_tf32(uint32_t m, uint32_t n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024u >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ float tf32_hi(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// D[tmem] (+)= A[smem] * B[smem]^T, M = 128, issued by one thread.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

// 3xTF32 product step: A_hi B_hi + A_hi B_lo + A_lo B_hi.
__device__ __forceinline__ void mma_tf32x3(uint32_t d_tmem, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi,
                                           uint32_t b_lo, uint32_t idesc, uint32_t acc) {
  mma_tf32(d_tmem, sw128_desc(a_hi), sw128_desc(b_hi), idesc, acc);
  mma_tf32(d_tmem, sw128_desc(a_hi), sw128_desc(b_lo), idesc, 1u);
  mma_tf32(d_tmem, sw128_desc(a_lo), sw128_desc(b_hi), idesc, 1u);
}

// D[tmem] (+)= A[tmem] * B[smem]^T: A's rows are the TMEM lanes, one fp32 K value per column.
__device__ __forceinline__ void mma_tf32_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}

// 3xTF32 step with A in TMEM (hi and lo column blocks) and B in shared memory.
__device__ __forceinline__ void mma_tf32x3_ta(uint32_t d_tmem, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi,
                                              uint32_t b_lo, uint32_t idesc, uint32_t acc) {
  mma_tf32_ta(d_tmem, a_hi, sw128_desc(b_hi), idesc, acc);
  mma_tf32_ta(d_tmem, a_hi, sw128_desc(b_lo), idesc, 1u);
  mma_tf32_ta(d_tmem, a_lo, sw128_desc(b_hi), idesc, 1u);
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Blocking probe: the thread is suspended in hardware until the phase completes or
// a short system-defined time passes (then it returns false).
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0u;
}

// Wait for the phase with the given parity to complete; false after `limit_ns`
// nanoseconds (or an absolute probe cap), so a lost arrival cannot hang the GPU.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t start = global_ns();
  for (uint32_t spin = 1; spin < (1u << 28); ++spin) {
    if (mbar_try(bar, parity)) return true;
    if ((spin & 63u) == 0u && global_ns() - start > limit_ns) return false;
  }
  return false;
}

// As mbar_wait, but also gives up as soon as `*abort` is non-zero (another thread
// of the CTA timed out), so one lost arrival ends the whole CTA quickly.
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t* bar, uint32_t parity, uint64_t limit_ns,
                                                   volatile int* abort) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t start = global_ns();
  for (uint32_t spin = 1; spin < (1u << 28); ++spin) {
    if (mbar_try(bar, parity)) return true;
    if ((spin & 15u) == 0u) {
      if (*abort) return false;
      if (global_ns() - start > limit_ns) {
        *abort = 1;
        return false;
      }
    }
  }
  *abort = 1;
  return false;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One arrival that also announces `bytes` of bulk-copy data the phase must wait for.
__device__ __forceinline__ void mbar_arrive_expect(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Bulk copy global -> shared (16-byte aligned, size a multiple of 16), completing on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Barrier among `count` threads (a multiple of 32) of the CTA, id 1..15.
__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Barrier among `count` threads that also ANDs `pred` over them (uniform result).
__device__ __forceinline__ bool named_barrier_all(uint32_t id, uint32_t count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return r != 0u;
}

// 8 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_load8(uint32_t taddr, float* v) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_store8(uint32_t taddr, const float* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
               "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
               "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
               "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
               : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// TMEM allocation (whole warp).  `slot` receives the base address.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t columns) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(columns)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(columns) : "memory");
}

// 16 consecutive fp32 columns of this thread's TMEM lane (warp w reads lanes 32w..32w+31).
__device__ __forceinline__ void tmem_load16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// tcgen05.st without waiting; tmem_store_wait() completes every store of the thread.
__device__ __forceinline__ void tmem_store16_async(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void tmem_store_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_store16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

}  // namespace tc
}  // namespace ictc
