// Thin inline-PTX wrappers for sm_100a: mbarriers, TMA tile loads (no multicast),
// tcgen05 tensor memory, MMA and loads.  Every wait is bounded by a wall-clock
// limit (the %globaltimer register) and by an abort word, so a kernel that loses
// a partner returns with an error status instead of spinning.
#pragma once

#include <cstdint>
#include <cuda.h>

namespace ungx
{
namespace ptx
{

__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
   return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer()
{
   uint64_t t;
   asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
   return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
   asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
   asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
   asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes)
{
   asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
   uint32_t ok;
   asm volatile("{\n\t.reg .pred p;\n\t"
                "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                "selp.u32 %0, 1, 0, p;\n\t}"
                : "=r"(ok)
                : "r"(smem_u32(bar)), "r"(parity)
                : "memory");
   return ok != 0;
}

// Same test, but the thread may be suspended by the hardware for up to `hint_ns`
// while the phase is incomplete (it resumes as soon as the phase completes), so a
// waiting thread neither spins nor takes issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t hint_ns)
{
   uint32_t ok;
   asm volatile("{\n\t.reg .pred p;\n\t"
                "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
                "selp.u32 %0, 1, 0, p;\n\t}"
                : "=r"(ok)
                : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
                : "memory");
   return ok != 0;
}

// Bounded wait for the phase with the given parity.  Returns false when the
// deadline passed or another thread raised the abort word (both checked each time
// the thread wakes, at least every 20 us).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_word,
                                          uint64_t timeout_ns)
{
   if (mbar_try_wait(bar, parity))
      return true;
   const uint64_t start = globaltimer();
   for (;;)
   {
      if (mbar_try_wait_sleep(bar, parity, 20000u))
         return true;
      if (abort_word && *abort_word)
         return false;
      if (globaltimer() - start > timeout_ns)
         return false;
   }
}

// ---------------------------------------------------------------- TMA
// 2-D tiled bulk tensor load, global -> this CTA's shared memory, completion
// counted in bytes on `bar`.  c0 is the inner (column) coordinate.
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map, uint64_t *bar, int32_t c0,
                                            int32_t c1)
{
   asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
                "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
                : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map)
{
   asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols)
{
   asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                "r"(ncols)
                : "memory");
}

__device__ __forceinline__ void tmem_relinquish()
{
   asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
   asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16 (fp16 operands, fp32 accumulator),
// one CTA.  A occupies TMEM lanes 0..127 (row = lane), two fp16 of K per 32-bit
// column: one K=16 step reads 8 columns from a_tmem.  accumulate = 0 overwrites D.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate)
{
   asm volatile("{\n\t.reg .pred p;\n\t"
                "setp.ne.b32 p, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
                "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
                : "memory");
}

// Copy 128 rows x 256 bits (16 fp16 of K) from shared memory, described by a matrix
// descriptor, into TMEM lanes 0..127 at columns [taddr, taddr + 8).  Ordered before
// the tcgen05.mma this thread issues next; a later copy into the same columns must
// wait for the MMAs that read them (tcgen05.commit + mbarrier).
__device__ __forceinline__ void tmem_cp_128x256b(uint32_t taddr, uint64_t sdesc)
{
   asm volatile("tcgen05.cp.cta_group::1.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Arrive once on `bar` when every tcgen05 op this thread issued so far completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar)
{
   asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                    smem_u32(bar))
                : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// TMEM lane (base lane + t), columns [col, col+32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32])
{
   asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                  "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
                  "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
                  "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
                  "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                : "r"(taddr)
                : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand in the canonical
// 128-byte-swizzle layout: rows of 128 B (64 fp16), 8-row atoms of 1024 B stacked
// contiguously (what a TMA load with SWIZZLE_128B and a 128-byte inner box writes).
// Fields: start address >> 4 [0,14), leading byte offset >> 4 [16,30) (unused for
// swizzled K-major, set to 1), stride byte offset >> 4 [32,46) = 1024 B between
// 8-row atoms, version 1 [46,48), layout SWIZZLE_128B = 2 [61,64).
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t saddr)
{
   uint64_t d = 0;
   d |= uint64_t((saddr >> 4) & 0x3FFFu);
   d |= uint64_t(1) << 16;
   d |= uint64_t(1024 >> 4) << 32;
   d |= uint64_t(1) << 46;
   d |= uint64_t(2) << 61;
   return d;
}

// Instruction descriptor, kind::f16 with fp16 A and B, fp32 accumulator, both
// operands K-major: c_format F32 = 1 at [4,6), a/b format F16 = 0 at [7,10) /
// [10,13), N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t M, uint32_t N)
{
   return (1u << 4) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

} // namespace ptx
} // namespace ungx
