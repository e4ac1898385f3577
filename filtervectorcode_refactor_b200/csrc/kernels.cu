// Device code of the B200 cross-edge builder (sm_100a).
//
//   colsum / scale /    resident operand build (a4): column sums and ranges, the mean
//   center              and a power-of-two scale s, then fp16(s * (x - mean)) padded to
//                       a multiple of 16 columns and fp32 norms of the centred rows.
//   tc_kernel           the hot path.  Persistent CTAs pull source-centric work items
//                       (<=128 rows of one source group x all its LNG target groups).
//                       TMA stages fp16 operand chunks (64 columns, 128-byte rows)
//                       through a shared-memory ring; one thread copies the item's
//                       source rows into TMEM (tcgen05.cp) and issues tcgen05.mma
//                       kind::f16 with A in TMEM and the target tile (<= 192 rows) in
//                       shared memory into two 192-column TMEM accumulators; twelve
//                       epilogue warps read TMEM rows (thread = source row), form the
//                       keys ||x||^2 - 2 q.x and keep a sorted register list per row
//                       and column third (tc_list_depth(KP) keys).  The three lists of
//                       every row go to a small candidate buffer; no distance matrix
//                       reaches global memory.
//   rerank_kernel       merges a row's lists, computes the exact reference distance
//                       of each candidate, sorts by (distance, id), writes the top-k and
//                       checks a rounding-error certificate that no column outside the
//                       list could enter the top-k; failing rows are queued.
//   exact_rows_kernel   CUDA-core exact scan in the reference's fp32 summation order
//                       (FloatL2DistanceHandler::compute, UNG/codes/src/distance.cpp:34-91)
//                       with its (distance, id) queue order (UNG/codes/include/search_queue.h:20-22):
//                       route EXACT, and the rescan of the queued rows (a block per row);
//                       exact_rows_warp_kernel, a warp per row, for short target lists.
#include <cfloat>
#include <cmath>
#include <cuda_fp16.h>

#include "kernels.h"
#include "ptx.cuh"

namespace ungx
{
namespace
{
constexpr uint32_t kEpiWarps = 12;                    // three per TMEM lane quarter
constexpr uint32_t kTcThreads = 96 + 32 * kEpiWarps;  // warp 0 TMA, 1 MMA, 2..13 epilogue, 14 MMA (MODE 2)
constexpr uint32_t kBN = 192;          // target columns per tile / TMEM accumulator
constexpr uint32_t kAccBufs = 2;       // TMEM accumulators at columns 128 + 192 b
constexpr uint32_t kAccCol0 = 128;     // TMEM columns [0, 128): four A slots
constexpr uint32_t kASlots = 4;        // A slot = 32 TMEM columns = 64 fp16 of K x 128 rows
constexpr uint32_t kItemSlots = 2;
constexpr uint32_t kChunkK = 64;          // fp16 columns per K chunk: 128-byte rows
constexpr uint32_t kAChunk = 128 * 128;   // 128 rows x 64 fp16, 128-byte swizzled
constexpr uint32_t kBChunk = kBN * 128;   // 192 rows x 64 fp16
constexpr uint32_t kMaxStages = 16;
constexpr uint32_t kKeyLd = 36;           // a lane's row of 32 chunk keys (16-byte stores hit distinct banks)
constexpr uint32_t kSmemLimit = 232448;   // per-block opt-in maximum on sm_100
constexpr uint32_t kNoItem = 0xFFFFFFFFu;
// Limit of the waits that retire work already in flight before the CTA exits
// (independent of the configurable pipeline wait limit, which tests set tiny).
constexpr uint64_t kDrainWaitNs = 2000000000ull;

struct TcLayout
{
   uint32_t stages, stage_off, stage_bytes, colv_off, norm_off, key_off, bar_off, misc_off, total;
};

// Stages of the ring: A resident (dp <= 256) -> one 24 KB target chunk per stage, the
// item's source chunks (16 KB) pass through the same ring once per item; A streamed
// -> 16 KB source + 24 KB target chunk per stage.  As many stages as fit (at most
// 16), then the epilogue's column table (12 warps x list-depth slots x 32 lanes), the chunk
// norms, the chunk keys (12 warps x 32 lanes x kKeyLd), barriers, and the item slots.
__host__ __device__ inline TcLayout tc_layout(uint32_t dp, bool a_res, uint32_t kp)
{
   (void)dp;
   TcLayout L;
   L.stage_off = 0;
   L.stage_bytes = a_res ? kBChunk : kAChunk + kBChunk;
   const uint32_t kd = uint32_t(tc_list_depth(int(kp)));
   const uint32_t fixed =
       kEpiWarps * kd * 32u * 4u + kEpiWarps * 32u * 4u + kEpiWarps * 32u * kKeyLd * 4u + 48u * 8u + 128u + 1024u;
   const uint32_t fit = fixed < kSmemLimit ? (kSmemLimit - fixed) / L.stage_bytes : 0u;
   L.stages = fit < kMaxStages ? fit : kMaxStages;
   L.colv_off = L.stage_off + L.stages * L.stage_bytes;
   L.norm_off = L.colv_off + kEpiWarps * kd * 32u * 4u;
   L.key_off = L.norm_off + kEpiWarps * 32u * 4u;
   L.bar_off = L.key_off + kEpiWarps * 32u * kKeyLd * 4u;
   L.misc_off = L.bar_off + 48u * 8u;
   L.total = L.misc_off + 128u;
   return L;
}

// Order-preserving map of a float to an unsigned key (for atomic min / max).
__device__ __forceinline__ uint32_t float_key(float f)
{
   const uint32_t u = __float_as_uint(f);
   return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k)
{
   return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Two fp32 lanes per instruction (sm_100 f32x2 arithmetic); each lane rounds exactly
// like the scalar __fmaf_rn / __fsub_rn.
__device__ __forceinline__ uint64_t pack2(float lo, float hi)
{
   return (uint64_t(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c)
{
   uint64_t d;
   asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
   return d;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b)
{
   uint64_t d;
   asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
   return d;
}

// Squared L2 in the reference's order: 8 accumulators over i mod 8 with the update
// rounded twice (mul, add), lanes folded hi+lo, a 4-wide tail and a masked tail
// each updated with one fused rounding, then two pairwise horizontal adds.
template <bool VEC4>
__device__ __forceinline__ float ref_l2(const float *__restrict__ a, const float *__restrict__ b, uint32_t d)
{
   float l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f, l4 = 0.f, l5 = 0.f, l6 = 0.f, l7 = 0.f;
   uint32_t i = 0;
#define UNGX_LANE(l, x, y)                                                                                       \
   {                                                                                                           \
      const float t = __fsub_rn((x), (y));                                                                     \
      l = __fadd_rn(l, __fmul_rn(t, t));                                                                       \
   }
   if (VEC4)
   {
      for (; i + 8 <= d; i += 8)
      {
         const float4 a0 = __ldg(reinterpret_cast<const float4 *>(a + i));
         const float4 a1 = __ldg(reinterpret_cast<const float4 *>(a + i + 4));
         const float4 b0 = __ldg(reinterpret_cast<const float4 *>(b + i));
         const float4 b1 = __ldg(reinterpret_cast<const float4 *>(b + i + 4));
         UNGX_LANE(l0, a0.x, b0.x);
         UNGX_LANE(l1, a0.y, b0.y);
         UNGX_LANE(l2, a0.z, b0.z);
         UNGX_LANE(l3, a0.w, b0.w);
         UNGX_LANE(l4, a1.x, b1.x);
         UNGX_LANE(l5, a1.y, b1.y);
         UNGX_LANE(l6, a1.z, b1.z);
         UNGX_LANE(l7, a1.w, b1.w);
      }
   }
   else
   {
      for (; i + 8 <= d; i += 8)
      {
         UNGX_LANE(l0, __ldg(a + i + 0), __ldg(b + i + 0));
         UNGX_LANE(l1, __ldg(a + i + 1), __ldg(b + i + 1));
         UNGX_LANE(l2, __ldg(a + i + 2), __ldg(b + i + 2));
         UNGX_LANE(l3, __ldg(a + i + 3), __ldg(b + i + 3));
         UNGX_LANE(l4, __ldg(a + i + 4), __ldg(b + i + 4));
         UNGX_LANE(l5, __ldg(a + i + 5), __ldg(b + i + 5));
         UNGX_LANE(l6, __ldg(a + i + 6), __ldg(b + i + 6));
         UNGX_LANE(l7, __ldg(a + i + 7), __ldg(b + i + 7));
      }
   }
#undef UNGX_LANE
   float s0 = __fadd_rn(l4, l0), s1 = __fadd_rn(l5, l1), s2 = __fadd_rn(l6, l2), s3 = __fadd_rn(l7, l3);
   if (d - i >= 4)
   {
      float t;
      t = __fsub_rn(__ldg(a + i + 0), __ldg(b + i + 0));
      s0 = __fmaf_rn(t, t, s0);
      t = __fsub_rn(__ldg(a + i + 1), __ldg(b + i + 1));
      s1 = __fmaf_rn(t, t, s1);
      t = __fsub_rn(__ldg(a + i + 2), __ldg(b + i + 2));
      s2 = __fmaf_rn(t, t, s2);
      t = __fsub_rn(__ldg(a + i + 3), __ldg(b + i + 3));
      s3 = __fmaf_rn(t, t, s3);
      i += 4;
   }
   if (d > i)
   {
      const uint32_t rem = d - i; // 1..3; masked lanes add 0*0, which leaves them unchanged
      float t = __fsub_rn(__ldg(a + i), __ldg(b + i));
      s0 = __fmaf_rn(t, t, s0);
      if (rem > 1)
      {
         t = __fsub_rn(__ldg(a + i + 1), __ldg(b + i + 1));
         s1 = __fmaf_rn(t, t, s1);
      }
      if (rem > 2)
      {
         t = __fsub_rn(__ldg(a + i + 2), __ldg(b + i + 2));
         s2 = __fmaf_rn(t, t, s2);
      }
   }
   return __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
}

// ref_l2 for one candidate per lane of a group of TPR lanes (lanes j of `gmask`), the
// candidate rows staged through shared memory: chunks of 32 dimensions of the group's
// TPR candidate rows are copied by cp.async in coalesced 128-byte row segments (two
// buffers of [TPR][36] floats, the next chunk in flight while this one is summed), so
// that each lane reads its own candidate from shared memory instead of gathering
// 16-byte pieces of TPR different rows from global memory.  The query row a is read from
// global memory (the same address for the whole group).  The arithmetic is ref_l2's,
// in its order: the 8-lane blocks in ascending dimension, then the tails, which all
// lie in the last chunk.  Every lane of the group calls it (crow = UINT32_MAX: no row,
// zeros staged, result unused).  W: copy bytes, 16 when d % 4 == 0 and X is 16-byte
// aligned, else 4.  Used for wide rows (d > 256), where the gathered reads cost most.
constexpr uint32_t kStLd = 36; // staged row stride (floats): 16-byte aligned, quarter-warp conflict-free

template <int W>
__device__ __forceinline__ void rr_copy(float *dst, const float *src, bool ok)
{
   const uint32_t sa = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
   const size_t ga = __cvta_generic_to_global(src);
   if constexpr (W == 16)
      asm volatile("cp.async.ca.shared.global [%0], [%1], 16, %2;\n" ::"r"(sa), "l"(ga), "r"(ok ? 16u : 0u) : "memory");
   else
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(sa), "l"(ga), "r"(ok ? 4u : 0u) : "memory");
}

template <int W, uint32_t TPR>
__device__ float ref_l2_staged(const float *__restrict__ a, const float *__restrict__ X, uint32_t d, uint32_t crow,
                               float *buf, uint32_t j, uint32_t gmask)
{
   constexpr uint32_t F = W / 4;          // floats per copy
   constexpr uint32_t PER_ROW = 32u / F;  // copies per staged row segment
   constexpr uint32_t STAGE = TPR * kStLd;
   const uint32_t nch = (d + 31u) / 32u;
   auto issue = [&](uint32_t c, uint32_t slot) {
      float *dst = buf + slot * STAGE;
#pragma unroll 8
      for (uint32_t k = 0; k < PER_ROW; ++k) // TPR rows x PER_ROW copies over TPR lanes
      {
         const uint32_t i = j + TPR * k, r = i / PER_ROW, o = (i % PER_ROW) * F;
         const uint32_t rr = __shfl_sync(gmask, crow, r, TPR);
         const uint32_t dim = 32u * c + o;
         const bool ok = rr != 0xFFFFFFFFu && dim < d;
         rr_copy<W>(dst + r * kStLd + o, ok ? X + size_t(rr) * d + dim : X, ok);
      }
   };
   float l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f, l4 = 0.f, l5 = 0.f, l6 = 0.f, l7 = 0.f;
#define UNGX_LANE(l, x, y)                                                                                       \
   {                                                                                                           \
      const float t = __fsub_rn((x), (y));                                                                     \
      l = __fadd_rn(l, __fmul_rn(t, t));                                                                       \
   }
   const uint32_t d8 = d & ~7u; // dims of the 8-lane blocks
   float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
   issue(0, 0);
   asm volatile("cp.async.commit_group;\n" ::: "memory");
   for (uint32_t c = 0; c < nch; ++c)
   {
      if (c + 1 < nch)
      {
         issue(c + 1, (c + 1) & 1u);
         asm volatile("cp.async.commit_group;\n" ::: "memory");
         asm volatile("cp.async.wait_group 1;\n" ::: "memory");
      }
      else
         asm volatile("cp.async.wait_group 0;\n" ::: "memory");
      __syncwarp(gmask);
      const float *b = buf + (c & 1u) * STAGE + j * kStLd; // this lane's row, dims 32c ..
      const uint32_t base = 32u * c;
#pragma unroll
      for (uint32_t blk = 0; blk < 4; ++blk)
      {
         const uint32_t i = base + 8u * blk;
         if (i + 8u <= d8)
         {
            const float4 b0 = *reinterpret_cast<const float4 *>(b + 8u * blk);
            const float4 b1 = *reinterpret_cast<const float4 *>(b + 8u * blk + 4u);
            if (W == 16)
            {
               const float4 a0 = __ldg(reinterpret_cast<const float4 *>(a + i));
               const float4 a1 = __ldg(reinterpret_cast<const float4 *>(a + i + 4));
               UNGX_LANE(l0, a0.x, b0.x);
               UNGX_LANE(l1, a0.y, b0.y);
               UNGX_LANE(l2, a0.z, b0.z);
               UNGX_LANE(l3, a0.w, b0.w);
               UNGX_LANE(l4, a1.x, b1.x);
               UNGX_LANE(l5, a1.y, b1.y);
               UNGX_LANE(l6, a1.z, b1.z);
               UNGX_LANE(l7, a1.w, b1.w);
            }
            else
            {
               UNGX_LANE(l0, __ldg(a + i + 0), b0.x);
               UNGX_LANE(l1, __ldg(a + i + 1), b0.y);
               UNGX_LANE(l2, __ldg(a + i + 2), b0.z);
               UNGX_LANE(l3, __ldg(a + i + 3), b0.w);
               UNGX_LANE(l4, __ldg(a + i + 4), b1.x);
               UNGX_LANE(l5, __ldg(a + i + 5), b1.y);
               UNGX_LANE(l6, __ldg(a + i + 6), b1.z);
               UNGX_LANE(l7, __ldg(a + i + 7), b1.w);
            }
         }
      }
      if (c + 1 == nch)
      {
         // the tails: dims d8 .. d - 1, all inside this last chunk
         s0 = __fadd_rn(l4, l0), s1 = __fadd_rn(l5, l1), s2 = __fadd_rn(l6, l2), s3 = __fadd_rn(l7, l3);
         uint32_t i = d8;
         if (d - i >= 4)
         {
            const float *bt = b + (i - base);
            float t;
            t = __fsub_rn(__ldg(a + i + 0), bt[0]);
            s0 = __fmaf_rn(t, t, s0);
            t = __fsub_rn(__ldg(a + i + 1), bt[1]);
            s1 = __fmaf_rn(t, t, s1);
            t = __fsub_rn(__ldg(a + i + 2), bt[2]);
            s2 = __fmaf_rn(t, t, s2);
            t = __fsub_rn(__ldg(a + i + 3), bt[3]);
            s3 = __fmaf_rn(t, t, s3);
            i += 4;
         }
         if (d > i)
         {
            const float *bt = b + (i - base);
            const uint32_t rem = d - i;
            float t = __fsub_rn(__ldg(a + i), bt[0]);
            s0 = __fmaf_rn(t, t, s0);
            if (rem > 1)
            {
               t = __fsub_rn(__ldg(a + i + 1), bt[1]);
               s1 = __fmaf_rn(t, t, s1);
            }
            if (rem > 2)
            {
               t = __fsub_rn(__ldg(a + i + 2), bt[2]);
               s2 = __fmaf_rn(t, t, s2);
            }
         }
      }
      __syncwarp(gmask); // this buffer is refilled two chunks on
   }
#undef UNGX_LANE
   return __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
}

__device__ __forceinline__ bool pair_less(float d0, uint32_t i0, float d1, uint32_t i1)
{
   return d0 < d1 || (d0 == d1 && i0 < i1);
}

// Sorted insert of (d, id) into an ascending (distance, id) list of K entries (the
// last entry drops out).  Branch-free; an entry that does not precede the last one
// leaves the list unchanged.  Static indices only, so the list stays in registers.
template <int K>
__device__ __forceinline__ void insert_pair(float (&kd)[K], uint32_t (&ki)[K], float d, uint32_t id)
{
#pragma unroll
   for (int i = K - 1; i > 0; --i)
   {
      const bool prev = pair_less(d, id, kd[i - 1], ki[i - 1]);
      const bool here = pair_less(d, id, kd[i], ki[i]);
      const float nd = prev ? kd[i - 1] : (here ? d : kd[i]);
      const uint32_t ni = prev ? ki[i - 1] : (here ? id : ki[i]);
      kd[i] = nd;
      ki[i] = ni;
   }
   if (pair_less(d, id, kd[0], ki[0]))
   {
      kd[0] = d;
      ki[0] = id;
   }
}

// ------------------------------------------------------------------ prep
// Column sums (fp64) and column ranges of X over a block of rows; thread = column,
// four rows in flight per thread.
// Column sums (fp64), minima and maxima over the rows i * stride (i < n sampled rows).
// With a gate, the kernel runs only when *gate is non-zero (the full pass after a
// sampled scale turned out too large for some element).
__global__ void colsum_kernel(const float *__restrict__ X, uint32_t n, uint32_t d, double *__restrict__ sums,
                              uint32_t *__restrict__ range, uint32_t rows_per_block, uint32_t stride,
                              const uint32_t *__restrict__ gate)
{
   if (gate && *gate == 0u)
      return;
   const uint64_t r0 = uint64_t(blockIdx.x) * rows_per_block;
   const uint64_t r1 = (r0 + rows_per_block < n) ? r0 + rows_per_block : uint64_t(n);
   const uint64_t sd = uint64_t(stride) * d;
   for (uint32_t j = threadIdx.x; j < d; j += blockDim.x)
   {
      double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
      float mn = INFINITY, mx = -INFINITY;
      uint64_t r = r0;
      for (; r + 4 <= r1; r += 4)
      {
         const float v0 = __ldg(X + r * sd + j), v1 = __ldg(X + (r + 1) * sd + j);
         const float v2 = __ldg(X + (r + 2) * sd + j), v3 = __ldg(X + (r + 3) * sd + j);
         a0 += (double)v0;
         a1 += (double)v1;
         a2 += (double)v2;
         a3 += (double)v3;
         mn = fminf(fminf(mn, v0), fminf(fminf(v1, v2), v3));
         mx = fmaxf(fmaxf(mx, v0), fmaxf(fmaxf(v1, v2), v3));
      }
      for (; r < r1; ++r)
      {
         const float v = __ldg(X + r * sd + j);
         a0 += (double)v;
         mn = fminf(mn, v);
         mx = fmaxf(mx, v);
      }
      atomicAdd(&sums[j], (a0 + a1) + (a2 + a3));
      atomicMax(&range[2 * j], ~float_key(mn)); // minimum kept as the complement (zero = none)
      atomicMax(&range[2 * j + 1], float_key(mx));
   }
}

// One block: the fp32 mean, the largest centred magnitude m = max_j max(fl(max_j -
// mean_j), fl(mean_j - min_j)) (rounding is monotone, so no centred element exceeds
// it), and the scale s = 2^e with 2^(14 - headroom) <= s m < 2^(15 - headroom): from a
// row sample, headroom bits leave room for elements beyond the sample's range.
__global__ void scale_kernel(const double *__restrict__ sums, const uint32_t *__restrict__ range, uint32_t n,
                             uint32_t d, float *__restrict__ mean, OperandScale *__restrict__ out, int headroom,
                             const uint32_t *__restrict__ gate)
{
   if (gate && *gate == 0u)
      return;
   __shared__ float s_m[32];
   float m = 0.f;
   bool bad = false;
   for (uint32_t j = threadIdx.x; j < d; j += blockDim.x)
   {
      const float mu = (float)(sums[j] / (double)n);
      mean[j] = mu;
      const float lo = key_float(~range[2 * j]), hi = key_float(range[2 * j + 1]);
      const float e = fmaxf(__fsub_rn(hi, mu), __fsub_rn(mu, lo));
      if (!(e <= FLT_MAX)) // inf or nan in the data
         bad = true;
      else
         m = fmaxf(m, e);
   }
   bad = __syncthreads_or(bad);
   for (int o = 16; o; o >>= 1)
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
   if ((threadIdx.x & 31) == 0)
      s_m[threadIdx.x >> 5] = m;
   __syncthreads();
   if (threadIdx.x == 0)
   {
      for (uint32_t w = 1; w < (blockDim.x + 31) / 32; ++w)
         m = fmaxf(m, s_m[w]);
      int e = 0;
      int exact_only = bad ? 1 : 0;
      if (m > 0.f && !bad)
      {
         e = 14 - headroom - ilogbf(m); // ilogb: floor(log2 m), also for subnormal m
         if (e > 60)
            e = 60; // tiny data: keep 1/s^2 a normal float (the certificate sees the loss)
         if (e < -60)
         {
            e = -60;
            exact_only = 1; // s m would overflow fp16
         }
      }
      OperandScale sc;
      sc.s = ldexpf(1.f, e);
      sc.neg2_inv_s2 = -ldexpf(1.f, 1 - 2 * e);
      sc.inv_s = ldexpf(1.f, -e);
      sc.exact_only = exact_only;
      *out = sc;
   }
}

// Warp per row: v = fl(x - mean), operand fp16(s v) (saturated; s v is exact), norm
// = fp32 sum of v^2.  Columns d..dp-1 of the operand are zero.  An element with |s v|
// above the fp16 range (or not finite) sets *saturated; with a gate the kernel runs
// only when *gate is non-zero.
__global__ void center_kernel(const float *__restrict__ X, const float *__restrict__ mean,
                              const OperandScale *__restrict__ scale, uint32_t n, uint32_t d, uint32_t dp,
                              __half *__restrict__ Xh, float *__restrict__ xnorm, uint32_t *__restrict__ saturated,
                              const uint32_t *__restrict__ gate)
{
   if (gate && *gate == 0u)
      return;
   extern __shared__ float s_mean[];
   for (uint32_t j = threadIdx.x; j < d; j += blockDim.x)
      s_mean[j] = mean[j];
   __syncthreads();
   const float sc = scale->s;
   const uint32_t lane = threadIdx.x & 31;
   const uint64_t warps = (uint64_t(gridDim.x) * blockDim.x) >> 5;
   for (uint64_t r = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < n; r += warps)
   {
      float acc = 0.f;
      for (uint32_t j = 2 * lane; j < dp; j += 64)
      {
         float v0 = 0.f, v1 = 0.f;
         if (j < d)
            v0 = __fsub_rn(X[r * d + j], s_mean[j]);
         if (j + 1 < d)
            v1 = __fsub_rn(X[r * d + j + 1], s_mean[j + 1]);
         if (saturated && !(fabsf(v0 * sc) <= 65504.f && fabsf(v1 * sc) <= 65504.f))
            *saturated = 1u;
         const float w0 = fminf(fmaxf(v0 * sc, -65504.f), 65504.f);
         const float w1 = fminf(fmaxf(v1 * sc, -65504.f), 65504.f);
         *reinterpret_cast<__half2 *>(Xh + r * dp + j) = __halves2half2(__float2half_rn(w0), __float2half_rn(w1));
         acc = __fmaf_rn(v0, v0, acc);
         acc = __fmaf_rn(v1, v1, acc);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1)
         acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0)
         xnorm[r] = acc;
   }
}

// The same operand rows and norms for d % 4 == 0 with X 16-byte aligned: a lane takes
// four consecutive columns (one 16-byte load, one 8-byte store), and a warp works on
// four rows at once so that four loads per lane are in flight.  Each lane's fma chain
// runs over its columns in ascending order before the warp's xor tree, as above.
__global__ void center4_kernel(const float *__restrict__ X, const float *__restrict__ mean,
                               const OperandScale *__restrict__ scale, uint32_t n, uint32_t d, uint32_t dp,
                               __half *__restrict__ Xh, float *__restrict__ xnorm, uint32_t *__restrict__ saturated,
                               const uint32_t *__restrict__ gate)
{
   if (gate && *gate == 0u)
      return;
   extern __shared__ float s_mean[];
   for (uint32_t j = threadIdx.x; j < dp; j += blockDim.x)
      s_mean[j] = j < d ? mean[j] : 0.f;
   __syncthreads();
   const float sc = scale->s;
   const uint32_t lane = threadIdx.x & 31;
   const uint64_t warps = (uint64_t(gridDim.x) * blockDim.x) >> 5;
   const uint32_t q4 = dp / 4u, d4 = d / 4u;
   constexpr uint32_t RW = 4; // rows per warp iteration
   for (uint64_t r0 = ((uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5) * RW; r0 < n; r0 += warps * RW)
   {
      float acc[RW] = {0.f, 0.f, 0.f, 0.f};
      for (uint32_t c = lane; c < q4; c += 32)
      {
         float4 x[RW];
#pragma unroll
         for (uint32_t i = 0; i < RW; ++i)
            x[i] = (r0 + i < n && c < d4) ? __ldg(reinterpret_cast<const float4 *>(X + (r0 + i) * d) + c)
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
         const float4 mu = reinterpret_cast<const float4 *>(s_mean)[c];
#pragma unroll
         for (uint32_t i = 0; i < RW; ++i)
         {
            if (r0 + i >= n)
               continue;
            const bool in = c < d4; // padding columns stay exact zeros
            const float v0 = in ? __fsub_rn(x[i].x, mu.x) : 0.f, v1 = in ? __fsub_rn(x[i].y, mu.y) : 0.f;
            const float v2 = in ? __fsub_rn(x[i].z, mu.z) : 0.f, v3 = in ? __fsub_rn(x[i].w, mu.w) : 0.f;
            if (saturated && !(fabsf(v0 * sc) <= 65504.f && fabsf(v1 * sc) <= 65504.f &&
                               fabsf(v2 * sc) <= 65504.f && fabsf(v3 * sc) <= 65504.f))
               *saturated = 1u;
            const __half2 h01 = __halves2half2(__float2half_rn(fminf(fmaxf(v0 * sc, -65504.f), 65504.f)),
                                               __float2half_rn(fminf(fmaxf(v1 * sc, -65504.f), 65504.f)));
            const __half2 h23 = __halves2half2(__float2half_rn(fminf(fmaxf(v2 * sc, -65504.f), 65504.f)),
                                               __float2half_rn(fminf(fmaxf(v3 * sc, -65504.f), 65504.f)));
            uint2 pk;
            pk.x = *reinterpret_cast<const uint32_t *>(&h01);
            pk.y = *reinterpret_cast<const uint32_t *>(&h23);
            *reinterpret_cast<uint2 *>(Xh + (r0 + i) * dp + 4u * c) = pk;
            acc[i] = __fmaf_rn(v0, v0, acc[i]);
            acc[i] = __fmaf_rn(v1, v1, acc[i]);
            acc[i] = __fmaf_rn(v2, v2, acc[i]);
            acc[i] = __fmaf_rn(v3, v3, acc[i]);
         }
      }
#pragma unroll
      for (uint32_t i = 0; i < RW; ++i)
      {
#pragma unroll
         for (int o = 16; o; o >>= 1)
            acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
         if (lane == 0 && r0 + i < n)
            xnorm[r0 + i] = acc[i];
      }
   }
}

// Warp per chunk (group, first row, rows <= 4096) of a group's rows: the chunk's largest
// norm into out[group] by an integer max on the float bits (norms are >= 0; out zeroed
// by the caller).  Chunks keep one large group from serialising on a single warp.
__global__ void group_maxnorm_kernel(const float *__restrict__ xnorm, const uint32_t *__restrict__ chunks,
                                     uint32_t nchunks, float *__restrict__ out)
{
   const uint32_t lane = threadIdx.x & 31;
   const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
   for (uint32_t c = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; c < nchunks; c += warps)
   {
      const uint32_t g = chunks[3 * c], a = chunks[3 * c + 1], b = a + chunks[3 * c + 2];
      float m = 0.f;
      for (uint32_t r = a + lane; r < b; r += 32)
         m = fmaxf(m, xnorm[r]);
#pragma unroll
      for (int o = 16; o; o >>= 1)
         m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0)
         atomicMax(reinterpret_cast<int *>(out + g), __float_as_int(m));
   }
}

__global__ void fill_empty_kernel(const RowRange *__restrict__ ranges, uint32_t k, uint32_t *__restrict__ ids,
                                  float *__restrict__ dists)
{
   const RowRange rr = ranges[blockIdx.x];
   const uint64_t base = uint64_t(rr.begin) * k, cnt = uint64_t(rr.count) * k;
   for (uint64_t i = threadIdx.x; i < cnt; i += blockDim.x)
   {
      ids[base + i] = 0xFFFFFFFFu;
      if (dists)
         dists[base + i] = INFINITY;
   }
}

__global__ void gather_rows_kernel(const CopyRange *__restrict__ ranges, uint32_t k,
                                  const uint32_t *__restrict__ ids, const float *__restrict__ dists,
                                  uint32_t *__restrict__ out_ids, float *__restrict__ out_dists)
{
   const CopyRange r = ranges[blockIdx.x];
   const uint64_t src = uint64_t(r.src_row) * k, dst = uint64_t(r.dst_row) * k, cnt = uint64_t(r.count) * k;
   for (uint64_t i = threadIdx.x; i < cnt; i += blockDim.x)
   {
      out_ids[dst + i] = ids[src + i];
      if (dists)
         out_dists[dst + i] = dists[src + i];
   }
}

__global__ void scatter_rows_kernel(const CopyRange *__restrict__ ranges, uint32_t k, const uint32_t *__restrict__ ids,
                                    const float *__restrict__ dists, uint32_t *__restrict__ out_ids,
                                    float *__restrict__ out_dists)
{
   const CopyRange r = ranges[blockIdx.x];
   const uint64_t dst = uint64_t(r.src_row) * k, src = uint64_t(r.dst_row) * k, cnt = uint64_t(r.count) * k;
   for (uint64_t i = threadIdx.x; i < cnt; i += blockDim.x)
   {
      out_ids[dst + i] = ids[src + i];
      if (dists)
         out_dists[dst + i] = dists[src + i];
   }
}

// Thread per source row of a pass (capacity path): the pass's top-k of the row (ids
// are rows of the pass buffer) merged with the row's running top-k over the earlier
// passes (global ids), both sorted by (distance, id); the k smallest go back to the
// running list.  Buffer row c is global row base_src + c below split, base_tgt +
// (c - split) from there.
template <int KM>
__global__ void merge_pass_kernel(const uint32_t *__restrict__ pass_ids, const float *__restrict__ pass_dists,
                                  uint32_t rows, uint32_t k, uint32_t base_src, uint32_t split, uint32_t base_tgt,
                                  uint32_t *__restrict__ ids, float *__restrict__ dists)
{
   for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x)
   {
      const uint64_t po = uint64_t(r) * k, go = uint64_t(base_src + r) * k;
      uint32_t a = 0, b = 0;
      uint32_t out_i[KM];
      float out_d[KM];
      for (uint32_t o = 0; o < k; ++o)
      {
         uint32_t pi = 0xFFFFFFFFu, gi = 0xFFFFFFFFu;
         float pd = INFINITY, gd = INFINITY;
         if (a < k && pass_ids[po + a] != 0xFFFFFFFFu)
         {
            const uint32_t c = pass_ids[po + a];
            pi = c < split ? base_src + c : base_tgt + (c - split);
            pd = pass_dists[po + a];
         }
         if (b < k && ids[go + b] != 0xFFFFFFFFu)
         {
            gi = ids[go + b];
            gd = dists[go + b];
         }
         if (pi != 0xFFFFFFFFu && (gi == 0xFFFFFFFFu || pair_less(pd, pi, gd, gi)))
         {
            out_i[o] = pi;
            out_d[o] = pd;
            ++a;
         }
         else
         {
            out_i[o] = gi;
            out_d[o] = gd;
            if (gi != 0xFFFFFFFFu)
               ++b;
         }
      }
      for (uint32_t o = 0; o < k; ++o)
      {
         ids[go + o] = out_i[o];
         dists[go + o] = out_d[o];
      }
   }
}

// ------------------------------------------------------------------ exact scan
// One block (8 warps) per row: the 256 threads stride over the row's candidate
// columns keeping a sorted top-KMAX each; every warp then emits its own top-k by k
// rounds of a warp arg-min over (distance, id), and one thread merges the 8 lists.
template <int KMAX, bool VEC4>
__global__ void __launch_bounds__(256) exact_rows_kernel(const ExactParams p)
{
   __shared__ float s_d[8][KMAX];
   __shared__ uint32_t s_i[8][KMAX];
   const uint32_t count = p.count_dev ? *(volatile const uint32_t *)p.count_dev : p.count_host;
   const uint32_t lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
   for (uint32_t w = blockIdx.x; w < count; w += gridDim.x)
   {
      const uint32_t row = p.rows[w];
      const WorkItem it = p.items[p.row_items[w]];
      float bd[KMAX];
      uint32_t bi[KMAX];
#pragma unroll
      for (int i = 0; i < KMAX; ++i)
      {
         bd[i] = INFINITY;
         bi[i] = 0xFFFFFFFFu;
      }
      const float *q = p.X + size_t(row) * p.d;
      for (uint32_t s = 0; s < it.seg_count; ++s)
      {
         const Segment sg = p.segs[it.seg_begin + s];
         const uint32_t end = sg.x_begin + sg.x_count;
         for (uint32_t x = sg.x_begin + threadIdx.x; x < end; x += blockDim.x)
         {
            const float D = ref_l2<VEC4>(q, p.X + size_t(x) * p.d, p.d);
            if (pair_less(D, x, bd[KMAX - 1], bi[KMAX - 1]))
               insert_pair<KMAX>(bd, bi, D, x);
         }
      }
      for (uint32_t o = 0; o < p.k; ++o)
      {
         float md = bd[0];
         uint32_t mi = bi[0];
#pragma unroll
         for (int off = 16; off; off >>= 1)
         {
            const float od = __shfl_xor_sync(0xffffffffu, md, off);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, mi, off);
            if (pair_less(od, oi, md, mi))
            {
               md = od;
               mi = oi;
            }
         }
         if (mi != 0xFFFFFFFFu && bi[0] == mi)
         {
#pragma unroll
            for (int i = 0; i < KMAX - 1; ++i)
            {
               bd[i] = bd[i + 1];
               bi[i] = bi[i + 1];
            }
            bd[KMAX - 1] = INFINITY;
            bi[KMAX - 1] = 0xFFFFFFFFu;
         }
         if (lane == 0)
         {
            s_d[wid][o] = md;
            s_i[wid][o] = mi;
         }
      }
      __syncthreads();
      if (threadIdx.x == 0)
      {
#pragma unroll
         for (int i = 0; i < KMAX; ++i)
         {
            bd[i] = INFINITY;
            bi[i] = 0xFFFFFFFFu;
         }
         for (uint32_t wv = 0; wv < 8; ++wv)
            for (uint32_t o = 0; o < p.k && s_i[wv][o] != 0xFFFFFFFFu; ++o)
               insert_pair<KMAX>(bd, bi, s_d[wv][o], s_i[wv][o]);
         const size_t slot = p.out_pos ? size_t(p.out_pos[w]) : size_t(row);
#pragma unroll
         for (int i = 0; i < KMAX; ++i)
            if (uint32_t(i) < p.k)
            {
               p.out_ids[slot * p.k + i] = bi[i];
               if (p.out_dists)
                  p.out_dists[slot * p.k + i] = bd[i];
            }
      }
      __syncthreads();
   }
}

// The same scan with the target columns staged through shared memory: warp w of the
// block takes the 32-column steps w, w + 8, ... of each segment, lane l column x0 + l.
// A step's 32 target rows pass through a two-buffer ring per warp in chunks of 32
// dimensions, copied by cp.async as coalesced 128-byte row segments (the threads of
// exact_rows_kernel each read their own target row, 32 rows per load instruction).
// Lane l then reads its own row from shared memory (row stride 36 floats: the 16-byte
// reads of a quarter warp hit distinct banks) and applies ref_l2's arithmetic in its
// order: the 8-lane blocks in ascending dimension, the accumulators carried from chunk
// to chunk, then the tails, which all lie in the last chunk.  The query row is staged
// once per row.  W: copy bytes, 16 when d % 4 == 0 and X is 16-byte aligned, else 4.
constexpr uint32_t kExLd = 36;                       // staged row stride (floats)
constexpr uint32_t kExStage = 32u * kExLd;           // one buffer of a warp
constexpr uint32_t kExWarpFloats = 2u * kExStage;    // a warp's two buffers
constexpr uint32_t kExMaxDim = 8192;                 // query row staged in shared memory

__device__ __forceinline__ void ex_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void ex_wait()
{
   asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
template <int W>
__device__ __forceinline__ void ex_copy(float *dst, const float *src, bool ok)
{
   const uint32_t sa = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
   const size_t ga = __cvta_generic_to_global(src);
   if constexpr (W == 16)
      asm volatile("cp.async.ca.shared.global [%0], [%1], 16, %2;\n" ::"r"(sa), "l"(ga), "r"(ok ? 16u : 0u) : "memory");
   else
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(sa), "l"(ga), "r"(ok ? 4u : 0u) : "memory");
}

template <int KMAX, int W>
__global__ void __launch_bounds__(256) exact_rows_staged_kernel(const ExactParams p)
{
   extern __shared__ __align__(16) float ex_smem[];
   __shared__ float s_d[8][KMAX];
   __shared__ uint32_t s_i[8][KMAX];
   const uint32_t count = p.count_dev ? *(volatile const uint32_t *)p.count_dev : p.count_host;
   const uint32_t lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
   float *buf = ex_smem + wid * kExWarpFloats;   // this warp's ring
   float *sq = ex_smem + 8u * kExWarpFloats;     // the query row
   const uint32_t d = p.d, d8 = d & ~7u, nch = (d + 31u) / 32u;
   constexpr uint32_t F = W / 4, PER_ROW = 32u / F, PER_LANE = PER_ROW; // 32 rows x PER_ROW copies / 32 lanes
   for (uint32_t w = blockIdx.x; w < count; w += gridDim.x)
   {
      const uint32_t row = p.rows[w];
      const WorkItem it = p.items[p.row_items[w]];
      __syncthreads(); // the previous row's query and lists are no longer read
      for (uint32_t j = threadIdx.x; j < d; j += blockDim.x)
         sq[j] = p.X[size_t(row) * d + j];
      __syncthreads();
      float bd[KMAX];
      uint32_t bi[KMAX];
#pragma unroll
      for (int i = 0; i < KMAX; ++i)
      {
         bd[i] = INFINITY;
         bi[i] = 0xFFFFFFFFu;
      }
      for (uint32_t s = 0; s < it.seg_count; ++s)
      {
         const Segment sg = p.segs[it.seg_begin + s];
         const uint32_t end = sg.x_begin + sg.x_count;
         const uint32_t nsteps = (sg.x_count + 31u) / 32u;
         const uint32_t mine = nsteps > wid ? (nsteps - wid + 7u) / 8u : 0u;
         const uint32_t U = mine * nch; // (step, chunk) stages of this warp
         auto issue = [&](uint32_t u) {
            const uint32_t i = u / nch, c = u - i * nch;
            const uint32_t x0 = sg.x_begin + 32u * (wid + 8u * i);
            float *dst = buf + (u & 1u) * kExStage;
#pragma unroll
            for (uint32_t k = 0; k < PER_LANE; ++k)
            {
               const uint32_t e = lane + 32u * k, r = e / PER_ROW, o = (e % PER_ROW) * F;
               const uint32_t dim = 32u * c + o;
               const bool ok = x0 + r < end && dim < d;
               ex_copy<W>(dst + r * kExLd + o, ok ? p.X + size_t(x0 + r) * d + dim : p.X, ok);
            }
         };
         if (U)
            issue(0u);
         ex_commit();
         float l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f, l4 = 0.f, l5 = 0.f, l6 = 0.f, l7 = 0.f;
         for (uint32_t u = 0; u < U; ++u)
         {
            if (u + 1u < U)
            {
               issue(u + 1u);
               ex_commit();
               ex_wait<1>();
            }
            else
               ex_wait<0>();
            __syncwarp();
            const uint32_t i = u / nch, c = u - i * nch;
            const float *b = buf + (u & 1u) * kExStage + lane * kExLd; // this lane's column, dims 32c ..
            const uint32_t base = 32u * c;
            if (c == 0u)
               l0 = l1 = l2 = l3 = l4 = l5 = l6 = l7 = 0.f;
#define UNGX_LANE(l, x, y)                                                                                       \
   {                                                                                                           \
      const float t = __fsub_rn((x), (y));                                                                     \
      l = __fadd_rn(l, __fmul_rn(t, t));                                                                       \
   }
#pragma unroll
            for (uint32_t blk = 0; blk < 4u; ++blk)
            {
               const uint32_t i0 = base + 8u * blk;
               if (i0 + 8u <= d8)
               {
                  const float4 b0 = *reinterpret_cast<const float4 *>(b + 8u * blk);
                  const float4 b1 = *reinterpret_cast<const float4 *>(b + 8u * blk + 4u);
                  const float *a = sq + i0;
                  UNGX_LANE(l0, a[0], b0.x);
                  UNGX_LANE(l1, a[1], b0.y);
                  UNGX_LANE(l2, a[2], b0.z);
                  UNGX_LANE(l3, a[3], b0.w);
                  UNGX_LANE(l4, a[4], b1.x);
                  UNGX_LANE(l5, a[5], b1.y);
                  UNGX_LANE(l6, a[6], b1.z);
                  UNGX_LANE(l7, a[7], b1.w);
               }
            }
#undef UNGX_LANE
            if (c + 1u == nch)
            {
               // the tails (dims d8 .. d - 1, inside this last chunk), then the column's place
               float s0 = __fadd_rn(l4, l0), s1 = __fadd_rn(l5, l1), s2 = __fadd_rn(l6, l2), s3 = __fadd_rn(l7, l3);
               uint32_t t0 = d8;
               if (d - t0 >= 4u)
               {
                  const float *bt = b + (t0 - base);
                  float t;
                  t = __fsub_rn(sq[t0 + 0], bt[0]);
                  s0 = __fmaf_rn(t, t, s0);
                  t = __fsub_rn(sq[t0 + 1], bt[1]);
                  s1 = __fmaf_rn(t, t, s1);
                  t = __fsub_rn(sq[t0 + 2], bt[2]);
                  s2 = __fmaf_rn(t, t, s2);
                  t = __fsub_rn(sq[t0 + 3], bt[3]);
                  s3 = __fmaf_rn(t, t, s3);
                  t0 += 4u;
               }
               if (d > t0)
               {
                  const float *bt = b + (t0 - base);
                  const uint32_t rem = d - t0;
                  float t = __fsub_rn(sq[t0], bt[0]);
                  s0 = __fmaf_rn(t, t, s0);
                  if (rem > 1u)
                  {
                     t = __fsub_rn(sq[t0 + 1], bt[1]);
                     s1 = __fmaf_rn(t, t, s1);
                  }
                  if (rem > 2u)
                  {
                     t = __fsub_rn(sq[t0 + 2], bt[2]);
                     s2 = __fmaf_rn(t, t, s2);
                  }
               }
               const float D = __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
               const uint32_t x = sg.x_begin + 32u * (wid + 8u * i) + lane;
               if (x < end && pair_less(D, x, bd[KMAX - 1], bi[KMAX - 1]))
                  insert_pair<KMAX>(bd, bi, D, x);
            }
            __syncwarp(); // this buffer is refilled two stages on
         }
      }
      // every warp's top-k by k rounds of a warp arg-min over (distance, id), then one
      // thread merges the 8 lists (as exact_rows_kernel)
      for (uint32_t o = 0; o < p.k; ++o)
      {
         float md = bd[0];
         uint32_t mi = bi[0];
#pragma unroll
         for (int off = 16; off; off >>= 1)
         {
            const float od = __shfl_xor_sync(0xffffffffu, md, off);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, mi, off);
            if (pair_less(od, oi, md, mi))
            {
               md = od;
               mi = oi;
            }
         }
         if (mi != 0xFFFFFFFFu && bi[0] == mi)
         {
#pragma unroll
            for (int i = 0; i < KMAX - 1; ++i)
            {
               bd[i] = bd[i + 1];
               bi[i] = bi[i + 1];
            }
            bd[KMAX - 1] = INFINITY;
            bi[KMAX - 1] = 0xFFFFFFFFu;
         }
         if (lane == 0)
         {
            s_d[wid][o] = md;
            s_i[wid][o] = mi;
         }
      }
      __syncthreads();
      if (threadIdx.x == 0)
      {
#pragma unroll
         for (int i = 0; i < KMAX; ++i)
         {
            bd[i] = INFINITY;
            bi[i] = 0xFFFFFFFFu;
         }
         for (uint32_t wv = 0; wv < 8; ++wv)
            for (uint32_t o = 0; o < p.k && s_i[wv][o] != 0xFFFFFFFFu; ++o)
               insert_pair<KMAX>(bd, bi, s_d[wv][o], s_i[wv][o]);
         const size_t slot = p.out_pos ? size_t(p.out_pos[w]) : size_t(row);
#pragma unroll
         for (int i = 0; i < KMAX; ++i)
            if (uint32_t(i) < p.k)
            {
               p.out_ids[slot * p.k + i] = bi[i];
               if (p.out_dists)
                  p.out_dists[slot * p.k + i] = bd[i];
            }
      }
   }
}

// A warp per row, for rows whose candidate columns are few (the additional-edge
// queries scan one target group each): lanes stride over the columns keeping a sorted
// top-KMAX each, then k rounds of a warp arg-min over (distance, id) give the row's
// top-k in order, written by lane 0.  No block barrier.
template <int KMAX, bool VEC4>
__global__ void __launch_bounds__(256) exact_rows_warp_kernel(const ExactParams p)
{
   const uint32_t count = p.count_dev ? *(volatile const uint32_t *)p.count_dev : p.count_host;
   const uint32_t lane = threadIdx.x & 31;
   const uint32_t per_block = blockDim.x >> 5;
   for (uint32_t w = blockIdx.x * per_block + (threadIdx.x >> 5); w < count; w += gridDim.x * per_block)
   {
      const uint32_t row = p.rows[w];
      const WorkItem it = p.items[p.row_items[w]];
      float bd[KMAX];
      uint32_t bi[KMAX];
#pragma unroll
      for (int i = 0; i < KMAX; ++i)
      {
         bd[i] = INFINITY;
         bi[i] = 0xFFFFFFFFu;
      }
      const float *q = p.X + size_t(row) * p.d;
      for (uint32_t s = 0; s < it.seg_count; ++s)
      {
         const Segment sg = p.segs[it.seg_begin + s];
         const uint32_t end = sg.x_begin + sg.x_count;
         for (uint32_t x = sg.x_begin + lane; x < end; x += 32)
         {
            const float D = ref_l2<VEC4>(q, p.X + size_t(x) * p.d, p.d);
            if (pair_less(D, x, bd[KMAX - 1], bi[KMAX - 1]))
               insert_pair<KMAX>(bd, bi, D, x);
         }
      }
      const size_t slot = p.out_pos ? size_t(p.out_pos[w]) : size_t(row);
      for (uint32_t o = 0; o < p.k; ++o)
      {
         float md = bd[0];
         uint32_t mi = bi[0];
#pragma unroll
         for (int off = 16; off; off >>= 1)
         {
            const float od = __shfl_xor_sync(0xffffffffu, md, off);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, mi, off);
            if (pair_less(od, oi, md, mi))
            {
               md = od;
               mi = oi;
            }
         }
         if (mi != 0xFFFFFFFFu && bi[0] == mi)
         {
#pragma unroll
            for (int i = 0; i < KMAX - 1; ++i)
            {
               bd[i] = bd[i + 1];
               bi[i] = bi[i + 1];
            }
            bd[KMAX - 1] = INFINITY;
            bi[KMAX - 1] = 0xFFFFFFFFu;
         }
         if (lane == 0)
         {
            p.out_ids[slot * p.k + o] = mi;
            if (p.out_dists)
               p.out_dists[slot * p.k + o] = md;
         }
      }
   }
}

// ------------------------------------------------------------------ tensor-core path
__device__ __forceinline__ void raise_abort(volatile int *abort_word, int *status, int code)
{
   *abort_word = 1;
   atomicCAS(status, 0, code);
}

// Narrowest target box covering `valid` (1..192) columns: 16 (i + 1) rows.
__device__ __forceinline__ uint32_t box_index(uint32_t valid) { return (valid + 15u) / 16u - 1u; }

// Walks the 192-column tiles of a work item: segment by segment, 192 columns at a
// time.  The descriptor of the following segment is always loaded one segment
// ahead, so crossing into a new segment never waits on global memory.
struct TileIter
{
   const Segment *segs;
   uint32_t seg, nseg, t0;
   uint2 cur, nxt; // (x_begin, x_count)
   __device__ __forceinline__ uint2 load(uint32_t s) const
   {
      if (s >= nseg)
         return make_uint2(0, 0);
      const uint4 v = __ldg(reinterpret_cast<const uint4 *>(segs + s));
      return make_uint2(v.x, v.y);
   }
   __device__ __forceinline__ void start(const Segment *s, uint32_t begin, uint32_t count)
   {
      segs = s + begin;
      seg = 0;
      nseg = count;
      t0 = 0;
      cur = load(0);
      nxt = load(1);
   }
   __device__ __forceinline__ bool valid_tile() const { return seg < nseg; }
   __device__ __forceinline__ uint32_t x0() const { return cur.x + t0; }
   __device__ __forceinline__ uint32_t cols() const { return min(kBN, cur.y - t0); }
   __device__ __forceinline__ void next()
   {
      t0 += kBN;
      if (t0 >= cur.y)
      {
         t0 = 0;
         ++seg;
         cur = nxt;
         nxt = load(seg + 1);
      }
   }
};

// Candidate keys carry, in their 5 lowest mantissa bits, the slot of the entry in a
// per-thread column array.  A sorted list of such keys is updated with min/max only;
// the packing moves a key by at most 32 ulp (relative 2^-18), which the certificate
// accounts for.
constexpr uint32_t kSlotMask = 31u;

__device__ __forceinline__ float packed_init(int i)
{
   return __uint_as_float((0x7F7FFFFFu & ~kSlotMask) | uint32_t(i)); // huge, finite, ascending
}

template <int K>
__device__ __forceinline__ void insert_packed(float (&L)[K], float v)
{
#pragma unroll
   for (int i = K - 1; i > 0; --i)
      L[i] = fmaxf(L[i - 1], fminf(L[i], v));
   L[0] = fminf(L[0], v);
}

// MODE 0: A streamed per K chunk (dp > 256), one MMA issuer.
// MODE 1: A resident per item (128 < dp <= 256), one MMA issuer.
// MODE 2: A resident (dp <= 128), two MMA issuers (warps 1 and 14) on alternate tiles,
//         each with its own ring of stages and its own two A slots: one thread's
//         barrier waits and bookkeeping overlap the other's MMAs (tcgen05.mma issue
//         hardly queues, and a tile is only dp / 16 MMAs).
template <int KP, int MODE>
__global__ void __launch_bounds__(kTcThreads, 1) tc_kernel(const __grid_constant__ TcMaps maps, const TcParams p)
{
   constexpr bool A_RES = MODE >= 1;
   constexpr bool DUAL = MODE == 2;
   constexpr uint32_t R = DUAL ? 2u : 1u; // rings of stages
   extern __shared__ uint8_t smem_raw[];
   const uint32_t raw_u32 = ptx::smem_u32(smem_raw);
   uint8_t *smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
   const TcLayout L = tc_layout(p.dp, A_RES, KP);
   const uint32_t SR = L.stages / R; // stages per ring
   uint8_t *sStage = smem + L.stage_off;
   float *sNorm = reinterpret_cast<float *>(smem + L.norm_off);
   float *sKey = reinterpret_cast<float *>(smem + L.key_off);
   uint32_t *sColv = reinterpret_cast<uint32_t *>(smem + L.colv_off);
   uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bar_off);
   uint64_t *full = bars;              // [R * SR <= 16], ring r = stages [r SR, r SR + SR)
   uint64_t *empty = bars + 16;        // [R * SR]
   uint64_t *acc_full = bars + 32;     // [2]
   uint64_t *acc_empty = bars + 34;    // [2]
   uint64_t *a_free = bars + 36;       // [4]: MMAs reading A slot s completed (MODE 2: [issuer])
   uint64_t *item_full = bars + 40;    // [2]
   uint64_t *item_empty = bars + 42;   // [2]
   uint64_t *done_bar = bars + 44;     // [2]: one per issuer
   volatile uint32_t *item_slot = reinterpret_cast<volatile uint32_t *>(smem + L.misc_off);
   uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L.misc_off + 16);
   volatile int *abort_word = reinterpret_cast<volatile int *>(smem + L.misc_off + 32);
   WorkItem *item_desc = reinterpret_cast<WorkItem *>(smem + L.misc_off + 64); // [kItemSlots]

   const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
   const uint32_t nch = (p.dp + kChunkK - 1) / kChunkK;
   const uint64_t tmo = p.timeout_ns;

   if (threadIdx.x == 0)
   {
      for (uint32_t s = 0; s < R * SR; ++s)
      {
         ptx::mbar_init(&full[s], 1);
         ptx::mbar_init(&empty[s], 1);
      }
      for (uint32_t b = 0; b < kAccBufs; ++b)
      {
         ptx::mbar_init(&acc_full[b], 1);
         ptx::mbar_init(&acc_empty[b], kEpiWarps);
      }
      for (uint32_t s = 0; s < kASlots; ++s)
         ptx::mbar_init(&a_free[s], 1);
      for (uint32_t s = 0; s < kItemSlots; ++s)
      {
         ptx::mbar_init(&item_full[s], 1);
         ptx::mbar_init(&item_empty[s], R + kEpiWarps); // MMA issuers + epilogue warps
      }
      ptx::mbar_init(&done_bar[0], 1);
      ptx::mbar_init(&done_bar[1], 1);
      *abort_word = 0;
      ptx::fence_mbar_init();
   }
   if (warp == 0 && lane == 0)
   {
      ptx::prefetch_tmap(&maps.a);
      for (uint32_t i = 0; i < kTcBoxes; ++i)
         ptx::prefetch_tmap(&maps.b[i]);
   }
   if (warp == 1)
   {
      ptx::tmem_alloc(tmem_slot, 512);
      ptx::tmem_relinquish();
   }
   ptx::tc_fence_before();
   __syncthreads();
   ptx::tc_fence_after();
   const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t *>(tmem_slot);

   if (warp == 0)
   {
      // ------------------------------------------------ TMA producer
      if (lane == 0 && !(p.inject & UNGX_INJECT_WITHHOLD_WORK))
      {
         uint32_t it[R], pst[R], pph[R]; // per ring: stages issued, position, phase
         for (uint32_t r = 0; r < R; ++r)
            it[r] = pst[r] = pph[r] = 0;
         uint32_t iseq = 0, tseq = 0;
         bool ok = true;
         auto next_stage = [&](uint32_t r, uint32_t bytes) -> uint8_t * {
            const uint32_t g = r * SR + pst[r];
            if (!ptx::mbar_wait(&empty[g], pph[r] ^ 1u, abort_word, tmo))
               return nullptr;
            ptx::mbar_arrive_expect_tx(&full[g], bytes);
            return sStage + g * L.stage_bytes;
         };
         auto advance = [&](uint32_t r) {
            ++it[r];
            if (++pst[r] == SR) // ring position and phase kept without division
            {
               pst[r] = 0;
               pph[r] ^= 1u;
            }
         };
         for (;;)
         {
            const uint32_t idx = atomicAdd(p.item_counter, 1u);
            const uint32_t slot = iseq % kItemSlots;
            if (!ptx::mbar_wait(&item_empty[slot], ((iseq / kItemSlots) & 1u) ^ 1u, abort_word, tmo))
            {
               ok = false;
               break;
            }
            WorkItem w{};
            if (idx < p.num_items)
               w = p.items[idx];
            item_desc[slot] = w;
            item_slot[slot] = idx < p.num_items ? idx : kNoItem;
            ptx::mbar_arrive(&item_full[slot]);
            ++iseq;
            if (idx >= p.num_items)
               break;
            if (A_RES) // the item's source chunks, once per ring
               for (uint32_t r = 0; r < R && ok; ++r)
                  for (uint32_t c = 0; c < nch; ++c)
                  {
                     uint8_t *dst = next_stage(r, kAChunk);
                     if (!dst)
                     {
                        ok = false;
                        break;
                     }
                     ptx::tma_load_2d(dst, &maps.a, &full[r * SR + pst[r]], int32_t(c * kChunkK),
                                      int32_t(w.row_begin));
                     advance(r);
                  }
            TileIter ti;
            for (ti.start(p.segs, w.seg_begin, w.seg_count); ti.valid_tile() && ok; ti.next(), ++tseq)
            {
               const uint32_t r = DUAL ? (tseq & 1u) : 0u;
               const uint32_t bix = box_index(ti.cols());
               const uint32_t brows = 16u * (bix + 1u);
               for (uint32_t c = 0; c < nch; ++c)
               {
                  uint8_t *dst = next_stage(r, (A_RES ? 0u : kAChunk) + brows * 128u);
                  if (!dst)
                  {
                     ok = false;
                     break;
                  }
                  uint64_t *fb = &full[r * SR + pst[r]];
                  if (!A_RES)
                     ptx::tma_load_2d(dst, &maps.a, fb, int32_t(c * kChunkK), int32_t(w.row_begin));
                  ptx::tma_load_2d(dst + (A_RES ? 0u : kAChunk), &maps.b[bix], fb, int32_t(c * kChunkK),
                                   int32_t(ti.x0()));
                  advance(r);
               }
            }
            if (!ok)
               break;
         }
         if (!ok)
         {
            raise_abort(abort_word, p.status, UNGX_ERR_TIMEOUT);
            // drain: every load already issued must land before the CTA exits
            for (uint32_t r = 0; r < R; ++r)
               for (uint32_t st = 0; st < SR; ++st)
               {
                  const uint32_t issued = it[r] / SR + (st < it[r] % SR ? 1u : 0u);
                  if (issued)
                     ptx::mbar_wait(&full[r * SR + st], (issued - 1) & 1u, nullptr, kDrainWaitNs);
               }
         }
      }
      __syncwarp();
   }
   else if (warp == 1 || (DUAL && warp == kEpiWarps + 2u))
   {
      // ------------------------------------------------ MMA issuer(s)
      const uint32_t m = warp == 1 ? 0u : 1u; // issuer: ring m, accumulator (tile parity) m
      if (lane == 0)
      {
         uint32_t tseq = 0, iseq = 0, mst = 0, mph = 0, items = 0;
         uint32_t apos = 0; // MODE 0/1: A slots used so far (slot = apos % 4, use count = apos / 4)
         bool ok = true;
         auto take_slot = [&]() -> int {
            const uint32_t s = apos % kASlots, u = apos / kASlots;
            if (u && !ptx::mbar_wait(&a_free[s], (u - 1u) & 1u, abort_word, tmo))
               return -1;
            ++apos;
            return int(s);
         };
         auto wait_full = [&]() -> uint8_t * {
            const uint32_t g = m * SR + mst;
            if (!ptx::mbar_wait(&full[g], mph, abort_word, tmo))
               return nullptr;
            return sStage + g * L.stage_bytes;
         };
         auto release = [&]() {
            ptx::mma_commit(&empty[m * SR + mst]);
            if (++mst == SR)
            {
               mst = 0;
               mph ^= 1u;
            }
         };
         // four 128x256b copies: 128 rows x 64 fp16 -> TMEM columns [32 s, 32 s + 32)
         auto copy_a = [&](const uint8_t *src, uint32_t s) {
            const uint64_t ad = ptx::sdesc_k_sw128(ptx::smem_u32(src));
#pragma unroll
            for (uint32_t ks = 0; ks < 4; ++ks)
               ptx::tmem_cp_128x256b(tmem_base + s * 32u + ks * 8u, ad + 2u * ks);
         };
         for (;;)
         {
            const uint32_t slot = iseq % kItemSlots;
            if (!ptx::mbar_wait(&item_full[slot], (iseq / kItemSlots) & 1u, abort_word, tmo))
            {
               ok = false;
               break;
            }
            const uint32_t idx = item_slot[slot];
            ++iseq;
            if (idx == kNoItem)
               break;
            const WorkItem w = item_desc[slot];
            const uint32_t abase = apos;
            if (DUAL)
            {
               // this issuer's A slots 2m, 2m + 1 are free once its previous item's MMAs completed
               if (items && !ptx::mbar_wait(&a_free[m], (items - 1u) & 1u, abort_word, tmo))
               {
                  ok = false;
                  break;
               }
               for (uint32_t c = 0; c < nch && ok; ++c)
               {
                  const uint8_t *stage = wait_full();
                  if (!stage)
                  {
                     ok = false;
                     break;
                  }
                  ptx::tc_fence_after();
                  copy_a(stage, 2u * m + c);
                  release();
               }
            }
            else if (A_RES)
               for (uint32_t c = 0; c < nch; ++c)
               {
                  const int s = take_slot();
                  const uint8_t *stage = s < 0 ? nullptr : wait_full();
                  if (!stage)
                  {
                     ok = false;
                     break;
                  }
                  ptx::tc_fence_after();
                  copy_a(stage, uint32_t(s));
                  release();
               }
            TileIter ti;
            for (ti.start(p.segs, w.seg_begin, w.seg_count); ti.valid_tile() && ok; ti.next(), ++tseq)
            {
               const uint32_t b = tseq & 1u;
               if (DUAL && b != m)
                  continue; // the other issuer's tile
               if (!ptx::mbar_wait(&acc_empty[b], ((tseq >> 1) & 1u) ^ 1u, abort_word, tmo))
               {
                  ok = false;
                  break;
               }
               ptx::tc_fence_after();
               const uint32_t N = 16u * (box_index(ti.cols()) + 1u);
               const uint32_t idesc = ptx::idesc_f16(128, N);
               const uint32_t dt = tmem_base + kAccCol0 + b * kBN;
               if (DUAL)
               {
                  // dp <= 128: one or two chunks of four K = 16 steps (the last may be partial)
                  const uint32_t at = tmem_base + 64u * m;
                  const uint8_t *st0 = wait_full();
                  if (!st0)
                  {
                     ok = false;
                     break;
                  }
                  const uint64_t bd0 = ptx::sdesc_k_sw128(ptx::smem_u32(st0));
                  const uint32_t k0 = p.dp >= kChunkK ? 4u : p.dp / 16u;
                  ptx::mma_f16_ts(dt, at, bd0, idesc, 0u);
#pragma unroll
                  for (uint32_t ks = 1; ks < 4; ++ks)
                     if (ks < k0)
                        ptx::mma_f16_ts(dt, at + ks * 8u, bd0 + 2u * ks, idesc, 1u);
                  release();
                  if (nch > 1)
                  {
                     const uint8_t *st1 = wait_full();
                     if (!st1)
                     {
                        ok = false;
                        break;
                     }
                     const uint64_t bd1 = ptx::sdesc_k_sw128(ptx::smem_u32(st1));
                     const uint32_t k1 = (p.dp - kChunkK) / 16u;
#pragma unroll
                     for (uint32_t ks = 0; ks < 4; ++ks)
                        if (ks < k1)
                           ptx::mma_f16_ts(dt, at + 32u + ks * 8u, bd1 + 2u * ks, idesc, 1u);
                     release();
                  }
               }
               else
                  for (uint32_t c = 0; c < nch; ++c)
                  {
                     int s;
                     if (A_RES)
                        s = int((abase + c) % kASlots);
                     else if ((s = take_slot()) < 0)
                     {
                        ok = false;
                        break;
                     }
                     const uint8_t *stage = wait_full();
                     if (!stage)
                     {
                        ok = false;
                        break;
                     }
                     if (!A_RES)
                     {
                        ptx::tc_fence_after();
                        copy_a(stage, uint32_t(s));
                     }
                     const uint64_t bd = ptx::sdesc_k_sw128(ptx::smem_u32(stage + (A_RES ? 0u : kAChunk)));
                     const uint32_t kleft = p.dp - c * kChunkK; // multiple of 16
                     const uint32_t ksteps = kleft >= kChunkK ? 4u : kleft / 16u;
                     const uint32_t at = tmem_base + uint32_t(s) * 32u;
                     for (uint32_t ks = 0; ks < ksteps; ++ks) // K = 16 per MMA (+32 B, +8 TMEM columns)
                        ptx::mma_f16_ts(dt, at + ks * 8u, bd + 2u * ks, idesc, (c | ks) != 0u);
                     release();
                     if (!A_RES)
                        ptx::mma_commit(&a_free[s]);
                  }
               if (!ok)
                  break;
               ptx::mma_commit(&acc_full[b]);
            }
            if (DUAL)
               ptx::mma_commit(&a_free[m]);
            else if (A_RES) // the item's A slots are free once its MMAs complete
               for (uint32_t c = 0; c < nch && abase + c < apos; ++c)
                  ptx::mma_commit(&a_free[(abase + c) % kASlots]);
            ++items;
            if (!ok)
               break;
            ptx::mbar_arrive(&item_empty[slot]);
         }
         if (!ok)
            raise_abort(abort_word, p.status, UNGX_ERR_TIMEOUT);
         // every MMA / copy issued by this thread (and its arrivals) completes before teardown
         ptx::mma_commit(&done_bar[m]);
         ptx::mbar_wait(&done_bar[m], 0, nullptr, kDrainWaitNs);
      }
      __syncwarp();
   }
   else if (warp == kEpiWarps + 2u)
   {
      // spare warp (single-issuer modes)
   }
   else
   {
      // ------------------------------------------------ epilogue: one thread per source row
      // Warp w reads TMEM lane quarter w % 4 (rows 32q..32q+31) and, of every 192-column
      // tile, the 32-column chunks h and h + 3 (h = 0, 1, 2: its column third).
      const uint32_t q = warp & 3u;
      const uint32_t h = (warp - 2u) >> 2;
      const uint32_t r = q * 32u + lane;
      float *nrm = sNorm + (warp - 2u) * 32u;
      float *mykey = sKey + ((warp - 2u) * 32u + lane) * kKeyLd; // this lane's keys of the chunk
      const float nis = p.scale->neg2_inv_s2; // keys in the unscaled centred domain
      uint32_t tseq = 0, iseq = 0;
      bool ok = true;
      for (;;)
      {
         const uint32_t slot = iseq % kItemSlots;
         if (!ptx::mbar_wait(&item_full[slot], (iseq / kItemSlots) & 1u, abort_word, tmo))
         {
            ok = false;
            break;
         }
         const uint32_t idx = item_slot[slot];
         ++iseq;
         if (idx == kNoItem)
            break;
         const WorkItem w = item_desc[slot];
         const bool row_ok = r < w.row_count;
         const bool warp_ok = q * 32u < w.row_count;
         constexpr int KD = tc_list_depth(KP);
         float key[KD]; // ascending packed keys (slot in the low bits)
         // column of each slot: colv[slot * 32 + lane] (bank = lane, conflict-free)
         uint32_t *colv = sColv + (warp - 2u) * (KD * 32u) + lane;
#pragma unroll
         for (int i = 0; i < KD; ++i)
         {
            key[i] = packed_init(i);
            colv[i * 32] = 0xFFFFFFFFu;
         }
         float thr = row_ok ? key[KD - 1] : -INFINITY; // rows past the item never take candidates
         TileIter ti;
         ti.start(p.segs, w.seg_begin, w.seg_count);
         // norms of this warp's two chunks of the current tile; the next tile's are
         // loaded while the current one is processed
         float n0 = INFINITY, n1 = INFINITY;
         if (ti.valid_tile())
         {
            const uint32_t c0 = h * 32u + lane, c1 = c0 + 96u, v = ti.cols(), x0 = ti.x0();
            n0 = c0 < v ? __ldg(p.xnorm + x0 + c0) : INFINITY;
            n1 = c1 < v ? __ldg(p.xnorm + x0 + c1) : INFINITY;
         }
         for (; ti.valid_tile(); ++tseq)
         {
            const uint32_t valid = ti.cols(), x0 = ti.x0();
            const float cn0 = n0, cn1 = n1;
            ti.next();
            if (ti.valid_tile())
            {
               const uint32_t c0 = h * 32u + lane, c1 = c0 + 96u, v = ti.cols(), nx0 = ti.x0();
               n0 = c0 < v ? __ldg(p.xnorm + nx0 + c0) : INFINITY;
               n1 = c1 < v ? __ldg(p.xnorm + nx0 + c1) : INFINITY;
            }
            const uint32_t b = tseq & 1u;
            if (!ptx::mbar_wait(&acc_full[b], (tseq >> 1) & 1u, abort_word, tmo))
            {
               ok = false;
               break;
            }
            ptx::tc_fence_after();
#pragma unroll 1
            for (uint32_t i = 0; i < 2; ++i)
            {
               const uint32_t j = h + 3u * i;
               if (!warp_ok || j * 32u >= valid)
                  break;
               __syncwarp();
               nrm[lane] = i ? cn1 : cn0;
               __syncwarp();
               uint32_t raw[32];
               ptx::tmem_ld32(tmem_base + ((q * 32u) << 16) + kAccCol0 + b * kBN + j * 32u, raw);
               ptx::tmem_wait_ld();
               // key = fl(norm + nis * acc); the sign of fl(key - thr) is set exactly when
               // key < thr (an exact zero difference is +0): element jj goes to bit 31 - jj.
               // When some lane has a candidate, the keys go to the lane's row in shared
               // memory, where the inserts read them.
               const float4 *n4 = reinterpret_cast<const float4 *>(nrm);
               const uint64_t nis2 = pack2(nis, nis), thr2 = pack2(thr, thr);
               uint32_t mask = 0;
               uint64_t kv[16];
#pragma unroll
               for (int g = 0; g < 8; ++g)
               {
                  const float4 nv = n4[g];
                  const uint64_t k01 = fma2(nis2, pack2(__uint_as_float(raw[4 * g]), __uint_as_float(raw[4 * g + 1])),
                                            pack2(nv.x, nv.y));
                  const uint64_t k23 =
                      fma2(nis2, pack2(__uint_as_float(raw[4 * g + 2]), __uint_as_float(raw[4 * g + 3])),
                           pack2(nv.z, nv.w));
                  kv[2 * g] = k01;
                  kv[2 * g + 1] = k23;
                  const uint64_t d01 = sub2(k01, thr2), d23 = sub2(k23, thr2);
                  mask = __funnelshift_l(uint32_t(d01), mask, 1);
                  mask = __funnelshift_l(uint32_t(d01 >> 32), mask, 1);
                  mask = __funnelshift_l(uint32_t(d23), mask, 1);
                  mask = __funnelshift_l(uint32_t(d23 >> 32), mask, 1);
               }
               // every lane inserts its passing keys; the loop runs as often as the
               // busiest lane needs, lanes without a candidate insert +inf (a no-op)
               const uint32_t cbase = x0 + j * 32u;
               if (p.exclude_self) // self-join: the row's own column never passes
               {
                  const uint32_t off = w.row_begin + r - cbase;
                  if (off < 32u)
                     mask &= ~(0x80000000u >> off);
               }
               if (__any_sync(0xffffffffu, mask != 0u))
               {
#pragma unroll
                  for (int g = 0; g < 8; ++g)
                     *reinterpret_cast<uint4 *>(mykey + 4 * g) = make_uint4(
                         uint32_t(kv[2 * g]), uint32_t(kv[2 * g] >> 32), uint32_t(kv[2 * g + 1]), uint32_t(kv[2 * g + 1] >> 32));
               }
               while (__any_sync(0xffffffffu, mask != 0u))
               {
                  const uint32_t jj = mask ? uint32_t(__clz(mask)) : 0u;
                  const float kk = mykey[jj];
                  const uint32_t ev = __float_as_uint(key[KD - 1]) & kSlotMask; // slot that drops out
                  const float v = __uint_as_float((__float_as_uint(kk) & ~kSlotMask) | ev);
                  const bool ins = mask != 0u && v < key[KD - 1];
                  if (ins)
                     colv[ev * 32u] = cbase + jj;
                  insert_packed<KD>(key, ins ? v : INFINITY);
                  mask &= ~(0x80000000u >> jj);
               }
               thr = row_ok ? key[KD - 1] : -INFINITY;
            }
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0)
               ptx::mbar_arrive(&acc_empty[b]);
         }
         if (!ok)
            break;
         if (row_ok)
         {
            float4 *kd = reinterpret_cast<float4 *>(p.cand_key + (size_t(w.row_begin + r) * kTcLists + h) * KD);
            uint4 *cd = reinterpret_cast<uint4 *>(p.cand_col + (size_t(w.row_begin + r) * kTcLists + h) * KD);
#pragma unroll
            for (int i = 0; i < KD / 4; ++i)
            {
               kd[i] = make_float4(key[4 * i], key[4 * i + 1], key[4 * i + 2], key[4 * i + 3]);
               cd[i] = make_uint4(colv[(__float_as_uint(key[4 * i]) & kSlotMask) * 32u],
                                  colv[(__float_as_uint(key[4 * i + 1]) & kSlotMask) * 32u],
                                  colv[(__float_as_uint(key[4 * i + 2]) & kSlotMask) * 32u],
                                  colv[(__float_as_uint(key[4 * i + 3]) & kSlotMask) * 32u]);
            }
         }
         __syncwarp();
         if (lane == 0)
            ptx::mbar_arrive(&item_empty[slot]);
      }
      if (!ok)
         raise_abort(abort_word, p.status, UNGX_ERR_TIMEOUT);
      __syncwarp();
   }

   ptx::tc_fence_before();
   __syncthreads();
   if (warp == 1)
   {
      ptx::tc_fence_after();
      ptx::tmem_dealloc(tmem_base, 512);
   }
}

// ------------------------------------------------------------------ rerank + certificate
// One block per work item.  A row belongs to a group of KP lanes (a half warp for
// KP = 16, a warp for KP = 32) that never waits on the rest of the block:
//   1. the lanes rank the row's 3 x KD list entries (packed prefilter keys, within
//      2^-17 relative of the fp32 key) by counting over shuffles, ties by entry index,
//      and the KP smallest go to one lane each (the merged list);
//   2. each lane computes the exact reference distance of its candidate unless its
//      key shows it cannot reach the top-k;
//   3. the lanes rank their (distance, id) pairs the same way and write the first k;
//   4. the certificate is evaluated by every lane, recorded by lane 0.
template <int KP, bool STAGED>
__global__ void __launch_bounds__(256, STAGED ? 3 : 4) rerank_kernel(const RerankParams p)
{
   constexpr uint32_t TPR = KP;           // lanes per row
   constexpr int KD = tc_list_depth(KP);  // depth of each of the row's lists
   constexpr int NE = int(kTcLists) * KD; // list entries per row
   constexpr int EPL = (NE + int(TPR) - 1) / int(TPR);
   constexpr uint32_t RPB = 256u / TPR; // rows in flight per block
   static_assert(TPR == 16 || TPR == 32, "a row group is a half warp or a warp");
   __shared__ uint2 s_slot[RPB][KP]; // merged list: (key bits, column) by rank
   __shared__ float s_maxn2;
   __shared__ uint32_t s_total;
   __shared__ unsigned long long s_cnt[2];
   // an aborted prefilter left the candidate buffer unwritten: touch nothing
   if (*reinterpret_cast<const volatile int *>(p.status) != 0)
      return;
   const WorkItem w = p.items[blockIdx.x];
   const uint32_t tid = threadIdx.x;
   if (tid < 32)
   {
      float m = 0.f;
      uint32_t tot = 0;
      for (uint32_t s = tid; s < w.seg_count; s += 32)
      {
         const Segment sg = p.segs[w.seg_begin + s];
         m = fmaxf(m, p.group_maxn2[sg.group_id]);
         tot += sg.x_count;
      }
#pragma unroll
      for (int o = 16; o; o >>= 1)
      {
         m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
         tot += __shfl_xor_sync(0xffffffffu, tot, o);
      }
      if (tid == 0)
      {
         s_maxn2 = m;
         s_total = tot;
         s_cnt[0] = s_cnt[1] = 0;
      }
   }
   __syncthreads();
   const uint32_t total = s_total;
   const uint32_t grp = tid / TPR, j = tid % TPR;
   const uint32_t gmask = TPR == 32u ? 0xffffffffu : (0xffffu << (tid & 16u));
   const bool vec4 = (p.d & 3u) == 0;
   const bool w16 = vec4 && reinterpret_cast<uintptr_t>(p.X) % 16u == 0;
   extern __shared__ __align__(16) float rr_stage[]; // STAGED: [256 / TPR groups][2][TPR][kStLd]
   float *stage = rr_stage + grp * (2u * TPR * kStLd);
   const double pk = 1.0 / 131072.0; // packed-key tolerance, 2^-17 relative
   const double bmax = sqrt((double)s_maxn2 * (1.0 + p.gd));
   const double inv_s = (double)p.scale->inv_s;
   const bool exact_only = p.scale->exact_only != 0;
   const uint32_t k = p.k;
   uint32_t n_cert = 0, n_fail = 0;
   for (uint32_t r = grp; r < w.row_count; r += RPB)
   {
      const uint32_t row = w.row_begin + r;
      const float *kp = p.cand_key + size_t(row) * NE;
      const uint32_t *cp = p.cand_col + size_t(row) * NE;
      float ek[EPL];
      uint32_t ec[EPL];
#pragma unroll
      for (int e = 0; e < EPL; ++e)
      {
         const int idx = int(j) + e * int(TPR);
         ek[e] = idx < NE ? kp[idx] : INFINITY;
         ec[e] = idx < NE ? cp[idx] : 0xFFFFFFFFu;
      }
      // 1. rank among the NE entries: (key, entry index) order
      uint32_t rk[EPL];
#pragma unroll
      for (int e = 0; e < EPL; ++e)
         rk[e] = 0;
#pragma unroll
      for (int src = 0; src < NE; ++src)
      {
         const float v = __shfl_sync(gmask, ek[src / int(TPR)], src % int(TPR), TPR);
#pragma unroll
         for (int e = 0; e < EPL; ++e)
            rk[e] += (v < ek[e] || (v == ek[e] && src < int(j) + e * int(TPR))) ? 1u : 0u;
      }
      // a column a list dropped has a key at least that list's last one
      float lmin = INFINITY;
#pragma unroll
      for (int l = 0; l < int(kTcLists); ++l)
      {
         const int src = l * KD + KD - 1;
         lmin = fminf(lmin, __shfl_sync(gmask, ek[src / int(TPR)], src % int(TPR), TPR));
      }
#pragma unroll
      for (int e = 0; e < EPL; ++e)
         if (rk[e] < uint32_t(KP))
            s_slot[grp][rk[e]] = make_uint2(__float_as_uint(ek[e]), ec[e]);
      __syncwarp(gmask);
      const uint2 mine = s_slot[grp][j];
      __syncwarp(gmask);
      const float key = __uint_as_float(mine.x);
      const float kk = __shfl_sync(gmask, key, k - 1u, TPR);      // k-th merged key
      const float klast = __shfl_sync(gmask, key, TPR - 1u, TPR); // KP-th merged key

      const double qn = (double)__ldg(p.xnorm + row);
      const double ahi = sqrt(qn * (1.0 + p.gd));
      // |key - (||b||^2 - 2 a.b)| <= bound for every column of this row
      const double bound =
          (p.c1 * ahi * bmax + p.c2 * bmax * bmax + p.c3 * inv_s * (ahi + bmax) + p.c4 * inv_s * inv_s) *
          (1.0 + 1.0 / 1024.0);
      // 2. a candidate whose smallest possible reference distance exceeds the largest
      // possible one of the k-th candidate cannot enter the top-k: it is not reranked
      const double khi = (double)kk + fabs((double)kk) * pk;
      const double lim = (khi + qn * (1.0 + p.gd) + bound) * (1.0 + p.gref);
      const double a2lo = qn * (1.0 - p.gd);
      const double kc = (double)key;
      const double lo = fmax(0.0, kc - fabs(kc) * pk + a2lo - bound) * (1.0 - p.gref);
      float D = INFINITY;
      const bool need = !(lo > lim) && mine.y < p.n; // a column outside the matrix is never read
      if constexpr (STAGED)
      {
         if (__any_sync(gmask, need))
         {
            const float *qv = p.X + size_t(row) * p.d;
            const uint32_t crow = need ? mine.y : 0xFFFFFFFFu;
            const float Dv = w16 ? ref_l2_staged<16, TPR>(qv, p.X, p.d, crow, stage, j, gmask)
                                 : ref_l2_staged<4, TPR>(qv, p.X, p.d, crow, stage, j, gmask);
            if (need)
               D = Dv;
         }
      }
      else if (need)
      {
         const float *qv = p.X + size_t(row) * p.d;
         const float *xv = p.X + size_t(mine.y) * p.d;
         D = vec4 ? ref_l2<true>(qv, xv, p.d) : ref_l2<false>(qv, xv, p.d);
      }
      const uint32_t id = D != INFINITY ? mine.y : 0xFFFFFFFFu; // not reranked: an empty slot
      // 3. rank of (D, id) among the row's candidates, ties by lane; the first k are the row
      uint32_t orank = 0;
#pragma unroll
      for (int src = 0; src < int(TPR); ++src)
      {
         const float d2 = __shfl_sync(gmask, D, src, TPR);
         const uint32_t i2 = __shfl_sync(gmask, id, src, TPR);
         orank += (pair_less(d2, i2, D, id) || (d2 == D && i2 == id && src < int(j))) ? 1u : 0u;
      }
      if (orank < k)
      {
         p.out_ids[size_t(row) * k + orank] = id;
         if (p.out_dists)
            p.out_dists[size_t(row) * k + orank] = D;
      }
      // 4. certificate: every column outside the merged list has key >= T = min(KP-th
      // merged key, every list's last key) (up to the packing tolerance), hence true
      // squared distance >= ||a||^2 + T - bound and reference distance >= that *
      // (1 - gref); above the k-th exact distance, no excluded column can enter the
      // top-k.  With at most KD columns no list dropped any.
      const uint32_t at_k = __ballot_sync(gmask, orank == k - 1u) >> (TPR == 32u ? 0u : (tid & 16u));
      const float dk = __shfl_sync(gmask, D, __ffs(at_k) - 1, TPR);
      bool cert = !exact_only;
      if (cert && total > uint32_t(KD))
      {
         const double Tp = (double)fminf(klast, lmin);
         const double T = Tp - fabs(Tp) * pk;
         const double lhs = (a2lo + T - bound) * (1.0 - p.gref);
         cert = lhs > (double)dk;
      }
      if (j == 0)
      {
         if (!cert)
         {
            const uint32_t pos = atomicAdd(p.fb_count, 1u);
            p.fb_rows[pos] = row;
            p.fb_items[pos] = blockIdx.x + p.item_offset;
            ++n_fail;
         }
         else
            ++n_cert;
      }
   }
   if (j == 0)
   {
      if (n_cert)
         atomicAdd(&s_cnt[0], (unsigned long long)n_cert);
      if (n_fail)
         atomicAdd(&s_cnt[1], (unsigned long long)n_fail);
   }
   __syncthreads();
   if (tid == 0)
   {
      if (s_cnt[0])
         atomicAdd(&p.counters[0], s_cnt[0]);
      if (s_cnt[1])
         atomicAdd(&p.counters[1], s_cnt[1]);
   }
}

template <int KP, int MODE>
cudaError_t launch_tc_t(const TcMaps &maps, const TcParams &p, uint32_t grid, cudaStream_t s)
{
   const TcLayout L = tc_layout(p.dp, MODE >= 1, KP);
   if (L.stages < (MODE == 2 ? 4u : 2u))
      return cudaErrorInvalidValue;
   const size_t smem = L.total + 1024;
   cudaError_t e = cudaFuncSetAttribute(tc_kernel<KP, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
   if (e != cudaSuccess)
      return e;
   tc_kernel<KP, MODE><<<grid, kTcThreads, smem, s>>>(maps, p);
   return cudaGetLastError();
}

template <int KP>
cudaError_t launch_tc_kp(const TcMaps &maps, const TcParams &p, uint32_t grid, cudaStream_t s)
{
   if (p.dp <= 2u * kChunkK)
      return launch_tc_t<KP, 2>(maps, p, grid, s);
   if (tc_a_resident(p.dp))
      return launch_tc_t<KP, 1>(maps, p, grid, s);
   return launch_tc_t<KP, 0>(maps, p, grid, s);
}

template <int KMAX>
cudaError_t launch_exact_t(const ExactParams &p, uint32_t grid, cudaStream_t s)
{
   if (p.warp_per_row && KMAX <= 16)
   {
      // eight rows per block
      const uint32_t g = p.count_dev ? grid : std::max(1u, std::min(grid, (p.count_host + 7u) / 8u));
      if ((p.d & 3u) == 0)
         exact_rows_warp_kernel<KMAX <= 16 ? KMAX : 16, true><<<g, 256, 0, s>>>(p);
      else
         exact_rows_warp_kernel<KMAX <= 16 ? KMAX : 16, false><<<g, 256, 0, s>>>(p);
      return cudaGetLastError();
   }
   if (KMAX <= 64 && p.d <= kExMaxDim) // (lists of 128 per lane spill either way)
   {
      const size_t smem = (8u * kExWarpFloats + p.d) * sizeof(float);
      const bool w16 = (p.d & 3u) == 0 && reinterpret_cast<uintptr_t>(p.X) % 16u == 0;
      auto kern = w16 ? exact_rows_staged_kernel<KMAX, 16> : exact_rows_staged_kernel<KMAX, 4>;
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess)
         return e;
      kern<<<grid, 256, smem, s>>>(p);
      return cudaGetLastError();
   }
   if ((p.d & 3u) == 0)
      exact_rows_kernel<KMAX, true><<<grid, 256, 0, s>>>(p);
   else
      exact_rows_kernel<KMAX, false><<<grid, 256, 0, s>>>(p);
   return cudaGetLastError();
}

} // namespace

int tc_candidates_for_k(uint32_t k)
{
   // 16 entries up to k = 8, else 32: the certificate needs slack past k, more of it
   // for larger k and high-dimensional data (configuration 3, k = 16, d = 960: with 24
   // entries 0.47 % of rows fail and their exact rescan costs 3x the prefilter; with 32,
   // none fail)
   if (k == 0 || k > kTcMaxK)
      return 0;
   return k <= 8 ? 16 : 32;
}

uint32_t tc_operand_cols(uint32_t d)
{
   const uint32_t dp = (d + 15u) / 16u * 16u;
   return dp < kChunkK ? kChunkK : dp;
}

bool tc_a_resident(uint32_t dp) { return (dp + kChunkK - 1) / kChunkK <= kASlots; }

size_t tc_smem_bytes(uint32_t dp, uint32_t k)
{
   return tc_layout(dp, tc_a_resident(dp), (uint32_t)tc_candidates_for_k(k)).total + 1024;
}

void tc_certificate_constants(uint32_t d, uint32_t dp, RerankParams &p)
{
   const double u24 = std::ldexp(1.0, -24);
   // relative error of the fp16 operand (11-bit significand, nearest-even; the scale
   // by a power of two is exact) against the exact centred value, for elements in
   // the normal fp16 range
   const double ur = u24 + std::ldexp(1.0, -11) * (1.0 + u24);
   // fp16 x fp16 products are exact in fp32; the tensor-core fp32 accumulation over dp
   // products is taken as one 2^-23 relative error per product plus 16
   const double cacc = (double(dp) + 16.0) * std::ldexp(1.0, -23);
   p.c1 = 4.0 * ur + 2.0 * ur * ur + 2.0 * cacc * (1.0 + ur) * (1.0 + ur) + 2.0 * std::ldexp(1.0, -23);
   p.c2 = (double(d) + 4.0) * u24 + std::ldexp(1.0, -23) + u24;
   // elements below the normal fp16 range carry an absolute error <= 2^-25 in scaled
   // units: the key moves by at most 2 (1+ur) 2^-25 sqrt(d) (|a| + |b|) / s plus
   // 2 d 2^-50 / s^2, and the accumulation adds its relative share of both
   p.c3 = 2.0 * (1.0 + ur) * std::ldexp(1.0, -25) * std::sqrt(double(d)) * (1.0 + cacc) * (1.0 + std::ldexp(1.0, -20));
   p.c4 = 2.0 * double(d) * std::ldexp(1.0, -50) * (1.0 + cacc) * (1.0 + std::ldexp(1.0, -20));
   p.gd = (double(d) + 6.0) * u24;
   p.gref = (double(d) + 8.0) * u24;
}

namespace
{
// Zeroes the column statistics when *gate is non-zero (before the full pass).
__global__ void zero_stats_kernel(double *__restrict__ sums, uint32_t *__restrict__ range, uint32_t d,
                                  const uint32_t *__restrict__ gate)
{
   if (*gate == 0u)
      return;
   for (uint32_t j = threadIdx.x; j < d; j += blockDim.x)
   {
      sums[j] = 0.0;
      range[2 * j] = range[2 * j + 1] = 0u;
   }
}

cudaError_t colsum_pass(const float *X, uint32_t n, uint32_t d, uint32_t stride, double *sums, uint32_t *range,
                        const uint32_t *gate, cudaStream_t s)
{
   const uint32_t rows = (n + stride - 1) / stride;
   const uint32_t rows_per_block = 256;
   const uint32_t blocks = (rows + rows_per_block - 1) / rows_per_block;
   colsum_kernel<<<blocks, d < 256 ? ((d + 31) / 32) * 32 : 256, 0, s>>>(X, rows, d, sums, range, rows_per_block,
                                                                         stride, gate);
   return cudaGetLastError();
}

cudaError_t center_pass(const float *X, const float *mean, const OperandScale *scale, uint32_t n, uint32_t d,
                        uint32_t dp, uint16_t *Xh, float *xnorm, uint32_t *saturated, const uint32_t *gate,
                        cudaStream_t s)
{
   const size_t smem = sizeof(float) * dp;
   const bool vec = d % 4u == 0 && reinterpret_cast<uintptr_t>(X) % 16u == 0;
   auto kern = vec ? center4_kernel : center_kernel;
   if (smem > 48 * 1024)
   {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess)
         return e;
   }
   const uint32_t rows_per_block = vec ? 32u : 8u; // 8 warps of 4 rows, or of 1
   const uint32_t blocks = std::min<uint32_t>((n + rows_per_block - 1) / rows_per_block, 148 * 16);
   kern<<<blocks, 256, smem, s>>>(X, mean, scale, n, d, dp, reinterpret_cast<__half *>(Xh), xnorm, saturated, gate);
   return cudaGetLastError();
}
} // namespace

uint32_t operand_sample_stride(uint32_t n) { return n > (1u << 18) ? n / (1u << 16) : 1u; }

cudaError_t launch_prepare_operand(const float *X, uint32_t n, uint32_t d, uint32_t dp, double *sums, uint32_t *range,
                                   float *mean, OperandScale *scale, uint16_t *Xh, float *xnorm, uint32_t *flag,
                                   cudaStream_t s)
{
   if (n == 0)
      return cudaErrorInvalidValue;
   cudaError_t e;
   if ((e = cudaMemsetAsync(sums, 0, sizeof(double) * d, s)) != cudaSuccess ||
       (e = cudaMemsetAsync(range, 0, sizeof(uint32_t) * 2 * d, s)) != cudaSuccess ||
       (e = cudaMemsetAsync(flag, 0, sizeof(uint32_t), s)) != cudaSuccess)
      return e;
   const uint32_t stride = operand_sample_stride(n);
   const uint32_t rows = (n + stride - 1) / stride;
   if ((e = colsum_pass(X, n, d, stride, sums, range, nullptr, s)) != cudaSuccess)
      return e;
   scale_kernel<<<1, 256, 0, s>>>(sums, range, rows, d, mean, scale, stride > 1 ? 2 : 0, nullptr);
   if ((e = cudaGetLastError()) != cudaSuccess)
      return e;
   if ((e = center_pass(X, mean, scale, n, d, dp, Xh, xnorm, stride > 1 ? flag : nullptr, nullptr, s)) !=
       cudaSuccess)
      return e;
   if (stride == 1)
      return cudaSuccess; // every row was in the statistics: nothing can saturate
   // an element outside the sample's reach: the exact full pass, gated on the flag
   zero_stats_kernel<<<1, 256, 0, s>>>(sums, range, d, flag);
   if ((e = cudaGetLastError()) != cudaSuccess || (e = colsum_pass(X, n, d, 1, sums, range, flag, s)) != cudaSuccess)
      return e;
   scale_kernel<<<1, 256, 0, s>>>(sums, range, n, d, mean, scale, 0, flag);
   if ((e = cudaGetLastError()) != cudaSuccess)
      return e;
   return center_pass(X, mean, scale, n, d, dp, Xh, xnorm, nullptr, flag, s);
}

cudaError_t launch_group_maxnorm(const float *xnorm, const uint32_t *chunks, uint32_t nchunks, uint32_t G, float *out,
                                 cudaStream_t s)
{
   cudaError_t e = cudaMemsetAsync(out, 0, sizeof(float) * (size_t(G) + 1), s);
   if (e != cudaSuccess || nchunks == 0)
      return e;
   const uint32_t blocks = std::min<uint32_t>((nchunks + 7) / 8, 148 * 16);
   group_maxnorm_kernel<<<blocks, 256, 0, s>>>(xnorm, chunks, nchunks, out);
   return cudaGetLastError();
}

cudaError_t launch_fill_empty(const RowRange *ranges, uint32_t nranges, uint32_t k, uint32_t *ids, float *dists,
                              cudaStream_t s)
{
   if (nranges == 0)
      return cudaSuccess;
   fill_empty_kernel<<<nranges, 256, 0, s>>>(ranges, k, ids, dists);
   return cudaGetLastError();
}

cudaError_t launch_gather_rows(const CopyRange *ranges, uint32_t nranges, uint32_t k, const uint32_t *ids,
                               const float *dists, uint32_t *out_ids, float *out_dists, cudaStream_t s)
{
   if (nranges == 0)
      return cudaSuccess;
   gather_rows_kernel<<<nranges, 256, 0, s>>>(ranges, k, ids, dists, out_ids, out_dists);
   return cudaGetLastError();
}

cudaError_t launch_merge_pass(const uint32_t *pass_ids, const float *pass_dists, uint32_t rows, uint32_t k,
                              uint32_t base_src, uint32_t split, uint32_t base_tgt, uint32_t *ids, float *dists,
                              cudaStream_t s)
{
   if (rows == 0)
      return cudaSuccess;
   if (k > kMergeMaxK)
      return cudaErrorInvalidValue;
   const uint32_t blocks = std::min<uint32_t>((rows + 255) / 256, 148 * 8);
   if (k <= 8)
      merge_pass_kernel<8><<<blocks, 256, 0, s>>>(pass_ids, pass_dists, rows, k, base_src, split, base_tgt, ids, dists);
   else if (k <= 32)
      merge_pass_kernel<32><<<blocks, 256, 0, s>>>(pass_ids, pass_dists, rows, k, base_src, split, base_tgt, ids, dists);
   else
      merge_pass_kernel<kMergeMaxK>
          <<<blocks, 256, 0, s>>>(pass_ids, pass_dists, rows, k, base_src, split, base_tgt, ids, dists);
   return cudaGetLastError();
}

cudaError_t launch_scatter_rows(const CopyRange *ranges, uint32_t nranges, uint32_t k, const uint32_t *ids,
                                const float *dists, uint32_t *out_ids, float *out_dists, cudaStream_t s)
{
   if (nranges == 0)
      return cudaSuccess;
   scatter_rows_kernel<<<nranges, 256, 0, s>>>(ranges, k, ids, dists, out_ids, out_dists);
   return cudaGetLastError();
}

cudaError_t launch_exact(const ExactParams &p, uint32_t grid, cudaStream_t s)
{
   if (p.k <= 8)
      return launch_exact_t<8>(p, grid, s);
   if (p.k <= 16)
      return launch_exact_t<16>(p, grid, s);
   if (p.k <= 32)
      return launch_exact_t<32>(p, grid, s);
   if (p.k <= 64)
      return launch_exact_t<64>(p, grid, s);
   return launch_exact_t<128>(p, grid, s);
}

cudaError_t launch_tc(const TcMaps &maps, const TcParams &p, uint32_t kp, uint32_t grid, cudaStream_t s)
{
   if (kp == 16)
      return launch_tc_kp<16>(maps, p, grid, s);
   if (kp == 32)
      return launch_tc_kp<32>(maps, p, grid, s);
   return cudaErrorInvalidValue;
}

cudaError_t launch_rerank(const RerankParams &p, uint32_t kp, uint32_t num_items, cudaStream_t s)
{
   if (num_items == 0)
      return cudaSuccess;
   if (kp != 16 && kp != 32)
      return cudaErrorInvalidValue;
   // wide rows (d > 256): the candidate rows staged through shared memory (config 3,
   // d = 960: 13 vs 30 ms); narrow ones gather them from global memory (config 2: 0.96
   // vs 1.22 ms staged)
   if (p.d > 256)
   {
      const size_t smem = size_t(256) * 2 * kStLd * sizeof(float);
      auto kern = kp == 16 ? rerank_kernel<16, true> : rerank_kernel<32, true>;
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess)
         return e;
      kern<<<num_items, 256, smem, s>>>(p);
   }
   else if (kp == 16)
      rerank_kernel<16, false><<<num_items, 256, 0, s>>>(p);
   else
      rerank_kernel<32, false><<<num_items, 256, 0, s>>>(p);
   return cudaGetLastError();
}

} // namespace ungx
