// Device code of the B200 cross-edge builder (sm_100a).
//
//   colsum / center     resident operand build (a4): mean, centred + TF32-rounded
//                       copy padded to 32 columns, fp32 row norms.
//   exact_rows_kernel   CUDA-core exact scan, squared L2 in the reference's fp32
//                       summation order (FloatL2DistanceHandler::compute,
//                       UNG/codes/src/distance.cpp:34-91) and its (distance, id)
//                       queue order (UNG/codes/include/search_queue.h:20-22).
//                       Route EXACT, and the rescan of rows whose certificate failed.
//   tc_kernel           the hot path: persistent CTAs pull source-centric work items;
//                       TMA stages 128-row source tiles and target tiles through a
//                       4-stage shared-memory ring; one thread issues tcgen05.mma
//                       kind::tf32 into a double-buffered TMEM accumulator; eight
//                       epilogue warps read TMEM rows (one thread per source row),
//                       turn dot products into ||x||^2 - 2 q.x keys and keep a
//                       register top-KP per row; at the end of the item the KP
//                       candidates are re-ranked with the exact reference distance
//                       and a rounding-error certificate proves that no excluded
//                       column could enter the top-k.  Rows whose certificate fails
//                       are queued for exact_rows_kernel.  No distance matrix is ever
//                       written to global memory.
#include <cfloat>
#include <cmath>

#include "kernels.h"
#include "ptx.cuh"

namespace ungx
{
namespace
{
constexpr uint32_t kTcThreads = 320; // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr uint32_t kStages = 4;
constexpr uint32_t kItemSlots = 2;
constexpr uint32_t kAChunk = 128 * 128; // 128 rows x 32 fp32
constexpr uint32_t kBChunk = 256 * 128; // up to 256 rows x 32 fp32
constexpr uint32_t kNoItem = 0xFFFFFFFFu;
constexpr int kPushBuf = 4; // per-lane buffer of candidates awaiting a merge into the sorted list
// Limit of the waits that retire work already in flight before the CTA exits
// (independent of the configurable pipeline wait limit, which tests set tiny).
constexpr uint64_t kDrainWaitNs = 2000000000ull;

struct TcLayout
{
   uint32_t a_off, a_bytes, stage_off, stage_bytes, merge_off, norm_off, bar_off, misc_off, total;
};

__host__ __device__ inline TcLayout tc_layout(uint32_t dp, bool a_res, uint32_t kp)
{
   TcLayout L;
   L.a_off = 0;
   L.a_bytes = a_res ? (dp / 32) * kAChunk : 0;
   L.stage_off = L.a_bytes;
   L.stage_bytes = a_res ? kBChunk : kAChunk + kBChunk;
   L.merge_off = L.stage_off + kStages * L.stage_bytes;
   L.norm_off = L.merge_off + 128 * kp * 8;
   L.bar_off = L.norm_off + 8 * 32 * 4;
   L.misc_off = L.bar_off + 32 * 8;
   L.total = L.misc_off + 64;
   return L;
}

__device__ __forceinline__ float tf32_rne(float v)
{
   uint32_t u = __float_as_uint(v);
   if ((u & 0x7f800000u) == 0x7f800000u)
      return v;
   u += 0xFFFu + ((u >> 13) & 1u);
   return __uint_as_float(u & 0xFFFFE000u);
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

__device__ __forceinline__ bool pair_less(float d0, uint32_t i0, float d1, uint32_t i1)
{
   return d0 < d1 || (d0 == d1 && i0 < i1);
}

// Sorted insert of (d, id) into an ascending (distance, id) list; caller checked
// that (d, id) precedes the last entry.  Static indices only (stays in registers).
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

// Same on prefilter keys alone (their order among equal keys does not matter).
template <int K>
__device__ __forceinline__ void insert_key(float (&kd)[K], uint32_t (&ki)[K], float d, uint32_t id)
{
#pragma unroll
   for (int i = K - 1; i > 0; --i)
   {
      const bool prev = d < kd[i - 1];
      const bool here = d < kd[i];
      const float nd = prev ? kd[i - 1] : (here ? d : kd[i]);
      const uint32_t ni = prev ? ki[i - 1] : (here ? id : ki[i]);
      kd[i] = nd;
      ki[i] = ni;
   }
   if (d < kd[0])
   {
      kd[0] = d;
      ki[0] = id;
   }
}

// ------------------------------------------------------------------ prep
__global__ void colsum_kernel(const float *__restrict__ X, uint32_t n, uint32_t d, double *__restrict__ sums,
                              uint32_t rows_per_block)
{
   const uint64_t r0 = uint64_t(blockIdx.x) * rows_per_block;
   const uint64_t r1 = (r0 + rows_per_block < n) ? r0 + rows_per_block : uint64_t(n);
   for (uint32_t j = threadIdx.x; j < d; j += blockDim.x)
   {
      double acc = 0.0;
      for (uint64_t r = r0; r < r1; ++r)
         acc += (double)X[r * d + j];
      atomicAdd(&sums[j], acc);
   }
}

__global__ void center_kernel(const float *__restrict__ X, const double *__restrict__ sums, uint32_t n,
                              uint32_t d, uint32_t dp, float *__restrict__ mean, float *__restrict__ Xp,
                              float *__restrict__ xnorm)
{
   extern __shared__ float s_mean[];
   for (uint32_t j = threadIdx.x; j < d; j += blockDim.x)
      s_mean[j] = (float)(sums[j] / (double)n);
   __syncthreads();
   if (blockIdx.x == 0)
      for (uint32_t j = threadIdx.x; j < d; j += blockDim.x)
         mean[j] = s_mean[j];
   const uint32_t lane = threadIdx.x & 31;
   const uint64_t warps = (uint64_t(gridDim.x) * blockDim.x) >> 5;
   for (uint64_t r = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < n; r += warps)
   {
      float acc = 0.f;
      for (uint32_t j = lane; j < dp; j += 32)
      {
         float v = 0.f;
         if (j < d)
            v = __fsub_rn(X[r * d + j], s_mean[j]);
         Xp[r * dp + j] = tf32_rne(v);
         acc = __fmaf_rn(v, v, acc);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1)
         acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0)
         xnorm[r] = acc;
   }
}

__global__ void group_maxnorm_kernel(const float *__restrict__ xnorm, const uint32_t *__restrict__ ranges, uint32_t G,
                                     float *__restrict__ out)
{
   const uint32_t lane = threadIdx.x & 31;
   const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
   for (uint32_t g = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; g <= G; g += warps)
   {
      float m = 0.f;
      if (g > 0)
         for (uint32_t r = ranges[2 * g] + lane; r < ranges[2 * g + 1]; r += 32)
            m = fmaxf(m, xnorm[r]);
#pragma unroll
      for (int o = 16; o; o >>= 1)
         m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0)
         out[g] = m;
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

// ------------------------------------------------------------------ exact scan
// One warp per row: lanes stride over the row's candidate columns keeping a sorted
// top-KMAX each, then k rounds of a warp arg-min by (distance, id) emit the result.
template <int KMAX, bool VEC4>
__global__ void __launch_bounds__(256) exact_rows_kernel(const ExactParams p)
{
   const uint32_t count = p.count_dev ? *(volatile const uint32_t *)p.count_dev : p.count_host;
   const uint32_t lane = threadIdx.x & 31;
   const uint32_t nw = (gridDim.x * blockDim.x) >> 5;
   for (uint32_t w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < count; w += nw)
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
            p.out_ids[size_t(row) * p.k + o] = mi;
            if (p.out_dists)
               p.out_dists[size_t(row) * p.k + o] = (mi == 0xFFFFFFFFu) ? INFINITY : md;
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

__device__ __forceinline__ uint32_t box_index(uint32_t valid)
{
   return valid <= 16 ? 0u : valid <= 32 ? 1u : valid <= 64 ? 2u : valid <= 128 ? 3u : 4u;
}

template <int KP, bool A_RES>
__global__ void __launch_bounds__(kTcThreads, 1) tc_kernel(const __grid_constant__ TcMaps maps, const TcParams p)
{
   extern __shared__ uint8_t smem_raw[];
   const uint32_t raw_u32 = ptx::smem_u32(smem_raw);
   uint8_t *smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
   const TcLayout L = tc_layout(p.dp, A_RES, KP);
   uint8_t *sA = smem + L.a_off;
   uint8_t *sStage = smem + L.stage_off;
   float2 *sMerge = reinterpret_cast<float2 *>(smem + L.merge_off);
   float *sNorm = reinterpret_cast<float *>(smem + L.norm_off);
   uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bar_off);
   uint64_t *full = bars;
   uint64_t *empty = bars + kStages;
   uint64_t *acc_full = bars + 2 * kStages;
   uint64_t *acc_empty = acc_full + 2;
   uint64_t *a_full = acc_empty + 2;
   uint64_t *a_empty = a_full + 1;
   uint64_t *item_full = a_empty + 1;
   uint64_t *item_empty = item_full + kItemSlots;
   uint64_t *done_bar = item_empty + kItemSlots;
   uint64_t *merge_ready = done_bar + 1; // [4] per TMEM quarter: half 1 published its list
   uint64_t *merge_done = merge_ready + 4; // [4] per TMEM quarter: half 0 consumed it
   volatile uint32_t *item_slot = reinterpret_cast<volatile uint32_t *>(smem + L.misc_off);
   uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L.misc_off + 16);
   volatile int *abort_word = reinterpret_cast<volatile int *>(smem + L.misc_off + 32);

   const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
   const uint32_t nch = p.dp / 32;
   const uint64_t tmo = p.timeout_ns;

   if (threadIdx.x == 0)
   {
      for (uint32_t s = 0; s < kStages; ++s)
      {
         ptx::mbar_init(&full[s], 1);
         ptx::mbar_init(&empty[s], 1);
      }
      for (uint32_t b = 0; b < 2; ++b)
      {
         ptx::mbar_init(&acc_full[b], 1);
         ptx::mbar_init(&acc_empty[b], 8);
      }
      ptx::mbar_init(a_full, 1);
      ptx::mbar_init(a_empty, 1);
      for (uint32_t s = 0; s < kItemSlots; ++s)
      {
         ptx::mbar_init(&item_full[s], 1);
         ptx::mbar_init(&item_empty[s], 9); // MMA thread + 8 epilogue warps
      }
      ptx::mbar_init(done_bar, 1);
      for (uint32_t qq = 0; qq < 4; ++qq)
      {
         ptx::mbar_init(&merge_ready[qq], 1);
         ptx::mbar_init(&merge_done[qq], 1);
      }
      *abort_word = 0;
      ptx::fence_mbar_init();
   }
   if (warp == 0 && lane == 0)
   {
      ptx::prefetch_tmap(&maps.a);
      for (int i = 0; i < 5; ++i)
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
      if (lane == 0)
      {
         uint32_t it = 0, iseq = 0, aseq = 0;
         bool ok = true;
         for (;;)
         {
            const uint32_t idx = atomicAdd(p.item_counter, 1u);
            const uint32_t slot = iseq % kItemSlots;
            if (!ptx::mbar_wait(&item_empty[slot], ((iseq / kItemSlots) & 1u) ^ 1u, abort_word, tmo))
            {
               ok = false;
               break;
            }
            item_slot[slot] = idx < p.num_items ? idx : kNoItem;
            ptx::mbar_arrive(&item_full[slot]);
            ++iseq;
            if (idx >= p.num_items)
               break;
            const WorkItem w = p.items[idx];
            if (A_RES)
            {
               if (!ptx::mbar_wait(a_empty, (aseq & 1u) ^ 1u, abort_word, tmo))
               {
                  ok = false;
                  break;
               }
               ptx::mbar_arrive_expect_tx(a_full, nch * kAChunk);
               for (uint32_t c = 0; c < nch; ++c)
                  ptx::tma_load_2d(sA + c * kAChunk, &maps.a, a_full, int32_t(c * 32), int32_t(w.row_begin));
               ++aseq;
            }
            for (uint32_t s = 0; s < w.seg_count && ok; ++s)
            {
               const Segment sg = p.segs[w.seg_begin + s];
               for (uint32_t t0 = 0; t0 < sg.x_count && ok; t0 += 256)
               {
                  const uint32_t valid = min(256u, sg.x_count - t0);
                  const uint32_t bix = box_index(valid);
                  const uint32_t brows = 16u << bix;
                  for (uint32_t c = 0; c < nch; ++c)
                  {
                     const uint32_t st = it % kStages;
                     if (!ptx::mbar_wait(&empty[st], ((it / kStages) & 1u) ^ 1u, abort_word, tmo))
                     {
                        ok = false;
                        break;
                     }
                     uint8_t *dst = sStage + st * L.stage_bytes;
                     ptx::mbar_arrive_expect_tx(&full[st], (A_RES ? 0u : kAChunk) + brows * 128u);
                     if (!A_RES)
                        ptx::tma_load_2d(dst, &maps.a, &full[st], int32_t(c * 32), int32_t(w.row_begin));
                     ptx::tma_load_2d(dst + (A_RES ? 0u : kAChunk), &maps.b[bix], &full[st], int32_t(c * 32),
                                      int32_t(sg.x_begin + t0));
                     ++it;
                  }
               }
            }
            if (!ok)
               break;
         }
         if (!ok)
         {
            raise_abort(abort_word, p.status, UNGX_ERR_TIMEOUT);
            // drain: every load already issued must land before the CTA exits
            for (uint32_t st = 0; st < kStages; ++st)
            {
               const uint32_t issued = it / kStages + (st < it % kStages ? 1u : 0u);
               if (issued)
                  ptx::mbar_wait(&full[st], (issued - 1) & 1u, nullptr, kDrainWaitNs);
            }
            if (A_RES && aseq)
               ptx::mbar_wait(a_full, (aseq - 1) & 1u, nullptr, kDrainWaitNs);
         }
      }
      __syncwarp();
   }
   else if (warp == 1)
   {
      // ------------------------------------------------ MMA issuer
      if (lane == 0)
      {
         uint32_t it = 0, tseq = 0, iseq = 0, aseq = 0;
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
            const WorkItem w = p.items[idx];
            if (A_RES && !ptx::mbar_wait(a_full, aseq & 1u, abort_word, tmo))
            {
               ok = false;
               break;
            }
            for (uint32_t s = 0; s < w.seg_count && ok; ++s)
            {
               const Segment sg = p.segs[w.seg_begin + s];
               for (uint32_t t0 = 0; t0 < sg.x_count && ok; t0 += 256)
               {
                  const uint32_t valid = min(256u, sg.x_count - t0);
                  const uint32_t b = tseq & 1u;
                  if (!ptx::mbar_wait(&acc_empty[b], ((tseq >> 1) & 1u) ^ 1u, abort_word, tmo))
                  {
                     ok = false;
                     break;
                  }
                  ptx::tc_fence_after();
                  const uint32_t N = min(256u, (valid + 15u) & ~15u);
                  const uint32_t idesc = ptx::idesc_tf32(128, N);
                  const uint32_t dt = tmem_base + b * 256u;
                  for (uint32_t c = 0; c < nch; ++c)
                  {
                     const uint32_t st = it % kStages;
                     if (!ptx::mbar_wait(&full[st], (it / kStages) & 1u, abort_word, tmo))
                     {
                        ok = false;
                        break;
                     }
                     ptx::tc_fence_after();
                     uint8_t *stage = sStage + st * L.stage_bytes;
                     const uint64_t ad = ptx::sdesc_k_sw128(ptx::smem_u32(A_RES ? sA + c * kAChunk : stage));
                     const uint64_t bd = ptx::sdesc_k_sw128(ptx::smem_u32(stage + (A_RES ? 0u : kAChunk)));
#pragma unroll
                     for (uint32_t ks = 0; ks < 4; ++ks) // 4 x K=8 per 32-column chunk (+32 B each)
                        ptx::mma_tf32(dt, ad + 2u * ks, bd + 2u * ks, idesc, (c | ks) != 0u);
                     ptx::mma_commit(&empty[st]);
                     ++it;
                  }
                  if (!ok)
                     break;
                  ptx::mma_commit(&acc_full[b]);
                  ++tseq;
               }
            }
            if (!ok)
               break;
            if (A_RES)
            {
               ptx::mma_commit(a_empty);
               ++aseq;
            }
            ptx::mbar_arrive(&item_empty[slot]);
         }
         if (!ok)
            raise_abort(abort_word, p.status, UNGX_ERR_TIMEOUT);
         // every MMA issued by this thread (and its arrivals) completes before teardown
         ptx::mma_commit(done_bar);
         ptx::mbar_wait(done_bar, 0, nullptr, kDrainWaitNs);
      }
      __syncwarp();
   }
   else
   {
      // ------------------------------------------------ epilogue: one thread per source row
      const uint32_t q = warp & 3u;          // TMEM lane quarter this warp may read
      const uint32_t h = (warp - 2u) >> 2;   // which half of each tile's 32-column chunks
      const uint32_t r = q * 32u + lane;     // row inside the work item
      float *nrm = sNorm + (warp - 2u) * 32u;
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
         const WorkItem w = p.items[idx];
         const bool row_ok = r < w.row_count;
         const bool warp_ok = q * 32u < w.row_count;
         // Sorted candidate list (key, col) of the KP smallest keys seen, and a
         // small unsorted buffer of keys that beat the list's threshold as it was
         // at the last flush.  Pushes are branch-free; the buffer is merged into the
         // list only when some lane of the warp fills it, so all lanes merge together.
         float key[KP];
         uint32_t col[KP];
#pragma unroll
         for (int i = 0; i < KP; ++i)
         {
            key[i] = INFINITY;
            col[i] = 0xFFFFFFFFu;
         }
         float bk[kPushBuf];
         uint32_t bc[kPushBuf];
#pragma unroll
         for (int i = 0; i < kPushBuf; ++i)
         {
            bk[i] = INFINITY;
            bc[i] = 0xFFFFFFFFu;
         }
         uint32_t nb = 0;
         float thr = row_ok ? INFINITY : -INFINITY; // rows past the item never take candidates
         auto flush = [&]() {
#pragma unroll
            for (int i = 0; i < kPushBuf; ++i)
            {
               insert_key<KP>(key, col, bk[i], bc[i]); // +inf entries leave the list unchanged
               bk[i] = INFINITY;
            }
            nb = 0;
            thr = row_ok ? key[KP - 1] : -INFINITY;
         };
         float maxn2 = 0.f;
         uint32_t total = 0;
         for (uint32_t s = 0; s < w.seg_count && ok; ++s)
         {
            const Segment sg = p.segs[w.seg_begin + s];
            maxn2 = fmaxf(maxn2, p.group_maxn2[sg.group_id]);
            total += sg.x_count;
            for (uint32_t t0 = 0; t0 < sg.x_count; t0 += 256)
            {
               const uint32_t valid = min(256u, sg.x_count - t0);
               const uint32_t x0 = sg.x_begin + t0;
               const uint32_t b = tseq & 1u;
               const uint32_t nchunk = (valid + 31u) >> 5;
               // norms of this warp's chunks (j = h, h+2, ...), loaded before the wait
               float nreg[4];
#pragma unroll
               for (uint32_t i = 0; i < 4; ++i)
               {
                  const uint32_t c = (h + 2u * i) * 32u + lane;
                  nreg[i] = c < valid ? __ldg(p.xnorm + x0 + c) : INFINITY;
               }
               if (!ptx::mbar_wait(&acc_full[b], (tseq >> 1) & 1u, abort_word, tmo))
               {
                  ok = false;
                  break;
               }
               ptx::tc_fence_after();
#pragma unroll 1
               for (uint32_t i = 0; i < 4; ++i)
               {
                  const uint32_t j = h + 2u * i;
                  if (j >= nchunk)
                     break;
                  const float nv = i == 0 ? nreg[0] : i == 1 ? nreg[1] : i == 2 ? nreg[2] : nreg[3];
                  __syncwarp();
                  nrm[lane] = nv;
                  __syncwarp();
                  if (!warp_ok)
                     continue;
                  uint32_t v[32];
                  ptx::tmem_ld32(tmem_base + ((q * 32u) << 16) + b * 256u + j * 32u, v);
                  ptx::tmem_wait_ld();
                  const uint32_t cbase = x0 + j * 32u;
#pragma unroll
                  for (int jj = 0; jj < 32; ++jj)
                  {
                     const float kk = __fmaf_rn(-2.0f, __uint_as_float(v[jj]), nrm[jj]);
                     const bool pass = kk < thr;
                     if (__any_sync(0xffffffffu, pass))
                     {
#pragma unroll
                        for (int m = kPushBuf - 1; m > 0; --m)
                        {
                           bk[m] = pass ? bk[m - 1] : bk[m];
                           bc[m] = pass ? bc[m - 1] : bc[m];
                        }
                        bk[0] = pass ? kk : bk[0];
                        bc[0] = pass ? cbase + jj : bc[0];
                        nb += pass ? 1u : 0u;
                        if (__any_sync(0xffffffffu, nb == kPushBuf))
                           flush();
                     }
                  }
               }
               __syncwarp();
               ptx::tc_fence_before();
               __syncwarp();
               if (lane == 0)
                  ptx::mbar_arrive(&acc_empty[b]);
               ++tseq;
            }
         }
         if (!ok)
            break;
         flush();
         // ---- merge the two column halves of each row (bounded mbarrier handshake)
         const uint32_t mseq = iseq - 1; // items this warp has finished before this one
         if (h == 1)
         {
            if (!ptx::mbar_wait(&merge_done[q], (mseq & 1u) ^ 1u, abort_word, tmo))
            {
               ok = false;
               break;
            }
            if (row_ok)
            {
#pragma unroll
               for (int i = 0; i < KP; ++i)
                  sMerge[r * KP + i] = make_float2(key[i], __uint_as_float(col[i]));
            }
            __syncwarp();
            if (lane == 0)
               ptx::mbar_arrive(&merge_ready[q]);
         }
         else if (!ptx::mbar_wait(&merge_ready[q], mseq & 1u, abort_word, tmo))
         {
            ok = false;
            break;
         }
         bool cert = true;
         if (h == 0 && row_ok)
         {
            for (int i = 0; i < KP; ++i)
            {
               const float2 e = sMerge[r * KP + i];
               if (e.x < key[KP - 1])
                  insert_key<KP>(key, col, e.x, __float_as_uint(e.y));
            }
            // ---- exact rerank of the candidates in the reference's arithmetic
            const uint32_t row = w.row_begin + r;
            const uint32_t m = total < uint32_t(KP) ? total : uint32_t(KP);
            uint32_t cl[KP];
#pragma unroll
            for (int i = 0; i < KP; ++i)
               cl[i] = col[i];
            float sd[KP];
            uint32_t si[KP];
#pragma unroll
            for (int i = 0; i < KP; ++i)
            {
               sd[i] = INFINITY;
               si[i] = 0xFFFFFFFFu;
            }
            const float *qv = p.X + size_t(row) * p.d;
            const bool vec4 = (p.d & 3u) == 0;
#pragma unroll 1
            for (uint32_t i = 0; i < m; ++i)
            {
               const uint32_t x = cl[i];
               const float *xv = p.X + size_t(x) * p.d;
               const float D = vec4 ? ref_l2<true>(qv, xv, p.d) : ref_l2<false>(qv, xv, p.d);
               if (pair_less(D, x, sd[KP - 1], si[KP - 1]))
                  insert_pair<KP>(sd, si, D, x);
            }
            // ---- certificate: every column outside the list has key >= T, hence
            // true squared distance >= ||a||^2 + T - bound and reference distance
            // >= that * (1 - gref); if this exceeds the k-th exact distance no
            // excluded column can enter the top-k.
            if (total > uint32_t(KP))
            {
               float dk = INFINITY;
#pragma unroll
               for (int i = 0; i < KP; ++i)
                  if (uint32_t(i) == p.k - 1)
                     dk = sd[i];
               const double T = (double)key[KP - 1];
               const double qn = (double)__ldg(p.xnorm + row);
               const double a2lo = qn * (1.0 - p.gd);
               const double ahi = sqrt(qn * (1.0 + p.gd));
               const double bmax = sqrt((double)maxn2 * (1.0 + p.gd));
               const double bound = (p.c1 * ahi * bmax + p.c2 * bmax * bmax) * (1.0 + 1.0 / 1024.0);
               const double lhs = (a2lo + T - bound) * (1.0 - p.gref);
               cert = lhs > (double)dk;
            }
#pragma unroll
            for (int i = 0; i < KP; ++i)
               if (uint32_t(i) < p.k)
               {
                  p.out_ids[size_t(row) * p.k + i] = si[i];
                  if (p.out_dists)
                     p.out_dists[size_t(row) * p.k + i] = sd[i];
               }
            if (!cert)
            {
               const uint32_t pos = atomicAdd(p.fb_count, 1u);
               p.fb_rows[pos] = row;
               p.fb_items[pos] = idx;
            }
         }
         if (h == 0)
         {
            __syncwarp();
            if (lane == 0)
               ptx::mbar_arrive(&merge_done[q]);
            const uint32_t nrows = __popc(__ballot_sync(0xffffffffu, row_ok));
            const uint32_t nfail = __popc(__ballot_sync(0xffffffffu, row_ok && !cert));
            if (lane == 0)
            {
               if (nrows - nfail)
                  atomicAdd(&p.counters[0], (unsigned long long)(nrows - nfail));
               if (nfail)
                  atomicAdd(&p.counters[1], (unsigned long long)nfail);
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

template <int KP, bool A_RES>
cudaError_t launch_tc_t(const TcMaps &maps, const TcParams &p, uint32_t grid, cudaStream_t s)
{
   const TcLayout L = tc_layout(p.dp, A_RES, KP);
   const size_t smem = L.total + 1024;
   cudaError_t e = cudaFuncSetAttribute(tc_kernel<KP, A_RES>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
   if (e != cudaSuccess)
      return e;
   tc_kernel<KP, A_RES><<<grid, kTcThreads, smem, s>>>(maps, p);
   return cudaGetLastError();
}

template <int KMAX>
cudaError_t launch_exact_t(const ExactParams &p, uint32_t grid, cudaStream_t s)
{
   if ((p.d & 3u) == 0)
      exact_rows_kernel<KMAX, true><<<grid, 256, 0, s>>>(p);
   else
      exact_rows_kernel<KMAX, false><<<grid, 256, 0, s>>>(p);
   return cudaGetLastError();
}

} // namespace

int tc_candidates_for_k(uint32_t k)
{
   // the smallest candidate list with at least two entries of slack past k
   if (k == 0 || k > kTcMaxK)
      return 0;
   return k + 2 <= 8 ? 8 : k + 2 <= 16 ? 16 : k + 2 <= 24 ? 24 : 32;
}

bool tc_a_resident(uint32_t dp) { return dp <= 128; }

size_t tc_smem_bytes(uint32_t dp, uint32_t k)
{
   return tc_layout(dp, tc_a_resident(dp), (uint32_t)tc_candidates_for_k(k)).total + 1024;
}

void tc_certificate_constants(uint32_t d, uint32_t dp, TcParams &p)
{
   const double u24 = std::ldexp(1.0, -24);
   // relative error of a TF32-rounded centred value against the exact centred value
   const double ur = u24 + std::ldexp(1.0, -11) * (1.0 + u24);
   // tensor-core fp32 accumulation, taken 4x looser than one rounding per K=8 step
   const double cacc = (double(dp) / 2.0 + 8.0) * std::ldexp(1.0, -22);
   p.c1 = 4.0 * ur + 2.0 * ur * ur + 2.0 * cacc * (1.0 + ur) * (1.0 + ur) + 2.0 * std::ldexp(1.0, -23);
   p.c2 = (double(d) + 4.0) * u24 + std::ldexp(1.0, -23) + u24;
   p.gd = (double(d) + 6.0) * u24;
   p.gref = (double(d) + 8.0) * u24;
}

cudaError_t launch_colsum(const float *X, uint32_t n, uint32_t d, double *sums, cudaStream_t s)
{
   cudaError_t e = cudaMemsetAsync(sums, 0, sizeof(double) * d, s);
   if (e != cudaSuccess || n == 0)
      return e;
   const uint32_t rows_per_block = 2048;
   const uint32_t blocks = (n + rows_per_block - 1) / rows_per_block;
   colsum_kernel<<<blocks, 256, 0, s>>>(X, n, d, sums, rows_per_block);
   return cudaGetLastError();
}

cudaError_t launch_center(const float *X, const double *sums, uint32_t n, uint32_t d, uint32_t dp, float *mean,
                          float *Xp, float *xnorm, cudaStream_t s)
{
   const size_t smem = sizeof(float) * d;
   if (smem > 48 * 1024)
   {
      cudaError_t e = cudaFuncSetAttribute(center_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess)
         return e;
   }
   const uint32_t blocks = n ? std::min<uint32_t>((n + 7) / 8, 148 * 16) : 1;
   center_kernel<<<blocks, 256, smem, s>>>(X, sums, n, d, dp, mean, Xp, xnorm);
   return cudaGetLastError();
}

cudaError_t launch_group_maxnorm(const float *xnorm, const uint32_t *ranges, uint32_t G, float *out, cudaStream_t s)
{
   const uint32_t blocks = std::min<uint32_t>((G + 1 + 7) / 8, 148 * 16);
   group_maxnorm_kernel<<<blocks, 256, 0, s>>>(xnorm, ranges, G, out);
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

cudaError_t launch_tc(const TcMaps &maps, const TcParams &p, uint32_t grid, cudaStream_t s)
{
   const int kp = tc_candidates_for_k(p.k);
   const bool ares = tc_a_resident(p.dp);
   if (kp == 8)
      return ares ? launch_tc_t<8, true>(maps, p, grid, s) : launch_tc_t<8, false>(maps, p, grid, s);
   if (kp == 16)
      return ares ? launch_tc_t<16, true>(maps, p, grid, s) : launch_tc_t<16, false>(maps, p, grid, s);
   if (kp == 24)
      return ares ? launch_tc_t<24, true>(maps, p, grid, s) : launch_tc_t<24, false>(maps, p, grid, s);
   if (kp == 32)
      return ares ? launch_tc_t<32, true>(maps, p, grid, s) : launch_tc_t<32, false>(maps, p, grid, s);
   return cudaErrorInvalidValue;
}

} // namespace ungx
