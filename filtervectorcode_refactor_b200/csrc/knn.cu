// Large-group intra-graph exact kNN seeding on the device (sm_100a): the role of
// batched_exact_knn_graph_kernel (UNG/codes/src/tagore_graph_builder.cu:650-795) with
// the host defaults of make_fast_exact_batch_config
// (UNG/codes/src/tagore_cuda_config.cpp:23-45).
//
// Every point of a group keeps its cand_degree = min(64, K - 1, n - 1) nearest other
// points of the group, then writes one row [degree, local ids...] in the head / ring
// anchor / tail layout.  The distance is the reference's: built with --use_fast_math
// (UNG/codes/src/CMakeLists.txt:79-80), a 128-thread block sums per-thread partials
// acc = fma(diff, diff, acc) over dims t, t+128, ... by a __shfl_down tree inside each
// warp and (w0 + w2) + (w1 + w3) across the warps; every add, sub and fma flushes
// subnormals (.ftz).  A warp's shuffle tree is a balanced binary tree whose in-order
// leaves are the lanes in 5-bit bit-reversed order, so it is evaluated here as a
// recursive tree over those leaves, for a 4 x 2 block of (row, candidate) pairs per
// thread at once (register tiling; each shared-memory load feeds two to four pairs).
//
// Layout of a block (256 threads): 64 source rows x 32 candidates per step, both tiles
// transposed in shared memory ([dim][64]); distances of the step go to a shared tile,
// then each warp updates the sorted lists of 8 rows (kept in shared memory): the
// candidates that beat a row's last entry are inserted in ascending candidate order
// (strict <, the reference's tie rule), a ballot giving the position and a one-lane
// shift moving the tail, so that all 32 lanes work on one row's insert.  The tree code
// is one 8-leaf subtree body looped over the 16 (warp, subtree) positions: a kernel of
// a few hundred instructions (a fully unrolled tree missed the instruction cache).
#include <algorithm>
#include <cfloat>
#include <type_traits>

#include "kernels.h"

namespace ungx
{
namespace
{
constexpr int kKnnRows = 64;     // source rows per block
constexpr int kKnnCands = 32;    // candidates per step
constexpr int kKnnThreads = 256; // 16 x 16 threads, 4 x 2 pairs each
constexpr int kKnnMax = 64;      // longest candidate list
constexpr int kLd = kKnnCands + 1;     // distance tile row stride
constexpr int kLl = kKnnMax + 1;       // list row stride

__device__ __forceinline__ float add_ftz(float a, float b)
{
   float r;
   asm("add.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
   return r;
}
__device__ __forceinline__ float sub_ftz(float a, float b)
{
   float r;
   asm("sub.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
   return r;
}
__device__ __forceinline__ float fma_ftz(float a, float b, float c)
{
   float r;
   asm("fma.rn.ftz.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
   return r;
}

// Partial of thread t of the reference's block for the 4 x 2 pairs: fma chain over
// dims t, t + 128, ... (zero when t >= d).
__device__ __forceinline__ void leaf(float (&out)[8], const float *sq, const float *sx, int t, uint32_t d, int r0,
                                     int c0)
{
#pragma unroll
   for (int i = 0; i < 8; ++i)
      out[i] = 0.0f;
   for (uint32_t dim = t; dim < d; dim += 128)
   {
      const float4 q = *reinterpret_cast<const float4 *>(sq + dim * kKnnRows + r0);
      const float2 x = *reinterpret_cast<const float2 *>(sx + dim * kKnnCands + c0);
      const float qa[4] = {q.x, q.y, q.z, q.w}, xa[2] = {x.x, x.y};
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
         for (int b = 0; b < 2; ++b)
         {
            const float diff = sub_ftz(qa[a], xa[b]);
            out[a * 2 + b] = fma_ftz(diff, diff, out[a * 2 + b]);
         }
   }
}

__host__ __device__ constexpr int bitrev3(int k) { return ((k & 1) << 2) | (k & 2) | ((k & 4) >> 2); }

// Balanced tree over the in-order leaves [LO, LO + SIZE) of one 8-leaf subtree whose
// leaf i sits at dimension offset base + 4 bitrev3(i) (in-order leaf 8 g + i of a warp
// is lane bitrev5(8 g + i) = 4 bitrev3(i) + bitrev2(g)).
template <int LO, int SIZE>
__device__ __forceinline__ void sub_tree(float (&out)[8], const float *sq, const float *sx, int base, uint32_t d,
                                         int r0, int c0)
{
   if constexpr (SIZE == 1)
      leaf(out, sq, sx, base + 4 * bitrev3(LO), d, r0, c0);
   else
   {
      float l[8], r[8];
      sub_tree<LO, SIZE / 2>(l, sq, sx, base, d, r0, c0);
      sub_tree<LO + SIZE / 2, SIZE / 2>(r, sq, sx, base, d, r0, c0);
#pragma unroll
      for (int i = 0; i < 8; ++i)
         out[i] = add_ftz(l[i], r[i]);
   }
}

// The shuffle tree of warp j (lanes / dims 32 j ..): ((S0 + S1) + (S2 + S3)) over its
// four in-order 8-leaf subtrees g, each at dims 32 j + bitrev2(g) + 4 bitrev3(i).  The
// subtree body is shared by all 16 (warp, subtree) uses: small code.
__device__ __forceinline__ void warp_tree(float (&out)[8], const float *sq, const float *sx, int j, uint32_t d,
                                          int r0, int c0)
{
   float a[8], b[8];
#pragma unroll 1
   for (int g = 0; g < 4; ++g) // a = S0 + S1, b = S2 + S3 (g is uniform: no divergence)
   {
      float t[8];
      sub_tree<0, 8>(t, sq, sx, 32 * j + ((g & 1) << 1 | (g >> 1)), d, r0, c0);
#pragma unroll
      for (int i = 0; i < 8; ++i)
      {
         if (g == 0)
            a[i] = t[i];
         else if (g == 1)
            a[i] = add_ftz(a[i], t[i]);
         else if (g == 2)
            b[i] = t[i];
         else
            b[i] = add_ftz(b[i], t[i]);
      }
   }
#pragma unroll
   for (int i = 0; i < 8; ++i)
      out[i] = add_ftz(a[i], b[i]);
}

// The same sums on packed pairs (sm_100 f32x2 arithmetic: each half rounds and
// flushes exactly like the scalar instruction): pair P[b][h] holds rows 2h, 2h + 1 of
// the thread's 4 x 2 block against candidate b, so a leaf is four packed subtractions
// and four packed FMAs instead of eight of each.
__device__ __forceinline__ uint64_t pk2(float lo, float hi)
{
   return (uint64_t(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ uint64_t sub2_ftz(uint64_t a, uint64_t b)
{
   uint64_t d;
   asm("sub.rn.ftz.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
   return d;
}
__device__ __forceinline__ uint64_t add2_ftz(uint64_t a, uint64_t b)
{
   uint64_t d;
   asm("add.rn.ftz.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
   return d;
}
__device__ __forceinline__ uint64_t fma2_ftz(uint64_t a, uint64_t b, uint64_t c)
{
   uint64_t d;
   asm("fma.rn.ftz.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
   return d;
}

__device__ __forceinline__ uint64_t mul2_ftz(uint64_t a, uint64_t b)
{
   uint64_t d;
   asm("mul.rn.ftz.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
   return d;
}

__device__ __forceinline__ void leaf2(uint64_t (&out)[4], const float *sq, const float *sx, int t, uint32_t d, int r0,
                                     int c0)
{
   if (d <= 128u) // one dimension per leaf: fma(x, x, +0) == mul(x, x) for a square
   {
      if (uint32_t(t) < d)
      {
         const float4 q = *reinterpret_cast<const float4 *>(sq + t * kKnnRows + r0);
         const float2 x = *reinterpret_cast<const float2 *>(sx + t * kKnnCands + c0);
         const uint64_t q01 = pk2(q.x, q.y), q23 = pk2(q.z, q.w);
         const uint64_t x0 = pk2(x.x, x.x), x1 = pk2(x.y, x.y);
         const uint64_t d00 = sub2_ftz(q01, x0), d01 = sub2_ftz(q23, x0);
         const uint64_t d10 = sub2_ftz(q01, x1), d11 = sub2_ftz(q23, x1);
         out[0] = mul2_ftz(d00, d00);
         out[1] = mul2_ftz(d01, d01);
         out[2] = mul2_ftz(d10, d10);
         out[3] = mul2_ftz(d11, d11);
      }
      else
      {
#pragma unroll
         for (int i = 0; i < 4; ++i)
            out[i] = 0;
      }
      return;
   }
#pragma unroll
   for (int i = 0; i < 4; ++i)
      out[i] = 0;
   for (uint32_t dim = t; dim < d; dim += 128)
   {
      const float4 q = *reinterpret_cast<const float4 *>(sq + dim * kKnnRows + r0);
      const float2 x = *reinterpret_cast<const float2 *>(sx + dim * kKnnCands + c0);
      const uint64_t q01 = pk2(q.x, q.y), q23 = pk2(q.z, q.w);
      const uint64_t x0 = pk2(x.x, x.x), x1 = pk2(x.y, x.y);
      const uint64_t d00 = sub2_ftz(q01, x0), d01 = sub2_ftz(q23, x0);
      const uint64_t d10 = sub2_ftz(q01, x1), d11 = sub2_ftz(q23, x1);
      out[0] = fma2_ftz(d00, d00, out[0]);
      out[1] = fma2_ftz(d01, d01, out[1]);
      out[2] = fma2_ftz(d10, d10, out[2]);
      out[3] = fma2_ftz(d11, d11, out[3]);
   }
}

template <int LO, int SIZE>
__device__ __forceinline__ void sub_tree2(uint64_t (&out)[4], const float *sq, const float *sx, int base, uint32_t d,
                                          int r0, int c0)
{
   if constexpr (SIZE == 1)
      leaf2(out, sq, sx, base + 4 * bitrev3(LO), d, r0, c0);
   else
   {
      uint64_t l[4], r[4];
      sub_tree2<LO, SIZE / 2>(l, sq, sx, base, d, r0, c0);
      sub_tree2<LO + SIZE / 2, SIZE / 2>(r, sq, sx, base, d, r0, c0);
#pragma unroll
      for (int i = 0; i < 4; ++i)
         out[i] = add2_ftz(l[i], r[i]);
   }
}

__device__ __forceinline__ void warp_tree2(uint64_t (&out)[4], const float *sq, const float *sx, int j, uint32_t d,
                                           int r0, int c0)
{
   uint64_t a[4], b[4];
#pragma unroll 1
   for (int g = 0; g < 4; ++g) // a = S0 + S1, b = S2 + S3
   {
      uint64_t t[4];
      sub_tree2<0, 8>(t, sq, sx, 32 * j + ((g & 1) << 1 | (g >> 1)), d, r0, c0);
#pragma unroll
      for (int i = 0; i < 4; ++i)
      {
         if (g == 0)
            a[i] = t[i];
         else if (g == 1)
            a[i] = add2_ftz(a[i], t[i]);
         else if (g == 2)
            b[i] = t[i];
         else
            b[i] = add2_ftz(b[i], t[i]);
      }
   }
#pragma unroll
   for (int i = 0; i < 4; ++i)
      out[i] = add2_ftz(a[i], b[i]);
}

// One output row: [degree, head, ring anchors, tail, dedupe tail], padded with the point
// itself (the reference's layout of batched_exact_knn_graph_kernel's epilogue).
__device__ void write_row(const KnnParams &p, uint32_t group, uint32_t n, uint32_t s, uint32_t cand,
                          const uint32_t *top)
{
   uint32_t *row = p.graph + size_t(p.base[group] + s) * p.graph_stride;
   const uint32_t out_degree = min(p.final_degree, cand);
   row[0] = out_degree;
   uint32_t write = 0;
   if (out_degree > 0)
   {
      const uint32_t near_limit = min(out_degree, min(p.head_keep, p.final_degree));
      for (; write < near_limit; ++write)
         row[1 + write] = top[write];
      const uint32_t remaining = p.final_degree > write ? p.final_degree - write : 0;
      const uint32_t anchor_limit =
          p.anchor_tail ? (p.anchor_slots == 0 ? remaining : min(p.anchor_slots, remaining)) : 0;
      if (anchor_limit > 0 && n > 1)
         for (uint32_t t = 0; t < anchor_limit && write < out_degree; ++t)
         {
            const uint32_t hop = max(1u, uint32_t((uint64_t(t + 1) * n) / (anchor_limit + 1)));
            const bool backward = p.bidir_anchor && (t & 1u);
            uint32_t c = backward ? (s + n - (hop % n)) % n : (s + hop) % n;
            for (uint32_t retry = 0; retry < n && write < out_degree;
                 ++retry, c = backward ? (c + n - 1) % n : (c + 1) % n)
            {
               if (c == s)
                  continue;
               bool dup = false;
               for (uint32_t q = 0; q < write; ++q)
                  if (row[1 + q] == c)
                  {
                     dup = true;
                     break;
                  }
               if (!dup)
               {
                  row[1 + write++] = c;
                  break;
               }
            }
         }
      const uint32_t tail_start = near_limit;
      const uint32_t tail_count = cand > tail_start ? cand - tail_start : 0;
      const uint32_t step = tail_count > remaining && remaining > 0 ? (tail_count + remaining - 1) / remaining : 1;
      for (uint32_t sc = tail_start; sc < cand && write < out_degree; sc += step)
         row[1 + write++] = top[sc];
      for (uint32_t sc = tail_start; sc < cand && write < out_degree; ++sc)
      {
         const uint32_t c = top[sc];
         bool dup = false;
         for (uint32_t q = 0; q < write; ++q)
            if (row[1 + q] == c)
            {
               dup = true;
               break;
            }
         if (!dup)
            row[1 + write++] = c;
      }
   }
   for (uint32_t j = out_degree; j + 1 < p.graph_stride; ++j)
      row[1 + j] = s;
}

// The same row written by a whole warp (one row per call, warp-uniform control flow):
// lane i holds row entry i in h0 and entry 32 + i in h1, so "already in the row" is one
// vote instead of a scan, and the row goes out in coalesced stores.  hops[t] (from
// anchor_hops, or computed here when null) are the group's ring-anchor hops, which
// depend only on the group's size and the layout.
__device__ __forceinline__ uint32_t anchor_limit_of(const KnnParams &p, uint32_t cand)
{
   const uint32_t out_degree = min(p.final_degree, cand);
   if (out_degree == 0)
      return 0;
   const uint32_t near_limit = min(out_degree, min(p.head_keep, p.final_degree));
   const uint32_t remaining = p.final_degree > near_limit ? p.final_degree - near_limit : 0;
   return p.anchor_tail ? (p.anchor_slots == 0 ? remaining : min(p.anchor_slots, remaining)) : 0;
}

// hops[t] = max(1, (t + 1) n / (anchor_limit + 1)) for t < anchor_limit (<= kKnnMax), lane-parallel.
__device__ __forceinline__ void anchor_hops(const KnnParams &p, uint32_t n, uint32_t cand, uint32_t *hops,
                                            uint32_t lane)
{
   const uint32_t A = min(anchor_limit_of(p, cand), uint32_t(kKnnMax));
   for (uint32_t t = lane; t < A; t += 32)
      hops[t] = max(1u, uint32_t((uint64_t(t + 1) * n) / (A + 1)));
   __syncwarp();
}

__device__ void write_row_warp(const KnnParams &p, uint32_t group, uint32_t n, uint32_t s, uint32_t cand,
                               const uint32_t *top, const uint32_t *hops, uint32_t lane)
{
   uint32_t *row = p.graph + size_t(p.base[group] + s) * p.graph_stride;
   const uint32_t out_degree = min(p.final_degree, cand);
   uint32_t h0 = 0xFFFFFFFFu, h1 = 0xFFFFFFFFu;
   uint32_t write = 0;
   auto member = [&](uint32_t c) {
      return __any_sync(0xffffffffu, (lane < write && h0 == c) || (lane + 32u < write && h1 == c));
   };
   auto append = [&](uint32_t c) {
      if (lane == write)
         h0 = c;
      else if (lane + 32u == write)
         h1 = c;
      ++write;
   };
   if (out_degree > 0)
   {
      const uint32_t near_limit = min(out_degree, min(p.head_keep, p.final_degree));
      if (lane < near_limit)
         h0 = top[lane];
      if (lane + 32u < near_limit)
         h1 = top[lane + 32u];
      write = near_limit;
      const uint32_t remaining = p.final_degree > write ? p.final_degree - write : 0;
      const uint32_t anchor_limit =
          p.anchor_tail ? (p.anchor_slots == 0 ? remaining : min(p.anchor_slots, remaining)) : 0;
      if (anchor_limit > 0 && n > 1)
         for (uint32_t t = 0; t < anchor_limit && write < out_degree; ++t)
         {
            const uint32_t hop = hops && t < uint32_t(kKnnMax)
                                     ? hops[t]
                                     : max(1u, uint32_t((uint64_t(t + 1) * n) / (anchor_limit + 1)));
            const bool backward = p.bidir_anchor && (t & 1u);
            // hop < n: (s + hop) % n and (s + n - hop) % n by one conditional subtraction
            uint32_t c = backward ? s + n - hop : s + hop;
            c = c >= n ? c - n : c;
            for (uint32_t retry = 0; retry < n && write < out_degree;
                 ++retry, c = backward ? (c == 0 ? n - 1 : c - 1) : (c + 1 == n ? 0 : c + 1))
            {
               if (c == s || member(c))
                  continue;
               append(c);
               break;
            }
         }
      const uint32_t tail_start = near_limit;
      const uint32_t tail_count = cand > tail_start ? cand - tail_start : 0;
      const uint32_t step = tail_count > remaining && remaining > 0 ? (tail_count + remaining - 1) / remaining : 1;
      for (uint32_t sc = tail_start; sc < cand && write < out_degree; sc += step)
         append(top[sc]);
      for (uint32_t sc = tail_start; sc < cand && write < out_degree; ++sc)
      {
         const uint32_t c = top[sc];
         if (!member(c))
            append(c);
      }
   }
   if (lane == 0)
      row[0] = out_degree;
   // entries the layout wrote, then the padding (slots write .. out_degree - 1, if any
   // stayed empty, are left as they were, as write_row leaves them)
   for (uint32_t i = lane; i + 1 < p.graph_stride; i += 32)
      if (i < write)
         row[1 + i] = i < 32u ? h0 : h1;
      else if (i >= out_degree)
         row[1 + i] = s;
}

struct KnnTask
{
   uint32_t group, row0;
};

__global__ void __launch_bounds__(kKnnThreads) exact_knn_kernel(const KnnParams p, const KnnTask *__restrict__ tasks)
{
   extern __shared__ float smem_f[];
   float *sq = smem_f;                            // [d][64] source rows
   float *sx = sq + size_t(p.dpad) * kKnnRows;    // [d][64] candidates
   float *sd = sx + size_t(p.dpad) * kKnnCands;   // [64][33] distances of the step
   float *ld = sd + kKnnRows * kLd;               // [64][65] list distances
   uint32_t *li = reinterpret_cast<uint32_t *>(ld + kKnnRows * kLl); // [64][65] list ids

   const KnnTask task = tasks[blockIdx.x];
   const uint32_t first = p.ranges[2 * task.group], n = p.ranges[2 * task.group + 1] - first;
   const uint32_t tid = threadIdx.x;
   uint32_t cand = p.candidate_k > 0 ? p.candidate_k - 1 : 0;
   cand = min(cand, uint32_t(kKnnMax));
   cand = min(cand, n > 0 ? n - 1 : 0u);
   if (task.row0 == 0 && tid == 0 && p.entry_points)
      p.entry_points[task.group] = 0;

   // source rows, transposed; rows past the group read as zero.  With d % 4 == 0 each
   // thread reads four consecutive dims of a row (16-byte loads) and the stores of a
   // warp go to 32 consecutive rows of a dim (conflict-free).
   const bool vec4 = (p.d & 3u) == 0;
   if (vec4)
      for (uint32_t idx = tid; idx < uint32_t(kKnnRows) * (p.dpad / 4u); idx += kKnnThreads)
      {
         const uint32_t r = idx % kKnnRows, d4 = idx / kKnnRows, row = task.row0 + r;
         const float4 v = row < n ? __ldg(reinterpret_cast<const float4 *>(p.X + size_t(first + row) * p.d) + d4)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
         sq[(4 * d4 + 0) * kKnnRows + r] = v.x;
         sq[(4 * d4 + 1) * kKnnRows + r] = v.y;
         sq[(4 * d4 + 2) * kKnnRows + r] = v.z;
         sq[(4 * d4 + 3) * kKnnRows + r] = v.w;
      }
   else
      for (uint32_t idx = tid; idx < uint32_t(kKnnRows) * p.dpad; idx += kKnnThreads)
      {
         const uint32_t r = idx % kKnnRows, dim = idx / kKnnRows;
         const uint32_t row = task.row0 + r;
         sq[dim * kKnnRows + r] = (row < n && dim < p.d) ? p.X[size_t(first + row) * p.d + dim] : 0.0f;
      }
   for (uint32_t idx = tid; idx < uint32_t(kKnnRows) * kLl; idx += kKnnThreads)
   {
      ld[idx] = FLT_MAX;
      li[idx] = 0xFFFFFFFFu;
   }
   const int tr = int(tid / 16u), tc = int(tid % 16u);
   const int r0 = tr * 4, c0 = tc * 2;
   const uint32_t warp = tid >> 5, lane = tid & 31u;
   for (uint32_t x0 = 0; x0 < n; x0 += kKnnCands)
   {
      __syncthreads(); // previous step's candidate tile and distances are consumed
      if (vec4)
         for (uint32_t idx = tid; idx < uint32_t(kKnnCands) * (p.dpad / 4u); idx += kKnnThreads)
         {
            const uint32_t c = idx % kKnnCands, d4 = idx / kKnnCands, x = x0 + c;
            const float4 v = x < n ? __ldg(reinterpret_cast<const float4 *>(p.X + size_t(first + x) * p.d) + d4)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
            sx[(4 * d4 + 0) * kKnnCands + c] = v.x;
            sx[(4 * d4 + 1) * kKnnCands + c] = v.y;
            sx[(4 * d4 + 2) * kKnnCands + c] = v.z;
            sx[(4 * d4 + 3) * kKnnCands + c] = v.w;
         }
      else
         for (uint32_t idx = tid; idx < uint32_t(kKnnCands) * p.dpad; idx += kKnnThreads)
         {
            const uint32_t c = idx % kKnnCands, dim = idx / kKnnCands;
            const uint32_t x = x0 + c;
            sx[dim * kKnnCands + c] = (x < n && dim < p.d) ? p.X[size_t(first + x) * p.d + dim] : 0.0f;
         }
      __syncthreads();
      // (w0 + w2) + (w1 + w3); a warp block past d is +0 and is skipped
      float s02[8], s13[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
         s02[i] = s13[i] = 0.0f;
      const int nj = int(min(p.d, 128u) + 31u) / 32;
#pragma unroll 1
      for (int j = 0; j < nj; ++j)
      {
         float w[8];
         warp_tree(w, sq, sx, j, p.d, r0, c0);
#pragma unroll
         for (int i = 0; i < 8; ++i)
         {
            if (j == 0)
               s02[i] = w[i];
            else if (j == 1)
               s13[i] = w[i];
            else if (j == 2)
               s02[i] = add_ftz(s02[i], w[i]);
            else
               s13[i] = add_ftz(s13[i], w[i]);
         }
      }
      // a skipped warp total is +0, and every partial is +0 or normal: adding it changes nothing
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
         for (int b = 0; b < 2; ++b)
            sd[(r0 + a) * kLd + c0 + b] = add_ftz(s02[a * 2 + b], s13[a * 2 + b]);
      __syncthreads();
      // The reference's insert, one warp per row (8 rows per warp): the row's step
      // candidates that beat its last entry are taken in ascending local id; each goes
      // after every entry <= its distance (strict <), the last entry dropping out.  The
      // list's empty tail holds FLT_MAX / UINT32_MAX, so a distance of FLT_MAX or more
      // never enters.  Lane l holds entries l and l + 32 while the row is updated.
      if (cand > 0)
#pragma unroll 1
         for (uint32_t i = 0; i < uint32_t(kKnnRows) / (kKnnThreads / 32u); ++i)
         {
            const uint32_t r = warp * (uint32_t(kKnnRows) / (kKnnThreads / 32u)) + i;
            const uint32_t s = task.row0 + r;
            if (s >= n)
               break;
            const uint32_t x = x0 + lane;
            const float dist = sd[r * kLd + lane];
            uint32_t m = __ballot_sync(0xffffffffu, x < n && x != s && dist < ld[r * kLl + cand - 1]);
            if (!m)
               continue;
            float e0 = ld[r * kLl + lane], e1 = ld[r * kLl + 32u + lane];
            uint32_t i0 = li[r * kLl + lane], i1 = li[r * kLl + 32u + lane];
            const uint32_t lc = (cand - 1u) & 31u;
            while (m)
            {
               const uint32_t b = __ffs(m) - 1u;
               m &= m - 1u;
               const float nd = __shfl_sync(0xffffffffu, dist, b);
               const float last = __shfl_sync(0xffffffffu, cand > 32u ? e1 : e0, lc);
               if (!(nd < last))
                  continue;
               const uint32_t pos = __popc(__ballot_sync(0xffffffffu, lane < cand && e0 <= nd)) +
                                    __popc(__ballot_sync(0xffffffffu, lane + 32u < cand && e1 <= nd));
               const float u0 = __shfl_up_sync(0xffffffffu, e0, 1), u1 = __shfl_up_sync(0xffffffffu, e1, 1);
               const uint32_t v0 = __shfl_up_sync(0xffffffffu, i0, 1), v1 = __shfl_up_sync(0xffffffffu, i1, 1);
               const float t31 = __shfl_sync(0xffffffffu, e0, 31);
               const uint32_t j31 = __shfl_sync(0xffffffffu, i0, 31);
               const float p1 = lane ? u1 : t31;
               const uint32_t q1 = lane ? v1 : j31;
               const uint32_t nid = x0 + b;
               if (lane >= pos)
               {
                  e0 = lane == pos ? nd : u0;
                  i0 = lane == pos ? nid : v0;
               }
               if (lane + 32u >= pos)
               {
                  e1 = lane + 32u == pos ? nd : p1;
                  i1 = lane + 32u == pos ? nid : q1;
               }
            }
            ld[r * kLl + lane] = e0;
            ld[r * kLl + 32u + lane] = e1;
            li[r * kLl + lane] = i0;
            li[r * kLl + 32u + lane] = i1;
         }
   }
   __syncthreads();
   // the row layout: head, ring anchors, tail, padding with the point itself
   if (tid < uint32_t(kKnnRows) && task.row0 + tid < n)
      write_row(p, task.group, n, task.row0 + tid, cand, li + tid * kLl);
}

// ------------------------------------------------------------------ two-phase path
// The reference's block distance is symmetric bit for bit: swapping the two points
// negates every difference (exact in IEEE arithmetic, flush-to-zero included) and
// fma(-x, -x, acc) == fma(x, x, acc), so the leaves, the tree and the sum are the same.
// Phase 1 therefore evaluates only the 64 x 64 tiles on and above the diagonal of each
// group's distance matrix and writes every value at (i, j) and (j, i); phase 2 gives
// each row to a warp, which scans the row in ascending candidate order with the
// reference's insert.

struct KnnTile
{
   uint32_t group, bi, bj; // rows 64 bi .., columns 64 bj .., bj >= bi
};

__global__ void __launch_bounds__(kKnnThreads, 3) knn_dist_kernel(const KnnParams p, const KnnTile *__restrict__ tiles)
{
   extern __shared__ float smem_f[];
   float *sq = smem_f;                          // [d][64] source rows
   float *sx = sq + size_t(p.dpad) * kKnnRows;  // [d][32] candidates
   float *sd = sx + size_t(p.dpad) * kKnnCands; // [64][33] distances of the step
   const KnnTile task = tiles[blockIdx.x];
   const uint32_t first = p.ranges[2 * task.group], n = p.ranges[2 * task.group + 1] - first;
   const uint32_t row0 = task.bi * kKnnRows, col0 = task.bj * kKnnRows;
   float *D = p.dist + p.dbase[task.group]; // [n][n]
   const uint32_t tid = threadIdx.x;
   const bool vec4 = (p.d & 3u) == 0;
   if (vec4)
      for (uint32_t idx = tid; idx < uint32_t(kKnnRows) * (p.dpad / 4u); idx += kKnnThreads)
      {
         const uint32_t r = idx % kKnnRows, d4 = idx / kKnnRows, row = row0 + r;
         const float4 v = row < n ? __ldg(reinterpret_cast<const float4 *>(p.X + size_t(first + row) * p.d) + d4)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
         sq[(4 * d4 + 0) * kKnnRows + r] = v.x;
         sq[(4 * d4 + 1) * kKnnRows + r] = v.y;
         sq[(4 * d4 + 2) * kKnnRows + r] = v.z;
         sq[(4 * d4 + 3) * kKnnRows + r] = v.w;
      }
   else
      for (uint32_t idx = tid; idx < uint32_t(kKnnRows) * p.dpad; idx += kKnnThreads)
      {
         const uint32_t r = idx % kKnnRows, dim = idx / kKnnRows, row = row0 + r;
         sq[dim * kKnnRows + r] = (row < n && dim < p.d) ? p.X[size_t(first + row) * p.d + dim] : 0.0f;
      }
   const int r0 = int(tid / 16u) * 4, c0 = int(tid % 16u) * 2;
   for (uint32_t step = 0; step < 2; ++step)
   {
      const uint32_t x0 = col0 + step * kKnnCands;
      if (x0 >= n)
         break;
      __syncthreads(); // the previous step's candidates and distances are consumed
      if (vec4)
         for (uint32_t idx = tid; idx < uint32_t(kKnnCands) * (p.dpad / 4u); idx += kKnnThreads)
         {
            const uint32_t c = idx % kKnnCands, d4 = idx / kKnnCands, x = x0 + c;
            const float4 v = x < n ? __ldg(reinterpret_cast<const float4 *>(p.X + size_t(first + x) * p.d) + d4)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
            sx[(4 * d4 + 0) * kKnnCands + c] = v.x;
            sx[(4 * d4 + 1) * kKnnCands + c] = v.y;
            sx[(4 * d4 + 2) * kKnnCands + c] = v.z;
            sx[(4 * d4 + 3) * kKnnCands + c] = v.w;
         }
      else
         for (uint32_t idx = tid; idx < uint32_t(kKnnCands) * p.dpad; idx += kKnnThreads)
         {
            const uint32_t c = idx % kKnnCands, dim = idx / kKnnCands, x = x0 + c;
            sx[dim * kKnnCands + c] = (x < n && dim < p.d) ? p.X[size_t(first + x) * p.d + dim] : 0.0f;
         }
      __syncthreads();
      // (w0 + w2) + (w1 + w3); a warp block past d is +0 and is skipped
      uint64_t s02[4], s13[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
         s02[i] = s13[i] = 0;
      const int nj = int(min(p.d, 128u) + 31u) / 32;
#pragma unroll 1
      for (int j = 0; j < nj; ++j)
      {
         uint64_t w[4];
         warp_tree2(w, sq, sx, j, p.d, r0, c0);
#pragma unroll
         for (int i = 0; i < 4; ++i)
         {
            if (j == 0)
               s02[i] = w[i];
            else if (j == 1)
               s13[i] = w[i];
            else if (j == 2)
               s02[i] = add2_ftz(s02[i], w[i]);
            else
               s13[i] = add2_ftz(s13[i], w[i]);
         }
      }
      // pair P[b][h]: rows 2h (low half), 2h + 1 (high half), candidate b
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
         for (int h = 0; h < 2; ++h)
         {
            const uint64_t v = add2_ftz(s02[b * 2 + h], s13[b * 2 + h]);
            sd[(r0 + 2 * h) * kLd + c0 + b] = __uint_as_float(uint32_t(v));
            sd[(r0 + 2 * h + 1) * kLd + c0 + b] = __uint_as_float(uint32_t(v >> 32));
         }
      __syncthreads();
      // (i, j): 32-column row pieces; (j, i) off the diagonal: 64-row column pieces
      for (uint32_t idx = tid; idx < uint32_t(kKnnRows) * kKnnCands; idx += kKnnThreads)
      {
         const uint32_t r = idx / kKnnCands, c = idx % kKnnCands, row = row0 + r, col = x0 + c;
         if (row < n && col < n)
            D[size_t(row) * n + col] = sd[r * kLd + c];
      }
      if (task.bi != task.bj)
         for (uint32_t idx = tid; idx < uint32_t(kKnnRows) * kKnnCands; idx += kKnnThreads)
         {
            const uint32_t r = idx % kKnnRows, c = idx / kKnnRows, row = row0 + r, col = x0 + c;
            if (row < n && col < n)
               D[size_t(col) * n + row] = sd[r * kLd + c];
         }
   }
}

// (distance, id) order of the reference's lists; an empty slot (+inf, UINT32_MAX) is last
__device__ __forceinline__ bool pair_less_knn(float d0, uint32_t i0, float d1, uint32_t i1)
{
   return d0 < d1 || (d0 == d1 && i0 < i1);
}

constexpr int kRowWarps = 4; // warps per block of the row pass, 32 rows each

// Phase 2: a warp per 32 rows of a group.  Each row's list (lane l: entries l and
// l + 32) takes the row's candidates in ascending order; then every lane lays out one
// of the warp's rows (head, ring anchors, tail, padding with the point itself).
__global__ void __launch_bounds__(kRowWarps * 32) knn_rows_kernel(const KnnParams p, const KnnTask *__restrict__ tasks,
                                                                   uint32_t num_tasks)
{
   __shared__ uint32_t s_top[kRowWarps][32][kKnnMax];
   const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
   const uint32_t ti = blockIdx.x * kRowWarps + warp;
   if (ti >= num_tasks)
      return;
   const KnnTask task = tasks[ti];
   const uint32_t first = p.ranges[2 * task.group], n = p.ranges[2 * task.group + 1] - first;
   uint32_t cand = p.candidate_k > 0 ? p.candidate_k - 1 : 0;
   cand = min(cand, uint32_t(kKnnMax));
   cand = min(cand, n > 0 ? n - 1 : 0u);
   if (task.row0 == 0 && lane == 0 && p.entry_points)
      p.entry_points[task.group] = 0;
   const float *D = p.dist + p.dbase[task.group];
   const uint32_t lc = cand > 0 ? (cand - 1u) & 31u : 0u;
   for (uint32_t rr = 0; rr < 32u && task.row0 + rr < n; ++rr)
   {
      const uint32_t s = task.row0 + rr;
      float e0 = FLT_MAX, e1 = FLT_MAX;
      uint32_t i0 = 0xFFFFFFFFu, i1 = 0xFFFFFFFFu;
      if (cand > 0)
      {
         // Columns 0..63 at once.  Inserting candidates in ascending id with strict <
         // keeps the cand smallest by (distance, id) of those with a distance below
         // FLT_MAX, so the warp sorts the 64 by (distance, id) (bitonic, element l and
         // l + 32 in lane l) and keeps the first cand; the rest of the list holds
         // FLT_MAX / UINT32_MAX as the reference's does.
         {
            const uint32_t xa = lane, xb = lane + 32u;
            float da = xa < n ? D[size_t(s) * n + xa] : INFINITY;
            float db = xb < n ? D[size_t(s) * n + xb] : INFINITY;
            uint32_t ia = xa, ib = xb;
            if (!(xa < n && xa != s && da < FLT_MAX))
            {
               da = INFINITY;
               ia = 0xFFFFFFFFu;
            }
            if (!(xb < n && xb != s && db < FLT_MAX))
            {
               db = INFINITY;
               ib = 0xFFFFFFFFu;
            }
#pragma unroll
            for (uint32_t k = 2; k <= 64; k <<= 1)
#pragma unroll
               for (uint32_t j = k >> 1; j > 0; j >>= 1)
               {
                  if (j == 32)
                  {
                     // partner of element l is l + 32, in the same lane; k == 64: ascending
                     if (pair_less_knn(db, ib, da, ia))
                     {
                        const float td = da;
                        const uint32_t ti = ia;
                        da = db;
                        ia = ib;
                        db = td;
                        ib = ti;
                     }
                     continue;
                  }
                  const bool lower = (lane & j) == 0;
                  {
                     const float od = __shfl_xor_sync(0xffffffffu, da, j);
                     const uint32_t oi = __shfl_xor_sync(0xffffffffu, ia, j);
                     const bool asc = (lane & k) == 0;
                     const bool o_less = pair_less_knn(od, oi, da, ia);
                     if (lower == asc ? o_less : !o_less)
                     {
                        da = od;
                        ia = oi;
                     }
                  }
                  {
                     const float od = __shfl_xor_sync(0xffffffffu, db, j);
                     const uint32_t oi = __shfl_xor_sync(0xffffffffu, ib, j);
                     const bool asc = ((lane + 32u) & k) == 0;
                     const bool o_less = pair_less_knn(od, oi, db, ib);
                     if (lower == asc ? o_less : !o_less)
                     {
                        db = od;
                        ib = oi;
                     }
                  }
               }
            e0 = lane < cand && ia != 0xFFFFFFFFu ? da : FLT_MAX;
            i0 = lane < cand && ia != 0xFFFFFFFFu ? ia : 0xFFFFFFFFu;
            e1 = lane + 32u < cand && ib != 0xFFFFFFFFu ? db : FLT_MAX;
            i1 = lane + 32u < cand && ib != 0xFFFFFFFFu ? ib : 0xFFFFFFFFu;
         }
         // the row's distances are loaded four 32-column steps ahead of their use
         float pf[4];
#pragma unroll
         for (int j = 0; j < 4; ++j)
         {
            const uint32_t xj = 64u + 32u * uint32_t(j) + lane;
            pf[j] = xj < n ? D[size_t(s) * n + xj] : FLT_MAX;
         }
         for (uint32_t xb = 64; xb < n; xb += 128u)
#pragma unroll
         for (int j = 0; j < 4; ++j)
         {
            const uint32_t x0 = xb + 32u * uint32_t(j);
            if (x0 >= n)
               break;
            const uint32_t x = x0 + lane;
            const float dist = pf[j];
            {
               const uint32_t xn = x + 128u;
               pf[j] = xn < n ? D[size_t(s) * n + xn] : FLT_MAX;
            }
            const float last0 = __shfl_sync(0xffffffffu, cand > 32u ? e1 : e0, lc);
            uint32_t m = __ballot_sync(0xffffffffu, x < n && x != s && dist < last0);
            while (m)
            {
               const uint32_t b = __ffs(m) - 1u;
               m &= m - 1u;
               const float nd = __shfl_sync(0xffffffffu, dist, b);
               const float last = __shfl_sync(0xffffffffu, cand > 32u ? e1 : e0, lc);
               if (!(nd < last))
                  continue;
               const uint32_t pos = __popc(__ballot_sync(0xffffffffu, lane < cand && e0 <= nd)) +
                                    __popc(__ballot_sync(0xffffffffu, lane + 32u < cand && e1 <= nd));
               const float u0 = __shfl_up_sync(0xffffffffu, e0, 1), u1 = __shfl_up_sync(0xffffffffu, e1, 1);
               const uint32_t v0 = __shfl_up_sync(0xffffffffu, i0, 1), v1 = __shfl_up_sync(0xffffffffu, i1, 1);
               const float t31 = __shfl_sync(0xffffffffu, e0, 31);
               const uint32_t j31 = __shfl_sync(0xffffffffu, i0, 31);
               const float p1 = lane ? u1 : t31;
               const uint32_t q1 = lane ? v1 : j31;
               const uint32_t nid = x0 + b;
               if (lane >= pos)
               {
                  e0 = lane == pos ? nd : u0;
                  i0 = lane == pos ? nid : v0;
               }
               if (lane + 32u >= pos)
               {
                  e1 = lane + 32u == pos ? nd : p1;
                  i1 = lane + 32u == pos ? nid : q1;
               }
            }
         }
      }
      s_top[warp][rr][lane] = i0;
      s_top[warp][rr][32u + lane] = i1;
   }
   __syncwarp();
   if (task.row0 + lane < n)
      write_row(p, task.group, n, task.row0 + lane, cand, s_top[warp][lane]);
}

// ------------------------------------------------------------------ tensor-core route
// Distances of one query row to 32 gathered candidate rows (lane l: candidate l), in
// the reference's block summation.  The candidates' dimensions of reference warp j
// (dims 32 j + l + 128 c, c < C) pass through a ring of NB per-warp stages in shared
// memory, filled by cp.async: a row segment of 32 floats is 128 contiguous bytes
// whatever rows are gathered, so the loads are coalesced, and NB - 1 stages are in
// flight while one is summed.  W is the copy width: 16 bytes when d is a multiple of
// 4 and X 16-byte aligned (row stride 32 C + 4 floats: the 16-byte reads of a quarter
// warp, lane l reading its own candidate's row, hit 32 distinct banks), else 8 or 4
// bytes (stride 32 C + 2: the 8-byte reads of a half warp are conflict-free).  Lane l
// evaluates the 32 partials of reference warp j for its candidate as 16 packed f32x2
// pairs: the fma chains over c, the first one from a zero accumulator as in the
// reference, then the __shfl_down tree (offsets 16 .. 2 are packed adds of pairs m and
// m + off / 2; offset 1 adds the two halves), and the warp sums as (w0 + w2) + (w1 +
// w3).  Padding past d is zero: 0 - 0 = +0 and fma(+0, +0, acc) = acc for acc >= +0,
// so the padded sums equal the reference's.  The zero accumulator is a register the
// compiler cannot prove zero: a packed square written as a multiply (or an fma of a
// known zero) followed by the tree's first packed add was contracted by ptxas into one
// fma, one rounding fewer than the reference's, which moved about one distance in
// eight by an ulp.
__device__ __forceinline__ void cp_async16(float *dst, const float *src, uint32_t bytes)
{
   asm volatile("cp.async.ca.shared.global [%0], [%1], 16, %2;\n" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                "l"(__cvta_generic_to_global(src)), "r"(bytes)
                : "memory");
}
__device__ __forceinline__ void cp_async8(float *dst, const float *src, uint32_t bytes)
{
   asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                "l"(__cvta_generic_to_global(src)), "r"(bytes)
                : "memory");
}
__device__ __forceinline__ void cp_async4(float *dst, const float *src, uint32_t bytes)
{
   asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                "l"(__cvta_generic_to_global(src)), "r"(bytes)
                : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait()
{
   asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

constexpr uint32_t kNoRow = 0xFFFFFFFFu;

// Copy of W bytes (W / 4 floats) at dim of row rr of X into dst; zeros when rr is
// kNoRow or dim >= d (d a multiple of W / 4).
template <int W>
__device__ __forceinline__ void stage_copy(float *dst, const float *X, uint32_t d, uint32_t rr, uint32_t dim)
{
   const bool ok = rr != kNoRow && dim < d;
   const float *src = ok ? X + size_t(rr) * d + dim : X;
   if constexpr (W == 16)
      cp_async16(dst, src, ok ? 16u : 0u);
   else if constexpr (W == 8)
      cp_async8(dst, src, ok ? 8u : 0u);
   else
      cp_async4(dst, src, ok ? 4u : 0u);
}

// C = ceil(d / 128) segments per partial; W copy bytes; NB stages in the ring.
template <int C, int W, int NB>
struct WarpDist
{
   static constexpr int kF = W / 4;                     // floats per copy
   static constexpr int kLd = 32 * C + (W == 16 ? 4 : 2); // stage row stride (floats)
   static constexpr int kStage = 32 * kLd;             // one buffer
   static constexpr int kQ = 128 * C;                  // the query row, zero padded
   static constexpr int kWarpFloats = NB * kStage + 2 * kQ;
   static constexpr int kCopies = 32 * 32 * C / kF;    // copies of one stage (32 rows)

   float *st; // [NB][32][kLd]
   float *sq; // [2][kQ]
   const float *X;
   uint32_t d;
   uint64_t zero; // packed (+0, +0), not known to the compiler as a constant

   // Copy i of a stage: row r, float offset o within the row's 32 C staged floats.
   __device__ __forceinline__ static void copy_slot(uint32_t i, uint32_t &r, uint32_t &o)
   {
      r = i / (32u * C / kF);
      o = (i % (32u * C / kF)) * kF;
   }
   // Dimension of staged float o of reference warp j.
   __device__ __forceinline__ static uint32_t stage_dim(uint32_t j, uint32_t o)
   {
      return 32u * j + 128u * (o / 32u) + o % 32u;
   }

   // Copies of reference warp j's dimensions of candidate rows shfl(row, r) into stage buf.
   __device__ __forceinline__ void issue(uint32_t buf, uint32_t row, uint32_t j, uint32_t lane) const
   {
      float *dst = st + buf * kStage;
#pragma unroll 8
      for (int k = 0; k < kCopies / 32; ++k)
      {
         uint32_t r, o;
         copy_slot(lane + 32u * k, r, o);
         const uint32_t rr = __shfl_sync(0xffffffffu, row, r);
         stage_copy<W>(dst + r * kLd + o, X, d, rr, stage_dim(j, o));
      }
   }

   // The same copies for a block of `threads` threads (thread tid) and the contiguous
   // candidate rows first + x0 + r (r < 32, those at or past `end` are kNoRow).
   __device__ __forceinline__ void issue_block(uint32_t buf, uint32_t first, uint32_t x0, uint32_t n, uint32_t j,
                                               uint32_t tid, uint32_t threads) const
   {
      float *dst = st + buf * kStage;
      for (uint32_t i = tid; i < uint32_t(kCopies); i += threads)
      {
         uint32_t r, o;
         copy_slot(i, r, o);
         stage_copy<W>(dst + r * kLd + o, X, d, x0 + r < n ? first + x0 + r : kNoRow, stage_dim(j, o));
      }
   }

   // The query row into buffer qb (zero padded to kQ).
   __device__ __forceinline__ void issue_query(uint32_t qb, uint32_t row, uint32_t lane) const
   {
      float *dst = sq + qb * kQ;
#pragma unroll
      for (int k = 0; k < kQ / kF / 32; ++k)
      {
         const uint32_t dim = kF * (lane + 32u * k);
         stage_copy<W>(dst + dim, X, d, row, dim);
      }
   }

   // Sum w_j of reference warp j for this lane's candidate (stage buf, query qb).
   __device__ __forceinline__ float warp_sum(uint32_t buf, uint32_t qb, uint32_t j, uint32_t lane) const
   {
      const float *b = st + buf * kStage + lane * kLd;
      const float *a = sq + qb * kQ + 32u * j;
      uint64_t v[16];
#pragma unroll
      for (int c = 0; c < C; ++c)
#pragma unroll
         for (int m = 0; m < 16; m += (W == 16 ? 2 : 1))
         {
            uint64_t bv[2], av[2];
            if constexpr (W == 16)
            {
               const ulonglong2 b2 = *reinterpret_cast<const ulonglong2 *>(b + c * 32 + 2 * m);
               const ulonglong2 a2 = *reinterpret_cast<const ulonglong2 *>(a + c * 128 + 2 * m);
               bv[0] = b2.x, bv[1] = b2.y, av[0] = a2.x, av[1] = a2.y;
            }
            else
            {
               bv[0] = *reinterpret_cast<const uint64_t *>(b + c * 32 + 2 * m);
               av[0] = *reinterpret_cast<const uint64_t *>(a + c * 128 + 2 * m);
            }
#pragma unroll
            for (int h = 0; h < (W == 16 ? 2 : 1); ++h)
            {
               const uint64_t df = sub2_ftz(av[h], bv[h]);
               v[m + h] = fma2_ftz(df, df, c == 0 ? zero : v[m + h]);
            }
         }
#pragma unroll
      for (int h = 8; h >= 1; h >>= 1)
#pragma unroll
         for (int m = 0; m < h; ++m)
            v[m] = add2_ftz(v[m], v[m + h]);
      return add_ftz(__uint_as_float(uint32_t(v[0])), __uint_as_float(uint32_t(v[0] >> 32)));
   }
};

constexpr int kRrWarps = 4;         // a block per work item: 4 warps x 32 rows
constexpr int kRrLists = 3;         // the prefilter's lists per row (column thirds)
constexpr int kRrDepth = 32;        // entries per list
constexpr int kRrEntries = kRrLists * kRrDepth;
constexpr int kRrMaxDim = 352;      // three 128-dim segments per partial at most

// A block per work item (<= 128 rows of one group); warp w ranks rows 32 w .. 32 w + 31
// one after the other, then every lane lays out one of them.  Per row: the 96 list
// entries (list e: lane l holds entry l) get the reference's distance, list by list
// through the staged pipeline above (the next row's query and candidates are fetched
// while the current row's last list is summed); the cand smallest by (distance, local
// id) below FLT_MAX are the row's list (the reference's strict-< inserts in ascending
// id from FLT_MAX keep exactly those).  Certificate: every column outside the lists has
// a prefilter key >= T, the smallest last key of a list that dropped a column, so its
// reference distance is at least ((|a|^2 + T - bound)(1 - gref) - abs_err); when that
// exceeds the cand-th distance no such column can enter.  A row whose lists all saw
// every one of their columns is exact as it stands.  Rejected rows are queued for the
// exact kernel.
template <int C, int W, int NB>
__global__ void __launch_bounds__(kRrWarps * 32, C == 1 ? 5 : 1) knn_rerank_kernel(const KnnRerankParams rp)
{
   using WD = WarpDist<C, W, NB>;
   extern __shared__ __align__(16) float rr_smem[];
   if (*reinterpret_cast<const volatile int *>(rp.status) != 0)
      return; // an aborted prefilter left the lists unwritten
   const KnnParams &p = rp.p;
   const WorkItem w = rp.items[blockIdx.x];
   const Segment sg = rp.segs[w.seg_begin];
   const uint32_t group = sg.group_id - 1u;
   const uint32_t first = p.ranges[2 * group], end = p.ranges[2 * group + 1], n = end - first;
   const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
   const WD wd{rr_smem + warp * WD::kWarpFloats, rr_smem + warp * WD::kWarpFloats + NB * WD::kStage, p.X, p.d,
               uint64_t(p.d >> 31)};
   // the ranked list of the warp's current row, and the group's anchor hops
   uint32_t *s_top = reinterpret_cast<uint32_t *>(rr_smem + kRrWarps * WD::kWarpFloats) + warp * (2 * kKnnMax);
   uint32_t *s_hops = s_top + kKnnMax;
   uint32_t cand = p.candidate_k > 0 ? p.candidate_k - 1 : 0;
   cand = min(cand, uint32_t(kKnnMax));
   cand = min(cand, n > 0 ? n - 1 : 0u);
   if (w.row_begin == first && threadIdx.x == 0 && p.entry_points)
      p.entry_points[group] = 0;
   anchor_hops(p, n, cand, s_hops, lane);
   const double pk = 1.0 / 131072.0; // packed-key tolerance, 2^-17 relative
   const double bmax = sqrt((double)rp.group_maxn2[sg.group_id] * (1.0 + rp.gd));
   const double inv_s = (double)rp.scale->inv_s;
   const bool exact_only = rp.scale->exact_only != 0;
   // columns each list saw: the group's columns in tiles of 192 from its first row, chunks
   // of 32; list h takes chunks h and h + 3 of every tile (the row itself is excluded)
   uint32_t seen[kRrLists] = {0u, 0u, 0u};
   for (uint32_t t0 = 0; t0 < n; t0 += 192u)
#pragma unroll
      for (uint32_t c = 0; c < 6u; ++c)
      {
         const uint32_t a = t0 + 32u * c;
         seen[c % 3u] += a < n ? min(32u, n - a) : 0u;
      }
   uint32_t n_cert = 0, n_fail = 0;
   const uint32_t r0 = warp * 32u;
   const uint32_t nrows = r0 < w.row_count ? min(32u, w.row_count - r0) : 0u;
   // this lane's candidate row of each list of a row (kNoRow: empty, outside, itself)
   auto cand_rows = [&](uint32_t rr, uint32_t (&c)[kRrLists]) {
      const uint32_t row = w.row_begin + r0 + rr;
      const uint32_t *cp = rp.cand_col + size_t(row) * kRrEntries;
#pragma unroll
      for (int e = 0; e < kRrLists; ++e)
      {
         const uint32_t v = cp[lane + 32u * e];
         c[e] = v < end && v >= first && v != row ? v : kNoRow;
      }
   };
   // the certificate's inputs of a row: each list's last key (+inf when the list saw every
   // one of its columns) and the row's squared norm, loaded a row ahead
   auto cert_inputs = [&](uint32_t rr, float (&lk)[kRrLists], float &qn) {
      const uint32_t row = w.row_begin + r0 + rr, sl = row - first;
      const uint32_t self_list = ((sl % 192u) / 32u) % 3u;
      const float *kp = rp.cand_key + size_t(row) * kRrEntries;
#pragma unroll
      for (int f = 0; f < kRrLists; ++f)
         // list f dropped a column only when it saw more than 32 (every column it
         // dropped has a key >= its last one)
         lk[f] = seen[f] - (uint32_t(f) == self_list ? 1u : 0u) > uint32_t(kRrDepth) ? __ldg(kp + 32 * f + 31)
                                                                                         : INFINITY;
      qn = __ldg(rp.xnorm + row);
   };
   uint32_t cur[kRrLists], nxt[kRrLists];
   float ck[kRrLists], nk[kRrLists], cqn = 0.f, nqn = 0.f;
   // stage t1 of row rr1 (the current row rr or the next one) into its ring slot
   static_assert(NB == 2, "the rerank's stage loop is written for a two-stage ring");
   if (nrows)
   {
      cand_rows(0, cur);
      cert_inputs(0, ck, cqn);
      if (nrows > 1)
      {
         cand_rows(1, nxt);
         cert_inputs(1, nk, nqn);
      }
      // row 0's query and its first stage (list 0, reference warp 0) into slot 0
      wd.issue_query(0u, w.row_begin + r0, lane);
      wd.issue(0u, cur[0], 0u, lane);
   }
   cp_commit();
   float D[kRrLists] = {INFINITY, INFINITY, INFINITY};
   // stages of a row: list e (run-time loop) x reference warp j (unrolled); stage 4 e + j
   // sits in ring slot j & 1 (a row has 12 stages, an even count), and each iteration
   // first puts the following stage in flight: the next reference warp, the next list
   // or the next row's first list with its query
   for (uint32_t rr = 0; rr < nrows; ++rr)
   {
      const uint32_t qb = rr & 1u;
      for (uint32_t e = 0; e < uint32_t(kRrLists); ++e)
      {
         const uint32_t my = e == 0u ? cur[0] : (e == 1u ? cur[1] : cur[2]);
         float s02 = 0.f, s13 = 0.f;
#pragma unroll
         for (uint32_t j = 0; j < 4u; ++j)
         {
            if (j < 3u)
               wd.issue((j + 1u) & 1u, my, j + 1u, lane);
            else if (e + 1u < uint32_t(kRrLists))
               wd.issue(0u, e == 0u ? cur[1] : cur[2], 0u, lane);
            else if (rr + 1u < nrows)
            {
               wd.issue_query(qb ^ 1u, w.row_begin + r0 + rr + 1u, lane);
               wd.issue(0u, nxt[0], 0u, lane);
            }
            cp_commit();
            cp_wait<1>(); // this stage has landed (the next may be in flight)
            __syncwarp();
            const float ws = wd.warp_sum(j & 1u, qb, j, lane);
            __syncwarp();
            if (j == 0u)
               s02 = ws;
            else if (j == 1u)
               s13 = ws;
            else if (j == 2u)
               s02 = add_ftz(s02, ws);
            else
            {
               const float dd = add_ftz(s02, add_ftz(s13, ws));
               const float dv = my != kNoRow && dd < FLT_MAX ? dd : INFINITY;
               if (e == 0u)
                  D[0] = dv;
               else if (e == 1u)
                  D[1] = dv;
               else
                  D[2] = dv;
            }
         }
      }
      // ---- row rr complete: rank, lay out, certify
      const uint32_t row = w.row_begin + r0 + rr; // global row of X
      const uint32_t s = row - first;             // local row
      uint32_t db[kRrLists], id[kRrLists];
      const float T = fminf(ck[0], fminf(ck[1], ck[2])); // smallest last key of a list that dropped a column
      const float qn_row = cqn;
#pragma unroll
      for (int f = 0; f < kRrLists; ++f)
      {
         id[f] = D[f] != INFINITY ? cur[f] - first : 0xFFFFFFFFu;
         db[f] = __float_as_uint(D[f]); // non-negative: the bits order as the values
      }
      // rank of each entry by (distance, local id): first by distance alone; equal
      // distances of valid entries share a rank then, which shows as a rank sum below
      // 0 + 1 + ... + (nvalid - 1), and a second pass breaks those ties by id
      uint32_t rk[kRrLists] = {0u, 0u, 0u};
#pragma unroll 4
      for (int src = 0; src < 32; ++src)
#pragma unroll
         for (int f = 0; f < kRrLists; ++f)
         {
            const uint32_t d2 = __shfl_sync(0xffffffffu, db[f], src);
#pragma unroll
            for (int e2 = 0; e2 < kRrLists; ++e2)
               rk[e2] += d2 < db[e2] ? 1u : 0u;
         }
      {
         uint32_t nv = 0, rsum = 0;
#pragma unroll
         for (int f = 0; f < kRrLists; ++f)
         {
            const bool valid = id[f] != 0xFFFFFFFFu;
            nv += valid ? 1u : 0u;
            rsum += valid ? rk[f] : 0u;
         }
         nv = __reduce_add_sync(0xffffffffu, nv);
         rsum = __reduce_add_sync(0xffffffffu, rsum);
         if (nv > 0 && rsum != nv * (nv - 1u) / 2u)
#pragma unroll 1
            for (int src = 0; src < 32; ++src)
#pragma unroll
               for (int f = 0; f < kRrLists; ++f)
               {
                  const uint32_t d2 = __shfl_sync(0xffffffffu, db[f], src);
                  const uint32_t i2 = __shfl_sync(0xffffffffu, id[f], src);
#pragma unroll
                  for (int e2 = 0; e2 < kRrLists; ++e2)
                     rk[e2] += d2 == db[e2] && i2 < id[e2] ? 1u : 0u;
               }
      }
      uint32_t nvalid = 0, have_k = 0;
      float dk = INFINITY;
#pragma unroll
      for (int f = 0; f < kRrLists; ++f)
      {
         const bool valid = id[f] != 0xFFFFFFFFu;
         nvalid += __popc(__ballot_sync(0xffffffffu, valid));
         if (valid && rk[f] < cand)
            s_top[rk[f]] = id[f];
         const uint32_t at = __ballot_sync(0xffffffffu, valid && cand > 0 && rk[f] == cand - 1u);
         if (at)
         {
            have_k = 1;
            dk = __shfl_sync(0xffffffffu, D[f], __ffs(at) - 1);
         }
      }
      for (uint32_t q = nvalid + lane; q < cand; q += 32)
         s_top[q] = 0xFFFFFFFFu; // the reference's unfilled list slots
      // certificate (warp-uniform), list by list: list f passes when it dropped no
      // column or its last key clears the cand-th distance; one failing list is
      // rescanned alone (its columns only, merged with the other lists' entries),
      // more (or no usable bound) send the row to the full rescan
      uint32_t bad = 0; // bit f: list f fails; 8: the row needs the full rescan
      if (cand == 0)
         bad = 0; // nothing to rank
      else if (exact_only)
         bad = 8; // keys of data outside the fp16 operand's range prove nothing
      else if (T == INFINITY)
         bad = 0; // no list dropped a column: every column was ranked
      else if (!have_k)
         bad = 8;
      else
      {
         const double qn = (double)qn_row;
         const double ahi = sqrt(qn * (1.0 + rp.gd));
         const double bound = (rp.c1 * ahi * bmax + rp.c2 * bmax * bmax + rp.c3 * inv_s * (ahi + bmax) +
                               rp.c4 * inv_s * inv_s) *
                              (1.0 + 1.0 / 1024.0);
#pragma unroll
         for (int f = 0; f < kRrLists; ++f)
         {
            const float Tf = ck[f];
            if (Tf == INFINITY)
               continue;
            const double Tp = (double)Tf - fabs((double)Tf) * pk;
            const double lhs = (qn * (1.0 - rp.gd) + Tp - bound) * (1.0 - rp.gref) - rp.abs_err;
            if (!(lhs > (double)dk))
               bad |= 1u << f;
         }
      }
      uint32_t h = bad == 0 ? 4u : (bad == 8u || __popc(bad) > 1 ? 3u : uint32_t(__ffs(bad) - 1));
      uint32_t pidx = 0;
      if (h < 3u)
      {
         // the passing lists' entries by rank, for the partial rescan's merge
         if (lane == 0)
            pidx = atomicAdd(rp.fb_pend_count, 1u);
         pidx = __shfl_sync(0xffffffffu, pidx, 0);
         if (pidx >= rp.fb_pend_cap)
            h = 3u; // no room: the full rescan
         else
         {
            float2 *pe = rp.fb_pend + size_t(pidx) * kRrEntries;
#pragma unroll
            for (int f = 0; f < kRrLists; ++f)
            {
               const bool keep = id[f] != 0xFFFFFFFFu && uint32_t(f) != h;
               if (id[f] != 0xFFFFFFFFu)
                  pe[rk[f]] = keep ? make_float2(D[f], __uint_as_float(id[f]))
                                   : make_float2(INFINITY, __uint_as_float(0xFFFFFFFFu));
            }
            for (uint32_t q = nvalid + lane; q < uint32_t(kRrEntries); q += 32)
               pe[q] = make_float2(INFINITY, __uint_as_float(0xFFFFFFFFu));
         }
      }
      if (lane == 0)
      {
         if (h == 4u)
            ++n_cert;
         else
         {
            const uint32_t slot = atomicAdd(rp.fb_group_count + 4u * group + h, 1u);
            const size_t at = 4u * size_t(p.base[group]) + size_t(h) * n + slot;
            rp.fb_rows[at] = s;
            rp.fb_pend_idx[at] = pidx;
            ++n_fail;
         }
      }
      // the next row's candidates and certificate inputs, one row ahead of the pipeline
#pragma unroll
      for (int f = 0; f < kRrLists; ++f)
      {
         cur[f] = nxt[f];
         ck[f] = nk[f];
      }
      cqn = nqn;
      if (rr + 2u < nrows)
      {
         cand_rows(rr + 2u, nxt);
         cert_inputs(rr + 2u, nk, nqn);
      }
      __syncwarp();
      write_row_warp(p, group, n, s, cand, s_top, s_hops, lane);
      __syncwarp();
   }
   if (lane == 0)
   {
      if (n_cert)
         atomicAdd(&rp.counters[0], (unsigned long long)n_cert);
      if (n_fail)
         atomicAdd(&rp.counters[1], (unsigned long long)n_fail);
   }
}

// The reference's inserts of one 32-column step into a list of cand (<= 64) entries
// held by the warp (lane l: entries l and l + 32): the columns whose distance beats the
// last entry (strict <, FLT_MAX at first) are taken in ascending id; a ballot gives
// each one's position and one shuffle moves the tail.
__device__ __forceinline__ void list_insert(float dist, uint32_t x0, uint32_t cand, uint32_t lane, float &e0, float &e1,
                                            uint32_t &i0, uint32_t &i1)
{
   const uint32_t lc = cand > 0 ? (cand - 1u) & 31u : 0u;
   const float last0 = __shfl_sync(0xffffffffu, cand > 32u ? e1 : e0, lc);
   uint32_t m = __ballot_sync(0xffffffffu, dist < last0);
   while (m)
   {
      const uint32_t b = __ffs(m) - 1u;
      m &= m - 1u;
      const float nd = __shfl_sync(0xffffffffu, dist, b);
      const float last = __shfl_sync(0xffffffffu, cand > 32u ? e1 : e0, lc);
      if (!(nd < last))
         continue;
      const uint32_t pos = __popc(__ballot_sync(0xffffffffu, lane < cand && e0 <= nd)) +
                           __popc(__ballot_sync(0xffffffffu, lane + 32u < cand && e1 <= nd));
      const float u0 = __shfl_up_sync(0xffffffffu, e0, 1), u1 = __shfl_up_sync(0xffffffffu, e1, 1);
      const uint32_t v0 = __shfl_up_sync(0xffffffffu, i0, 1), v1 = __shfl_up_sync(0xffffffffu, i1, 1);
      const float t31 = __shfl_sync(0xffffffffu, e0, 31);
      const uint32_t j31 = __shfl_sync(0xffffffffu, i0, 31);
      const float p1 = lane ? u1 : t31;
      const uint32_t q1 = lane ? v1 : j31;
      const uint32_t nid = x0 + b;
      if (lane >= pos)
      {
         e0 = lane == pos ? nd : u0;
         i0 = lane == pos ? nid : v0;
      }
      if (lane + 32u >= pos)
      {
         e1 = lane + 32u == pos ? nd : p1;
         i1 = lane + 32u == pos ? nid : q1;
      }
   }
}

// The same insert for a list seeded out of column order (the partial rescan starts
// from the passing lists' entries): places and the threshold test compare (distance,
// id) pairs, and a column enters only below FLT_MAX, so the list ends as the cand
// smallest pairs below FLT_MAX, which is what the reference's inserts in ascending id
// keep.
__device__ __forceinline__ void list_insert_pair(float dist, uint32_t x0, uint32_t cand, uint32_t lane, float &e0,
                                                 float &e1, uint32_t &i0, uint32_t &i1)
{
   const uint32_t lc = cand > 0 ? (cand - 1u) & 31u : 0u;
   auto less = [](float da, uint32_t ia, float db, uint32_t ib) { return da < db || (da == db && ia < ib); };
   const float last0 = __shfl_sync(0xffffffffu, cand > 32u ? e1 : e0, lc);
   const uint32_t lid0 = __shfl_sync(0xffffffffu, cand > 32u ? i1 : i0, lc);
   uint32_t m = __ballot_sync(0xffffffffu, dist < FLT_MAX && less(dist, x0 + lane, last0, lid0));
   while (m)
   {
      const uint32_t b = __ffs(m) - 1u;
      m &= m - 1u;
      const float nd = __shfl_sync(0xffffffffu, dist, b);
      const uint32_t nid = x0 + b;
      const float last = __shfl_sync(0xffffffffu, cand > 32u ? e1 : e0, lc);
      const uint32_t lid = __shfl_sync(0xffffffffu, cand > 32u ? i1 : i0, lc);
      if (!less(nd, nid, last, lid))
         continue;
      const uint32_t pos = __popc(__ballot_sync(0xffffffffu, lane < cand && less(e0, i0, nd, nid))) +
                           __popc(__ballot_sync(0xffffffffu, lane + 32u < cand && less(e1, i1, nd, nid)));
      const float u0 = __shfl_up_sync(0xffffffffu, e0, 1), u1 = __shfl_up_sync(0xffffffffu, e1, 1);
      const uint32_t v0 = __shfl_up_sync(0xffffffffu, i0, 1), v1 = __shfl_up_sync(0xffffffffu, i1, 1);
      const float t31 = __shfl_sync(0xffffffffu, e0, 31);
      const uint32_t j31 = __shfl_sync(0xffffffffu, i0, 31);
      const float p1 = lane ? u1 : t31;
      const uint32_t q1 = lane ? v1 : j31;
      if (lane >= pos)
      {
         e0 = lane == pos ? nd : u0;
         i0 = lane == pos ? nid : v0;
      }
      if (lane + 32u >= pos)
      {
         e1 = lane + 32u == pos ? nd : p1;
         i1 = lane + 32u == pos ? nid : q1;
      }
   }
}

// Rows the certificate rejected, in tasks of up to kFbWarps rows of one group (task =
// (group, first slot, rows); the rows' local ids at fb_rows[base[group] + slot]): warp w
// takes the task's row w, and every 32-column step of the group passes once through a
// block-wide staged ring (NB stages, one barrier per stage) shared by the task's rows.
// Lane l sums column x0 + l for its warp's row; the passing columns of a step are
// inserted in ascending id (list_insert).  Then the row is laid out as every other row.
// A persistent grid takes the tasks in turn; their number is read on the device.
constexpr int kFbWarps = 8;

template <int C, int W, int NB>
__global__ void __launch_bounds__(kFbWarps * 32) knn_fallback_rows_kernel(const KnnParams p,
                                                                        const uint32_t *__restrict__ fb_rows,
                                                                        const uint32_t *__restrict__ fb_pend_idx,
                                                                        const float2 *__restrict__ fb_pend,
                                                                        const uint32_t *__restrict__ tasks,
                                                                        const uint32_t *__restrict__ num_tasks)
{
   using WD = WarpDist<C, W, NB>;
   extern __shared__ __align__(16) float fb_smem[];
   const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, tid = threadIdx.x;
   float *st = fb_smem;                  // [NB][32][kLd]
   float *sq = fb_smem + NB * WD::kStage; // [kFbWarps][kQ]
   uint32_t *s_top = reinterpret_cast<uint32_t *>(sq + kFbWarps * WD::kQ) + warp * (2 * kKnnMax);
   uint32_t *s_hops = s_top + kKnnMax; // the task's group's anchor hops
   const WD wd{st, sq, p.X, p.d, uint64_t(p.d >> 31)};
   const uint32_t ntask = *num_tasks;
   for (uint32_t task = blockIdx.x; task < ntask; task += gridDim.x)
   {
      __syncthreads(); // the previous task's ring is no longer read
      const uint32_t group = tasks[4 * task], h = tasks[4 * task + 1], slot0 = tasks[4 * task + 2],
                     cnt = tasks[4 * task + 3];
      const uint32_t first = p.ranges[2 * group], n = p.ranges[2 * group + 1] - first;
      const bool active = warp < cnt;
      const size_t at = 4u * size_t(p.base[group]) + size_t(h) * n + slot0 + warp;
      const uint32_t s = active ? fb_rows[at] : 0u;
      uint32_t cand = p.candidate_k > 0 ? p.candidate_k - 1 : 0;
      cand = min(cand, uint32_t(kKnnMax));
      cand = min(cand, n > 0 ? n - 1 : 0u);
      // bucket 3: every 32-column step; bucket h < 3: the steps of list h (k = h mod 3:
      // chunks h and h + 3 of each 192-column tile from the group's first row)
      const uint32_t all_steps = cand > 0 ? (n + 31u) / 32u : 0u;
      const uint32_t steps = h == 3u ? all_steps : (all_steps > h ? (all_steps - h + 2u) / 3u : 0u);
      const uint32_t sstep = h == 3u ? 1u : 3u, s0 = h == 3u ? 0u : h;
      const uint32_t stages = 4u * steps; // (32-column step, reference warp)
      if (active && stages)
         wd.issue_query(warp, first + s, lane);
      // the ring starts with stages 0 .. NB - 2 in flight (one commit group each)
#pragma unroll
      for (uint32_t t1 = 0; t1 + 1u < uint32_t(NB); ++t1)
      {
         if (t1 < stages)
            wd.issue_block(t1, first, 32u * (s0 + sstep * (t1 >> 2)), n, t1 & 3u, tid, kFbWarps * 32u);
         cp_commit();
      }
      float e0 = FLT_MAX, e1 = FLT_MAX; // list entries lane and lane + 32
      uint32_t i0 = 0xFFFFFFFFu, i1 = 0xFFFFFFFFu;
      if (active && h < 3u && cand > 0)
      {
         // the seed: the passing lists' entries in (distance, id) order, the failing
         // list's places empty; compacted to the first cand places (s_top and s_hops
         // hold the distances and ids meanwhile)
         const float2 *pe = fb_pend + size_t(fb_pend_idx[at]) * kRrEntries;
         float *sd = reinterpret_cast<float *>(s_top);
         uint32_t base_pos = 0;
#pragma unroll
         for (int q = 0; q < kRrEntries / 32; ++q)
         {
            const float2 v = pe[lane + 32u * q];
            const bool ok = __float_as_uint(v.y) != 0xFFFFFFFFu;
            const uint32_t bal = __ballot_sync(0xffffffffu, ok);
            const uint32_t pos = base_pos + __popc(bal & ((1u << lane) - 1u));
            base_pos += __popc(bal);
            if (ok && pos < cand)
            {
               sd[pos] = v.x;
               s_top[kKnnMax + pos] = __float_as_uint(v.y);
            }
         }
         __syncwarp();
         if (lane < cand && lane < base_pos)
         {
            e0 = sd[lane];
            i0 = s_top[kKnnMax + lane];
         }
         if (lane + 32u < cand && lane + 32u < base_pos)
         {
            e1 = sd[lane + 32u];
            i1 = s_top[kKnnMax + lane + 32u];
         }
         __syncwarp();
      }
      float s02 = 0.f, s13 = 0.f;
      for (uint32_t t = 0; t < stages; ++t)
      {
         cp_wait<NB - 2>(); // stage t has landed (the later ones may be in flight)
         __syncthreads();   // ... for every thread's copies; stage t - 1's slot is free
         const uint32_t t1 = t + uint32_t(NB) - 1u;
         if (t1 < stages)
            wd.issue_block(t1 % uint32_t(NB), first, 32u * (s0 + sstep * (t1 >> 2)), n, t1 & 3u, tid,
                           kFbWarps * 32u);
         cp_commit();
         const uint32_t j = t & 3u;
         if (active)
         {
            const float ws = wd.warp_sum(t % uint32_t(NB), warp, j, lane);
            if (j == 0u)
               s02 = ws;
            else if (j == 1u)
               s13 = ws;
            else if (j == 2u)
               s02 = add_ftz(s02, ws);
            else
            {
               const uint32_t x0 = 32u * (s0 + sstep * (t >> 2)), x = x0 + lane;
               if (h == 3u)
                  list_insert(x < n && x != s ? add_ftz(s02, add_ftz(s13, ws)) : FLT_MAX, x0, cand, lane, e0, e1,
                              i0, i1);
               else
                  list_insert_pair(x < n && x != s ? add_ftz(s02, add_ftz(s13, ws)) : INFINITY, x0, cand, lane, e0,
                                   e1, i0, i1);
            }
         }
      }
      cp_wait<0>();
      if (active)
      {
         s_top[lane] = lane < cand ? i0 : 0xFFFFFFFFu;
         s_top[32u + lane] = lane + 32u < cand ? i1 : 0xFFFFFFFFu;
         anchor_hops(p, n, cand, s_hops, lane);
         write_row_warp(p, group, n, s, cand, s_top, s_hops, lane);
         __syncwarp();
      }
   }
}

// One block: the rejected rows of bucket (g, h) (fb_group_count[4 g + h] of them)
// become ceil(count / kFbWarps) tasks (group, bucket, first slot, rows), in bucket
// order (a block-wide scan of the buckets' task counts gives each thread's first task).
constexpr uint32_t kFbTaskThreads = 1024;

__global__ void __launch_bounds__(kFbTaskThreads) knn_fallback_tasks_kernel(const uint32_t *__restrict__ group_count,
                                                                            uint32_t G, uint32_t *__restrict__ tasks,
                                                                            uint32_t max_tasks,
                                                                            uint32_t *__restrict__ num_tasks)
{
   __shared__ uint32_t s_sum[kFbTaskThreads];
   const uint32_t tid = threadIdx.x;
   const uint32_t B = 4u * G; // buckets
   const uint32_t per = (B + kFbTaskThreads - 1) / kFbTaskThreads;
   const uint32_t b0 = min(B, tid * per), b1 = min(B, b0 + per);
   uint32_t local = 0;
   for (uint32_t b = b0; b < b1; ++b)
      local += (group_count[b] + kFbWarps - 1) / kFbWarps;
   s_sum[tid] = local;
   __syncthreads();
   for (uint32_t off = 1; off < kFbTaskThreads; off <<= 1)
   {
      const uint32_t v = tid >= off ? s_sum[tid - off] : 0u;
      __syncthreads();
      s_sum[tid] += v;
      __syncthreads();
   }
   uint32_t at = s_sum[tid] - local;
   for (uint32_t b = b0; b < b1; ++b)
   {
      const uint32_t c = group_count[b];
      for (uint32_t k = 0; k < c; k += kFbWarps, ++at)
         if (at < max_tasks)
         {
            tasks[4 * at] = b >> 2;
            tasks[4 * at + 1] = b & 3u;
            tasks[4 * at + 2] = k;
            tasks[4 * at + 3] = min(uint32_t(kFbWarps), c - k);
         }
   }
   if (tid == kFbTaskThreads - 1)
      *num_tasks = min(s_sum[tid], max_tasks);
}

template <int C, int W, int NB>
cudaError_t launch_rerank_nb(const KnnRerankParams &p, uint32_t num_items, cudaStream_t s)
{
   const size_t smem = kRrWarps * (size_t(WarpDist<C, W, NB>::kWarpFloats) * sizeof(float) +
                                   2 * kKnnMax * sizeof(uint32_t));
   cudaError_t e =
       cudaFuncSetAttribute(knn_rerank_kernel<C, W, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
   if (e != cudaSuccess)
      return e;
   knn_rerank_kernel<C, W, NB><<<num_items, kRrWarps * 32, smem, s>>>(p);
   return cudaGetLastError();
}

// A two-stage ring: occupancy (five blocks of four warps per SM for C = 1) hides more
// latency than deeper rings at fewer warps.
template <int C, int W>
cudaError_t launch_rerank_t(const KnnRerankParams &p, uint32_t num_items, cudaStream_t s)
{
   return launch_rerank_nb<C, W, 2>(p, num_items, s);
}

template <int C, int W>
cudaError_t launch_fallback_t(const KnnParams &p, const uint32_t *d_fb_rows, const uint32_t *d_pend_idx,
                              const float2 *d_pend, const uint32_t *d_tasks, const uint32_t *d_num_tasks,
                              uint32_t num_sms, cudaStream_t s)
{
   constexpr int NB = 4;
   using WD = WarpDist<C, W, NB>;
   static_assert(WD::kWarpFloats > 0, "the fallback's block shares one ring");
   const size_t smem = (NB * size_t(WD::kStage) + kFbWarps * size_t(WD::kQ)) * sizeof(float) +
                       kFbWarps * 2 * kKnnMax * sizeof(uint32_t);
   auto kern = knn_fallback_rows_kernel<C, W, NB>;
   cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
   if (e != cudaSuccess)
      return e;
   int per_sm = 0;
   if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kFbWarps * 32, smem)) != cudaSuccess)
      return e;
   const uint32_t grid = std::max<uint32_t>(1u, num_sms) * uint32_t(std::max(per_sm, 1));
   kern<<<grid, kFbWarps * 32, smem, s>>>(p, d_fb_rows, d_pend_idx, d_pend, d_tasks, d_num_tasks);
   return cudaGetLastError();
}

// Copy width: 16 bytes when every row starts 16-byte aligned, else 8 or 4.
int rr_width(const KnnParams &p)
{
   const uintptr_t x = reinterpret_cast<uintptr_t>(p.X);
   if (p.d % 4u == 0 && x % 16u == 0)
      return 16;
   if (p.d % 2u == 0 && x % 8u == 0)
      return 8;
   return 4;
}

// f(integral_constant<C>, integral_constant<W>) for the call's dimension and width.
template <class F>
cudaError_t by_dim(uint32_t d, int width, F &&f)
{
   const uint32_t c = (d + 127) / 128;
   auto by_w = [&](auto C) -> cudaError_t {
      if (width == 16)
         return f(C, std::integral_constant<int, 16>{});
      if (width == 8)
         return f(C, std::integral_constant<int, 8>{});
      return f(C, std::integral_constant<int, 4>{});
   };
   if (c == 1)
      return by_w(std::integral_constant<int, 1>{});
   if (c == 2)
      return by_w(std::integral_constant<int, 2>{});
   return by_w(std::integral_constant<int, 3>{});
}

} // namespace

cudaError_t launch_knn_fallback_tasks(const uint32_t *d_group_count, uint32_t num_groups, uint32_t *d_tasks,
                                      uint32_t max_tasks, uint32_t *d_num_tasks, cudaStream_t s)
{
   knn_fallback_tasks_kernel<<<1, kFbTaskThreads, 0, s>>>(d_group_count, num_groups, d_tasks, max_tasks, d_num_tasks);
   return cudaGetLastError();
}

cudaError_t launch_knn_fallback_rows(const KnnParams &p, const uint32_t *d_fb_rows, const uint32_t *d_pend_idx,
                                     const float2 *d_pend, const uint32_t *d_tasks, const uint32_t *d_num_tasks,
                                     uint32_t num_sms, cudaStream_t s)
{
   if (p.d > uint32_t(kRrMaxDim) || p.d == 0)
      return cudaErrorInvalidValue;
   return by_dim(p.d, rr_width(p), [&](auto C, auto W) {
      return launch_fallback_t<decltype(C)::value, decltype(W)::value>(p, d_fb_rows, d_pend_idx, d_pend, d_tasks,
                                                                       d_num_tasks, num_sms, s);
   });
}

cudaError_t launch_knn_rerank(const KnnRerankParams &p, uint32_t num_items, cudaStream_t s)
{
   if (num_items == 0)
      return cudaSuccess;
   if (p.p.d > uint32_t(kRrMaxDim) || p.p.d == 0)
      return cudaErrorInvalidValue;
   return by_dim(p.p.d, rr_width(p.p), [&](auto C, auto W) {
      return launch_rerank_t<decltype(C)::value, decltype(W)::value>(p, num_items, s);
   });
}

size_t knn_smem_bytes(uint32_t d)
{
   const uint32_t dpad = (d + 3) / 4 * 4;
   return (size_t(dpad) * (kKnnRows + kKnnCands) + kKnnRows * kLd + 2 * kKnnRows * kLl) * sizeof(float);
}

size_t knn_task_count(const uint32_t *ranges, uint32_t num_groups)
{
   size_t t = 0;
   for (uint32_t g = 0; g < num_groups; ++g)
      t += (ranges[2 * g + 1] - ranges[2 * g] + kKnnRows - 1) / kKnnRows;
   return t;
}

void knn_tasks(const uint32_t *ranges, uint32_t num_groups, uint32_t *tasks)
{
   size_t i = 0;
   for (uint32_t g = 0; g < num_groups; ++g)
      for (uint32_t r = 0; r < ranges[2 * g + 1] - ranges[2 * g]; r += kKnnRows)
      {
         tasks[2 * i] = g;
         tasks[2 * i + 1] = r;
         ++i;
      }
}

cudaError_t launch_exact_knn(const KnnParams &p, const uint32_t *d_tasks, uint32_t num_tasks, cudaStream_t s)
{
   if (num_tasks == 0)
      return cudaSuccess;
   const size_t smem = knn_smem_bytes(p.d);
   cudaError_t e = cudaFuncSetAttribute(exact_knn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
   if (e != cudaSuccess)
      return e;
   exact_knn_kernel<<<num_tasks, kKnnThreads, smem, s>>>(p, reinterpret_cast<const KnnTask *>(d_tasks));
   return cudaGetLastError();
}

cudaError_t launch_knn_two_phase(const KnnParams &p, const uint32_t *d_tiles, uint32_t num_tiles,
                                 const uint32_t *d_rows, uint32_t num_rows, cudaStream_t s)
{
   if (num_tiles)
   {
      const uint32_t dpad = (p.d + 3) / 4 * 4;
      const size_t smem = (size_t(dpad) * (kKnnRows + kKnnCands) + kKnnRows * kLd) * sizeof(float);
      cudaError_t e = cudaFuncSetAttribute(knn_dist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess)
         return e;
      knn_dist_kernel<<<num_tiles, kKnnThreads, smem, s>>>(p, reinterpret_cast<const KnnTile *>(d_tiles));
      if ((e = cudaGetLastError()) != cudaSuccess)
         return e;
   }
   if (num_rows)
      knn_rows_kernel<<<(num_rows + kRowWarps - 1) / kRowWarps, kRowWarps * 32, 0, s>>>(
          p, reinterpret_cast<const KnnTask *>(d_rows), num_rows);
   return cudaGetLastError();
}

} // namespace ungx
