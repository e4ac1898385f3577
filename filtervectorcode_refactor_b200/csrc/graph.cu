// Graph assembly on the device (sm_100a): the row -> group map, the LNG edges that
// cross edges reach (input of the additional-edge rule of
// UNG/codes/src/uni_nav_graph_cross_edges.cpp:442-596), and the whole-graph
// adjacency as CSR in the reference's per-point order (intra-group edges, cross
// edges in queue order, additional edges; UNG/codes/src/uni_nav_graph.cpp:285-297 and
// UNG/codes/src/ung_cross_edge_output_writer.cpp:17-149).  All of it is integer,
// HBM-bound work: coalesced grid-stride loops, one pass over each array.
#include <algorithm>

#include "kernels.h"

namespace ungx
{
namespace
{
constexpr uint32_t kScanThreads = 512;
constexpr uint32_t kScanItems = 4;
constexpr uint32_t kScanTile = kScanThreads * kScanItems;

__global__ void fill_u32_kernel(uint32_t *p, uint32_t n, uint32_t v)
{
   for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
      p[i] = v;
}

// One block per group: its rows get the group id.
__global__ void group_of_kernel(const uint32_t *__restrict__ ranges, uint32_t G, uint32_t n,
                                uint32_t *__restrict__ group_of)
{
   for (uint32_t g = blockIdx.x + 1; g <= G; g += gridDim.x)
   {
      const uint32_t a = ranges[2 * g], b = min(ranges[2 * g + 1], n);
      for (uint32_t v = a + threadIdx.x; v < b; v += blockDim.x)
         group_of[v] = g;
   }
}

// Thread per row: every non-empty cross-edge slot marks the LNG edge from the row's
// group to the neighbour's group (out lists are short: a linear search).
__global__ void mark_reached_kernel(const uint32_t *__restrict__ cross_ids, uint32_t n, uint32_t k,
                                    const uint32_t *__restrict__ group_of, uint32_t G,
                                    const uint64_t *__restrict__ out_offsets, const uint32_t *__restrict__ out_ids,
                                    uint8_t *__restrict__ flags)
{
   for (uint32_t v = blockIdx.x * blockDim.x + threadIdx.x; v < n; v += gridDim.x * blockDim.x)
   {
      const uint32_t f = group_of[v];
      if (f == 0 || f > G)
         continue;
      const uint64_t e0 = out_offsets[f], e1 = out_offsets[f + 1];
      for (uint32_t j = 0; j < k; ++j)
      {
         const uint32_t id = cross_ids[size_t(v) * k + j];
         if (id >= n)
            continue; // empty slot
         const uint32_t g = group_of[id];
         for (uint64_t e = e0; e < e1; ++e)
            if (out_ids[e] == g)
            {
               flags[e] = 1;
               break;
            }
      }
   }
}

__device__ __forceinline__ uint32_t cross_count(const uint32_t *cross_ids, uint32_t v, uint32_t k)
{
   uint32_t c = 0;
   while (c < k && cross_ids[size_t(v) * k + c] != 0xFFFFFFFFu)
      ++c;
   return c;
}

__global__ void graph_degrees_kernel(uint32_t n, uint32_t k, const uint64_t *__restrict__ intra_off,
                                     const uint32_t *__restrict__ cross_ids, const uint64_t *__restrict__ add_off,
                                     uint64_t *__restrict__ offsets)
{
   for (uint32_t v = blockIdx.x * blockDim.x + threadIdx.x; v <= n; v += gridDim.x * blockDim.x)
   {
      uint64_t deg = 0;
      if (v < n)
      {
         if (intra_off)
            deg += intra_off[v + 1] - intra_off[v];
         if (cross_ids)
            deg += cross_count(cross_ids, v, k);
         if (add_off)
            deg += add_off[v + 1] - add_off[v];
      }
      offsets[v] = deg;
   }
}

// Exclusive scan, phase 1: each block scans a tile of kScanTile values in place and
// leaves the tile's total in sums[block].
__global__ void __launch_bounds__(kScanThreads) scan_tiles_kernel(uint64_t *__restrict__ data, uint32_t count,
                                                                  uint64_t *__restrict__ sums)
{
   __shared__ uint64_t warp_tot[kScanThreads / 32];
   const uint32_t base = blockIdx.x * kScanTile + threadIdx.x * kScanItems;
   uint64_t v[kScanItems], run = 0;
#pragma unroll
   for (uint32_t i = 0; i < kScanItems; ++i)
   {
      v[i] = base + i < count ? data[base + i] : 0;
      const uint64_t t = v[i];
      v[i] = run; // exclusive within the thread
      run += t;
   }
   // exclusive scan of the thread totals across the block
   const uint32_t lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
   uint64_t inc = run;
#pragma unroll
   for (int o = 1; o < 32; o <<= 1)
   {
      const uint64_t y = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= uint32_t(o))
         inc += y;
   }
   if (lane == 31)
      warp_tot[wid] = inc;
   __syncthreads();
   if (wid == 0)
   {
      uint64_t w = lane < kScanThreads / 32 ? warp_tot[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1)
      {
         const uint64_t y = __shfl_up_sync(0xffffffffu, w, o);
         if (lane >= uint32_t(o))
            w += y;
      }
      if (lane < kScanThreads / 32)
         warp_tot[lane] = w; // inclusive over warps
   }
   __syncthreads();
   const uint64_t before = (inc - run) + (wid ? warp_tot[wid - 1] : 0);
#pragma unroll
   for (uint32_t i = 0; i < kScanItems; ++i)
      if (base + i < count)
         data[base + i] = v[i] + before;
   if (threadIdx.x == kScanThreads - 1)
      sums[blockIdx.x] = before + run;
}

// Phase 2: one block turns the tile totals into exclusive tile offsets.
__global__ void __launch_bounds__(1024) scan_sums_kernel(uint64_t *__restrict__ sums, uint32_t tiles)
{
   __shared__ uint64_t part[1024];
   const uint32_t per = (tiles + 1023) / 1024;
   const uint32_t a = threadIdx.x * per, b = min(a + per, tiles);
   uint64_t run = 0;
   for (uint32_t i = a; i < b; ++i)
      run += sums[i];
   part[threadIdx.x] = run;
   __syncthreads();
   for (uint32_t o = 1; o < 1024; o <<= 1)
   {
      const uint64_t y = threadIdx.x >= o ? part[threadIdx.x - o] : 0;
      __syncthreads();
      part[threadIdx.x] += y;
      __syncthreads();
   }
   uint64_t off = threadIdx.x ? part[threadIdx.x - 1] : 0;
   for (uint32_t i = a; i < b; ++i)
   {
      const uint64_t t = sums[i];
      sums[i] = off;
      off += t;
   }
}

// Phase 3: tile offsets added to every value.
__global__ void scan_add_kernel(uint64_t *__restrict__ data, uint32_t count, const uint64_t *__restrict__ sums)
{
   const uint64_t add = sums[blockIdx.x];
   const uint32_t base = blockIdx.x * kScanTile;
   for (uint32_t i = threadIdx.x; i < kScanTile && base + i < count; i += blockDim.x)
      data[base + i] += add;
}

// Warp per point: intra edges, cross edges up to the first sentinel, additional edges.
// The point's offsets and its first 32 cross slots are loaded together up front (one
// slot per lane); the cross count is the position of the first sentinel, found by a
// ballot instead of a serial walk of the row.
// With group_of / ranges given, intra columns are group-local ids and get the first
// row of the point's group added (add_offset_for_uni_nav_graph,
// UNG/codes/src/uni_nav_graph.cpp:285-297).
__global__ void graph_fill_kernel(uint32_t n, uint32_t k, const uint64_t *__restrict__ intra_off,
                                  const uint32_t *__restrict__ intra_cols, const uint32_t *__restrict__ group_of,
                                  const uint32_t *__restrict__ ranges, const uint32_t *__restrict__ cross_ids,
                                  const uint64_t *__restrict__ add_off, const uint32_t *__restrict__ add_cols,
                                  const uint64_t *__restrict__ offsets, uint32_t *__restrict__ cols)
{
   const uint32_t lane = threadIdx.x & 31;
   const uint64_t warps = (uint64_t(gridDim.x) * blockDim.x) >> 5;
   for (uint64_t v = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; v < n; v += warps)
   {
      uint64_t w = offsets[v];
      const uint64_t ia = intra_off ? intra_off[v] : 0, ib = intra_off ? intra_off[v + 1] : 0;
      const uint64_t aa = add_off ? add_off[v] : 0, ab = add_off ? add_off[v + 1] : 0;
      const uint32_t x0 = cross_ids && lane < k ? cross_ids[v * k + lane] : 0xFFFFFFFFu;
      if (intra_off)
      {
         const uint32_t shift = group_of ? ranges[2 * group_of[v]] : 0u;
         for (uint64_t i = ia + lane; i < ib; i += 32)
            cols[w + (i - ia)] = intra_cols[i] + shift;
         w += ib - ia;
      }
      if (cross_ids)
      {
         uint32_t x = x0;
         for (uint32_t base = 0;; base += 32) // warp-uniform: every lane sees the same ballot
         {
            const uint32_t empty = __ballot_sync(0xffffffffu, x == 0xFFFFFFFFu);
            const uint32_t cnt = empty ? uint32_t(__ffs(empty) - 1) : 32u;
            if (lane < cnt)
               cols[w + base + lane] = x;
            if (cnt < 32 || base + 32 >= k)
            {
               w += base + cnt;
               break;
            }
            x = base + 32 + lane < k ? cross_ids[v * k + base + 32 + lane] : 0xFFFFFFFFu;
         }
      }
      if (add_off)
         for (uint64_t i = aa + lane; i < ab; i += 32)
            cols[w + (i - aa)] = add_cols[i];
   }
}

// ------------------------------------------------------------------ additional edges
// The reference's loop over LNG edges f -> f' that no cross edge reaches
// (UNG/codes/src/uni_nav_graph_cross_edges.cpp:442-596) as device passes over the edges
// of each source group, in the reference's order (groups ascending, out-groups in
// order, vectors ascending).  Only the first k vectors of a group can get edges.

// Thread per source group: q_e queries for each unreached edge e (each vector of f adds
// m = min(|f'|, k/2) edges, so ceil(k / m) vectors, |f| at most), 0 otherwise; the
// reference's counters of missing edges and scanned vectors.
__global__ void add_edge_queries_kernel(const uint32_t *__restrict__ ranges, uint32_t G,
                                        const uint64_t *__restrict__ out_off, const uint32_t *__restrict__ out_ids,
                                        const uint8_t *__restrict__ reached, uint32_t k, uint64_t *__restrict__ qcnt,
                                        unsigned long long *__restrict__ stats)
{
   unsigned long long miss = 0, scanned = 0;
   for (uint32_t f = blockIdx.x * blockDim.x + threadIdx.x + 1; f <= G; f += gridDim.x * blockDim.x)
   {
      const uint32_t fs = ranges[2 * f + 1] - ranges[2 * f];
      for (uint64_t e = out_off[f]; e < out_off[f + 1]; ++e)
      {
         uint64_t q = 0;
         if (!reached[e])
         {
            const uint32_t t = out_ids[e];
            const uint32_t m = min(ranges[2 * t + 1] - ranges[2 * t], k / 2u);
            ++miss;
            if (m == 0)
               scanned += fs; // the reference scans every vector of f, adding nothing
            else
            {
               q = min(fs, (k + m - 1u) / m);
               scanned += q;
            }
         }
         qcnt[e] = q;
      }
   }
#pragma unroll
   for (int o = 16; o; o >>= 1)
   {
      miss += __shfl_xor_sync(0xffffffffu, miss, o);
      scanned += __shfl_xor_sync(0xffffffffu, scanned, o);
   }
   if ((threadIdx.x & 31u) == 0 && (miss | scanned))
   {
      atomicAdd(&stats[0], miss);
      atomicAdd(&stats[1], scanned);
   }
}

// Thread per source group: edge e's queries are rows qf .. qf + q_e - 1 at qoff[e]: a
// work item (rows, one target segment) per edge and the per-query row, item and slot.
__global__ void add_query_fill_kernel(const uint32_t *__restrict__ ranges, uint32_t G,
                                      const uint64_t *__restrict__ out_off, const uint32_t *__restrict__ out_ids,
                                      const uint64_t *__restrict__ qoff, WorkItem *__restrict__ items,
                                      Segment *__restrict__ segs, uint32_t *__restrict__ rows,
                                      uint32_t *__restrict__ row_items, uint32_t *__restrict__ pos)
{
   for (uint32_t f = blockIdx.x * blockDim.x + threadIdx.x + 1; f <= G; f += gridDim.x * blockDim.x)
   {
      const uint32_t qf = ranges[2 * f];
      for (uint64_t e = out_off[f]; e < out_off[f + 1]; ++e)
      {
         const uint32_t q = uint32_t(qoff[e + 1] - qoff[e]);
         if (q == 0)
            continue;
         const uint32_t t = out_ids[e];
         items[e] = {qf, q, uint32_t(e), 1u};
         segs[e] = {ranges[2 * t], ranges[2 * t + 1] - ranges[2 * t], t, 0u};
         for (uint32_t i = 0; i < q; ++i)
         {
            const uint32_t w = uint32_t(qoff[e]) + i;
            rows[w] = qf + i;
            row_items[w] = uint32_t(e);
            pos[w] = w;
         }
      }
   }
}

// Per query: the entries of its top-(k/2) before the first empty slot.
__global__ void add_count_kernel(const uint32_t *__restrict__ res, uint32_t nq, uint32_t kh, uint64_t *__restrict__ lcnt)
{
   for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < nq; i += gridDim.x * blockDim.x)
   {
      uint32_t c = 0;
      while (c < kh && res[size_t(i) * kh + c] != 0xFFFFFFFFu)
         ++c;
      lcnt[i] = c;
   }
}

// Per query: its entries into the (from, to) list at loff[i].
__global__ void add_list_kernel(const uint32_t *__restrict__ res, const uint32_t *__restrict__ rows, uint32_t nq,
                                uint32_t kh, const uint64_t *__restrict__ loff, uint32_t *__restrict__ from,
                                uint32_t *__restrict__ to)
{
   for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < nq; i += gridDim.x * blockDim.x)
   {
      const uint64_t a = loff[i], c = loff[i + 1] - a;
      for (uint32_t r = 0; r < c; ++r)
      {
         from[a + r] = rows[i];
         to[a + r] = res[size_t(i) * kh + r];
      }
   }
}

// Thread per (source group f, vector t < k): vector v = qf + t's entries over f's edges
// in order.  COUNT: their number into deg[v]; else: the entries at off[v].
template <bool COUNT>
__global__ void add_point_kernel(const uint32_t *__restrict__ ranges, uint32_t G, uint32_t k,
                                 const uint64_t *__restrict__ out_off, const uint64_t *__restrict__ qoff,
                                 const uint64_t *__restrict__ loff, const uint32_t *__restrict__ to,
                                 uint64_t *__restrict__ deg_or_off, uint32_t *__restrict__ cols)
{
   const uint64_t total = uint64_t(G) * k;
   for (uint64_t idx = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
        idx += uint64_t(gridDim.x) * blockDim.x)
   {
      const uint32_t f = uint32_t(idx / k) + 1u, t = uint32_t(idx % k);
      const uint32_t qf = ranges[2 * f];
      if (t >= ranges[2 * f + 1] - qf)
         continue;
      const uint32_t v = qf + t;
      uint64_t c = 0, w = COUNT ? 0 : deg_or_off[v];
      for (uint64_t e = out_off[f]; e < out_off[f + 1]; ++e)
      {
         if (qoff[e + 1] - qoff[e] <= t)
            continue;
         const uint64_t i = qoff[e] + t;
         if (COUNT)
            c += loff[i + 1] - loff[i];
         else
            for (uint64_t j = loff[i]; j < loff[i + 1]; ++j)
               cols[w++] = to[j];
      }
      if (COUNT)
         deg_or_off[v] = c;
   }
}

uint32_t grid_for(uint64_t work, uint32_t threads)
{
   const uint64_t g = (work + threads - 1) / threads;
   return uint32_t(std::max<uint64_t>(1, std::min<uint64_t>(g, 148ull * 32)));
}
} // namespace

cudaError_t launch_group_of(const uint32_t *ranges, uint32_t G, uint32_t n, uint32_t *group_of, cudaStream_t s)
{
   if (n == 0)
      return cudaSuccess;
   fill_u32_kernel<<<grid_for(n, 256), 256, 0, s>>>(group_of, n, G + 1);
   if (G)
      group_of_kernel<<<std::min<uint32_t>(G, 148u * 64), 128, 0, s>>>(ranges, G, n, group_of);
   return cudaGetLastError();
}

cudaError_t launch_mark_reached(const uint32_t *cross_ids, uint32_t n, uint32_t k, const uint32_t *group_of,
                                uint32_t G, const uint64_t *out_offsets, const uint32_t *out_ids, uint8_t *flags,
                                cudaStream_t s)
{
   if (n == 0 || k == 0)
      return cudaSuccess;
   mark_reached_kernel<<<grid_for(n, 256), 256, 0, s>>>(cross_ids, n, k, group_of, G, out_offsets, out_ids, flags);
   return cudaGetLastError();
}

size_t csr_scan_scratch_bytes(uint32_t n) { return (size_t(n) + 1 + kScanTile) / kScanTile * sizeof(uint64_t); }

cudaError_t launch_graph_degrees(uint32_t n, uint32_t k, const uint64_t *intra_off, const uint32_t *cross_ids,
                                 const uint64_t *add_off, uint64_t *offsets, cudaStream_t s)
{
   graph_degrees_kernel<<<grid_for(uint64_t(n) + 1, 256), 256, 0, s>>>(n, k, intra_off, cross_ids, add_off, offsets);
   return cudaGetLastError();
}

cudaError_t launch_exclusive_scan_u64(uint64_t *data, uint32_t count, void *scratch, cudaStream_t s)
{
   if (count == 0)
      return cudaSuccess;
   const uint32_t tiles = (count + kScanTile - 1) / kScanTile;
   uint64_t *sums = static_cast<uint64_t *>(scratch);
   scan_tiles_kernel<<<tiles, kScanThreads, 0, s>>>(data, count, sums);
   scan_sums_kernel<<<1, 1024, 0, s>>>(sums, tiles);
   scan_add_kernel<<<tiles, 256, 0, s>>>(data, count, sums);
   return cudaGetLastError();
}

cudaError_t launch_add_edge_queries(const uint32_t *ranges, uint32_t G, const uint64_t *out_off, const uint32_t *out_ids,
                                    const uint8_t *reached, uint32_t k, uint64_t *qcnt, unsigned long long *stats,
                                    cudaStream_t s)
{
   if (G == 0)
      return cudaSuccess;
   add_edge_queries_kernel<<<grid_for(G, 128), 128, 0, s>>>(ranges, G, out_off, out_ids, reached, k, qcnt, stats);
   return cudaGetLastError();
}

cudaError_t launch_add_query_fill(const uint32_t *ranges, uint32_t G, const uint64_t *out_off, const uint32_t *out_ids,
                                  const uint64_t *qoff, WorkItem *items, Segment *segs, uint32_t *rows,
                                  uint32_t *row_items, uint32_t *pos, cudaStream_t s)
{
   if (G == 0)
      return cudaSuccess;
   add_query_fill_kernel<<<grid_for(G, 128), 128, 0, s>>>(ranges, G, out_off, out_ids, qoff, items, segs, rows,
                                                          row_items, pos);
   return cudaGetLastError();
}

cudaError_t launch_add_list(const uint32_t *res, const uint32_t *rows, uint32_t nq, uint32_t kh, uint64_t *loff,
                            uint32_t *from, uint32_t *to, void *scratch, cudaStream_t s)
{
   if (nq == 0)
      return cudaSuccess;
   add_count_kernel<<<grid_for(nq, 256), 256, 0, s>>>(res, nq, kh, loff);
   cudaError_t e = cudaMemsetAsync(loff + nq, 0, sizeof(uint64_t), s);
   if (e == cudaSuccess)
      e = launch_exclusive_scan_u64(loff, nq + 1, scratch, s);
   if (e != cudaSuccess)
      return e;
   add_list_kernel<<<grid_for(nq, 256), 256, 0, s>>>(res, rows, nq, kh, loff, from, to);
   return cudaGetLastError();
}

cudaError_t launch_add_points(const uint32_t *ranges, uint32_t G, uint32_t n, uint32_t k, const uint64_t *out_off,
                              const uint64_t *qoff, const uint64_t *loff, const uint32_t *to, uint64_t *off,
                              uint32_t *cols, void *scratch, cudaStream_t s)
{
   cudaError_t e = cudaMemsetAsync(off, 0, (size_t(n) + 1) * sizeof(uint64_t), s);
   if (e != cudaSuccess || G == 0)
      return e;
   const uint32_t grid = grid_for(uint64_t(G) * k, 256);
   add_point_kernel<true><<<grid, 256, 0, s>>>(ranges, G, k, out_off, qoff, loff, to, off, cols);
   if ((e = launch_exclusive_scan_u64(off, n + 1, scratch, s)) != cudaSuccess)
      return e;
   add_point_kernel<false><<<grid, 256, 0, s>>>(ranges, G, k, out_off, qoff, loff, to, off, cols);
   return cudaGetLastError();
}

cudaError_t launch_graph_fill(uint32_t n, uint32_t k, const uint64_t *intra_off, const uint32_t *intra_cols,
                              const uint32_t *cross_ids, const uint64_t *add_off, const uint32_t *add_cols,
                              const uint64_t *offsets, uint32_t *cols, cudaStream_t s, const uint32_t *group_of,
                              const uint32_t *ranges)
{
   if (n == 0)
      return cudaSuccess;
   graph_fill_kernel<<<grid_for(uint64_t(n) * 32, 256), 256, 0, s>>>(n, k, intra_off, intra_cols, group_of, ranges,
                                                                      cross_ids, add_off, add_cols, offsets, cols);
   return cudaGetLastError();
}

} // namespace ungx
