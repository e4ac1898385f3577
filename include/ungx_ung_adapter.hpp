/*
 * ungx_ung_adapter.hpp -- header-only C++ glue between the reference's UniNavGraph
 * and the C ABI of include/ungx.h.
 *
 * It replaces the device work of
 *   bool UniNavGraph::build_cross_edges_generate_gpu_optimized(
 *       std::vector<SearchQueue>&, const CrossEdgeGpuRuntimeConfig&,
 *       std::vector<std::vector<IdxType>>*, std::vector<IdxType>*, CrossEdgeBuildTiming&)
 * (UNG/codes/include/uni_nav_graph.h:403-407, UNG/codes/src/uni_nav_graph_cross_edges.cpp:334-440)
 * and materialises the result in whichever writeback the reference asked for
 * (CrossEdgeGpuWritebackMode, UNG/codes/include/ung_cross_edge_config.h:17-22):
 *   - FlatId:      flat ids, UINT32_MAX = empty (ung_cross_edge_output_writer.cpp:78-88);
 *   - IdVector:    the valid ids of each point, nearest first;
 *   - SearchQueue: SearchQueue::insert of each (id, distance), after reserve(k), as the
 *                  reference's finaliser does (UNG/codes/src/gpu_cross_edge_output.cuh:120-132).
 * The types are template parameters, so the header compiles without the reference's
 * headers and binds to ANNS::SearchQueue / ANNS::IdxType / std::pair ranges as they are.
 */
#ifndef UNGX_UNG_ADAPTER_HPP
#define UNGX_UNG_ADAPTER_HPP

#include <cstdint>
#include <limits>
#include <string>
#include <vector>

#include "ungx.h"

namespace ungx_adapter
{

enum class Writeback
{
   SearchQueue = UNGX_WRITEBACK_SEARCH_QUEUE,
   IdVector = UNGX_WRITEBACK_ID_VECTOR,
   FlatId = UNGX_WRITEBACK_FLAT_ID
};

// Out-neighbours std::vector<std::vector<Idx>> (index = group id, 0 unused) to CSR.
template <class Idx>
inline void flatten_lng(const std::vector<std::vector<Idx>> &out_neighbors, uint32_t num_groups,
                        std::vector<uint64_t> &offsets, std::vector<uint32_t> &ids)
{
   offsets.assign(size_t(num_groups) + 2, 0);
   ids.clear();
   for (uint32_t g = 0; g <= num_groups; ++g)
   {
      offsets[g] = ids.size();
      if (g < out_neighbors.size())
         for (Idx t : out_neighbors[g])
            ids.push_back(uint32_t(t));
   }
   offsets[size_t(num_groups) + 1] = ids.size();
}

struct Result
{
   bool ok = false;
   int status = UNGX_OK;
   std::string error;
   ungx_cross_edge_timing timing{};
};

// One call = the whole seam: upload + operand build + planning + kernels + D2H.
//   base_vectors      reordered n x d fp32 rows (_base_storage->get_vector(0))
//   group_id_to_range std::vector<std::pair<Idx, Idx>> of G+1 entries (entry 0 unused)
//   lng_out           _label_nav_graph->out_neighbors
// Exactly one of the three outputs is written, per `mode`.
template <class SearchQueueT, class Idx, class RangePair>
Result generate_cross_edges(ungx_context *ctx, const float *base_vectors, uint32_t n, uint32_t d, uint32_t k,
                            const std::vector<RangePair> &group_id_to_range,
                            const std::vector<std::vector<Idx>> &lng_out, Writeback mode,
                            std::vector<SearchQueueT> *search_queues, std::vector<std::vector<Idx>> *id_vectors,
                            std::vector<Idx> *flat_ids)
{
   Result res;
   const uint32_t G = group_id_to_range.empty() ? 0u : uint32_t(group_id_to_range.size() - 1);
   std::vector<uint32_t> ranges(2 * size_t(G + 1), 0);
   for (uint32_t g = 1; g <= G; ++g)
   {
      ranges[2 * g] = uint32_t(group_id_to_range[g].first);
      ranges[2 * g + 1] = uint32_t(group_id_to_range[g].second);
   }
   std::vector<uint64_t> off;
   std::vector<uint32_t> ids;
   flatten_lng(lng_out, G, off, ids);

   ungx_cross_edge_problem p{};
   p.num_points = n;
   p.dim = d;
   p.topk = k;
   p.num_groups = G;
   p.group_ranges = ranges.data();
   p.lng_out_offsets = off.data();
   p.lng_out_ids = ids.empty() ? nullptr : ids.data();
   p.route = UNGX_ROUTE_AUTO;
   p.shard_rank = 0;
   p.shard_count = 1;

   std::vector<uint32_t> out_ids(size_t(n) * k);
   std::vector<float> out_d(size_t(n) * k);
   res.status = ungx_cross_edges_build(ctx, base_vectors, &p, out_ids.data(), out_d.data(), &res.timing);
   if (res.status != UNGX_OK)
   {
      res.error = ungx_last_error(ctx);
      return res; // the reference then falls back to its CPU path or throws in strict mode
   }
   const uint32_t EMPTY = std::numeric_limits<uint32_t>::max();
   if (mode == Writeback::FlatId && flat_ids)
   {
      flat_ids->resize(size_t(n) * k);
      for (size_t i = 0; i < out_ids.size(); ++i)
         (*flat_ids)[i] = Idx(out_ids[i]);
   }
   else if (mode == Writeback::IdVector && id_vectors)
   {
      id_vectors->resize(n);
      for (uint32_t v = 0; v < n; ++v)
      {
         auto &dst = (*id_vectors)[v];
         dst.clear();
         for (uint32_t i = 0; i < k; ++i)
            if (out_ids[size_t(v) * k + i] != EMPTY)
               dst.push_back(Idx(out_ids[size_t(v) * k + i]));
      }
   }
   else if (search_queues)
   {
      search_queues->resize(n);
      for (uint32_t v = 0; v < n; ++v)
      {
         auto &q = (*search_queues)[v];
         q.reserve(int32_t(k));
         for (uint32_t i = 0; i < k; ++i)
            if (out_ids[size_t(v) * k + i] != EMPTY)
               q.insert(Idx(out_ids[size_t(v) * k + i]), out_d[size_t(v) * k + i]);
      }
   }
   res.ok = true;
   return res;
}

} // namespace ungx_adapter

#endif // UNGX_UNG_ADAPTER_HPP
