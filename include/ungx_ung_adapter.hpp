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
 * generate_with_additional_edges adds build_cross_edges_generate_additional (exact
 * variant) with the cross edges kept in device memory, and build_cross_group_edges runs
 * the whole UniNavGraph::build_cross_group_edges step into the graph's neighbour lists.
 * The types are template parameters, so the header compiles without the reference's
 * headers and binds to ANNS::SearchQueue / ANNS::NeighborList / ANNS::IdxType /
 * std::pair ranges as they are.
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

// The problem arrays of the C ABI built from the reference's containers.
struct ProblemArrays
{
   std::vector<uint32_t> ranges;
   std::vector<uint64_t> off;
   std::vector<uint32_t> ids;
   ungx_cross_edge_problem p{};
};

template <class Idx, class RangePair>
inline void make_problem(uint32_t n, uint32_t d, uint32_t k, const std::vector<RangePair> &group_id_to_range,
                         const std::vector<std::vector<Idx>> &lng_out, ProblemArrays &a)
{
   const uint32_t G = group_id_to_range.empty() ? 0u : uint32_t(group_id_to_range.size() - 1);
   a.ranges.assign(2 * size_t(G + 1), 0);
   for (uint32_t g = 1; g <= G; ++g)
   {
      a.ranges[2 * g] = uint32_t(group_id_to_range[g].first);
      a.ranges[2 * g + 1] = uint32_t(group_id_to_range[g].second);
   }
   flatten_lng(lng_out, G, a.off, a.ids);
   a.p = ungx_cross_edge_problem{};
   a.p.num_points = n;
   a.p.dim = d;
   a.p.topk = k;
   a.p.num_groups = G;
   a.p.group_ranges = a.ranges.data();
   a.p.lng_out_offsets = a.off.data();
   a.p.lng_out_ids = a.ids.empty() ? nullptr : a.ids.data();
   a.p.route = UNGX_ROUTE_AUTO;
   a.p.shard_rank = 0;
   a.p.shard_count = 1;
}

// Flat ids / distances [n*k] into the writeback container `mode` names.
template <class SearchQueueT, class Idx>
inline void write_back(const std::vector<uint32_t> &out_ids, const std::vector<float> &out_d, uint32_t n, uint32_t k,
                       Writeback mode, std::vector<SearchQueueT> *search_queues,
                       std::vector<std::vector<Idx>> *id_vectors, std::vector<Idx> *flat_ids)
{
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
}

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
   ProblemArrays a;
   make_problem(n, d, k, group_id_to_range, lng_out, a);
   std::vector<uint32_t> out_ids(size_t(n) * k);
   std::vector<float> out_d(size_t(n) * k);
   res.status = ungx_cross_edges_build(ctx, base_vectors, &a.p, out_ids.data(), out_d.data(), &res.timing);
   if (res.status != UNGX_OK)
   {
      res.error = ungx_last_error(ctx);
      return res; // the reference then falls back to its CPU path or throws in strict mode
   }
   write_back(out_ids, out_d, n, k, mode, search_queues, id_vectors, flat_ids);
   res.ok = true;
   return res;
}

// The generate step and build_cross_edges_generate_additional with CpuExactScan
// (UNG/codes/src/uni_nav_graph_cross_edges.cpp:442-596) in one library call: the cross
// edges stay in device memory between the two.  The cross edges go to the writeback
// container `mode` names, the additional edges to materialized[group of from] as
// (from, to) pairs in the reference's order -- the lists
// append_materialized_additional_edges (UNG/codes/src/ung_cross_edge_output_writer.cpp:30-42)
// appends.  `new_vec_id_to_group_id` is the reference's map of the same name.
template <class SearchQueueT, class Idx, class RangePair, class PairT>
Result generate_with_additional_edges(ungx_context *ctx, const float *base_vectors, uint32_t n, uint32_t d,
                                      uint32_t k, const std::vector<RangePair> &group_id_to_range,
                                      const std::vector<std::vector<Idx>> &lng_out, Writeback mode,
                                      std::vector<SearchQueueT> *search_queues,
                                      std::vector<std::vector<Idx>> *id_vectors, std::vector<Idx> *flat_ids,
                                      const std::vector<Idx> &new_vec_id_to_group_id,
                                      std::vector<std::vector<PairT>> *materialized)
{
   Result res;
   ProblemArrays a;
   make_problem(n, d, k, group_id_to_range, lng_out, a);
   std::vector<uint32_t> out_ids(size_t(n) * k);
   std::vector<float> out_d(size_t(n) * k);
   ungx_cross_group_stats st{};
   res.status = ungx_build_cross_group_edges(ctx, base_vectors, &a.p, nullptr, nullptr, UNGX_BUILD_ADDITIONAL,
                                             out_ids.data(), out_d.data(), &st);
   std::vector<uint32_t> from, to;
   if (res.status == UNGX_OK)
   {
      from.resize(st.additional.edges);
      to.resize(st.additional.edges);
      res.status = ungx_additional_edges_copy(ctx, from.data(), to.data(), nullptr, nullptr);
   }
   if (res.status != UNGX_OK)
   {
      res.error = ungx_last_error(ctx);
      return res;
   }
   res.timing = st.cross;
   write_back(out_ids, out_d, n, k, mode, search_queues, id_vectors, flat_ids);
   if (materialized)
   {
      materialized->resize(a.p.num_groups + size_t(1));
      for (size_t i = 0; i < from.size(); ++i)
         (*materialized)[new_vec_id_to_group_id[from[i]]].emplace_back(Idx(from[i]), Idx(to[i]));
   }
   res.ok = true;
   return res;
}

// The whole of UniNavGraph::build_cross_group_edges
// (UNG/codes/src/uni_nav_graph_cross_edges.cpp:613-913) on the device: cross edges,
// exact additional edges, add_offset_for_uni_nav_graph (UNG/codes/src/uni_nav_graph.cpp:285-297)
// and the merge into the graph.  `neighbors[0..n)` (_graph->neighbors: any container
// with begin/end, clear and push_back) holds the intra-group edges on entry -- group-local
// ids unless `intra_ids_are_global` -- and each point's final adjacency on return: intra
// edges with global ids, cross edges nearest first, additional edges.
template <class NeighborListT, class Idx, class RangePair>
Result build_cross_group_edges(ungx_context *ctx, const float *base_vectors, uint32_t n, uint32_t d, uint32_t k,
                               const std::vector<RangePair> &group_id_to_range,
                               const std::vector<std::vector<Idx>> &lng_out, NeighborListT *neighbors,
                               bool intra_ids_are_global)
{
   Result res;
   ProblemArrays a;
   make_problem(n, d, k, group_id_to_range, lng_out, a);
   std::vector<uint64_t> ioff(size_t(n) + 1, 0);
   for (uint32_t v = 0; v < n; ++v)
      ioff[v + 1] = ioff[v] + uint64_t(neighbors[v].end() - neighbors[v].begin());
   std::vector<uint32_t> icols(ioff[n]);
   for (uint32_t v = 0; v < n; ++v)
   {
      uint64_t w = ioff[v];
      for (auto it = neighbors[v].begin(); it != neighbors[v].end(); ++it)
         icols[w++] = uint32_t(*it);
   }
   ungx_cross_group_stats st{};
   const uint32_t flags = UNGX_BUILD_ADDITIONAL | (intra_ids_are_global ? 0u : uint32_t(UNGX_BUILD_INTRA_LOCAL_IDS));
   res.status = ungx_build_cross_group_edges(ctx, base_vectors, &a.p, ioff.data(), icols.empty() ? nullptr : icols.data(),
                                             flags, nullptr, nullptr, &st);
   if (res.status != UNGX_OK)
   {
      res.error = ungx_last_error(ctx);
      return res;
   }
   std::vector<uint64_t> off(size_t(n) + 1);
   std::vector<uint32_t> cols(st.num_cols);
   res.status = ungx_graph_copy(ctx, off.data(), cols.data());
   if (res.status != UNGX_OK)
   {
      res.error = ungx_last_error(nullptr); // calls on a const context report globally
      return res;
   }
   res.timing = st.cross;
   for (uint32_t v = 0; v < n; ++v)
   {
      neighbors[v].clear();
      for (uint64_t i = off[v]; i < off[v + 1]; ++i)
         neighbors[v].push_back(Idx(cols[i]));
   }
   res.ok = true;
   return res;
}

} // namespace ungx_adapter

#endif // UNGX_UNG_ADAPTER_HPP
