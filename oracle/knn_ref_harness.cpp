// TEST INFRASTRUCTURE ONLY -- the reference's own GPU exact kNN seeding, for the parity
// tests of the device kNN seeding (tests/test_knn_gpu.py).
//
// Linked with UNG/codes/src/tagore_graph_builder.cu compiled where it lies (oracle/Makefile,
// target `ref`, with the reference's --use_fast_math and the stand-in header of
// oracle/tagore_stub for the absent external Tagore library).  ungref_knn_batch calls
// the reference's public ANNS::build_tagore_vamana_cuda_batch with prune mode FastGrnnd
// and a fast-exact threshold above every group, so every group goes through
// build_fast_exact_cuda_batch and batched_exact_knn_graph_kernel
// (UNG/codes/src/tagore_graph_builder.cu:650-795, 1058-1340): the rows it returns are
// the reference's.
#include <cstdint>
#include <cstring>
#include <exception>
#include <limits>
#include <vector>

#include "tagore_graph_builder.h"

extern "C" int ungref_knn_batch(const float *data, uint32_t dim, uint32_t num_groups, const uint32_t *group_sizes,
                                uint32_t candidate_k, uint32_t final_degree, uint32_t head_keep, uint32_t anchor_tail,
                                uint32_t anchor_slots, uint32_t bidir_anchor, uint32_t graph_stride, uint32_t *graph,
                                uint32_t *entry_points)
{
   try
   {
      std::vector<ANNS::TagoreGroupRequest> groups(num_groups);
      const float *p = data;
      uint64_t total = 0;
      for (uint32_t g = 0; g < num_groups; ++g)
      {
         groups[g].data = p;
         groups[g].num_points = group_sizes[g];
         p += size_t(group_sizes[g]) * dim;
         total += group_sizes[g];
      }
      ANNS::TagoreCudaRuntimeConfig cfg;
      cfg.fast_exact_batch_threshold = std::numeric_limits<uint32_t>::max();
      cfg.requested_streams = 1;
      cfg.fast_exact.head_keep = head_keep;
      cfg.fast_exact.anchor_tail = anchor_tail;
      cfg.fast_exact.anchor_slots = anchor_slots;
      cfg.fast_exact.bidir_anchor = bidir_anchor;
      cfg.fast_exact.reverse_cap = 0;
      cfg.fast_exact.reverse_slots = 0;
      cfg.fast_exact.graph_stride = graph_stride;
      cfg.fast_exact.use_warp_kernel = false;
      const ANNS::TagoreBatchBuildResult r = ANNS::build_tagore_vamana_cuda_batch(
          groups, dim, candidate_k, final_degree, /*top_m=*/1, /*iterations=*/1, /*alpha=*/1.2f,
          ANNS::TagorePruneMode::FastGrnnd, cfg);
      if (r.packed_graph.size() != total * graph_stride || r.groups.size() != num_groups)
         return -2;
      std::memcpy(graph, r.packed_graph.data(), r.packed_graph.size() * sizeof(uint32_t));
      if (entry_points)
         for (uint32_t g = 0; g < num_groups; ++g)
            entry_points[g] = r.groups[g].entry_point;
      return 0;
   }
   catch (const std::exception &)
   {
      return -1;
   }
}
