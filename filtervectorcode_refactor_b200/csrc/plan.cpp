// Host planning of the cross-edge work (a5) and the flat->CSR materialisation (a14).
//
// The reference plans target-centrically: per target group f' it gathers every
// query of every in-group into one batch (plan_cross_edge_target_workload,
// UNG/codes/src/gpu_cross_edge_planning.cuh:66-141) and later merges the per-target
// top-k of each query on the host or under a device spin lock
// (UNG/codes/src/gpu_gemm_topk.cu:252-309).  Here the plan is source-centric: a
// work item is <=128 consecutive rows of one source group with the list of its
// target groups, so every row's union top-k is finished inside one CTA and written
// once.  Rows are contiguous after the reorder, so no query gather exists.
#include <algorithm>
#include <cstring>
#include <numeric>

#include "ungx_internal.h"

namespace ungx
{

int build_plan(const ungx_cross_edge_problem &p, Plan &plan, std::string &err)
{
   plan = Plan();
   const uint32_t n = p.num_points, G = p.num_groups;
   if (p.dim == 0 || p.topk == 0)
   {
      err = "dim and topk must be positive";
      return UNGX_ERR_INVALID_ARG;
   }
   if (p.shard_count == 0 || p.shard_rank >= p.shard_count)
   {
      err = "shard_rank must be < shard_count";
      return UNGX_ERR_INVALID_ARG;
   }
   if (G > 0 && (!p.group_ranges || !p.lng_out_offsets))
   {
      err = "group_ranges / lng_out_offsets must not be null";
      return UNGX_ERR_INVALID_ARG;
   }
   for (uint32_t g = 1; g <= G; ++g)
   {
      const uint32_t a = p.group_ranges[2 * g], b = p.group_ranges[2 * g + 1];
      if (a > b || b > n)
      {
         err = "group " + std::to_string(g) + " has an invalid row range";
         return UNGX_ERR_INVALID_ARG;
      }
      if (p.lng_out_offsets[g + 1] < p.lng_out_offsets[g])
      {
         err = "lng_out_offsets not monotone at group " + std::to_string(g);
         return UNGX_ERR_INVALID_ARG;
      }
   }
   const uint64_t nnz = G ? p.lng_out_offsets[G + 1] : 0;
   if (nnz > 0 && !p.lng_out_ids)
   {
      err = "lng_out_ids must not be null";
      return UNGX_ERR_INVALID_ARG;
   }
   for (uint64_t e = G ? p.lng_out_offsets[1] : 0; e < nnz; ++e)
      if (p.lng_out_ids[e] == 0 || p.lng_out_ids[e] > G)
      {
         err = "lng_out_ids holds a group id outside 1..G";
         return UNGX_ERR_INVALID_ARG;
      }

   struct Cand
   {
      WorkItem item;
      uint64_t cost;
      uint64_t pairs;
   };
   std::vector<Cand> all;
   std::vector<std::pair<RowRange, uint32_t>> empties; // (range, group)
   for (uint32_t f = 1; f <= G; ++f)
   {
      const uint32_t a = p.group_ranges[2 * f], b = p.group_ranges[2 * f + 1];
      if (a == b)
         continue;
      if (p.skip_source_group && p.skip_source_group[f])
      {
         empties.push_back({{a, b - a}, f});
         continue;
      }
      const uint32_t seg_begin = (uint32_t)plan.segs.size();
      uint64_t cols = 0, cost_cols = 0;
      for (uint64_t e = p.lng_out_offsets[f]; e < p.lng_out_offsets[f + 1]; ++e)
      {
         const uint32_t t = p.lng_out_ids[e];
         const uint32_t ta = p.group_ranges[2 * t], tb = p.group_ranges[2 * t + 1];
         if (ta == tb)
            continue;
         plan.segs.push_back({ta, tb - ta, t, 0});
         cols += tb - ta;
         // MMA columns (16-granular) plus a per-tile overhead of ~32 columns
         const uint64_t full = (tb - ta) / 256, rem = (tb - ta) % 256;
         cost_cols += full * (256 + 32) + (rem ? ((rem + 15) / 16) * 16 + 32 : 0);
      }
      const uint32_t seg_count = (uint32_t)plan.segs.size() - seg_begin;
      if (seg_count == 0)
      {
         empties.push_back({{a, b - a}, f});
         continue;
      }
      for (uint32_t r = a; r < b; r += kRowsPerItem)
      {
         const uint32_t cnt = std::min(kRowsPerItem, b - r);
         all.push_back({{r, cnt, seg_begin, seg_count}, cost_cols, uint64_t(cnt) * cols});
      }
      plan.max_item_cols = (uint32_t)std::max<uint64_t>(plan.max_item_cols, cols);
   }
   // longest processing time first; ties broken by row for determinism
   std::stable_sort(all.begin(), all.end(), [](const Cand &x, const Cand &y) {
      if (x.cost != y.cost)
         return x.cost > y.cost;
      return x.item.row_begin < y.item.row_begin;
   });
   const uint32_t S = p.shard_count;
   std::vector<uint64_t> load(S, 0);
   for (const Cand &c : all)
   {
      uint32_t best = 0;
      for (uint32_t s = 1; s < S; ++s)
         if (load[s] < load[best])
            best = s;
      load[best] += c.cost + 1;
      if (best == p.shard_rank)
      {
         plan.items.push_back(c.item);
         plan.pairs += c.pairs;
         plan.padded_cols += c.cost;
      }
   }
   for (const auto &e : empties)
      if (e.second % S == p.shard_rank)
         plan.empty_rows.push_back(e.first);
   return UNGX_OK;
}

} // namespace ungx

extern "C"
{

int ungx_shard_rows(const ungx_cross_edge_problem *problem, uint32_t *rows, uint64_t *count)
{
   if (!problem || !count)
   {
      ungx::set_global_error("ungx_shard_rows: null argument");
      return UNGX_ERR_INVALID_ARG;
   }
   ungx::Plan plan;
   std::string err;
   const int st = ungx::build_plan(*problem, plan, err);
   if (st != UNGX_OK)
   {
      ungx::set_global_error("ungx_shard_rows: " + err);
      return st;
   }
   std::vector<uint32_t> out;
   for (const auto &it : plan.items)
      for (uint32_t r = 0; r < it.row_count; ++r)
         out.push_back(it.row_begin + r);
   for (const auto &e : plan.empty_rows)
      for (uint32_t r = 0; r < e.count; ++r)
         out.push_back(e.begin + r);
   std::sort(out.begin(), out.end());
   *count = out.size();
   if (rows)
      std::memcpy(rows, out.data(), out.size() * sizeof(uint32_t));
   return UNGX_OK;
}

int ungx_flat_to_csr(const uint32_t *flat_ids, uint32_t num_points, uint32_t topk, uint64_t *row_offsets,
                     uint32_t *col_indices)
{
   if ((!flat_ids && num_points) || !row_offsets)
   {
      ungx::set_global_error("ungx_flat_to_csr: null argument");
      return UNGX_ERR_INVALID_ARG;
   }
   row_offsets[0] = 0;
   for (uint32_t v = 0; v < num_points; ++v)
   {
      uint64_t c = 0;
      for (uint32_t i = 0; i < topk; ++i)
         c += flat_ids[(size_t)v * topk + i] != 0xffffffffu;
      row_offsets[v + 1] = row_offsets[v] + c;
   }
   if (col_indices)
      ungx::parallel_for(num_points, 0, 65536, [&](int64_t v) {
         uint64_t w = row_offsets[v];
         for (uint32_t i = 0; i < topk; ++i)
         {
            const uint32_t id = flat_ids[(size_t)v * topk + i];
            if (id != 0xffffffffu)
               col_indices[w++] = id;
         }
      });
   return UNGX_OK;
}

} // extern "C"
