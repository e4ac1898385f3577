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
   plan.items.clear();
   plan.segs.clear();
   plan.empty_rows.clear();
   plan.pairs = plan.padded_cols = 0;
   plan.max_item_cols = 0;
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

   // Pass 1, per source group f: its non-empty targets (segments), their columns and
   // the item cost (MMA columns, 16-granular, plus ~32 columns of per-tile overhead).
   // Pass 2 writes segments and items at offsets from prefix sums, so both passes can
   // run over groups in parallel and the result equals the sequential construction.
   plan.g_nseg.assign(size_t(G) + 1, 0u);
   plan.g_item0.assign(size_t(G) + 2, 0u);
   plan.g_seg0.assign(size_t(G) + 2, 0u);
   plan.g_cols.assign(size_t(G) + 1, 0u);
   plan.g_cost.assign(size_t(G) + 1, 0u);
   const bool par = nnz > 262144 || G > 65536; // thread start-up costs more on small plans
   auto over_groups = [&](auto &&body) {
      if (par)
         parallel_for(int64_t(G), 0, 4096, [&](int64_t i) { body(uint32_t(i) + 1u); });
      else
         for (uint32_t f = 1; f <= G; ++f)
            body(f);
   };
   over_groups([&](uint32_t f) {
      const uint32_t a = p.group_ranges[2 * f], b = p.group_ranges[2 * f + 1];
      if (a == b || (p.skip_source_group && p.skip_source_group[f]))
         return;
      uint32_t ns = 0;
      uint64_t cols = 0, cost = 0;
      for (uint64_t e = p.lng_out_offsets[f]; e < p.lng_out_offsets[f + 1]; ++e)
      {
         const uint32_t t = p.lng_out_ids[e];
         const uint32_t ta = p.group_ranges[2 * t], tb = p.group_ranges[2 * t + 1];
         if (ta == tb)
            continue;
         ++ns;
         cols += tb - ta;
         const uint64_t full = (tb - ta) / 256, rem = (tb - ta) % 256;
         cost += full * (256 + 32) + (rem ? ((rem + 15) / 16) * 16 + 32 : 0);
      }
      plan.g_nseg[f] = ns;
      plan.g_cols[f] = cols;
      plan.g_cost[f] = cost;
   });
   uint64_t nsegs = 0, nitems = 0;
   for (uint32_t f = 1; f <= G; ++f)
   {
      plan.g_seg0[f] = uint32_t(nsegs);
      plan.g_item0[f] = uint32_t(nitems);
      if (plan.g_nseg[f])
      {
         const uint32_t rows = p.group_ranges[2 * f + 1] - p.group_ranges[2 * f];
         nsegs += plan.g_nseg[f];
         nitems += (rows + kRowsPerItem - 1) / kRowsPerItem;
         plan.max_item_cols = (uint32_t)std::max<uint64_t>(plan.max_item_cols, plan.g_cols[f]);
      }
   }
   if (nsegs > UINT32_MAX || nitems > UINT32_MAX)
   {
      err = "plan exceeds 2^32 segments or items";
      return UNGX_ERR_INVALID_ARG;
   }
   plan.segs.resize(nsegs);
   plan.all.resize(nitems);
   plan.key.resize(nitems);
   plan.item_pairs.resize(nitems);
   over_groups([&](uint32_t f) {
      const uint32_t ns = plan.g_nseg[f];
      if (!ns)
         return;
      const uint32_t seg_begin = plan.g_seg0[f];
      Segment *sg = plan.segs.data() + seg_begin;
      for (uint64_t e = p.lng_out_offsets[f]; e < p.lng_out_offsets[f + 1]; ++e)
      {
         const uint32_t t = p.lng_out_ids[e];
         const uint32_t ta = p.group_ranges[2 * t], tb = p.group_ranges[2 * t + 1];
         if (ta != tb)
            *sg++ = {ta, tb - ta, t, 0};
      }
      const uint32_t a = p.group_ranges[2 * f], b = p.group_ranges[2 * f + 1];
      uint32_t i = plan.g_item0[f];
      for (uint32_t r = a; r < b; r += kRowsPerItem, ++i)
      {
         plan.all[i] = {r, std::min(kRowsPerItem, b - r), seg_begin, ns};
         plan.key[i] = plan.g_cost[f];
         plan.item_pairs[i] = uint64_t(plan.all[i].row_count) * plan.g_cols[f];
      }
   });

   // Longest processing time first, ties by first row: a stable LSD radix sort, first
   // by row (skipped when the groups' rows already ascend) and then by descending cost.
   const uint32_t N = uint32_t(nitems);
   plan.order.resize(N);
   plan.order2.resize(N);
   std::iota(plan.order.begin(), plan.order.end(), 0u);
   auto radix = [&](auto &&digit_of, int bits) {
      constexpr int kDigit = 11;
      std::vector<uint32_t> hist(size_t(1) << kDigit);
      for (int shift = 0; shift < bits; shift += kDigit)
      {
         std::fill(hist.begin(), hist.end(), 0u);
         for (uint32_t i = 0; i < N; ++i)
            ++hist[(digit_of(plan.order[i]) >> shift) & ((1u << kDigit) - 1u)];
         uint32_t sum = 0;
         for (auto &h : hist)
         {
            const uint32_t c = h;
            h = sum;
            sum += c;
         }
         for (uint32_t i = 0; i < N; ++i)
         {
            const uint32_t o = plan.order[i];
            plan.order2[hist[(digit_of(o) >> shift) & ((1u << kDigit) - 1u)]++] = o;
         }
         plan.order.swap(plan.order2);
      }
   };
   bool rows_ascend = true;
   for (uint32_t i = 1; i < N && rows_ascend; ++i)
      rows_ascend = plan.all[i - 1].row_begin < plan.all[i].row_begin;
   if (!rows_ascend)
      radix([&](uint32_t o) { return uint64_t(plan.all[o].row_begin); }, 32);
   uint64_t max_cost = 0;
   for (uint32_t i = 0; i < N; ++i)
      max_cost = std::max(max_cost, plan.key[i]);
   int cost_bits = 0;
   while (cost_bits < 64 && (max_cost >> cost_bits))
      ++cost_bits;
   radix([&](uint32_t o) { return max_cost - plan.key[o]; }, cost_bits);

   // greedy assignment to the least-loaded shard, in that order
   const uint32_t S = p.shard_count;
   std::vector<uint64_t> &load = plan.shard_load;
   load.assign(S, 0);
   plan.item_shard.resize(N);
   plan.items.reserve(S == 1 ? N : N / S + 1);
   for (uint32_t i = 0; i < N; ++i)
   {
      const uint32_t o = plan.order[i];
      uint32_t best = 0;
      for (uint32_t s = 1; s < S; ++s)
         if (load[s] < load[best])
            best = s;
      load[best] += plan.key[o] + 1;
      plan.item_shard[o] = best;
      if (best == p.shard_rank)
      {
         const WorkItem &it = plan.all[o];
         plan.items.push_back(it);
         plan.pairs += plan.item_pairs[o];
         plan.padded_cols += plan.key[o];
      }
   }
   // rows with no candidates: skipped source groups and groups without targets; and
   // every group's rows in chunks for the per-group norm maxima
   plan.norm_chunks.clear();
   for (uint32_t f = 1; f <= G; ++f)
   {
      const uint32_t a = p.group_ranges[2 * f], b = p.group_ranges[2 * f + 1];
      if (a != b && plan.g_nseg[f] == 0 && f % S == p.shard_rank)
         plan.empty_rows.push_back({a, b - a});
      for (uint32_t r = a; r < b; r += 4096u)
         plan.norm_chunks.insert(plan.norm_chunks.end(), {f, r, std::min(4096u, b - r)});
   }
   return UNGX_OK;
}

void shard_runs(const ungx_cross_edge_problem &p, const Plan &plan, std::vector<std::vector<CopyRange>> &runs,
                std::vector<uint32_t> &rows)
{
   const uint32_t S = p.shard_count, G = p.num_groups;
   runs.assign(S, {});
   rows.assign(S, 0u);
   // (first row, rows, shard) of every item and every group without targets
   struct Piece
   {
      uint32_t begin, count, shard;
   };
   std::vector<Piece> pieces;
   pieces.reserve(plan.all.size() + G);
   for (uint32_t f = 1; f <= G; ++f)
   {
      const uint32_t a = p.group_ranges[2 * f], b = p.group_ranges[2 * f + 1];
      if (a == b)
         continue;
      if (plan.g_nseg[f] == 0)
      {
         pieces.push_back({a, b - a, f % S});
         continue;
      }
      const uint32_t i0 = plan.g_item0[f], ni = (b - a + kRowsPerItem - 1) / kRowsPerItem;
      for (uint32_t i = i0; i < i0 + ni; ++i)
         pieces.push_back({plan.all[i].row_begin, plan.all[i].row_count, plan.item_shard[i]});
   }
   bool ascend = true;
   for (size_t i = 1; i < pieces.size() && ascend; ++i)
      ascend = pieces[i - 1].begin < pieces[i].begin;
   if (!ascend)
      std::sort(pieces.begin(), pieces.end(), [](const Piece &x, const Piece &y) { return x.begin < y.begin; });
   for (const Piece &pc : pieces)
   {
      auto &r = runs[pc.shard];
      if (!r.empty() && r.back().src_row + r.back().count == pc.begin)
         r.back().count += pc.count;
      else
         r.push_back({pc.begin, rows[pc.shard], pc.count, 0});
      rows[pc.shard] += pc.count;
   }
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
