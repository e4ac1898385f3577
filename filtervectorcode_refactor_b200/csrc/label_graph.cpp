// Input side of the cross-edge path (a16): grouping by exact label set, the
// group-contiguous reorder, and the label navigating graph (LNG) of minimal
// strict supersets.
//
//   grouping  -- build_trie_and_divide_groups, UNG/codes/src/uni_nav_graph_label_graph.cpp:21-43:
//                a group per distinct SORTED label sequence, numbered 1.. in the
//                order of first appearance over the original vector ids.
//   reorder   -- prepare_group_storages_graphs, UNG/codes/src/uni_nav_graph.cpp:148-169:
//                new id = position in the concatenation of groups 1..G, each group
//                keeping ascending original ids.
//   LNG       -- get_min_super_sets_optimized_bucket + build_label_nav_graph_optimized_phase1,
//                UNG/codes/src/uni_nav_graph_label_graph.cpp:103-206, 851-911: out(f) =
//                groups whose label set strictly includes f's and includes no other
//                such group's set.  The reference finds candidates by walking its
//                trie; here candidates come from an inverted index (label -> groups)
//                and inclusion is a bitset test.  Same set, different search.
//                in(f') is out() transposed, ascending source id (:889-906).
#include <algorithm>
#include <cstring>
#include <mutex>
#include <numeric>
#include <unordered_map>

#include "ungx_internal.h"

namespace ungx
{
namespace
{
thread_local std::string g_error;
}
void set_global_error(const std::string &msg) { g_error = msg; }
const char *global_error() { return g_error.c_str(); }
} // namespace ungx

struct ungx_label_graph
{
   uint32_t num_points = 0;
   uint32_t num_groups = 0;
   std::vector<uint32_t> new_to_old;
   std::vector<uint32_t> ranges;      // 2*(G+1)
   std::vector<uint64_t> set_off;     // G+2
   std::vector<uint32_t> set_labels;  // sorted label sequence per group
   std::vector<uint64_t> out_off, in_off;
   std::vector<uint32_t> out_ids, in_ids;
};

namespace
{
using ungx::parallel_for;

inline uint64_t hash_seq(const uint32_t *s, uint32_t len)
{
   uint64_t h = 0x9ae16a3b2f90404full ^ (uint64_t(len) * 0xc3a5c85c97cb3127ull);
   for (uint32_t i = 0; i < len; ++i)
   {
      h ^= uint64_t(s[i]) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
      h *= 0xff51afd7ed558ccdull;
   }
   return h ^ (h >> 31);
}

// Groups by exact label sequence, numbered 1.. in the order they are first added.
// Open addressing over the groups (not the points): it starts small and doubles at
// half load.  Each slot keeps its group's hash, and each group's labels go to a compact
// store when the group is created, so a probe reads only the table and that store.
struct GroupTable
{
   uint64_t cap = 1024;
   std::vector<uint64_t> slot_hash = std::vector<uint64_t>(1024, 0);
   std::vector<uint32_t> slot_gid = std::vector<uint32_t>(1024, 0);
   std::vector<uint64_t> hash = std::vector<uint64_t>(1, 0); // per group, index 0 unused
   std::vector<uint64_t> set_off = std::vector<uint64_t>(2, 0); // group g: [set_off[g], set_off[g+1])
   std::vector<uint32_t> set;
   uint32_t count = 0;

   uint32_t find_or_add(uint64_t h, const uint32_t *s, uint32_t len)
   {
      uint64_t p = h & (cap - 1);
      for (;;)
      {
         const uint32_t gid = slot_gid[p];
         if (gid == 0)
         {
            slot_gid[p] = ++count;
            slot_hash[p] = h;
            hash.push_back(h);
            set.insert(set.end(), s, s + len);
            set_off.push_back(set.size());
            if (2ull * count > cap)
               grow();
            return count;
         }
         if (slot_hash[p] == h && set_off[gid + 1] - set_off[gid] == len &&
             std::memcmp(set.data() + set_off[gid], s, len * sizeof(uint32_t)) == 0)
            return gid;
         p = (p + 1) & (cap - 1);
      }
   }

   void grow()
   {
      cap <<= 1;
      slot_hash.assign(cap, 0);
      slot_gid.assign(cap, 0);
      for (uint32_t gid = 1; gid <= count; ++gid)
      {
         uint64_t q = hash[gid] & (cap - 1);
         while (slot_gid[q] != 0)
            q = (q + 1) & (cap - 1);
         slot_gid[q] = gid;
         slot_hash[q] = hash[gid];
      }
   }
};

void build_lng(ungx_label_graph &g, int threads)
{
   const uint32_t G = g.num_groups;
   // dense label ids
   std::vector<uint32_t> uniq(g.set_labels);
   std::sort(uniq.begin(), uniq.end());
   uniq.erase(std::unique(uniq.begin(), uniq.end()), uniq.end());
   const uint32_t L = (uint32_t)uniq.size();
   bool has_dup = false;
   for (uint32_t f = 1; f <= G && !has_dup; ++f)
      for (uint64_t i = g.set_off[f] + 1; i < g.set_off[f + 1]; ++i)
         if (g.set_labels[i] == g.set_labels[i - 1])
         {
            has_dup = true;
            break;
         }
   const uint32_t W = std::max<uint32_t>(1, (L + 63) / 64);
   std::vector<uint64_t> masks((size_t)(G + 1) * W, 0);
   std::vector<uint32_t> dense(g.set_labels.size());
   for (size_t i = 0; i < g.set_labels.size(); ++i)
      dense[i] = (uint32_t)(std::lower_bound(uniq.begin(), uniq.end(), g.set_labels[i]) - uniq.begin());
   for (uint32_t f = 1; f <= G; ++f)
      for (uint64_t i = g.set_off[f]; i < g.set_off[f + 1]; ++i)
         masks[(size_t)f * W + dense[i] / 64] |= 1ull << (dense[i] % 64);
   // inverted index: dense label -> groups (ascending)
   std::vector<uint64_t> inv_off(L + 1, 0);
   for (uint32_t f = 1; f <= G; ++f)
      for (uint64_t i = g.set_off[f]; i < g.set_off[f + 1]; ++i)
         if (i == g.set_off[f] || dense[i] != dense[i - 1])
            inv_off[dense[i] + 1]++;
   for (uint32_t l = 0; l < L; ++l)
      inv_off[l + 1] += inv_off[l];
   std::vector<uint32_t> inv(inv_off[L]);
   {
      std::vector<uint64_t> fill(inv_off.begin(), inv_off.end() - 1);
      for (uint32_t f = 1; f <= G; ++f)
         for (uint64_t i = g.set_off[f]; i < g.set_off[f + 1]; ++i)
            if (i == g.set_off[f] || dense[i] != dense[i - 1])
               inv[fill[dense[i]]++] = f;
   }
   auto set_len = [&](uint32_t f) { return (uint32_t)(g.set_off[f + 1] - g.set_off[f]); };
   // includes(a ⊇ b)
   auto includes = [&](uint32_t a, uint32_t b) -> bool {
      if (has_dup)
         return std::includes(g.set_labels.begin() + g.set_off[a], g.set_labels.begin() + g.set_off[a + 1],
                              g.set_labels.begin() + g.set_off[b], g.set_labels.begin() + g.set_off[b + 1]);
      const uint64_t *ma = &masks[(size_t)a * W], *mb = &masks[(size_t)b * W];
      for (uint32_t w = 0; w < W; ++w)
         if ((ma[w] & mb[w]) != mb[w])
            return false;
      return true;
   };
   std::vector<uint32_t> all_groups(G);
   std::iota(all_groups.begin(), all_groups.end(), 1u);
   uint32_t max_len = 0;
   for (uint32_t f = 1; f <= G; ++f)
      max_len = std::max(max_len, set_len(f));

   // label sets of at most 64 distinct labels without repeats: the inverted lists carry
   // each group's label mask, so the superset test is a sequential scan of 8-byte words.
   // Each list is ordered by (set length, group id), the reference's visiting order, so
   // a group scans only the entries longer than its own set and they come out in that
   // order; a group of the longest length scans nothing.
   const bool fast = !has_dup && W == 1;
   std::vector<uint64_t> inv_mask(fast ? inv.size() : 0);
   std::vector<uint32_t> inv_len(fast ? inv.size() : 0);
   if (fast)
   {
      parallel_for(L, threads, 1, [&](int64_t l) {
         std::stable_sort(inv.begin() + inv_off[l], inv.begin() + inv_off[l + 1],
                          [&](uint32_t a, uint32_t b) { return set_len(a) < set_len(b); });
      });
      for (size_t j = 0; j < inv.size(); ++j)
      {
         inv_mask[j] = masks[inv[j]];
         inv_len[j] = set_len(inv[j]);
      }
   }
   std::vector<std::vector<uint32_t>> outs(G + 1);
   parallel_for(G, threads, 64, [&](int64_t i) {
      const uint32_t f = (uint32_t)i + 1;
      const uint32_t flen = set_len(f);
      if (fast)
      {
         // candidates: strict supersets among the groups holding one of f's labels, in
         // the reference's visiting order (label-set length, then group id); a candidate
         // is kept unless a kept shorter one is included in it
         // candidates: the entries longer than f's set in the list, among f's labels,
         // that has the fewest of them
         const uint64_t mf = masks[f];
         uint64_t best_n = UINT64_MAX, best_off = 0;
         for (uint64_t j = g.set_off[f]; j < g.set_off[f + 1]; ++j)
         {
            const uint32_t l = dense[j];
            const uint32_t *lb = inv_len.data() + inv_off[l], *le = inv_len.data() + inv_off[l + 1];
            const uint64_t a = inv_off[l] + (std::upper_bound(lb, le, flen) - lb);
            if (inv_off[l + 1] - a < best_n)
            {
               best_n = inv_off[l + 1] - a;
               best_off = a;
            }
         }
         std::vector<std::pair<uint32_t, uint32_t>> sup; // (length, group)
         if (best_n == UINT64_MAX) // the empty set: every other group is a superset
         {
            for (uint32_t c = 1; c <= G; ++c)
               if (c != f)
                  sup.push_back({set_len(c), c});
            std::sort(sup.begin(), sup.end());
         }
         else
         {
            for (uint64_t j = best_off; j < best_off + best_n; ++j)
            {
               const uint64_t m = inv_mask[j];
               if ((m & mf) == mf)
                  sup.push_back({inv_len[j], inv[j]});
            }
         }
         std::vector<uint32_t> kept;
         std::vector<uint64_t> kept_mask;
         std::vector<uint32_t> kept_len;
         for (const auto &lc : sup)
         {
            const uint64_t mc = masks[lc.second];
            bool is_min = true;
            for (size_t q = 0; q < kept.size(); ++q)
               if (kept_len[q] < lc.first && (mc & kept_mask[q]) == kept_mask[q])
               {
                  is_min = false;
                  break;
               }
            if (is_min)
            {
               kept.push_back(lc.second);
               kept_mask.push_back(mc);
               kept_len.push_back(lc.first);
            }
         }
         std::sort(kept.begin(), kept.end());
         outs[f].swap(kept);
         return;
      }
      // candidate source list: the inverted list of f's rarest label
      const uint32_t *lst = all_groups.data();
      uint64_t lst_n = G;
      for (uint64_t j = g.set_off[f]; j < g.set_off[f + 1]; ++j)
      {
         const uint32_t l = dense[j];
         if (inv_off[l + 1] - inv_off[l] < lst_n)
         {
            lst = inv.data() + inv_off[l];
            lst_n = inv_off[l + 1] - inv_off[l];
         }
      }
      // bucket candidates by label-set length (the reference's visiting order)
      std::vector<std::vector<uint32_t>> buckets(max_len + 1);
      for (uint64_t j = 0; j < lst_n; ++j)
      {
         const uint32_t c = lst[j];
         if (c == f || set_len(c) < flen)
            continue;
         if (includes(c, f))
            buckets[set_len(c)].push_back(c);
      }
      std::vector<uint32_t> kept;
      for (uint32_t len = flen; len <= max_len; ++len)
         for (uint32_t c : buckets[len])
         {
            bool is_min = true;
            for (uint32_t m : kept)
               if (set_len(m) < len && includes(c, m))
               {
                  is_min = false;
                  break;
               }
            if (is_min)
               kept.push_back(c);
         }
      std::sort(kept.begin(), kept.end());
      outs[f].swap(kept);
   });
   g.out_off.assign(G + 2, 0);
   for (uint32_t f = 1; f <= G; ++f)
      g.out_off[f + 1] = g.out_off[f] + outs[f].size();
   g.out_ids.resize(g.out_off[G + 1]);
   for (uint32_t f = 1; f <= G; ++f)
      std::copy(outs[f].begin(), outs[f].end(), g.out_ids.begin() + g.out_off[f]);
   // in-neighbours: serial over sources so each list is ascending
   g.in_off.assign(G + 2, 0);
   for (uint32_t e = 0; e < g.out_ids.size(); ++e)
      g.in_off[g.out_ids[e] + 1]++;
   for (uint32_t f = 0; f <= G; ++f)
      g.in_off[f + 1] += g.in_off[f];
   g.in_ids.resize(g.out_ids.size());
   std::vector<uint64_t> fill(g.in_off.begin(), g.in_off.end() - 1);
   for (uint32_t f = 1; f <= G; ++f)
      for (uint64_t e = g.out_off[f]; e < g.out_off[f + 1]; ++e)
         g.in_ids[fill[g.out_ids[e]]++] = f;
}
} // namespace

extern "C"
{

int ungx_label_graph_build(uint32_t n, const uint64_t *label_offsets, const uint32_t *labels, int threads,
                           ungx_label_graph **out)
{
   if (!out || (n > 0 && !label_offsets) || (n > 0 && label_offsets[n] > 0 && !labels))
   {
      ungx::set_global_error("ungx_label_graph_build: null argument");
      return UNGX_ERR_INVALID_ARG;
   }
   *out = nullptr;
   try
   {
      auto g = std::make_unique<ungx_label_graph>();
      g->num_points = n;
      const uint64_t total = n ? label_offsets[n] : 0;
      for (uint32_t v = 0; v < n; ++v)
         if (label_offsets[v + 1] < label_offsets[v])
         {
            ungx::set_global_error("ungx_label_graph_build: label_offsets not monotone");
            return UNGX_ERR_INVALID_ARG;
         }
      // sorted label sequence per point, and its hash
      std::vector<uint32_t> sl(labels, labels + total);
      std::vector<uint64_t> h(n);
      parallel_for(n, threads, 4096, [&](int64_t v) {
         uint32_t *b = sl.data() + label_offsets[v], *e = sl.data() + label_offsets[v + 1];
         std::sort(b, e);
         h[v] = hash_seq(b, (uint32_t)(e - b));
      });
      // first-appearance group ids.  The order is the definition, so the points are cut
      // into contiguous chunks, each numbered by its own table in parallel (local ids in
      // first-appearance order within the chunk), and the chunks' groups are then added
      // to one table in chunk order and local-id order: a group first seen at point v
      // gets its id after every group first seen before v, as in one serial pass.
      std::vector<uint32_t> point_gid(n);
      const int hw = threads > 0 ? threads : (int)std::max(1u, std::thread::hardware_concurrency());
      const uint32_t nchunks = n >= (1u << 18) ? (uint32_t)std::min<int64_t>(hw, n >> 16) : 1u;
      std::vector<GroupTable> local(nchunks);
      auto chunk_lo = [&](uint32_t c) { return (uint32_t)((uint64_t)n * c / nchunks); };
      parallel_for(nchunks, threads, 1, [&](int64_t c) {
         GroupTable &t = local[c];
         for (uint32_t v = chunk_lo((uint32_t)c); v < chunk_lo((uint32_t)c + 1); ++v)
            point_gid[v] = t.find_or_add(h[v], sl.data() + label_offsets[v],
                                         (uint32_t)(label_offsets[v + 1] - label_offsets[v]));
      });
      GroupTable global;
      std::vector<std::vector<uint32_t>> to_global(nchunks);
      for (uint32_t c = 0; c < nchunks; ++c)
      {
         const GroupTable &t = local[c];
         to_global[c].resize(t.count + 1, 0);
         for (uint32_t lg = 1; lg <= t.count; ++lg)
            to_global[c][lg] = global.find_or_add(t.hash[lg], t.set.data() + t.set_off[lg],
                                                  (uint32_t)(t.set_off[lg + 1] - t.set_off[lg]));
      }
      if (nchunks > 1)
         parallel_for(nchunks, threads, 1, [&](int64_t c) {
            const std::vector<uint32_t> &m = to_global[c];
            for (uint32_t v = chunk_lo((uint32_t)c); v < chunk_lo((uint32_t)c + 1); ++v)
               point_gid[v] = m[point_gid[v]];
         });
      local.clear();
      const uint32_t G = global.count;
      std::vector<uint64_t> gset_off = std::move(global.set_off);
      std::vector<uint32_t> gset = std::move(global.set);
      g->num_groups = G;
      // reorder
      std::vector<uint32_t> first(G + 2, 0);
      for (uint32_t v = 0; v < n; ++v)
         first[point_gid[v] + 1]++;
      for (uint32_t gid = 0; gid <= G; ++gid)
         first[gid + 1] += first[gid];
      g->ranges.assign(2 * (size_t)(G + 1), 0);
      for (uint32_t gid = 1; gid <= G; ++gid)
      {
         g->ranges[2 * gid] = first[gid];
         g->ranges[2 * gid + 1] = first[gid + 1];
      }
      g->new_to_old.resize(n);
      {
         std::vector<uint32_t> fill(first.begin(), first.end() - 1);
         for (uint32_t v = 0; v < n; ++v)
            g->new_to_old[fill[point_gid[v]]++] = v;
      }
      // group label sets: the store the grouping pass filled
      g->set_off = std::move(gset_off);
      g->set_labels = std::move(gset);
      build_lng(*g, threads);
      *out = g.release();
      return UNGX_OK;
   }
   catch (const std::bad_alloc &)
   {
      ungx::set_global_error("ungx_label_graph_build: out of host memory");
      return UNGX_ERR_OOM;
   }
   catch (const std::exception &e)
   {
      ungx::set_global_error(std::string("ungx_label_graph_build: ") + e.what());
      return UNGX_ERR_INVALID_ARG;
   }
}

int ungx_label_graph_destroy(ungx_label_graph *lg)
{
   delete lg;
   return UNGX_OK;
}

uint32_t ungx_label_graph_num_groups(const ungx_label_graph *lg) { return lg ? lg->num_groups : 0; }

uint64_t ungx_label_graph_num_edges(const ungx_label_graph *lg) { return lg ? lg->out_ids.size() : 0; }

int ungx_label_graph_copy_groups(const ungx_label_graph *lg, uint32_t *new_to_old, uint32_t *group_ranges)
{
   if (!lg)
      return UNGX_ERR_INVALID_ARG;
   if (new_to_old)
      std::copy(lg->new_to_old.begin(), lg->new_to_old.end(), new_to_old);
   if (group_ranges)
      std::copy(lg->ranges.begin(), lg->ranges.end(), group_ranges);
   return UNGX_OK;
}

int ungx_label_graph_copy_out_neighbors(const ungx_label_graph *lg, uint64_t *offsets, uint32_t *ids)
{
   if (!lg)
      return UNGX_ERR_INVALID_ARG;
   if (offsets)
      std::copy(lg->out_off.begin(), lg->out_off.end(), offsets);
   if (ids)
      std::copy(lg->out_ids.begin(), lg->out_ids.end(), ids);
   return UNGX_OK;
}

int ungx_label_graph_copy_in_neighbors(const ungx_label_graph *lg, uint64_t *offsets, uint32_t *ids)
{
   if (!lg)
      return UNGX_ERR_INVALID_ARG;
   if (offsets)
      std::copy(lg->in_off.begin(), lg->in_off.end(), offsets);
   if (ids)
      std::copy(lg->in_ids.begin(), lg->in_ids.end(), ids);
   return UNGX_OK;
}

uint64_t ungx_label_graph_num_set_labels(const ungx_label_graph *lg) { return lg ? lg->set_labels.size() : 0; }

int ungx_label_graph_copy_label_sets(const ungx_label_graph *lg, uint64_t *offsets, uint32_t *labels)
{
   if (!lg)
      return UNGX_ERR_INVALID_ARG;
   if (offsets)
      std::copy(lg->set_off.begin(), lg->set_off.end(), offsets);
   if (labels)
      std::copy(lg->set_labels.begin(), lg->set_labels.end(), labels);
   return UNGX_OK;
}

} // extern "C"
