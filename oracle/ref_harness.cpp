// TEST INFRASTRUCTURE ONLY -- never linked into the product library.
//
// Harness around the reference's own compiled leaf code (TrieIndex, SearchQueue,
// FloatL2DistanceHandler) from panjd123/FilterVectorCode_refactor.  It restates,
// step by step, the UniNavGraph member functions that the cross-edge path reads
// and runs, so that the reference's numerics and tie rules decide the oracle's
// answers:
//
//   grouping   UNG/codes/src/uni_nav_graph_label_graph.cpp:21-43  (build_trie_and_divide_groups)
//   reorder    UNG/codes/src/uni_nav_graph.cpp:148-169            (prepare_group_storages_graphs)
//   LNG        UNG/codes/src/uni_nav_graph_label_graph.cpp:103-206, 851-911
//              (get_min_super_sets_optimized_bucket + build_label_nav_graph_optimized_phase1)
//   cross scan UNG/codes/src/uni_nav_graph_cross_edges.cpp:32-57, 154-220
//              (append_cross_edges_from_target_range + build_cross_edges_generate_cpu_exact_scan)
//   additional UNG/codes/src/uni_nav_graph_cross_edges.cpp:442-596
//              (build_cross_edges_generate_additional, exact variant)
//   search     UNG/codes/src/uni_nav_graph_search_backend.cpp:242-283 (iterate_to_fixed_point)
//   truth      UNG/codes/src/filtered_scan.cpp:157-194          (FilteredScan::answer_one_query)
//
// The reference sources themselves are compiled from where they lie by
// oracle/Makefile into oracle/_ref/; nothing from them is copied here.
#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <memory>
#include <vector>

#include "distance.h"
#include "graph.h"
#include "search_queue.h"
#include "trie.h"

using ANNS::IdxType;
using ANNS::LabelType;

namespace
{
struct RefLabelGraph
{
   uint32_t num_points = 0;
   uint32_t num_groups = 0;
   ANNS::TrieIndex trie;
   std::vector<std::vector<IdxType>> group_vec_ids;        // [G+1]
   std::vector<std::vector<LabelType>> group_label_set;    // [G+1]
   std::vector<uint32_t> new_to_old;                       // [n]
   std::vector<uint32_t> group_first;                      // [G+2]
   std::vector<std::vector<IdxType>> out_neighbors;        // [G+1]
};

// Minimal-superset filter in the bucket order the reference uses
// (uni_nav_graph_label_graph.cpp:103-206): candidates come from the reference
// trie's own superset search; they are visited by increasing label-set size and a
// candidate is kept unless it includes an already kept set.
void min_super_sets(const RefLabelGraph &g, const std::vector<LabelType> &query, std::vector<IdxType> &out)
{
   out.clear();
   std::vector<std::shared_ptr<ANNS::TrieNode>> cands;
   g.trie.get_super_set_entrances(query, cands, true, true);
   if (cands.empty())
      return;
   if (cands.size() == 1)
   {
      out.push_back(cands[0]->group_id);
      return;
   }
   LabelType min_size = cands[0]->label_set_size, max_size = min_size;
   for (auto &c : cands)
   {
      min_size = std::min(min_size, c->label_set_size);
      max_size = std::max(max_size, c->label_set_size);
   }
   std::vector<const std::vector<LabelType> *> kept;
   auto consider = [&](const ANNS::TrieNode *c) {
      const auto &ls = g.group_label_set[c->group_id];
      bool is_min = true;
      if (c->label_set_size > min_size)
         for (auto *m : kept)
            if (std::includes(ls.begin(), ls.end(), m->begin(), m->end()))
            {
               is_min = false;
               break;
            }
      if (is_min)
      {
         out.push_back(c->group_id);
         kept.push_back(&ls);
      }
   };
   if (max_size - min_size <= 256)
   {
      std::vector<std::vector<const ANNS::TrieNode *>> buckets(max_size - min_size + 1);
      for (auto &c : cands)
         buckets[c->label_set_size - min_size].push_back(c.get());
      for (auto &b : buckets)
         for (auto *c : b)
            consider(c);
   }
   else
   {
      std::vector<const ANNS::TrieNode *> sorted;
      for (auto &c : cands)
         sorted.push_back(c.get());
      std::sort(sorted.begin(), sorted.end(),
                [](const ANNS::TrieNode *a, const ANNS::TrieNode *b) { return a->label_set_size < b->label_set_size; });
      for (auto *c : sorted)
         consider(c);
   }
}
} // namespace

extern "C"
{

// Labels arrive as CSR: point i owns labels[label_offsets[i] .. label_offsets[i+1]).
// Each point's labels are sorted ascending first, as Storage::load_from_file does
// (UNG/codes/src/storage.cpp:133-146).
void *ungref_label_graph_build(uint32_t num_points, const uint64_t *label_offsets, const uint32_t *labels)
{
   auto *g = new RefLabelGraph();
   g->num_points = num_points;
   IdxType next_group_id = 1;
   std::vector<LabelType> ls;
   for (uint32_t v = 0; v < num_points; ++v)
   {
      ls.assign(labels + label_offsets[v], labels + label_offsets[v + 1]);
      std::sort(ls.begin(), ls.end());
      IdxType gid = g->trie.insert(ls, next_group_id);
      if (gid + 1 > g->group_vec_ids.size())
      {
         g->group_vec_ids.resize(gid + 1);
         g->group_label_set.resize(gid + 1);
         g->group_label_set[gid] = ls;
      }
      g->group_vec_ids[gid].push_back(v);
   }
   g->num_groups = next_group_id - 1;
   g->group_vec_ids.resize(g->num_groups + 1);
   g->group_label_set.resize(g->num_groups + 1);

   g->new_to_old.resize(num_points);
   g->group_first.assign(g->num_groups + 2, 0);
   uint32_t nid = 0;
   for (uint32_t gid = 1; gid <= g->num_groups; ++gid)
   {
      g->group_first[gid] = nid;
      for (auto old : g->group_vec_ids[gid])
         g->new_to_old[nid++] = old;
   }
   g->group_first[g->num_groups + 1] = nid;

   g->out_neighbors.assign(g->num_groups + 1, {});
#pragma omp parallel for schedule(dynamic, 64)
   for (long long gid = 1; gid <= (long long)g->num_groups; ++gid)
      min_super_sets(*g, g->group_label_set[gid], g->out_neighbors[gid]);
   return g;
}

uint32_t ungref_num_groups(void *h) { return static_cast<RefLabelGraph *>(h)->num_groups; }

void ungref_copy_groups(void *h, uint32_t *new_to_old, uint32_t *group_first)
{
   auto *g = static_cast<RefLabelGraph *>(h);
   std::memcpy(new_to_old, g->new_to_old.data(), g->new_to_old.size() * sizeof(uint32_t));
   std::memcpy(group_first, g->group_first.data(), g->group_first.size() * sizeof(uint32_t));
}

uint64_t ungref_lng_nnz(void *h)
{
   auto *g = static_cast<RefLabelGraph *>(h);
   uint64_t nnz = 0;
   for (auto &o : g->out_neighbors)
      nnz += o.size();
   return nnz;
}

// out_offsets has G+2 entries (group 0 is empty); ids are in the reference's order.
void ungref_copy_lng_out(void *h, uint64_t *out_offsets, uint32_t *out_ids)
{
   auto *g = static_cast<RefLabelGraph *>(h);
   uint64_t pos = 0;
   out_offsets[0] = 0;
   for (uint32_t gid = 0; gid <= g->num_groups; ++gid)
   {
      out_offsets[gid] = pos;
      for (auto t : g->out_neighbors[gid])
         out_ids[pos++] = t;
   }
   out_offsets[g->num_groups + 1] = pos;
}

void ungref_label_graph_free(void *h) { delete static_cast<RefLabelGraph *>(h); }

float ungref_l2(const float *a, const float *b, uint32_t dim)
{
   static ANNS::FloatL2DistanceHandler h;
   return h.compute(reinterpret_cast<const char *>(a), reinterpret_cast<const char *>(b), dim);
}

// Exact cross-edge scan over the reordered base vectors X[n x d].
// Groups are 1..G with rows [group_first[g], group_first[g+1]).  LNG out-neighbours
// come as CSR over groups.  In-neighbours are derived serially in ascending source
// order (uni_nav_graph_label_graph.cpp:889-906) and the scan order is the
// reference's: target groups ascending, their in-groups in order, an OpenMP
// dynamic,1 loop over the source vectors.  When source_mask is non-null only
// source groups with a non-zero mask entry are scanned (used to time a bounded
// sample).  Row v of ids/dists receives the queue of point v in queue order;
// unused slots hold UINT32_MAX / +inf.  Returns the algorithmic pair count
// (the reference's dim_ops / dim).
uint64_t ungref_cross_exact(const float *X, uint32_t n, uint32_t d, uint32_t k, uint32_t num_groups,
                            const uint32_t *group_first, const uint64_t *out_offsets, const uint32_t *out_ids,
                            const uint8_t *source_mask, int num_threads, uint32_t *ids, float *dists)
{
   std::vector<std::vector<IdxType>> in_neighbors(num_groups + 1);
   for (uint32_t f = 1; f <= num_groups; ++f)
      for (uint64_t e = out_offsets[f]; e < out_offsets[f + 1]; ++e)
         in_neighbors[out_ids[e]].push_back(f);

   std::vector<ANNS::SearchQueue> queues(n);
   for (uint32_t v = 0; v < n; ++v)
      queues[v].reserve(k);
   ANNS::FloatL2DistanceHandler dist;
   if (num_threads > 0)
      omp_set_num_threads(num_threads);
   uint64_t pairs = 0;
   for (uint32_t t = 1; t <= num_groups; ++t)
   {
      if (in_neighbors[t].empty())
         continue;
      const IdxType tf = group_first[t], ts = group_first[t + 1];
      if (ts == tf)
         continue;
      for (IdxType f : in_neighbors[t])
      {
         if (source_mask && !source_mask[f])
            continue;
         const IdxType qf = group_first[f], qs = group_first[f + 1];
         pairs += uint64_t(qs - qf) * uint64_t(ts - tf);
#pragma omp parallel for schedule(dynamic, 1)
         for (long long v = qf; v < (long long)qs; ++v)
         {
            ANNS::SearchQueue local;
            local.reserve(k);
            const char *q = reinterpret_cast<const char *>(X + size_t(v) * d);
            for (IdxType x = tf; x < ts; ++x)
               local.insert(x, dist.compute(q, reinterpret_cast<const char *>(X + size_t(x) * d), d));
            for (int i = 0; i < local.size(); ++i)
               queues[v].insert(local[i].id, local[i].distance);
         }
      }
   }
   for (uint32_t v = 0; v < n; ++v)
   {
      const auto &q = queues[v];
      for (uint32_t i = 0; i < k; ++i)
      {
         const bool have = i < uint32_t(q.size());
         ids[size_t(v) * k + i] = have ? q[i].id : std::numeric_limits<uint32_t>::max();
         dists[size_t(v) * k + i] = have ? q[i].distance : std::numeric_limits<float>::infinity();
      }
   }
   return pairs;
}

// Additional edges, exact variant (UngAdditionalEdgesImpl::CpuExactScan), restating
// UniNavGraph::build_cross_edges_generate_additional
// (UNG/codes/src/uni_nav_graph_cross_edges.cpp:442-596) around the reference's own
// SearchQueue and FloatL2DistanceHandler.  cross_ids is the flat cross-edge output
// [n x k] (UINT32_MAX = empty slot).  For every group f, the groups its vectors'
// cross edges reach are marked; every LNG out-group f' of f that is not marked gets
// edges from f's vectors in ascending order, each contributing the first k/2 entries
// of its exact top-k over f', until k edges were added for that f'.  The (from, to)
// pairs come out in the reference's materialised order (group ascending; per group
// its out-groups in LNG order, vectors ascending, queue rank).  Returns the pair
// count; the pairs are written only when the count does not exceed cap.
uint64_t ungref_additional_edges(const float *X, uint32_t n, uint32_t d, uint32_t k, uint32_t num_groups,
                                 const uint32_t *group_first, const uint64_t *out_offsets, const uint32_t *out_ids,
                                 const uint32_t *cross_ids, uint64_t cap, uint32_t *from_ids, uint32_t *to_ids)
{
   std::vector<uint32_t> group_of(n, num_groups + 1);
   for (uint32_t g = 1; g <= num_groups; ++g)
      for (uint32_t v = group_first[g]; v < group_first[g + 1]; ++v)
         group_of[v] = g;
   std::vector<std::pair<uint32_t, uint32_t>> edges;
   std::vector<uint32_t> connected(size_t(num_groups) + 2, 0);
   ANNS::FloatL2DistanceHandler dist;
   uint32_t epoch = 0;
   for (uint32_t f = 1; f <= num_groups; ++f)
   {
      ++epoch;
      const uint32_t qf = group_first[f], qs = group_first[f + 1];
      for (uint32_t v = qf; v < qs; ++v)
         for (uint32_t j = 0; j < k; ++j)
         {
            const uint32_t id = cross_ids[size_t(v) * k + j];
            if (id == std::numeric_limits<uint32_t>::max())
               continue;
            const uint32_t g = group_of[id];
            if (g <= num_groups)
               connected[g] = epoch;
         }
      for (uint64_t e = out_offsets[f]; e < out_offsets[f + 1]; ++e)
      {
         const uint32_t t = out_ids[e];
         if (t <= num_groups && connected[t] == epoch)
            continue;
         uint32_t cnt = 0;
         for (uint32_t v = qf; v < qs && cnt < k; ++v)
         {
            ANNS::SearchQueue local;
            local.reserve(k);
            const char *q = reinterpret_cast<const char *>(X + size_t(v) * d);
            for (uint32_t x = group_first[t]; x < group_first[t + 1]; ++x)
               local.insert(x, dist.compute(q, reinterpret_cast<const char *>(X + size_t(x) * d), d));
            for (int r = 0; r < local.size() && r < int(k / 2); ++r)
            {
               edges.emplace_back(v, local[r].id);
               ++cnt;
            }
         }
      }
   }
   if (edges.size() <= cap)
      for (size_t i = 0; i < edges.size(); ++i)
      {
         from_ids[i] = edges[i].first;
         to_ids[i] = edges[i].second;
      }
   return edges.size();
}


// The reference's own graph writer: the CSR rows pushed into an ANNS::Graph
// (NeighborList per point) and written by Graph::save (UNG/codes/include/graph.h:207-216).
int ungref_graph_save_text(const char *path, uint32_t num_points, const uint64_t *offsets, const uint32_t *cols)
{
   ANNS::Graph g(num_points);
   for (uint32_t v = 0; v < num_points; ++v)
      for (uint64_t e = offsets[v]; e < offsets[v + 1]; ++e)
         g.neighbors[v].push_back(cols[e]);
   std::string fn(path);
   g.save(fn);
   g.clean();
   return 0;
}

// Greedy search of a built index, step for step iterate_to_fixed_point over the
// reference's own SearchQueue (capacity L, expanded flags) and distance handler:
// the given entry points, then the closest unexpanded candidate is expanded and every
// unvisited neighbour inserted, until none is left.  Result: the queue's first K ids.
void ungref_ung_search(const float *X, uint32_t n, uint32_t d, const uint64_t *offsets, const uint32_t *cols,
                       const float *Q, uint32_t nq, const uint64_t *entry_offsets, const uint32_t *entry_ids,
                       uint32_t L, uint32_t K, uint32_t *ids)
{
   ANNS::FloatL2DistanceHandler dist;
   const char *base = reinterpret_cast<const char *>(X);
   const size_t row = size_t(d) * sizeof(float);
   std::vector<uint8_t> visited(n);
   ANNS::SearchQueue sq;
   sq.reserve(int32_t(L));
   for (uint32_t qi = 0; qi < nq; ++qi)
   {
      const char *query = reinterpret_cast<const char *>(Q + size_t(qi) * d);
      sq.clear();
      std::fill(visited.begin(), visited.end(), 0);
      for (uint64_t e = entry_offsets[qi]; e < entry_offsets[qi + 1]; ++e)
         sq.insert(entry_ids[e], dist.compute(query, base + entry_ids[e] * row, d));
      while (sq.has_unexpanded_node())
      {
         const IdxType u = sq.get_closest_unexpanded().id;
         for (uint64_t j = offsets[u]; j < offsets[u + 1]; ++j)
         {
            const IdxType w = cols[j];
            if (visited[w])
               continue;
            visited[w] = 1;
            sq.insert(w, dist.compute(query, base + w * row, d));
         }
      }
      for (uint32_t r = 0; r < K; ++r)
         ids[size_t(qi) * K + r] = int32_t(r) < sq.size() ? sq[r].id : UINT32_MAX;
   }
}

// Filtered ground truth: every vector of the query's target groups into a
// reference SearchQueue of capacity K, groups in the given order.
void ungref_filtered_scan(const float *X, uint32_t d, const uint32_t *group_first, const float *Q, uint32_t nq,
                          const uint64_t *target_offsets, const uint32_t *target_ids, uint32_t K, uint32_t *ids,
                          float *dists)
{
   ANNS::FloatL2DistanceHandler dist;
   const char *base = reinterpret_cast<const char *>(X);
   const size_t row = size_t(d) * sizeof(float);
#pragma omp parallel for schedule(dynamic, 1)
   for (int64_t qi = 0; qi < int64_t(nq); ++qi)
   {
      const char *query = reinterpret_cast<const char *>(Q + size_t(qi) * d);
      ANNS::SearchQueue sq;
      sq.reserve(int32_t(K));
      for (uint64_t t = target_offsets[qi]; t < target_offsets[qi + 1]; ++t)
         for (uint32_t x = group_first[target_ids[t]]; x < group_first[target_ids[t] + 1]; ++x)
            sq.insert(x, dist.compute(query, base + x * row, d));
      for (uint32_t r = 0; r < K; ++r)
      {
         const bool have = int32_t(r) < sq.size();
         ids[size_t(qi) * K + r] = have ? sq[r].id : UINT32_MAX;
         dists[size_t(qi) * K + r] = have ? sq[r].distance : std::numeric_limits<float>::infinity();
      }
   }
}
} // extern "C"
