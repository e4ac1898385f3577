/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the UNG cross-edge build.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it;
 * the product library never links or calls it.
 *
 * Plain-C restatement of the reference algorithm (panjd123/FilterVectorCode_refactor):
 *
 *   orc_l2            FloatL2DistanceHandler::compute, UNG/codes/src/distance.cpp:34-91
 *                     (8 AVX2 lanes, hi+lo 128-bit fold, 4-wide tail, masked tail,
 *                     two horizontal adds).  `fused` is a bit mask: bit 0 makes the
 *                     8-lane loop update one rounding (fma), bit 1 does the same for
 *                     the 4-wide and masked tails.  The reference's release build
 *                     (GCC 13, -Ofast -mfma) rounds the loop update twice (mul, add)
 *                     and fuses the tails: mode ORC_L2_REFERENCE_BUILD = 2, checked
 *                     bit-for-bit against the compiled reference in the tests.
 *   orc_queue_insert  SearchQueue::insert, UNG/codes/src/search_queue.cpp:26-53 with
 *                     the (distance, id) order of UNG/codes/include/search_queue.h:20-22.
 *   orc_cross_exact   build_cross_edges_generate_cpu_exact_scan +
 *                     append_cross_edges_from_target_range,
 *                     UNG/codes/src/uni_nav_graph_cross_edges.cpp:32-57, 154-220.
 *   orc_label_graph_* build_trie_and_divide_groups (uni_nav_graph_label_graph.cpp:21-43),
 *                     prepare_group_storages_graphs (uni_nav_graph.cpp:148-169) and the
 *                     minimal-superset LNG (uni_nav_graph_label_graph.cpp:103-206, 851-911).
 *                     Out-neighbours are produced as a set (ascending group id); the
 *                     cross-edge result depends only on the set.
 *
 * Compiled with -ffp-contract=off so that every multiply and add rounds exactly
 * where the restatement says.
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct
{
   uint32_t id;
   float dist;
} orc_cand;

static int cmp_u32(const void *a, const void *b);

float orc_l2(const float *a, const float *b, uint32_t dim, int fused)
{
   float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
   uint32_t i = 0;
   while (dim - i >= 8)
   {
      for (int j = 0; j < 8; ++j)
      {
         const float t = a[i + j] - b[i + j];
         lane[j] = (fused & 1) ? fmaf(t, t, lane[j]) : lane[j] + t * t;
      }
      i += 8;
   }
   float s[4];
   for (int j = 0; j < 4; ++j)
      s[j] = lane[4 + j] + lane[j];
   if (dim - i >= 4)
   {
      for (int j = 0; j < 4; ++j)
      {
         const float t = a[i + j] - b[i + j];
         s[j] = (fused & 2) ? fmaf(t, t, s[j]) : s[j] + t * t;
      }
      i += 4;
   }
   if (dim > i)
   {
      for (uint32_t j = 0; j < 4; ++j)
      {
         const float t = (i + j < dim) ? a[i + j] - b[i + j] : 0.0f;
         s[j] = (fused & 2) ? fmaf(t, t, s[j]) : s[j] + t * t;
      }
   }
   const float h0 = s[0] + s[1], h1 = s[2] + s[3];
   return h0 + h1;
}

static int cand_less(orc_cand x, orc_cand y)
{
   return x.dist < y.dist || (x.dist == y.dist && x.id < y.id);
}

/* q has room for cap + 1 entries, *size <= cap. */
void orc_queue_insert(orc_cand *q, int32_t *size, int32_t cap, uint32_t id, float dist)
{
   orc_cand c = {id, dist};
   if (*size == cap && cand_less(q[*size - 1], c))
      return;
   int32_t lo = 0, hi = *size;
   while (lo < hi)
   {
      int32_t mid = (lo + hi) >> 1;
      if (cand_less(c, q[mid]))
         hi = mid;
      else if (q[mid].id == c.id)
         return;
      else
         lo = mid + 1;
   }
   if (lo < cap)
      memmove(&q[lo + 1], &q[lo], (size_t)(*size - lo) * sizeof(orc_cand));
   q[lo] = c;
   if (*size < cap)
      (*size)++;
}

/* See ungref_cross_exact in ref_harness.cpp for the argument contract. */
uint64_t orc_cross_exact(const float *X, uint32_t n, uint32_t d, uint32_t k, uint32_t num_groups,
                         const uint32_t *group_first, const uint64_t *out_offsets, const uint32_t *out_ids,
                         const uint8_t *source_mask, int num_threads, int fused, uint32_t *ids, float *dists)
{
   /* in-neighbours, ascending source id */
   uint64_t *in_off = (uint64_t *)calloc((size_t)num_groups + 2, sizeof(uint64_t));
   uint64_t nnz = out_offsets[num_groups + 1];
   uint32_t *in_ids = (uint32_t *)malloc((nnz ? nnz : 1) * sizeof(uint32_t));
   for (uint32_t f = 1; f <= num_groups; ++f)
      for (uint64_t e = out_offsets[f]; e < out_offsets[f + 1]; ++e)
         in_off[out_ids[e] + 1]++;
   for (uint32_t g = 0; g <= num_groups; ++g)
      in_off[g + 1] += in_off[g];
   uint64_t *fill = (uint64_t *)malloc(((size_t)num_groups + 1) * sizeof(uint64_t));
   memcpy(fill, in_off, ((size_t)num_groups + 1) * sizeof(uint64_t));
   for (uint32_t f = 1; f <= num_groups; ++f)
      for (uint64_t e = out_offsets[f]; e < out_offsets[f + 1]; ++e)
         in_ids[fill[out_ids[e]]++] = f;
   free(fill);

   orc_cand *queues = (orc_cand *)malloc((size_t)n * (k + 1) * sizeof(orc_cand));
   int32_t *qsize = (int32_t *)calloc(n ? n : 1, sizeof(int32_t));
   if (num_threads > 0)
      omp_set_num_threads(num_threads);
   uint64_t pairs = 0;
   for (uint32_t t = 1; t <= num_groups; ++t)
   {
      const uint32_t tf = group_first[t], ts = group_first[t + 1];
      if (in_off[t] == in_off[t + 1] || ts == tf)
         continue;
      for (uint64_t e = in_off[t]; e < in_off[t + 1]; ++e)
      {
         const uint32_t f = in_ids[e];
         if (source_mask && !source_mask[f])
            continue;
         const uint32_t qf = group_first[f], qs = group_first[f + 1];
         pairs += (uint64_t)(qs - qf) * (uint64_t)(ts - tf);
#pragma omp parallel for schedule(dynamic, 1)
         for (long long v = qf; v < (long long)qs; ++v)
         {
            orc_cand local[257];
            orc_cand *loc = k + 1 <= 257 ? local : (orc_cand *)malloc((k + 1) * sizeof(orc_cand));
            int32_t lsize = 0;
            const float *q = X + (size_t)v * d;
            for (uint32_t x = tf; x < ts; ++x)
               orc_queue_insert(loc, &lsize, (int32_t)k, x, orc_l2(q, X + (size_t)x * d, d, fused));
            for (int32_t i = 0; i < lsize; ++i)
               orc_queue_insert(queues + (size_t)v * (k + 1), &qsize[v], (int32_t)k, loc[i].id, loc[i].dist);
            if (loc != local)
               free(loc);
         }
      }
   }
   for (uint32_t v = 0; v < n; ++v)
      for (uint32_t i = 0; i < k; ++i)
      {
         const int have = (int32_t)i < qsize[v];
         ids[(size_t)v * k + i] = have ? queues[(size_t)v * (k + 1) + i].id : 0xffffffffu;
         dists[(size_t)v * k + i] = have ? queues[(size_t)v * (k + 1) + i].dist : INFINITY;
      }
   free(queues);
   free(qsize);
   free(in_off);
   free(in_ids);
   return pairs;
}

/* ---------------- grouping + LNG ---------------- */

typedef struct
{
   uint32_t num_points, num_groups;
   uint32_t *new_to_old;     /* [n] */
   uint32_t *group_first;    /* [G+2] */
   uint64_t *set_off;        /* [G+2] label set of group g: set_lab[set_off[g]..set_off[g+1]) */
   uint32_t *set_lab;
   uint64_t *out_off;        /* [G+2] */
   uint32_t *out_ids;
} orc_label_graph;

static int cmp_u32(const void *a, const void *b)
{
   uint32_t x = *(const uint32_t *)a, y = *(const uint32_t *)b;
   return (x > y) - (x < y);
}

static uint64_t hash_seq(const uint32_t *s, uint32_t len)
{
   uint64_t h = 1469598103934665603ull ^ len;
   for (uint32_t i = 0; i < len; ++i)
   {
      h ^= s[i] + 0x9e3779b97f4a7c15ull;
      h *= 1099511628211ull;
   }
   return h;
}

/* std::includes over sorted sequences (multiset semantics). */
static int seq_includes(const uint32_t *a, uint32_t na, const uint32_t *b, uint32_t nb)
{
   uint32_t i = 0, j = 0;
   while (j < nb)
   {
      if (i == na || b[j] < a[i])
         return 0;
      if (!(a[i] < b[j]))
         ++j;
      ++i;
   }
   return 1;
}

void *orc_label_graph_build(uint32_t n, const uint64_t *label_offsets, const uint32_t *labels)
{
   orc_label_graph *g = (orc_label_graph *)calloc(1, sizeof(orc_label_graph));
   g->num_points = n;
   /* sorted copy of every point's labels */
   uint64_t total = label_offsets[n];
   uint32_t *sl = (uint32_t *)malloc((total ? total : 1) * sizeof(uint32_t));
   memcpy(sl, labels, total * sizeof(uint32_t));
   for (uint32_t v = 0; v < n; ++v)
      qsort(sl + label_offsets[v], label_offsets[v + 1] - label_offsets[v], sizeof(uint32_t), cmp_u32);

   /* open-addressing table: label sequence -> group id, first appearance order */
   uint64_t cap = 16;
   while (cap < 2ull * n + 16)
      cap <<= 1;
   uint32_t *slot_point = (uint32_t *)malloc(cap * sizeof(uint32_t)); /* representative point */
   uint32_t *slot_group = (uint32_t *)calloc(cap, sizeof(uint32_t));
   uint32_t *point_group = (uint32_t *)malloc((n ? n : 1) * sizeof(uint32_t));
   uint32_t *rep = (uint32_t *)malloc(((size_t)n + 2) * sizeof(uint32_t));
   uint32_t G = 0;
   for (uint32_t v = 0; v < n; ++v)
   {
      const uint32_t *s = sl + label_offsets[v];
      const uint32_t len = (uint32_t)(label_offsets[v + 1] - label_offsets[v]);
      uint64_t h = hash_seq(s, len) & (cap - 1);
      for (;;)
      {
         if (slot_group[h] == 0)
         {
            slot_group[h] = ++G;
            slot_point[h] = v;
            rep[G] = v;
            point_group[v] = G;
            break;
         }
         const uint32_t r = slot_point[h];
         const uint32_t rlen = (uint32_t)(label_offsets[r + 1] - label_offsets[r]);
         if (rlen == len && memcmp(sl + label_offsets[r], s, len * sizeof(uint32_t)) == 0)
         {
            point_group[v] = slot_group[h];
            break;
         }
         h = (h + 1) & (cap - 1);
      }
   }
   free(slot_point);
   free(slot_group);
   g->num_groups = G;

   /* reorder: groups 1..G concatenated, original order inside a group */
   g->group_first = (uint32_t *)calloc((size_t)G + 2, sizeof(uint32_t));
   uint32_t *cnt = (uint32_t *)calloc((size_t)G + 2, sizeof(uint32_t));
   for (uint32_t v = 0; v < n; ++v)
      cnt[point_group[v]]++;
   uint32_t acc = 0;
   for (uint32_t gid = 1; gid <= G; ++gid)
   {
      g->group_first[gid] = acc;
      acc += cnt[gid];
   }
   g->group_first[G + 1] = acc;
   g->new_to_old = (uint32_t *)malloc((n ? n : 1) * sizeof(uint32_t));
   memset(cnt, 0, ((size_t)G + 2) * sizeof(uint32_t));
   for (uint32_t v = 0; v < n; ++v)
   {
      const uint32_t gid = point_group[v];
      g->new_to_old[g->group_first[gid] + cnt[gid]++] = v;
   }
   free(cnt);
   free(point_group);

   /* label set per group */
   g->set_off = (uint64_t *)calloc((size_t)G + 2, sizeof(uint64_t));
   for (uint32_t gid = 1; gid <= G; ++gid)
      g->set_off[gid + 1] = g->set_off[gid] + (label_offsets[rep[gid] + 1] - label_offsets[rep[gid]]);
   g->set_lab = (uint32_t *)malloc((g->set_off[G + 1] ? g->set_off[G + 1] : 1) * sizeof(uint32_t));
   for (uint32_t gid = 1; gid <= G; ++gid)
      memcpy(g->set_lab + g->set_off[gid], sl + label_offsets[rep[gid]],
             (g->set_off[gid + 1] - g->set_off[gid]) * sizeof(uint32_t));
   free(rep);
   free(sl);

   /* groups ordered by label-set size (stable), then minimal strict supersets */
   uint32_t *by_size = (uint32_t *)malloc(((size_t)G + 1) * sizeof(uint32_t));
   {
      uint32_t maxlen = 0;
      for (uint32_t gid = 1; gid <= G; ++gid)
      {
         uint32_t l = (uint32_t)(g->set_off[gid + 1] - g->set_off[gid]);
         if (l > maxlen)
            maxlen = l;
      }
      uint32_t *bc = (uint32_t *)calloc((size_t)maxlen + 2, sizeof(uint32_t));
      for (uint32_t gid = 1; gid <= G; ++gid)
         bc[g->set_off[gid + 1] - g->set_off[gid] + 1]++;
      for (uint32_t l = 0; l <= maxlen; ++l)
         bc[l + 1] += bc[l];
      for (uint32_t gid = 1; gid <= G; ++gid)
         by_size[bc[g->set_off[gid + 1] - g->set_off[gid]]++] = gid;
      free(bc);
   }
   uint32_t **mins = (uint32_t **)calloc((size_t)G + 1, sizeof(uint32_t *));
   uint32_t *nmins = (uint32_t *)calloc((size_t)G + 1, sizeof(uint32_t));
#pragma omp parallel for schedule(dynamic, 16)
   for (long long fl = 1; fl <= (long long)G; ++fl)
   {
      const uint32_t f = (uint32_t)fl;
      const uint32_t *fs = g->set_lab + g->set_off[f];
      const uint32_t fn = (uint32_t)(g->set_off[f + 1] - g->set_off[f]);
      uint32_t *kept = (uint32_t *)malloc(((size_t)G + 1) * sizeof(uint32_t));
      uint32_t nk = 0;
      for (uint32_t i = 0; i < G; ++i)
      {
         const uint32_t c = by_size[i];
         if (c == f)
            continue;
         const uint32_t *cs = g->set_lab + g->set_off[c];
         const uint32_t cn = (uint32_t)(g->set_off[c + 1] - g->set_off[c]);
         if (!seq_includes(cs, cn, fs, fn))
            continue;
         int is_min = 1;
         for (uint32_t m = 0; m < nk && is_min; ++m)
         {
            const uint32_t *ms = g->set_lab + g->set_off[kept[m]];
            const uint32_t mn = (uint32_t)(g->set_off[kept[m] + 1] - g->set_off[kept[m]]);
            if (mn < cn && seq_includes(cs, cn, ms, mn))
               is_min = 0;
         }
         if (is_min)
            kept[nk++] = c;
      }
      qsort(kept, nk, sizeof(uint32_t), cmp_u32);
      mins[f] = kept;
      nmins[f] = nk;
   }
   free(by_size);
   g->out_off = (uint64_t *)calloc((size_t)G + 2, sizeof(uint64_t));
   for (uint32_t f = 1; f <= G; ++f)
      g->out_off[f + 1] = g->out_off[f] + nmins[f];
   g->out_ids = (uint32_t *)malloc((g->out_off[G + 1] ? g->out_off[G + 1] : 1) * sizeof(uint32_t));
   for (uint32_t f = 1; f <= G; ++f)
   {
      memcpy(g->out_ids + g->out_off[f], mins[f], nmins[f] * sizeof(uint32_t));
      free(mins[f]);
   }
   free(mins);
   free(nmins);
   return g;
}

uint32_t orc_num_groups(void *h) { return ((orc_label_graph *)h)->num_groups; }

void orc_copy_groups(void *h, uint32_t *new_to_old, uint32_t *group_first)
{
   orc_label_graph *g = (orc_label_graph *)h;
   memcpy(new_to_old, g->new_to_old, (size_t)g->num_points * sizeof(uint32_t));
   memcpy(group_first, g->group_first, ((size_t)g->num_groups + 2) * sizeof(uint32_t));
}

uint64_t orc_lng_nnz(void *h)
{
   orc_label_graph *g = (orc_label_graph *)h;
   return g->out_off[g->num_groups + 1];
}

void orc_copy_lng_out(void *h, uint64_t *out_offsets, uint32_t *out_ids)
{
   orc_label_graph *g = (orc_label_graph *)h;
   memcpy(out_offsets, g->out_off, ((size_t)g->num_groups + 2) * sizeof(uint64_t));
   memcpy(out_ids, g->out_ids, g->out_off[g->num_groups + 1] * sizeof(uint32_t));
}

void orc_label_graph_free(void *h)
{
   orc_label_graph *g = (orc_label_graph *)h;
   if (!g)
      return;
   free(g->new_to_old);
   free(g->group_first);
   free(g->set_off);
   free(g->set_lab);
   free(g->out_off);
   free(g->out_ids);
   free(g);
}

/* Exact cross edges for a list of rows only (same result as orc_cross_exact on those
 * rows): every target group of the row's source group is scanned into the row's
 * queue in ascending target-group order, like the reference's outer loop. */
void orc_cross_rows(const float *X, uint32_t n, uint32_t d, uint32_t k, uint32_t num_groups,
                    const uint32_t *group_first, const uint64_t *out_offsets, const uint32_t *out_ids,
                    const uint32_t *rows, uint64_t nrows, int num_threads, int fused, uint32_t *ids, float *dists)
{
   (void)n;
   if (num_threads > 0)
      omp_set_num_threads(num_threads);
#pragma omp parallel for schedule(dynamic, 1)
   for (long long i = 0; i < (long long)nrows; ++i)
   {
      const uint32_t v = rows[i];
      /* source group of v: largest g with group_first[g] <= v and a non-empty range */
      uint32_t lo = 1, hi = num_groups;
      while (lo < hi)
      {
         uint32_t mid = (lo + hi + 1) / 2;
         if (group_first[mid] <= v)
            lo = mid;
         else
            hi = mid - 1;
      }
      while (lo > 1 && group_first[lo] == group_first[lo + 1])
         --lo;
      const uint32_t f = lo;
      orc_cand *q = (orc_cand *)malloc((k + 1) * sizeof(orc_cand));
      orc_cand *loc = (orc_cand *)malloc((k + 1) * sizeof(orc_cand));
      int32_t qs = 0;
      /* targets in ascending group order */
      uint64_t nt = out_offsets[f + 1] - out_offsets[f];
      uint32_t *tg = (uint32_t *)malloc((nt ? nt : 1) * sizeof(uint32_t));
      memcpy(tg, out_ids + out_offsets[f], nt * sizeof(uint32_t));
      qsort(tg, nt, sizeof(uint32_t), cmp_u32);
      for (uint64_t e = 0; e < nt; ++e)
      {
         const uint32_t t = tg[e];
         int32_t ls = 0;
         for (uint32_t x = group_first[t]; x < group_first[t + 1]; ++x)
            orc_queue_insert(loc, &ls, (int32_t)k, x, orc_l2(X + (size_t)v * d, X + (size_t)x * d, d, fused));
         for (int32_t j = 0; j < ls; ++j)
            orc_queue_insert(q, &qs, (int32_t)k, loc[j].id, loc[j].dist);
      }
      for (uint32_t j = 0; j < k; ++j)
      {
         ids[(size_t)i * k + j] = (int32_t)j < qs ? q[j].id : 0xffffffffu;
         dists[(size_t)i * k + j] = (int32_t)j < qs ? q[j].dist : INFINITY;
      }
      free(tg);
      free(q);
      free(loc);
   }
}

/* Additional edges, exact variant: the restatement of
 * UniNavGraph::build_cross_edges_generate_additional
 * (UNG/codes/src/uni_nav_graph_cross_edges.cpp:442-596) that ungref_additional_edges
 * in ref_harness.cpp runs on the reference's own SearchQueue and distance.  Same
 * contract: (from, to) pairs in the reference's materialised order, count returned,
 * pairs written only when the count does not exceed cap. */
uint64_t orc_additional_edges(const float *X, uint32_t n, uint32_t d, uint32_t k, uint32_t num_groups,
                              const uint32_t *group_first, const uint64_t *out_offsets, const uint32_t *out_ids,
                              const uint32_t *cross_ids, int fused, uint64_t cap, uint32_t *from_ids,
                              uint32_t *to_ids)
{
   uint32_t *group_of = (uint32_t *)malloc((n ? n : 1) * sizeof(uint32_t));
   for (uint32_t v = 0; v < n; ++v)
      group_of[v] = num_groups + 1;
   for (uint32_t g = 1; g <= num_groups; ++g)
      for (uint32_t v = group_first[g]; v < group_first[g + 1]; ++v)
         group_of[v] = g;
   uint32_t *connected = (uint32_t *)calloc((size_t)num_groups + 2, sizeof(uint32_t));
   orc_cand *loc = (orc_cand *)malloc(((size_t)k + 1) * sizeof(orc_cand));
   uint64_t count = 0;
   uint32_t epoch = 0;
   for (uint32_t f = 1; f <= num_groups; ++f)
   {
      ++epoch;
      const uint32_t qf = group_first[f], qs = group_first[f + 1];
      for (uint32_t v = qf; v < qs; ++v)
         for (uint32_t j = 0; j < k; ++j)
         {
            const uint32_t id = cross_ids[(size_t)v * k + j];
            if (id == 0xffffffffu)
               continue;
            if (group_of[id] <= num_groups)
               connected[group_of[id]] = epoch;
         }
      for (uint64_t e = out_offsets[f]; e < out_offsets[f + 1]; ++e)
      {
         const uint32_t t = out_ids[e];
         if (t <= num_groups && connected[t] == epoch)
            continue;
         uint32_t cnt = 0;
         for (uint32_t v = qf; v < qs && cnt < k; ++v)
         {
            int32_t ls = 0;
            for (uint32_t x = group_first[t]; x < group_first[t + 1]; ++x)
               orc_queue_insert(loc, &ls, (int32_t)k, x, orc_l2(X + (size_t)v * d, X + (size_t)x * d, d, fused));
            for (int32_t r = 0; r < ls && r < (int32_t)(k / 2); ++r)
            {
               if (count < cap)
               {
                  from_ids[count] = v;
                  to_ids[count] = loc[r].id;
               }
               ++count;
               ++cnt;
            }
         }
      }
   }
   free(loc);
   free(connected);
   free(group_of);
   return count;
}

/* ---------------- large-group intra-graph exact kNN seeding ----------------
 * Restatement of batched_exact_knn_graph_kernel (the default 128-thread block
 * variant) and of its host defaults, UNG/codes/src/tagore_graph_builder.cu:650-795
 * and make_fast_exact_batch_config (UNG/codes/src/tagore_cuda_config.cpp:23-45).
 * PARITY UNPINNED: that source includes the external Tagore_src.cuh, which is not
 * present, so the reference cannot be built or run here; this restatement was made
 * by reading the kernel.  The reference is compiled with --use_fast_math
 * (UNG/codes/src/CMakeLists.txt:79-80): every fp32 add, sub and fma flushes
 * subnormal inputs and results to zero, and `acc += diff * diff` is one fma.
 *
 * Distance of (src, dst): thread t of 128 accumulates acc = fma(diff, diff, acc) over
 * dims t, t+128, ... ; each warp sums its 32 partials by __shfl_down (offsets 16..1),
 * then warp 0 sums the four warp totals the same way: (w0 + w2) + (w1 + w3). */
static inline float ftz(float x) { return fabsf(x) < 1.17549435e-38f ? copysignf(0.0f, x) : x; }
static inline float add_ftz(float a, float b) { return ftz(ftz(a) + ftz(b)); }
static inline float sub_ftz(float a, float b) { return ftz(ftz(a) - ftz(b)); }
static inline float fma_ftz(float a, float b, float c) { return ftz(fmaf(ftz(a), ftz(b), ftz(c))); }

static float warp_tree32(const float *p)
{
   float v[32];
   for (int i = 0; i < 32; ++i)
      v[i] = p[i];
   for (int off = 16; off > 0; off >>= 1)
      for (int i = 0; i < off; ++i)
         v[i] = add_ftz(v[i], v[i + off]);
   return v[0];
}

float orc_block_l2(const float *a, const float *b, uint32_t dim)
{
   float part[128];
   for (uint32_t t = 0; t < 128; ++t)
   {
      float acc = 0.0f;
      for (uint32_t d = t; d < dim; d += 128)
      {
         const float diff = sub_ftz(a[d], b[d]);
         acc = fma_ftz(diff, diff, acc);
      }
      part[t] = acc;
   }
   const float w0 = warp_tree32(part), w1 = warp_tree32(part + 32), w2 = warp_tree32(part + 64),
               w3 = warp_tree32(part + 96);
   return add_ftz(add_ftz(w0, w2), add_ftz(w1, w3));
}

/* One point's output row (graph_stride uint32: [degree, local ids..., padding]) from
 * its candidate list top_idx[0 .. cand_degree); the head / anchor / tail layout. */
static void knn_row_layout(uint32_t *row, const uint32_t *top_idx, uint32_t cand_degree, uint32_t n,
                           uint32_t local_src, uint32_t final_degree, uint32_t head_keep, uint32_t anchor_tail,
                           uint32_t anchor_slots, uint32_t bidir_anchor, uint32_t graph_stride)
{
   const uint32_t out_degree = final_degree < cand_degree ? final_degree : cand_degree;
   row[0] = out_degree;
   if (out_degree > 0)
   {
      uint32_t near_limit = head_keep < final_degree ? head_keep : final_degree;
      if (out_degree < near_limit)
         near_limit = out_degree;
      uint32_t write = 0;
      for (; write < near_limit; ++write)
         row[1 + write] = top_idx[write];
      const uint32_t remaining = final_degree > write ? final_degree - write : 0;
      const uint32_t anchor_limit =
          anchor_tail ? (anchor_slots == 0 ? remaining : (anchor_slots < remaining ? anchor_slots : remaining)) : 0;
      if (anchor_limit > 0 && n > 1)
      {
         for (uint32_t t = 0; t < anchor_limit && write < out_degree; ++t)
         {
            uint32_t hop = (uint32_t)(((uint64_t)(t + 1) * n) / (anchor_limit + 1));
            if (hop < 1)
               hop = 1;
            const int backward = bidir_anchor && (t & 1u);
            uint32_t cand = backward ? (local_src + n - (hop % n)) % n : (local_src + hop) % n;
            for (uint32_t retry = 0; retry < n && write < out_degree;
                 ++retry, cand = backward ? (cand + n - 1) % n : (cand + 1) % n)
            {
               if (cand == local_src)
                  continue;
               int dup = 0;
               for (uint32_t p = 0; p < write; ++p)
                  if (row[1 + p] == cand)
                  {
                     dup = 1;
                     break;
                  }
               if (!dup)
               {
                  row[1 + write++] = cand;
                  break;
               }
            }
         }
      }
      const uint32_t tail_start = near_limit;
      const uint32_t tail_count = cand_degree > tail_start ? cand_degree - tail_start : 0;
      const uint32_t step = tail_count > remaining && remaining > 0 ? (tail_count + remaining - 1) / remaining : 1;
      for (uint32_t s = tail_start; s < cand_degree && write < out_degree; s += step)
         row[1 + write++] = top_idx[s];
      for (uint32_t s = tail_start; s < cand_degree && write < out_degree; ++s)
      {
         const uint32_t cand = top_idx[s];
         int dup = 0;
         for (uint32_t p = 0; p < write; ++p)
            if (row[1 + p] == cand)
            {
               dup = 1;
               break;
            }
         if (!dup)
            row[1 + write++] = cand;
      }
   }
   for (uint32_t j = out_degree; j + 1 < graph_stride; ++j)
      row[1 + j] = local_src;
}

/* Groups g = 0 .. num_groups-1 are rows [ranges[2g], ranges[2g+1]) of X [* x d];
 * graph receives one row of graph_stride uint32 per point, groups in order (local ids);
 * entry_points[g] = 0.  candidate_k is the K of the reference (cand_degree =
 * min(64, K - 1, n - 1)). */
void orc_exact_knn_graph(const float *X, uint32_t d, uint32_t num_groups, const uint32_t *ranges,
                         uint32_t candidate_k, uint32_t final_degree, uint32_t head_keep, uint32_t anchor_tail,
                         uint32_t anchor_slots, uint32_t bidir_anchor, uint32_t graph_stride, int num_threads,
                         uint32_t *graph, uint32_t *entry_points)
{
   uint64_t *base = (uint64_t *)malloc(((size_t)num_groups + 1) * sizeof(uint64_t));
   base[0] = 0;
   for (uint32_t g = 0; g < num_groups; ++g)
      base[g + 1] = base[g] + (ranges[2 * g + 1] - ranges[2 * g]);
   if (num_threads > 0)
      omp_set_num_threads(num_threads);
   for (uint32_t g = 0; g < num_groups; ++g)
   {
      const uint32_t first = ranges[2 * g], n = ranges[2 * g + 1] - ranges[2 * g];
      if (n == 0)
         continue; /* no point writes anything (the reference refuses empty groups) */
      if (entry_points)
         entry_points[g] = 0;
      uint32_t cand_degree = candidate_k > 0 ? candidate_k - 1 : 0;
      if (cand_degree > 64)
         cand_degree = 64;
      if (cand_degree > n - 1)
         cand_degree = n - 1;
#pragma omp parallel for schedule(dynamic, 16)
      for (long long s = 0; s < (long long)n; ++s)
      {
         uint32_t top_idx[64];
         float top_dist[64];
         for (int i = 0; i < 64; ++i)
         {
            top_idx[i] = 0xffffffffu;
            top_dist[i] = 3.402823466e+38f;
         }
         const float *src = X + (size_t)(first + s) * d;
         for (uint32_t x = 0; x < n; ++x)
         {
            if (x == (uint32_t)s)
               continue;
            const float dist = orc_block_l2(src, X + (size_t)(first + x) * d, d);
            if (cand_degree > 0 && dist < top_dist[cand_degree - 1])
            {
               uint32_t pos = cand_degree;
               while (pos > 0 && dist < top_dist[pos - 1])
               {
                  if (pos < cand_degree)
                  {
                     top_dist[pos] = top_dist[pos - 1];
                     top_idx[pos] = top_idx[pos - 1];
                  }
                  --pos;
               }
               top_dist[pos] = dist;
               top_idx[pos] = x;
            }
         }
         knn_row_layout(graph + (size_t)(base[g] + s) * graph_stride, top_idx, cand_degree, n, (uint32_t)s,
                        final_degree, head_keep, anchor_tail, anchor_slots, bidir_anchor, graph_stride);
      }
   }
   free(base);
}

/* ------------------------------------------------------------------ filtered search
 * Downstream check of a built index (benchmark configuration 5): UNG greedy search
 * over a CSR graph, and the brute-force filtered ground truth.
 *
 *   orc_ung_search      UniNavGraph::iterate_to_fixed_point,
 *                       UNG/codes/src/uni_nav_graph_search_backend.cpp:242-283, with the
 *                       expanded-flag queue of SearchQueue (search_queue.cpp:26-69):
 *                       capacity L, the closest unexpanded candidate is expanded, every
 *                       unvisited neighbour is inserted; the result is the first K
 *                       entries.  Entry points come from the caller (one list per query).
 *   orc_filtered_scan   FilteredScan::answer_one_query, UNG/codes/src/filtered_scan.cpp:
 *                       157-194: every vector of the target groups into a queue of K.
 *
 * Ids are the reordered ids of X throughout. */
typedef struct
{
   uint32_t id;
   float dist;
   uint8_t expanded;
} orc_scand;

static void orc_squeue_insert(orc_scand *q, int32_t *size, int32_t cap, int32_t *cur, uint32_t id, float dist)
{
   orc_cand c = {id, dist};
   if (*size == cap)
   {
      orc_cand last = {q[*size - 1].id, q[*size - 1].dist};
      if (cand_less(last, c))
         return;
   }
   int32_t lo = 0, hi = *size;
   while (lo < hi)
   {
      int32_t mid = (lo + hi) >> 1;
      orc_cand m = {q[mid].id, q[mid].dist};
      if (cand_less(c, m))
         hi = mid;
      else if (m.id == c.id)
         return;
      else
         lo = mid + 1;
   }
   if (lo < cap)
      memmove(&q[lo + 1], &q[lo], (size_t)(*size - lo) * sizeof(orc_scand));
   q[lo].id = id;
   q[lo].dist = dist;
   q[lo].expanded = 0;
   if (*size < cap)
      (*size)++;
   if (lo < *cur)
      *cur = lo;
}

/* Per query q: entries entry_ids[entry_offsets[q] .. entry_offsets[q+1]), search queue
 * of capacity L (L >= K), result ids[q*K .. +K) (UINT32_MAX where the queue holds fewer)
 * and the number of distance computations per query in cmps (may be NULL). */
void orc_ung_search(const float *X, uint32_t n, uint32_t d, const uint64_t *offsets, const uint32_t *cols,
                    const float *Q, uint32_t nq, const uint64_t *entry_offsets, const uint32_t *entry_ids,
                    uint32_t L, uint32_t K, int fused, int num_threads, uint32_t *ids, uint32_t *cmps)
{
   if (num_threads > 0)
      omp_set_num_threads(num_threads);
#pragma omp parallel
   {
      orc_scand *q = (orc_scand *)malloc(sizeof(orc_scand) * ((size_t)L + 1));
      uint32_t *stamp = (uint32_t *)calloc(n ? n : 1, sizeof(uint32_t));
      uint32_t epoch = 0;
#pragma omp for schedule(dynamic, 16)
      for (int64_t qi = 0; qi < (int64_t)nq; ++qi)
      {
         const float *qv = Q + (size_t)qi * d;
         int32_t size = 0, cur = 0;
         uint32_t ncmp = 0;
         ++epoch; /* a fresh visited set per query (clear_visited_set) */
         for (uint64_t e = entry_offsets[qi]; e < entry_offsets[qi + 1]; ++e)
         {
            const uint32_t v = entry_ids[e];
            orc_squeue_insert(q, &size, (int32_t)L, &cur, v, orc_l2(qv, X + (size_t)v * d, d, fused));
            ++ncmp;
         }
         while (cur < size)
         {
            const int32_t pre = cur;
            q[cur].expanded = 1;
            while (cur < size && q[cur].expanded)
               ++cur;
            const uint32_t u = q[pre].id;
            for (uint64_t j = offsets[u]; j < offsets[u + 1]; ++j)
            {
               const uint32_t w = cols[j];
               if (stamp[w] == epoch)
                  continue;
               stamp[w] = epoch;
               orc_squeue_insert(q, &size, (int32_t)L, &cur, w, orc_l2(qv, X + (size_t)w * d, d, fused));
               ++ncmp;
            }
         }
         for (uint32_t r = 0; r < K; ++r)
            ids[(size_t)qi * K + r] = (int32_t)r < size ? q[r].id : UINT32_MAX;
         if (cmps)
            cmps[qi] = ncmp;
      }
      free(q);
      free(stamp);
   }
}

/* Per query q: the K nearest vectors over the row ranges of its target groups,
 * target_ids[target_offsets[q] .. target_offsets[q+1]) (group ids 1..G, rows
 * [group_first[g], group_first[g+1])), in that order.  ids/dists [nq x K]. */
void orc_filtered_scan(const float *X, uint32_t d, const uint32_t *group_first, const float *Q, uint32_t nq,
                       const uint64_t *target_offsets, const uint32_t *target_ids, uint32_t K, int fused,
                       int num_threads, uint32_t *ids, float *dists)
{
   if (num_threads > 0)
      omp_set_num_threads(num_threads);
#pragma omp parallel
   {
      orc_cand *q = (orc_cand *)malloc(sizeof(orc_cand) * ((size_t)K + 1));
#pragma omp for schedule(dynamic, 1)
      for (int64_t qi = 0; qi < (int64_t)nq; ++qi)
      {
         const float *qv = Q + (size_t)qi * d;
         int32_t size = 0;
         for (uint64_t t = target_offsets[qi]; t < target_offsets[qi + 1]; ++t)
         {
            const uint32_t g = target_ids[t];
            for (uint32_t x = group_first[g]; x < group_first[g + 1]; ++x)
               orc_queue_insert(q, &size, (int32_t)K, x, orc_l2(qv, X + (size_t)x * d, d, fused));
         }
         for (uint32_t r = 0; r < K; ++r)
         {
            ids[(size_t)qi * K + r] = (int32_t)r < size ? q[r].id : UINT32_MAX;
            dists[(size_t)qi * K + r] = (int32_t)r < size ? q[r].dist : INFINITY;
         }
      }
      free(q);
   }
}
