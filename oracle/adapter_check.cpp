// TEST INFRASTRUCTURE ONLY -- the drop-in boundary checked against the reference's own
// types.  Compiled by `make -C oracle ref` with the reference's headers
// (UNG/codes/include: search_queue.h, graph.h, config.h) and linked with the reference's
// compiled SearchQueue (oracle/_ref/search_queue.o) and the product library.  It runs the
// C++ adapter (include/ungx_ung_adapter.hpp) the way the reference's UniNavGraph would:
//
//   1. generate_cross_edges<ANNS::SearchQueue, ANNS::IdxType> in the three writeback
//      modes (CrossEdgeGpuWritebackMode, UNG/codes/include/ung_cross_edge_config.h:17-22);
//   2. generate_with_additional_edges: cross edges into SearchQueues and the additional
//      edges into materialized[group] (UNG/codes/src/uni_nav_graph_cross_edges.cpp:442-596);
//   3. build_cross_group_edges into an ANNS::Graph whose neighbour lists hold the
//      group-local intra edges (UNG/codes/src/uni_nav_graph_cross_edges.cpp:613-913).
//
// usage: adapter_check <input.bin> <output.bin>
// input:  u32 n, d, k, G; u64 nnz_out, nnz_intra; f32 X[n*d]; u32 ranges[2(G+1)];
//         u64 out_off[G+2]; u32 out_ids[nnz_out]; u64 intra_off[n+1]; u32 intra_cols[nnz_intra];
//         u32 group_of[n]
// output: blocks of (u64 count, u32 words[count]) in the order written below.
// Without a usable device it prints "NO_CONTEXT <status>" and exits 0.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <utility>
#include <vector>

#include "graph.h"
#include "search_queue.h"
#include "ungx_ung_adapter.hpp"

namespace
{
template <class T>
bool read_n(FILE *f, std::vector<T> &v, size_t count)
{
   v.resize(count);
   return count == 0 || std::fread(v.data(), sizeof(T), count, f) == count;
}

void put_block(FILE *f, const std::vector<uint32_t> &w)
{
   const uint64_t c = w.size();
   std::fwrite(&c, sizeof(c), 1, f);
   if (c)
      std::fwrite(w.data(), sizeof(uint32_t), c, f);
}

uint32_t bits(float x)
{
   uint32_t u;
   std::memcpy(&u, &x, 4);
   return u;
}

// A SearchQueue's content as [n*k] ids and distance bits (empty slots: UINT32_MAX, +inf).
void queues_block(FILE *f, const std::vector<ANNS::SearchQueue> &qs, uint32_t n, uint32_t k)
{
   std::vector<uint32_t> ids(size_t(n) * k, std::numeric_limits<uint32_t>::max());
   std::vector<uint32_t> d(size_t(n) * k, bits(INFINITY));
   for (uint32_t v = 0; v < n; ++v)
      for (int32_t i = 0; i < qs[v].size() && i < int32_t(k); ++i)
      {
         ids[size_t(v) * k + i] = qs[v][i].id;
         d[size_t(v) * k + i] = bits(qs[v][i].distance);
      }
   put_block(f, ids);
   put_block(f, d);
}
} // namespace

int main(int argc, char **argv)
{
   if (argc != 3)
   {
      std::fprintf(stderr, "usage: %s <input.bin> <output.bin>\n", argv[0]);
      return 2;
   }
   FILE *in = std::fopen(argv[1], "rb");
   if (!in)
      return 2;
   uint32_t hdr[4];
   uint64_t nnz[2];
   if (std::fread(hdr, 4, 4, in) != 4 || std::fread(nnz, 8, 2, in) != 2)
      return 2;
   const uint32_t n = hdr[0], d = hdr[1], k = hdr[2], G = hdr[3];
   std::vector<float> X;
   std::vector<uint32_t> ranges, out_ids, intra_cols, group_of;
   std::vector<uint64_t> out_off, intra_off;
   if (!read_n(in, X, size_t(n) * d) || !read_n(in, ranges, 2 * size_t(G + 1)) || !read_n(in, out_off, G + size_t(2)) ||
       !read_n(in, out_ids, nnz[0]) || !read_n(in, intra_off, n + size_t(1)) || !read_n(in, intra_cols, nnz[1]) ||
       !read_n(in, group_of, n))
      return 2;
   std::fclose(in);

   // the reference's containers: _group_id_to_range, _label_nav_graph->out_neighbors
   std::vector<std::pair<ANNS::IdxType, ANNS::IdxType>> group_id_to_range(G + 1);
   std::vector<std::vector<ANNS::IdxType>> lng_out(G + 1);
   for (uint32_t g = 1; g <= G; ++g)
   {
      group_id_to_range[g] = {ranges[2 * g], ranges[2 * g + 1]};
      lng_out[g].assign(out_ids.begin() + out_off[g], out_ids.begin() + out_off[g + 1]);
   }
   std::vector<ANNS::IdxType> new_vec_id_to_group_id(group_of.begin(), group_of.end());

   ungx_context *ctx = nullptr;
   const int st = ungx_context_create(0, &ctx);
   if (st != UNGX_OK)
   {
      std::printf("NO_CONTEXT %d %s\n", st, ungx_last_error(nullptr));
      return 0;
   }
   FILE *out = std::fopen(argv[2], "wb");
   if (!out)
      return 2;
   using ungx_adapter::Writeback;
   int failures = 0;
   auto check = [&](const ungx_adapter::Result &r, const char *what) {
      if (!r.ok)
      {
         std::printf("FAILED %s %d %s\n", what, r.status, r.error.c_str());
         ++failures;
      }
   };

   // 1. the three writeback modes
   {
      std::vector<ANNS::SearchQueue> qs;
      check(ungx_adapter::generate_cross_edges<ANNS::SearchQueue, ANNS::IdxType>(
                ctx, X.data(), n, d, k, group_id_to_range, lng_out, Writeback::SearchQueue, &qs, nullptr, nullptr),
            "search_queue");
      qs.resize(n);
      queues_block(out, qs, n, k);
      std::vector<uint32_t> cap(n);
      for (uint32_t v = 0; v < n; ++v)
         cap[v] = uint32_t(qs[v].capacity());
      put_block(out, cap);
   }
   {
      std::vector<std::vector<ANNS::IdxType>> idv;
      check(ungx_adapter::generate_cross_edges<ANNS::SearchQueue, ANNS::IdxType>(
                ctx, X.data(), n, d, k, group_id_to_range, lng_out, Writeback::IdVector, nullptr, &idv, nullptr),
            "id_vector");
      idv.resize(n);
      std::vector<uint32_t> ids(size_t(n) * k, std::numeric_limits<uint32_t>::max());
      for (uint32_t v = 0; v < n; ++v)
         for (size_t i = 0; i < idv[v].size() && i < k; ++i)
            ids[size_t(v) * k + i] = idv[v][i];
      put_block(out, ids);
   }
   {
      std::vector<ANNS::IdxType> flat;
      check(ungx_adapter::generate_cross_edges<ANNS::SearchQueue, ANNS::IdxType>(
                ctx, X.data(), n, d, k, group_id_to_range, lng_out, Writeback::FlatId, nullptr, nullptr, &flat),
            "flat_id");
      flat.resize(size_t(n) * k, std::numeric_limits<uint32_t>::max());
      put_block(out, std::vector<uint32_t>(flat.begin(), flat.end()));
   }
   // 2. cross edges + additional edges, materialized per source group
   {
      std::vector<ANNS::SearchQueue> qs;
      std::vector<std::vector<std::pair<ANNS::IdxType, ANNS::IdxType>>> materialized;
      check(ungx_adapter::generate_with_additional_edges<ANNS::SearchQueue, ANNS::IdxType>(
                ctx, X.data(), n, d, k, group_id_to_range, lng_out, Writeback::SearchQueue, &qs, nullptr, nullptr,
                new_vec_id_to_group_id, &materialized),
            "with_additional");
      qs.resize(n);
      materialized.resize(G + 1);
      queues_block(out, qs, n, k);
      std::vector<uint32_t> from, to;
      for (uint32_t g = 1; g <= G; ++g) // merge_additional_edges_to_graph's order
         for (const auto &e : materialized[g])
         {
            from.push_back(e.first);
            to.push_back(e.second);
         }
      put_block(out, from);
      put_block(out, to);
   }
   // 3. the whole build_cross_group_edges step into the reference's Graph
   {
      ANNS::Graph graph(n);
      for (uint32_t v = 0; v < n; ++v)
         for (uint64_t i = intra_off[v]; i < intra_off[v + 1]; ++i)
            graph.neighbors[v].push_back(intra_cols[i]);
      check(ungx_adapter::build_cross_group_edges<ANNS::NeighborList, ANNS::IdxType>(
                ctx, X.data(), n, d, k, group_id_to_range, lng_out, graph.neighbors, false),
            "build_cross_group_edges");
      std::vector<uint32_t> off(1, 0), cols;
      for (uint32_t v = 0; v < n; ++v)
      {
         for (auto x : graph.neighbors[v])
            cols.push_back(x);
         off.push_back(uint32_t(cols.size()));
      }
      put_block(out, off);
      put_block(out, cols);
      graph.clean();
   }
   std::fclose(out);
   ungx_context_destroy(ctx);
   std::printf("DONE %d\n", failures);
   return failures ? 1 : 0;
}
