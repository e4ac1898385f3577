// The reference's on-disk graph text (ANNS::Graph::save, UNG/codes/include/graph.h:207-216,
// written by UniNavGraph::save as <prefix>graph, UNG/codes/src/uni_nav_graph_io.cpp:383-386)
// from a CSR adjacency: one line per point, "<id> " then "<neighbour> " for each
// neighbour in order, then a newline.  Rows are formatted in parallel chunks and
// written in order.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "ungx_internal.h"

namespace
{
// decimal digits of v appended at p, followed by a space; returns the new end
inline char *put_u32(char *p, uint32_t v)
{
   char tmp[10];
   int k = 0;
   do
   {
      tmp[k++] = char('0' + v % 10u);
      v /= 10u;
   } while (v);
   while (k)
      *p++ = tmp[--k];
   *p++ = ' ';
   return p;
}
} // namespace

extern "C"
{

int ungx_graph_save_text(const char *path, uint32_t num_points, const uint64_t *offsets, const uint32_t *cols)
{
   if (!path || (num_points && !offsets) || (num_points && offsets[num_points] > offsets[0] && !cols))
   {
      ungx::set_global_error("ungx_graph_save_text: null argument");
      return UNGX_ERR_INVALID_ARG;
   }
   for (uint32_t v = 0; v < num_points; ++v)
      if (offsets[v + 1] < offsets[v])
      {
         ungx::set_global_error("ungx_graph_save_text: offsets not monotone");
         return UNGX_ERR_INVALID_ARG;
      }
   FILE *f = std::fopen(path, "wb");
   if (!f)
   {
      ungx::set_global_error(std::string("ungx_graph_save_text: cannot open ") + path);
      return UNGX_ERR_INVALID_ARG;
   }
   // chunks of rows; each number takes at most 11 bytes with its space
   constexpr uint32_t kRows = 65536;
   const uint32_t nchunks = (num_points + kRows - 1) / kRows;
   constexpr uint32_t kBatch = 64; // chunks formatted per round (bounded host memory)
   int st = UNGX_OK;
   std::vector<std::string> buf(kBatch);
   for (uint32_t c0 = 0; c0 < nchunks && st == UNGX_OK; c0 += kBatch)
   {
      const uint32_t cn = std::min(kBatch, nchunks - c0);
      ungx::parallel_for(cn, 0, 1, [&](int64_t i) {
         const uint32_t a = (c0 + uint32_t(i)) * kRows, b = std::min(num_points, a + kRows);
         const uint64_t words = (b - a) + (offsets[b] - offsets[a]);
         std::string &s = buf[i];
         s.resize(words * 11 + (b - a));
         char *p = &s[0];
         for (uint32_t v = a; v < b; ++v)
         {
            p = put_u32(p, v);
            for (uint64_t e = offsets[v]; e < offsets[v + 1]; ++e)
               p = put_u32(p, cols[e]);
            *p++ = '\n';
         }
         s.resize(size_t(p - &s[0]));
      });
      for (uint32_t i = 0; i < cn; ++i)
         if (std::fwrite(buf[i].data(), 1, buf[i].size(), f) != buf[i].size())
         {
            ungx::set_global_error(std::string("ungx_graph_save_text: write failed on ") + path);
            st = UNGX_ERR_INVALID_ARG;
            break;
         }
   }
   if (std::fclose(f) != 0 && st == UNGX_OK)
   {
      ungx::set_global_error(std::string("ungx_graph_save_text: close failed on ") + path);
      st = UNGX_ERR_INVALID_ARG;
   }
   return st;
}

} // extern "C"
