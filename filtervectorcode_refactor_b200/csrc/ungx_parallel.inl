// std::thread parallel loop (the library carries no OpenMP runtime, so it can be
// loaded next to any other OpenMP copy in the host process).
#pragma once

#include <algorithm>
#include <atomic>

namespace ungx
{
template <class F>
void parallel_for(int64_t count, int threads, int64_t chunk, F &&body)
{
   if (count <= 0)
      return;
   if (threads <= 0)
      threads = (int)std::max(1u, std::thread::hardware_concurrency());
   if (chunk <= 0)
      chunk = 1;
   const int64_t nchunks = (count + chunk - 1) / chunk;
   threads = (int)std::min<int64_t>(threads, nchunks);
   std::atomic<int64_t> next{0};
   auto worker = [&]() {
      for (;;)
      {
         const int64_t c = next.fetch_add(1);
         if (c >= nchunks)
            return;
         const int64_t lo = c * chunk, hi = std::min(count, lo + chunk);
         for (int64_t i = lo; i < hi; ++i)
            body(i);
      }
   };
   if (threads <= 1)
   {
      worker();
      return;
   }
   std::vector<std::thread> pool;
   pool.reserve(threads - 1);
   for (int t = 1; t < threads; ++t)
      pool.emplace_back(worker);
   worker();
   for (auto &t : pool)
      t.join();
}
} // namespace ungx
