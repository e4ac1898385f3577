// The exact cross-edge route for callers that cannot allocate device memory.
//
// Some callers cannot call cudaMalloc at the moment they need the cross edges:
// a caller whose device memory is owned by another allocator (a framework's
// caching allocator, a pool with a hard budget) that must not see foreign
// allocations, or a service that must not grow its device footprint once it is
// serving.  ungx_cross_edges_exact_noalloc serves them: the caller passes the
// device-resident base vectors and device output buffers, and the work plan the
// kernels read (work items, target segments, the row list, the rows without
// targets) goes into one fixed scratch array that this file owns.
//
// The array is a file-scope __device__ variable of kScratchBytes (64 MiB).  It
// belongs to the library's device module, which the CUDA runtime loads on a device
// at the library's first use there (lazily, with CUDA_MODULE_LOADING=LAZY, at the
// first cudaGetSymbolAddress or kernel launch); the device then holds it until the
// process exits.  Host code cannot use its name as a device address, so the
// address is fetched once per device with cudaGetSymbolAddress, with that device
// current, by the first call on the device.
//
// Nothing in the array has to start at zero: each call overwrites every byte its
// kernels read.  Every call shares the one array, so calls that overlap on the GPU
// (on different streams, or from different host threads) race on it.  A call that
// returns UNGX_ERR_TIMEOUT may leave its copies and kernels running on the array;
// the caller synchronises the stream before calling again.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "kernels.h"
#include "ungx_internal.h"

namespace
{
constexpr size_t kScratchBytes = size_t(64) << 20; // 64 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_setup_mutex;
void *g_scratch_addr[kMaxDevices] = {};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

int fail(int code, const std::string &msg)
{
   ungx::set_global_error("ungx_cross_edges_exact_noalloc: " + msg);
   return code;
}
} // namespace

extern "C" int ungx_cross_edges_exact_noalloc(const ungx_cross_edge_problem *problem, const float *d_vectors,
                                              uint32_t *d_out_ids, float *d_out_dists, void *stream)
{
   if (!problem || (problem->num_points && (!d_vectors || !d_out_ids)))
      return fail(UNGX_ERR_INVALID_ARG, "null argument");
   if (problem->topk > ungx::kExactMaxK)
      return fail(UNGX_ERR_INVALID_ARG, "k above " + std::to_string(ungx::kExactMaxK) + " is not supported");

   int dev = 0;
   cudaError_t e = cudaGetDevice(&dev);
   if (e != cudaSuccess)
      return fail(UNGX_ERR_NO_DEVICE, std::string("no current device: ") + cudaGetErrorString(e));
   if (dev < 0 || dev >= kMaxDevices)
      return fail(UNGX_ERR_INVALID_ARG, "device index beyond the supported range");

   // host plan first: its size decides whether the problem fits the scratch array
   ungx::Plan plan;
   std::string err;
   int st = ungx::build_plan(*problem, plan, err);
   if (st != UNGX_OK)
      return fail(st, "invalid problem: " + err);
   std::vector<uint32_t> rows, row_items;
   for (uint32_t i = 0; i < plan.items.size(); ++i)
      for (uint32_t r = 0; r < plan.items[i].row_count; ++r)
      {
         rows.push_back(plan.items[i].row_begin + r);
         row_items.push_back(i);
      }
   const size_t b_items = align256(plan.items.size() * sizeof(ungx::WorkItem));
   const size_t b_segs = align256(plan.segs.size() * sizeof(ungx::Segment));
   const size_t b_empty = align256(plan.empty_rows.size() * sizeof(ungx::RowRange));
   const size_t b_rows = align256(rows.size() * sizeof(uint32_t));
   const size_t need = b_items + b_segs + b_empty + 2 * b_rows;
   if (need > kScratchBytes)
      return fail(UNGX_ERR_INVALID_ARG, "the problem's work plan needs " + std::to_string(need) +
                                            " bytes of scratch; this entry point holds at most " +
                                            std::to_string(kScratchBytes) +
                                            " bytes (about 8 bytes per source row plus 16 per item and segment)");

   // once per device, with that device current: the device address of the array
   void *base = nullptr;
   {
      std::lock_guard<std::mutex> lock(g_setup_mutex);
      if (!g_scratch_addr[dev])
      {
         e = cudaGetSymbolAddress(&g_scratch_addr[dev], g_noalloc_scratch);
         if (e != cudaSuccess)
         {
            g_scratch_addr[dev] = nullptr;
            return fail(UNGX_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
         }
      }
      base = g_scratch_addr[dev];
   }
   unsigned char *p = static_cast<unsigned char *>(base);
   auto *d_items = reinterpret_cast<ungx::WorkItem *>(p);
   auto *d_segs = reinterpret_cast<ungx::Segment *>(p + b_items);
   auto *d_empty = reinterpret_cast<ungx::RowRange *>(p + b_items + b_segs);
   auto *d_rows = reinterpret_cast<uint32_t *>(p + b_items + b_segs + b_empty);
   auto *d_row_items = reinterpret_cast<uint32_t *>(p + b_items + b_segs + b_empty + b_rows);

   cudaStream_t s = static_cast<cudaStream_t>(stream);
   auto copy = [&](void *dst, const void *src, size_t bytes) -> cudaError_t {
      return bytes ? cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s) : cudaSuccess;
   };
   if ((e = copy(d_items, plan.items.data(), plan.items.size() * sizeof(ungx::WorkItem))) != cudaSuccess ||
       (e = copy(d_segs, plan.segs.data(), plan.segs.size() * sizeof(ungx::Segment))) != cudaSuccess ||
       (e = copy(d_empty, plan.empty_rows.data(), plan.empty_rows.size() * sizeof(ungx::RowRange))) !=
           cudaSuccess ||
       (e = copy(d_rows, rows.data(), rows.size() * sizeof(uint32_t))) != cudaSuccess ||
       (e = copy(d_row_items, row_items.data(), row_items.size() * sizeof(uint32_t))) != cudaSuccess)
      return fail(UNGX_ERR_CUDA, std::string("plan copy: ") + cudaGetErrorString(e));

   e = ungx::launch_fill_empty(d_empty, (uint32_t)plan.empty_rows.size(), problem->topk, d_out_ids, d_out_dists, s);
   if (e == cudaSuccess && !rows.empty())
   {
      ungx::ExactParams ep{};
      ep.items = d_items;
      ep.segs = d_segs;
      ep.X = d_vectors;
      ep.d = problem->dim;
      ep.k = problem->topk;
      ep.rows = d_rows;
      ep.row_items = d_row_items;
      ep.count_dev = nullptr;
      ep.count_host = (uint32_t)rows.size();
      ep.out_ids = d_out_ids;
      ep.out_dists = d_out_dists;
      int sms = 148;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      const uint32_t grid = (uint32_t)std::min<uint64_t>(rows.size(), uint64_t(sms) * 8);
      e = ungx::launch_exact(ep, grid, s);
   }
   if (e != cudaSuccess)
      return fail(UNGX_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(e));

   // bounded wait: the host plan vectors live until the copies and kernels are done
   const auto t0 = std::chrono::steady_clock::now();
   for (uint32_t spin = 0;; ++spin)
   {
      e = cudaStreamQuery(s);
      if (e == cudaSuccess)
         break;
      if (e != cudaErrorNotReady)
         return fail(UNGX_ERR_CUDA, std::string("device work: ") + cudaGetErrorString(e));
      if (std::chrono::steady_clock::now() - t0 > std::chrono::minutes(10))
         return fail(UNGX_ERR_TIMEOUT, "device work exceeded 10 minutes");
      if (spin > 64)
         std::this_thread::sleep_for(std::chrono::microseconds(50));
   }
   return UNGX_OK;
}
