// C ABI entry points: context, resident base vectors, and the cross-edge generate
// step (UniNavGraph::build_cross_edges_generate_gpu_optimized's device work,
// UNG/codes/src/uni_nav_graph_cross_edges.cpp:334-440).
//
// Error behaviour follows the reference's seam: it throws inside and returns false
// to build_cross_group_edges, which falls back to the CPU or rethrows in strict mode
// (cross_edges.cpp:394-428, 775-789).  Here every failure is a negative status plus
// ungx_last_error(); the library itself has no CPU fallback.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <thread>

#include "kernels.h"
#include "nccl_dl.h"
#include "ungx_internal.h"

using ungx::Plan;

namespace
{
struct DevBuf
{
   void *p = nullptr;
   size_t bytes = 0;
   cudaError_t ensure(size_t need)
   {
      if (need <= bytes && p)
         return cudaSuccess;
      if (p)
         cudaFree(p);
      p = nullptr;
      bytes = 0;
      const size_t alloc = std::max<size_t>(need, 256);
      cudaError_t e = cudaMalloc(&p, alloc);
      if (e == cudaSuccess)
         bytes = alloc;
      return e;
   }
   void release()
   {
      if (p)
         cudaFree(p);
      p = nullptr;
      bytes = 0;
   }
   template <class T>
   T *as() const
   {
      return static_cast<T *>(p);
   }
};

// Page-locked host buffer that grows on demand (cudaHostAlloc).
struct PinnedBuf
{
   void *p = nullptr;
   size_t bytes = 0;
   cudaError_t ensure(size_t need)
   {
      if (need <= bytes && p)
         return cudaSuccess;
      if (p)
         cudaFreeHost(p);
      p = nullptr;
      bytes = 0;
      const size_t alloc = std::max<size_t>(need, 4096);
      cudaError_t e = cudaHostAlloc(&p, alloc, cudaHostAllocDefault);
      if (e == cudaSuccess)
         bytes = alloc;
      return e;
   }
   void release()
   {
      if (p)
         cudaFreeHost(p);
      p = nullptr;
      bytes = 0;
   }
};

double ms_since(std::chrono::steady_clock::time_point t0)
{
   return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}
} // namespace

// The problem a cached plan was made for; a call whose arrays are byte-identical (and
// whose shard is the same) reuses the plan and its device copy.
struct PlanKey
{
   uint32_t n = 0, G = 0, rank = 0, count = 0;
   bool skip = false;
   std::vector<uint32_t> ranges, ids;
   std::vector<uint64_t> off;
   std::vector<uint8_t> skipv;
};

struct ungx_context
{
   Plan plan; // the last generate call's plan and the planner's working storage
   PlanKey plan_key;
   bool plan_valid = false;     // `plan` was made for `plan_key`
   bool plan_on_device = false; // its arrays are in items / segs / empties / ranges / norm_chunks
   // every shard's rows as runs (multi-GPU gather), for the cached plan
   std::vector<std::vector<ungx::CopyRange>> runs;
   std::vector<uint32_t> run_rows;
   bool runs_valid = false;
   // multi-GPU: communicator of this context's device
   const ungx::NcclApi *nccl = nullptr;
   ncclComm_t comm = nullptr;
   int world = 1, rank = 0;
   DevBuf own_runs, all_runs, recv;
   cudaEvent_t dev_ev[8] = {};
   // a plan made while ungx_cross_edges_build uploaded the vectors, for that problem
   const ungx_cross_edge_problem *preplanned = nullptr;
   int preplan_status = 0;
   std::string preplan_err;
   double preplan_ms = 0;
   int device = 0;
   int num_sms = 148;
   cudaStream_t stream = nullptr;
   std::string err;
   uint32_t timeout_ms = 120000;
   uint64_t device_wait_ns = 4000000000ull;
   uint64_t mem_limit = 0; // device budget of ungx_cross_edges_build (0: free memory)
   DevBuf pass_x, pass_ids, pass_dists, pass_ranges; // capacity path
   Plan knn_plan; // tensor-core kNN seeding: items of the groups' self-joins
   DevBuf knn_items, knn_segs, knn_chunks, knn_gmax, knn_fb, knn_fbp, knn_fbt, knn_fbc, knn_pend, knn_cnt;
   uint32_t inject = UNGX_INJECT_NONE;
   PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
   // resident base vectors (a4)
   bool have_vectors = false;
   const float *X = nullptr; // device, n x d
   DevBuf X_owned, Xh, xnorm, mean, sums, range, scale, prep_flag; // Xh: fp16 operand [n x dp]
   uint32_t n = 0, d = 0, dp = 0;
   // per-call scratch
   DevBuf items, segs, empties, ranges, gmax, norm_chunks, counters, fb_rows, fb_items, rows, row_items, out_ids,
       out_dists;
   DevBuf cand_key, cand_col;
   DevBuf stage[2];
   DevBuf copy_ranges, compact; // a shard's rows gathered for one device -> host copy
   PinnedBuf host_stage;
   // additional edges and graph emission
   DevBuf g_ranges, g_out_off, g_out_ids, group_of, reach, add_items, add_segs, add_rows, add_row_items, add_pos,
       add_res, add_off, add_cols, add_qoff, add_loff, add_from, add_to, add_stats, scan_scratch, knn_ranges, knn_base,
       knn_tasks, knn_dist, knn_dbase, knn_tiles, knn_rows;
   uint64_t knn_rejected = 0; // rows the last tensor-route kNN seeding sent to the exact kernel
   double knn_phase_ms[6] = {}; // last kNN seeding: prefilter, rerank, fallback, whole call,
                                // start to prefilter, rerank to fallback
   uint32_t add_n = 0;     // points of the last additional-edge build
   uint64_t add_edges = 0; // its edges
   // merged adjacency of the last ungx_build_cross_group_edges call
   DevBuf intra_off, intra_cols, graph_off, graph_cols;
   uint32_t graph_n = 0;
   uint64_t graph_nnz = 0;
   uint32_t *h_counters = nullptr; // pinned
   cudaEvent_t ev[11] = {}; // ev[10]: end of the last vector preparation
};

namespace
{
int fail(ungx_context *ctx, int code, const std::string &msg)
{
   if (ctx)
      ctx->err = msg;
   ungx::set_global_error(msg);
   return code;
}

int cuda_fail(ungx_context *ctx, cudaError_t e, const char *what)
{
   const int code = (e == cudaErrorMemoryAllocation) ? UNGX_ERR_OOM : UNGX_ERR_CUDA;
   return fail(ctx, code, std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

#define UNGX_CUDA(ctx, expr, what)                                                                               \
   do                                                                                                          \
   {                                                                                                           \
      cudaError_t _e = (expr);                                                                                 \
      if (_e != cudaSuccess)                                                                                   \
         return cuda_fail((ctx), _e, (what));                                                                  \
   } while (0)

// Host wait on an event with a deadline (the device work itself carries bounded
// spin waits, so a timeout here means the GPU is far slower than expected).
int wait_event(ungx_context *ctx, cudaEvent_t ev, const char *what)
{
   const auto t0 = std::chrono::steady_clock::now();
   for (uint32_t spin = 0;; ++spin)
   {
      const cudaError_t e = cudaEventQuery(ev);
      if (e == cudaSuccess)
         return UNGX_OK;
      if (e != cudaErrorNotReady)
         return cuda_fail(ctx, e, what);
      if (ms_since(t0) > ctx->timeout_ms)
         return fail(ctx, UNGX_ERR_TIMEOUT, std::string(what) + ": device work exceeded the timeout");
      // spin for the first 2 ms (short kernels), then sleep in 20 us slices
      if (spin > 64 && ms_since(t0) > 2.0)
         std::this_thread::sleep_for(std::chrono::microseconds(20));
   }
}

// Tensor map of the fp16 operand [rows x cols]: boxes of 64 columns (128 bytes,
// 128-byte swizzle) by box_rows rows; out-of-range elements read as zero.
int make_map(ungx_context *ctx, CUtensorMap *map, void *base, uint32_t rows, uint32_t cols, uint32_t box_rows)
{
   cuuint64_t dims[2] = {cols, rows};
   cuuint64_t strides[1] = {cuuint64_t(cols) * sizeof(uint16_t)};
   cuuint32_t box[2] = {64, box_rows};
   cuuint32_t estr[2] = {1, 1};
   const CUresult r = ctx->encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims, strides, box, estr,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
   if (r != CUDA_SUCCESS)
      return fail(ctx, UNGX_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r));
   return UNGX_OK;
}

// Copy host vectors to the device.  Pinned (or registered) memory goes in one
// copy; pageable memory goes through two pinned staging buffers, alternating so the
// host memcpy of one chunk overlaps the DMA of the other.
int upload_vectors(ungx_context *ctx, float *dst, const float *src, size_t bytes)
{
   cudaPointerAttributes attr{};
   const cudaError_t ae = cudaPointerGetAttributes(&attr, src);
   if (ae == cudaSuccess && (attr.type == cudaMemoryTypeHost || attr.type == cudaMemoryTypeManaged))
   {
      UNGX_CUDA(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream), "vector upload");
      return UNGX_OK;
   }
   cudaGetLastError(); // clear a non-sticky attribute error for unregistered memory
   const size_t chunk = size_t(64) << 20;
   float *pin[2] = {nullptr, nullptr};
   cudaEvent_t done[2] = {nullptr, nullptr};
   int st = UNGX_OK;
   for (int i = 0; i < 2 && st == UNGX_OK; ++i)
   {
      if (cudaHostAlloc(&pin[i], chunk, cudaHostAllocDefault) != cudaSuccess ||
          cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming) != cudaSuccess)
         st = fail(ctx, UNGX_ERR_OOM, "pinned staging allocation failed");
   }
   for (size_t off = 0, i = 0; st == UNGX_OK && off < bytes; off += chunk, ++i)
   {
      const int b = int(i & 1);
      if (i >= 2)
         st = wait_event(ctx, done[b], "vector upload");
      if (st != UNGX_OK)
         break;
      const size_t len = std::min(chunk, bytes - off);
      std::memcpy(pin[b], reinterpret_cast<const char *>(src) + off, len);
      cudaError_t e = cudaMemcpyAsync(reinterpret_cast<char *>(dst) + off, pin[b], len, cudaMemcpyHostToDevice,
                                      ctx->stream);
      if (e == cudaSuccess)
         e = cudaEventRecord(done[b], ctx->stream);
      if (e != cudaSuccess)
         st = cuda_fail(ctx, e, "vector upload");
   }
   for (int i = 0; i < 2; ++i)
      if (done[i])
      {
         if (st == UNGX_OK)
            st = wait_event(ctx, done[i], "vector upload");
         cudaEventDestroy(done[i]);
      }
   for (int i = 0; i < 2; ++i)
      if (pin[i])
         cudaFreeHost(pin[i]);
   return st;
}

template <class T>
int upload(ungx_context *ctx, DevBuf &buf, const std::vector<T> &v, const char *what)
{
   UNGX_CUDA(ctx, buf.ensure(v.size() * sizeof(T)), what);
   if (!v.empty())
      UNGX_CUDA(ctx, cudaMemcpyAsync(buf.p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice, ctx->stream),
                what);
   return UNGX_OK;
}

bool same_problem(const PlanKey &k, const ungx_cross_edge_problem &p)
{
   if (k.n != p.num_points || k.G != p.num_groups || k.rank != p.shard_rank || k.count != p.shard_count ||
       k.skip != (p.skip_source_group != nullptr))
      return false;
   const size_t G = p.num_groups;
   if (G == 0)
      return true;
   if (std::memcmp(k.ranges.data(), p.group_ranges, 2 * (G + 1) * sizeof(uint32_t)) ||
       std::memcmp(k.off.data(), p.lng_out_offsets, (G + 2) * sizeof(uint64_t)))
      return false;
   const uint64_t nnz = p.lng_out_offsets[G + 1];
   if (k.ids.size() != nnz || (nnz && std::memcmp(k.ids.data(), p.lng_out_ids, nnz * sizeof(uint32_t))))
      return false;
   return !k.skip || !std::memcmp(k.skipv.data(), p.skip_source_group, G + 1);
}

// The context's plan for `p`: reused when the problem's arrays and shard equal the
// cached plan's, built (and the key stored) otherwise.
int ensure_plan(ungx_context *ctx, const ungx_cross_edge_problem &p, bool &reused, std::string &err)
{
   reused = false;
   if (p.dim == 0 || p.topk == 0)
   {
      err = "dim and topk must be positive";
      return UNGX_ERR_INVALID_ARG;
   }
   if (ctx->plan_valid && same_problem(ctx->plan_key, p))
   {
      reused = true;
      return UNGX_OK;
   }
   ctx->plan_valid = false;
   ctx->plan_on_device = false;
   ctx->runs_valid = false;
   const int st = ungx::build_plan(p, ctx->plan, err);
   if (st != UNGX_OK)
      return st;
   PlanKey &k = ctx->plan_key;
   const size_t G = p.num_groups;
   k.n = p.num_points;
   k.G = p.num_groups;
   k.rank = p.shard_rank;
   k.count = p.shard_count;
   k.skip = p.skip_source_group != nullptr;
   if (G)
   {
      k.ranges.assign(p.group_ranges, p.group_ranges + 2 * (G + 1));
      k.off.assign(p.lng_out_offsets, p.lng_out_offsets + G + 2);
      const uint64_t nnz = p.lng_out_offsets[G + 1];
      k.ids.assign(p.lng_out_ids, p.lng_out_ids + nnz);
      if (k.skip)
         k.skipv.assign(p.skip_source_group, p.skip_source_group + G + 1);
   }
   ctx->plan_valid = true;
   return UNGX_OK;
}

// The device half of generate: plan upload, kernels, counters.  Outputs are device
// pointers.  Fills `timing` with device times.
int run_generate(ungx_context *ctx, const ungx_cross_edge_problem &p, const Plan &plan, uint32_t *d_ids,
                 float *d_dists, cudaStream_t s, ungx_cross_edge_timing &t)
{
   const uint32_t k = p.topk;
   uint32_t route = p.route;
   const int kp = ungx::tc_candidates_for_k(k);
   if (route == UNGX_ROUTE_AUTO)
      route = kp ? UNGX_ROUTE_TENSOR : UNGX_ROUTE_EXACT;
   if (route == UNGX_ROUTE_TENSOR && !kp)
      return fail(ctx, UNGX_ERR_INVALID_ARG,
                  "tensor route supports k <= " + std::to_string(ungx::kTcMaxK) + "; use the exact route");
   if (route == UNGX_ROUTE_EXACT && k > ungx::kExactMaxK)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "k above " + std::to_string(ungx::kExactMaxK) + " is not supported");
   if (route != UNGX_ROUTE_TENSOR && route != UNGX_ROUTE_EXACT)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "unknown route");
   t.route_used = route;
   t.gpu_launches = 0;

   cudaEvent_t *ev = ctx->ev;
   if (s != ctx->stream) // the operand is prepared on the context's stream
      UNGX_CUDA(ctx, cudaStreamWaitEvent(s, ev[10], 0), "stream wait");
   UNGX_CUDA(ctx, cudaEventRecord(ev[0], s), "event");
   // plan upload (once per plan: the arrays stay on the device while the plan is reused)
   const bool cached = ctx->plan_on_device && &plan == &ctx->plan;
   int st;
   if (!cached)
   {
      std::vector<uint32_t> ranges(2 * size_t(p.num_groups + 1));
      if (p.num_groups)
         std::memcpy(ranges.data(), p.group_ranges, ranges.size() * sizeof(uint32_t));
      if ((st = upload(ctx, ctx->items, plan.items, "plan upload")) ||
          (st = upload(ctx, ctx->segs, plan.segs, "plan upload")) ||
          (st = upload(ctx, ctx->empties, plan.empty_rows, "plan upload")) ||
          (st = upload(ctx, ctx->ranges, ranges, "plan upload")) ||
          (st = upload(ctx, ctx->norm_chunks, plan.norm_chunks, "plan upload")))
         return st;
      ctx->plan_on_device = &plan == &ctx->plan;
   }
   uint64_t item_rows = 0;
   for (const auto &it : plan.items)
      item_rows += it.row_count;
   UNGX_CUDA(ctx, ctx->counters.ensure(64), "counters");
   UNGX_CUDA(ctx, cudaMemsetAsync(ctx->counters.p, 0, 64, s), "counters");
   UNGX_CUDA(ctx, cudaEventRecord(ev[1], s), "event");

   UNGX_CUDA(ctx, ungx::launch_fill_empty(ctx->empties.as<ungx::RowRange>(), (uint32_t)plan.empty_rows.size(), k,
                                          d_ids, d_dists, s),
             "fill kernel");
   t.gpu_launches += plan.empty_rows.empty() ? 0 : 1;
   uint32_t *cnt = ctx->counters.as<uint32_t>(); // [0] item counter [1] fb count [2] status, [4..7] u64 x2
   int *status = reinterpret_cast<int *>(cnt + 2);
   unsigned long long *stats = reinterpret_cast<unsigned long long *>(cnt + 4);

   UNGX_CUDA(ctx, cudaEventRecord(ev[2], s), "event");
   if (route == UNGX_ROUTE_TENSOR && !plan.items.empty())
   {
      UNGX_CUDA(ctx, ctx->gmax.ensure(sizeof(float) * (p.num_groups + 1)), "group norms");
      UNGX_CUDA(ctx,
                ungx::launch_group_maxnorm(ctx->xnorm.as<float>(), ctx->norm_chunks.as<uint32_t>(),
                                           (uint32_t)(plan.norm_chunks.size() / 3), p.num_groups,
                                           ctx->gmax.as<float>(), s),
                "group norm kernel");
      UNGX_CUDA(ctx, ctx->fb_rows.ensure(sizeof(uint32_t) * std::max<uint64_t>(item_rows, 1)), "fallback list");
      UNGX_CUDA(ctx, ctx->fb_items.ensure(sizeof(uint32_t) * std::max<uint64_t>(item_rows, 1)), "fallback list");
      // candidate lists [row][2][kp], indexed by the global row
      const size_t cand = size_t(ctx->n) * ungx::kTcLists * uint32_t(ungx::tc_list_depth(kp));
      UNGX_CUDA(ctx, ctx->cand_key.ensure(cand * sizeof(float)), "candidate buffer");
      UNGX_CUDA(ctx, ctx->cand_col.ensure(cand * sizeof(uint32_t)), "candidate buffer");
      ungx::TcMaps maps;
      if ((st = make_map(ctx, &maps.a, ctx->Xh.p, ctx->n, ctx->dp, 128)))
         return st;
      for (uint32_t i = 0; i < ungx::kTcBoxes; ++i)
         if ((st = make_map(ctx, &maps.b[i], ctx->Xh.p, ctx->n, ctx->dp, 16u * (i + 1u))))
            return st;
      ungx::TcParams tp{};
      tp.items = ctx->items.as<ungx::WorkItem>();
      tp.segs = ctx->segs.as<ungx::Segment>();
      tp.num_items = (uint32_t)plan.items.size();
      tp.item_counter = cnt + 0;
      tp.xnorm = ctx->xnorm.as<float>();
      tp.dp = ctx->dp;
      tp.scale = ctx->scale.as<ungx::OperandScale>();
      tp.cand_key = ctx->cand_key.as<float>();
      tp.cand_col = ctx->cand_col.as<uint32_t>();
      tp.status = status;
      tp.timeout_ns = ctx->device_wait_ns;
      tp.inject = ctx->inject;
      const uint32_t grid = (uint32_t)std::min<size_t>(plan.items.size(), (size_t)ctx->num_sms);
      UNGX_CUDA(ctx, ungx::launch_tc(maps, tp, (uint32_t)kp, grid, s), "tensor-core kernel launch");
      UNGX_CUDA(ctx, cudaEventRecord(ev[3], s), "event");
      ungx::RerankParams rp{};
      rp.items = tp.items;
      rp.segs = tp.segs;
      rp.item_offset = 0;
      rp.X = ctx->X;
      rp.xnorm = tp.xnorm;
      rp.group_maxn2 = ctx->gmax.as<float>();
      rp.n = ctx->n;
      rp.status = status;
      rp.d = ctx->d;
      rp.k = k;
      rp.cand_key = tp.cand_key;
      rp.cand_col = tp.cand_col;
      rp.out_ids = d_ids;
      rp.out_dists = d_dists;
      rp.fb_rows = ctx->fb_rows.as<uint32_t>();
      rp.fb_items = ctx->fb_items.as<uint32_t>();
      rp.fb_count = cnt + 1;
      rp.counters = stats;
      rp.scale = tp.scale;
      ungx::tc_certificate_constants(ctx->d, ctx->dp, rp);
      UNGX_CUDA(ctx, ungx::launch_rerank(rp, (uint32_t)kp, (uint32_t)plan.items.size(), s), "rerank kernel launch");
      UNGX_CUDA(ctx, cudaEventRecord(ev[8], s), "event");
      // rows the certificate rejected: exact rescan (count read on the device)
      ungx::ExactParams ep{};
      ep.items = tp.items;
      ep.segs = tp.segs;
      ep.X = ctx->X;
      ep.d = ctx->d;
      ep.k = k;
      ep.rows = rp.fb_rows;
      ep.row_items = rp.fb_items;
      ep.count_dev = rp.fb_count;
      ep.out_ids = d_ids;
      ep.out_dists = d_dists;
      UNGX_CUDA(ctx, ungx::launch_exact(ep, (uint32_t)ctx->num_sms * 8, s), "fallback kernel launch");
      t.gpu_launches += 4;
   }
   else if (!plan.items.empty())
   {
      std::vector<uint32_t> rows, row_items;
      rows.reserve(item_rows);
      row_items.reserve(item_rows);
      for (uint32_t i = 0; i < plan.items.size(); ++i)
         for (uint32_t r = 0; r < plan.items[i].row_count; ++r)
         {
            rows.push_back(plan.items[i].row_begin + r);
            row_items.push_back(i);
         }
      if ((st = upload(ctx, ctx->rows, rows, "row list")) || (st = upload(ctx, ctx->row_items, row_items, "row list")))
         return st;
      UNGX_CUDA(ctx, cudaEventRecord(ev[3], s), "event");
      ungx::ExactParams ep{};
      ep.items = ctx->items.as<ungx::WorkItem>();
      ep.segs = ctx->segs.as<ungx::Segment>();
      ep.X = ctx->X;
      ep.d = ctx->d;
      ep.k = k;
      ep.rows = ctx->rows.as<uint32_t>();
      ep.row_items = ctx->row_items.as<uint32_t>();
      ep.count_host = (uint32_t)rows.size();
      ep.out_ids = d_ids;
      ep.out_dists = d_dists;
      // one block per row, persistent over the row list
      const uint32_t grid = (uint32_t)std::min<uint64_t>(rows.size(), (uint64_t)ctx->num_sms * 8);
      UNGX_CUDA(ctx, ungx::launch_exact(ep, std::max(grid, 1u), s), "exact kernel launch");
      t.gpu_launches += 1;
   }
   else
   {
      UNGX_CUDA(ctx, cudaEventRecord(ev[3], s), "event");
   }
   UNGX_CUDA(ctx, cudaEventRecord(ev[4], s), "event");
   UNGX_CUDA(ctx, cudaMemcpyAsync(ctx->h_counters, ctx->counters.p, 64, cudaMemcpyDeviceToHost, s), "counters");
   UNGX_CUDA(ctx, cudaEventRecord(ev[5], s), "event");
   if ((st = wait_event(ctx, ev[5], "cross-edge kernels")))
      return st;
   float a = 0, b = 0, c = 0;
   cudaEventElapsedTime(&a, ev[0], ev[1]);
   cudaEventElapsedTime(&b, ev[2], ev[4]);
   cudaEventElapsedTime(&c, ev[2], ev[3]);
   t.gpu_h2d_ms += a;
   t.gpu_kernel_ms += b;
   if (route == UNGX_ROUTE_TENSOR && !plan.items.empty())
   {
      t.tc_kernel_ms += c;
      float rr = 0, f = 0;
      cudaEventElapsedTime(&rr, ev[3], ev[8]);
      cudaEventElapsedTime(&f, ev[8], ev[4]);
      t.rerank_ms += rr;
      t.fallback_ms += f;
   }
   const int dev_status = reinterpret_cast<const int *>(ctx->h_counters)[2];
   const unsigned long long *hs = reinterpret_cast<const unsigned long long *>(ctx->h_counters + 4);
   if (route == UNGX_ROUTE_TENSOR)
   {
      t.rows_certified = hs[0];
      t.rows_fallback = hs[1];
   }
   else
   {
      t.rows_certified = 0;
      t.rows_fallback = 0;
   }
   if (dev_status != 0)
      return fail(ctx, dev_status, "tensor-core kernel reported status " + std::to_string(dev_status) +
                                       " (a bounded device wait expired)");
   return UNGX_OK;
}
// Device bytes per point of the resident path: base vectors, tensor-core operand, norm,
// candidate lists, outputs and fallback lists.
uint64_t bytes_per_point(uint32_t d, uint32_t k)
{
   const uint64_t dp = ungx::tc_operand_cols(d);
   const int kp = ungx::tc_candidates_for_k(k);
   const uint64_t lists = kp ? uint64_t(ungx::kTcLists) * uint64_t(ungx::tc_list_depth(kp)) * 8u : 0u;
   return 4ull * d + 2 * dp + 4 + lists + 8ull * k + 8;
}

// The device budget of ungx_cross_edges_build: the set limit, else the free device memory
// plus what the context already holds (its buffers are reused by the call).
uint64_t device_budget(ungx_context *ctx)
{
   if (ctx->mem_limit)
      return ctx->mem_limit;
   size_t fr = 0, tot = 0;
   if (cudaMemGetInfo(&fr, &tot) != cudaSuccess)
   {
      cudaGetLastError();
      return UINT64_MAX;
   }
   uint64_t held = 0;
   for (const DevBuf *b : {&ctx->X_owned, &ctx->Xh, &ctx->xnorm, &ctx->cand_key, &ctx->cand_col, &ctx->out_ids,
                           &ctx->out_dists, &ctx->fb_rows, &ctx->fb_items, &ctx->pass_x, &ctx->pass_ids,
                           &ctx->pass_dists})
      held += b->bytes;
   return uint64_t(double(fr) * 0.92) + held;
}

// The capacity path of ungx_cross_edges_build (the reference's X-side streaming,
// UNG/codes/src/uni_nav_graph_cross_edges.cpp:402-418): rows in slices of m, one pass per
// (source slice i, target slice j) that some LNG edge needs, two slices on the device.  A
// pass is an ordinary generate over a sub-problem of the pass buffer (rows of slice i,
// then those of slice j): each group's rows in slice i are a source group whose targets
// are its LNG out-groups' rows in slice j.  Its exact per-row top-k is merged into the
// running top-k by (distance, id), so the result equals the resident one.
int run_passes(ungx_context *ctx, const float *vectors, const ungx_cross_edge_problem &p, uint64_t budget,
               uint32_t *out_ids, float *out_dists, ungx_cross_edge_timing &t)
{
   const uint32_t n = p.num_points, d = p.dim, k = p.topk, G = p.num_groups;
   if (k > ungx::kMergeMaxK)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "capacity path supports k <= " + std::to_string(ungx::kMergeMaxK));
   const uint64_t per = bytes_per_point(d, k);
   const uint64_t fixed = uint64_t(n) * k * 8 + (uint64_t(64) << 20);
   const uint64_t m64 = budget > fixed ? (budget - fixed) / (2 * per) : 0;
   if (m64 < 16)
      return fail(ctx, UNGX_ERR_OOM,
                  "device memory budget of " + std::to_string(budget) + " bytes holds less than two slices of 16 rows");
   const uint32_t m = uint32_t(std::min<uint64_t>(m64, n));
   const uint32_t S = (n + m - 1) / m;
   cudaStream_t s = ctx->stream;
   const size_t nk = size_t(n) * k;
   UNGX_CUDA(ctx, ctx->out_ids.ensure(nk * sizeof(uint32_t)), "output allocation");
   UNGX_CUDA(ctx, ctx->out_dists.ensure(nk * sizeof(float)), "output allocation");
   UNGX_CUDA(ctx, ctx->pass_x.ensure(size_t(2) * m * d * sizeof(float)), "pass buffer");
   UNGX_CUDA(ctx, ctx->pass_ids.ensure(size_t(2) * m * k * sizeof(uint32_t)), "pass outputs");
   UNGX_CUDA(ctx, ctx->pass_dists.ensure(size_t(2) * m * k * sizeof(float)), "pass outputs");
   uint32_t *g_ids = ctx->out_ids.as<uint32_t>(), *p_ids = ctx->pass_ids.as<uint32_t>();
   float *g_d = ctx->out_dists.as<float>(), *p_d = ctx->pass_dists.as<float>();
   float *X = ctx->pass_x.as<float>();
   // sentinel rows: the running result [0, n) once, the pass outputs [0, 2m) before each pass
   std::vector<ungx::RowRange> fill;
   for (uint32_t r = 0; r < n; r += 65536)
      fill.push_back({r, std::min<uint32_t>(65536, n - r)});
   const uint32_t n_global_ranges = uint32_t(fill.size());
   for (uint32_t r = 0; r < 2 * m; r += 65536)
      fill.push_back({r, std::min<uint32_t>(65536, 2 * m - r)});
   const uint32_t n_pass_ranges = uint32_t(fill.size()) - n_global_ranges;
   int st;
   if ((st = upload(ctx, ctx->pass_ranges, fill, "fill ranges")))
      return st;
   const ungx::RowRange *d_fill = ctx->pass_ranges.as<ungx::RowRange>();
   UNGX_CUDA(ctx, ungx::launch_fill_empty(d_fill, n_global_ranges, k, g_ids, g_d, s), "fill kernel");
   const uint32_t *R = p.group_ranges;
   const uint64_t *OO = p.lng_out_offsets;
   const uint32_t *OI = p.lng_out_ids;
   auto overlaps = [&](uint32_t g, uint32_t a, uint32_t b) { return R[2 * g] < b && R[2 * g + 1] > a && R[2 * g] < R[2 * g + 1]; };
   std::vector<uint32_t> tgt_id(size_t(G) + 1, 0u);
   std::vector<uint8_t> need(S);
   t.passes = 0;
   for (uint32_t i = 0; i < S; ++i)
   {
      const uint32_t si = i * m, ei = std::min(n, si + m), ni = ei - si;
      std::vector<uint32_t> src_groups;
      std::fill(need.begin(), need.end(), uint8_t(0));
      for (uint32_t g = 1; g <= G; ++g)
         if (overlaps(g, si, ei))
         {
            src_groups.push_back(g);
            if (p.skip_source_group && p.skip_source_group[g])
               continue;
            for (uint64_t e = OO[g]; e < OO[g + 1]; ++e)
            {
               const uint32_t ta = R[2 * OI[e]], tb = R[2 * OI[e] + 1];
               if (ta < tb)
                  for (uint32_t j = ta / m; j <= (tb - 1) / m; ++j)
                     need[j] = 1;
            }
         }
      if ((st = upload_vectors(ctx, X, vectors + size_t(si) * d, size_t(ni) * d * sizeof(float))))
         return st;
      for (uint32_t j = 0; j < S; ++j)
      {
         if (!need[j])
            continue;
         const uint32_t sj = j * m, ej = std::min(n, sj + m), nj = ej - sj;
         const uint32_t nbuf = j == i ? ni : ni + nj;
         if (j != i && (st = upload_vectors(ctx, X + size_t(ni) * d, vectors + size_t(sj) * d,
                                            size_t(nj) * d * sizeof(float))))
            return st;
         // the pass's sub-problem over the buffer rows
         std::vector<uint32_t> ranges(2, 0u), ids;
         std::vector<uint64_t> off(1, 0u);
         auto piece = [&](uint32_t g, uint32_t a, uint32_t b, uint32_t base) {
            ranges.push_back(base + std::max(R[2 * g], a) - a);
            ranges.push_back(base + std::min(R[2 * g + 1], b) - a);
         };
         std::vector<uint32_t> tgt_groups;
         if (j == i)
         {
            for (size_t q = 0; q < src_groups.size(); ++q)
               tgt_id[src_groups[q]] = uint32_t(q + 1);
         }
         else
         {
            for (uint32_t g = 1; g <= G; ++g)
               if (overlaps(g, sj, ej))
               {
                  tgt_groups.push_back(g);
                  tgt_id[g] = uint32_t(src_groups.size() + tgt_groups.size());
               }
         }
         for (uint32_t g : src_groups)
         {
            piece(g, si, ei, 0);
            off.push_back(ids.size());
            if (!(p.skip_source_group && p.skip_source_group[g]))
               for (uint64_t e = OO[g]; e < OO[g + 1]; ++e)
                  if (tgt_id[OI[e]])
                     ids.push_back(tgt_id[OI[e]]);
         }
         for (uint32_t g : tgt_groups)
         {
            piece(g, sj, ej, ni);
            off.push_back(ids.size());
         }
         off.push_back(ids.size()); // off[q] = first out id of group q (1..), off[0] = 0
         for (uint32_t g : src_groups)
            tgt_id[g] = 0;
         for (uint32_t g : tgt_groups)
            tgt_id[g] = 0;
         ungx_cross_edge_problem sub{};
         sub.num_points = nbuf;
         sub.dim = d;
         sub.topk = k;
         sub.num_groups = uint32_t(src_groups.size() + tgt_groups.size());
         sub.group_ranges = ranges.data();
         sub.lng_out_offsets = off.data();
         sub.lng_out_ids = ids.empty() ? nullptr : ids.data();
         sub.route = p.route;
         sub.shard_rank = 0;
         sub.shard_count = 1;
         if ((st = ungx_prepare_base_vectors(ctx, X, nbuf, d, 1)))
            return st;
         bool reused = false;
         std::string err;
         if ((st = ensure_plan(ctx, sub, reused, err)))
            return fail(ctx, st, "capacity pass: " + err);
         UNGX_CUDA(ctx, ungx::launch_fill_empty(d_fill + n_global_ranges, n_pass_ranges, k, p_ids, p_d, s),
                   "fill kernel");
         ungx_cross_edge_timing tp{};
         if ((st = run_generate(ctx, sub, ctx->plan, p_ids, p_d, s, tp)))
            return st;
         UNGX_CUDA(ctx, ungx::launch_merge_pass(p_ids, p_d, ni, k, si, ni, j == i ? si : sj, g_ids, g_d, s),
                   "merge kernel");
         t.gpu_h2d_ms += tp.gpu_h2d_ms;
         t.gpu_kernel_ms += tp.gpu_kernel_ms;
         t.tc_kernel_ms += tp.tc_kernel_ms;
         t.rerank_ms += tp.rerank_ms;
         t.fallback_ms += tp.fallback_ms;
         t.rows_certified += tp.rows_certified;
         t.rows_fallback += tp.rows_fallback;
         t.gpu_launches += tp.gpu_launches + 3 + 2; // + the operand kernels, the fill and the merge
         t.pairs += ctx->plan.pairs;
         t.route_used = tp.route_used;
         ++t.passes;
      }
   }
   UNGX_CUDA(ctx, cudaMemcpyAsync(out_ids, g_ids, nk * sizeof(uint32_t), cudaMemcpyDeviceToHost, s), "output copy");
   if (out_dists)
      UNGX_CUDA(ctx, cudaMemcpyAsync(out_dists, g_d, nk * sizeof(float), cudaMemcpyDeviceToHost, s), "output copy");
   UNGX_CUDA(ctx, cudaEventRecord(ctx->ev[7], s), "event");
   if ((st = wait_event(ctx, ctx->ev[7], "output copy")))
      return st;
   ctx->plan_valid = false; // the context's plan belongs to the last pass's sub-problem
   ctx->plan_on_device = false;
   return UNGX_OK;
}
// The tensor-core route of the exact kNN seeding: tc_kernel over the groups' self-joins
// (items of <= 128 rows of a group, the group itself the only target, the diagonal
// excluded; lists of 32 per column third), the rerank in the reference's distance with
// its certificate, then the exact kernel for the rows it rejected.  Every row is written
// by the rerank; the fallback rewrites the rejected ones.
int run_knn_tensor(ungx_context *ctx, const std::vector<uint32_t> &ranges, uint32_t num_groups,
                   const ungx::KnnParams &kp, cudaStream_t s, bool &launched)
{
   launched = false;
   // the self-join problem: group g (1-based) = the caller's group g - 1, out(g) = {g}
   std::vector<uint32_t> sr(2 * (size_t(num_groups) + 1), 0u), sid(num_groups);
   std::vector<uint64_t> so(size_t(num_groups) + 2, 0u);
   for (uint32_t g = 0; g < num_groups; ++g)
   {
      sr[2 * (g + 1)] = ranges[2 * g];
      sr[2 * (g + 1) + 1] = ranges[2 * g + 1];
      so[g + 1] = g;
      sid[g] = g + 1;
   }
   so[num_groups + 1] = num_groups;
   ungx_cross_edge_problem sp{};
   sp.num_points = ctx->n;
   sp.dim = ctx->d;
   sp.topk = 24;
   sp.num_groups = num_groups;
   sp.group_ranges = sr.data();
   sp.lng_out_offsets = so.data();
   sp.lng_out_ids = sid.data();
   sp.route = UNGX_ROUTE_TENSOR;
   sp.shard_rank = 0;
   sp.shard_count = 1;
   std::string err;
   ungx::Plan &plan = ctx->knn_plan;
   int st = ungx::build_plan(sp, plan, err);
   if (st)
      return fail(ctx, st, "kNN plan: " + err);
   if (plan.items.empty())
      return UNGX_OK;
   if ((st = upload(ctx, ctx->knn_items, plan.items, "kNN plan")) || (st = upload(ctx, ctx->knn_segs, plan.segs, "kNN plan")) ||
       (st = upload(ctx, ctx->knn_chunks, plan.norm_chunks, "kNN plan")))
      return st;
   constexpr int kp_lists = 32;
   UNGX_CUDA(ctx, ctx->knn_gmax.ensure(sizeof(float) * (size_t(num_groups) + 1)), "group norms");
   UNGX_CUDA(ctx,
             ungx::launch_group_maxnorm(ctx->xnorm.as<float>(), ctx->knn_chunks.as<uint32_t>(),
                                        (uint32_t)(plan.norm_chunks.size() / 3), num_groups, ctx->knn_gmax.as<float>(), s),
             "group norm kernel");
   const size_t cand = size_t(ctx->n) * ungx::kTcLists * uint32_t(ungx::tc_list_depth(kp_lists));
   UNGX_CUDA(ctx, ctx->cand_key.ensure(cand * sizeof(float)), "candidate buffer");
   UNGX_CUDA(ctx, ctx->cand_col.ensure(cand * sizeof(uint32_t)), "candidate buffer");
   uint64_t item_rows = 0;
   for (const auto &it : plan.items)
      item_rows += it.row_count;
   const uint64_t rows_max = std::max<uint64_t>(item_rows, 1);
   // rejected rows: four buckets per group (a failing list 0, 1, 2, or the full rescan),
   // each with room for the group's rows; pending entries for up to 2^17 partial rows
   const uint32_t pend_cap = (uint32_t)std::min<uint64_t>(rows_max, 1u << 17);
   UNGX_CUDA(ctx, ctx->knn_fb.ensure(4 * sizeof(uint32_t) * rows_max), "fallback list");
   UNGX_CUDA(ctx, ctx->knn_fbp.ensure(4 * sizeof(uint32_t) * rows_max), "fallback list");
   UNGX_CUDA(ctx, ctx->knn_fbt.ensure(4 * sizeof(uint32_t) * rows_max), "fallback tasks");
   UNGX_CUDA(ctx, ctx->knn_fbc.ensure(4 * sizeof(uint32_t) * std::max<uint32_t>(num_groups, 1)), "fallback counts");
   UNGX_CUDA(ctx, ctx->knn_pend.ensure(size_t(pend_cap) * 96 * sizeof(float2)), "fallback entries");
   UNGX_CUDA(ctx, cudaMemsetAsync(ctx->knn_fbc.p, 0, 4 * sizeof(uint32_t) * num_groups, s), "fallback counts");
   UNGX_CUDA(ctx, ctx->knn_cnt.ensure(64), "counters");
   UNGX_CUDA(ctx, cudaMemsetAsync(ctx->knn_cnt.p, 0, 64, s), "counters");
   // [0] item counter [1] partial rows with pending entries [2] status [3] fallback tasks,
   // [4..7] u64 x2: certified, rejected rows
   uint32_t *cnt = ctx->knn_cnt.as<uint32_t>();
   ungx::TcMaps maps;
   if ((st = make_map(ctx, &maps.a, ctx->Xh.p, ctx->n, ctx->dp, 128)))
      return st;
   for (uint32_t i = 0; i < ungx::kTcBoxes; ++i)
      if ((st = make_map(ctx, &maps.b[i], ctx->Xh.p, ctx->n, ctx->dp, 16u * (i + 1u))))
         return st;
   ungx::TcParams tp{};
   tp.items = ctx->knn_items.as<ungx::WorkItem>();
   tp.segs = ctx->knn_segs.as<ungx::Segment>();
   tp.num_items = (uint32_t)plan.items.size();
   tp.item_counter = cnt + 0;
   tp.xnorm = ctx->xnorm.as<float>();
   tp.dp = ctx->dp;
   tp.scale = ctx->scale.as<ungx::OperandScale>();
   tp.cand_key = ctx->cand_key.as<float>();
   tp.cand_col = ctx->cand_col.as<uint32_t>();
   tp.status = reinterpret_cast<int *>(cnt + 2);
   tp.timeout_ns = ctx->device_wait_ns;
   tp.inject = ctx->inject;
   tp.exclude_self = 1;
   const uint32_t grid = (uint32_t)std::min<size_t>(plan.items.size(), (size_t)ctx->num_sms);
   UNGX_CUDA(ctx, cudaEventRecord(ctx->ev[3], s), "event");
   UNGX_CUDA(ctx, ungx::launch_tc(maps, tp, (uint32_t)kp_lists, grid, s), "kNN tensor-core kernel launch");
   UNGX_CUDA(ctx, cudaEventRecord(ctx->ev[4], s), "event");
   ungx::KnnRerankParams rp{};
   rp.p = kp;
   rp.items = tp.items;
   rp.segs = tp.segs;
   rp.cand_key = tp.cand_key;
   rp.cand_col = tp.cand_col;
   rp.xnorm = tp.xnorm;
   rp.group_maxn2 = ctx->knn_gmax.as<float>();
   rp.scale = tp.scale;
   rp.status = tp.status;
   ungx::RerankParams cc{};
   ungx::tc_certificate_constants(ctx->d, ctx->dp, cc);
   rp.c1 = cc.c1;
   rp.c2 = cc.c2;
   rp.c3 = cc.c3;
   rp.c4 = cc.c4;
   rp.gd = cc.gd;
   // the reference's block distance: one rounding in the difference, at most ceil(d/128)
   // fused updates per partial, 7 levels of additions; flushed subnormals add at most
   // (d + 128) 2^-126 in absolute terms
   rp.gref = (16.0 + 2.0 * ((ctx->d + 127) / 128)) * std::ldexp(1.0, -24);
   rp.abs_err = (double(ctx->d) + 128.0) * std::ldexp(1.0, -126) * 2.0;
   rp.fb_rows = ctx->knn_fb.as<uint32_t>();
   rp.fb_pend_idx = ctx->knn_fbp.as<uint32_t>();
   rp.fb_group_count = ctx->knn_fbc.as<uint32_t>();
   rp.fb_pend = ctx->knn_pend.as<float2>();
   rp.fb_pend_count = cnt + 1;
   rp.fb_pend_cap = pend_cap;
   rp.counters = reinterpret_cast<unsigned long long *>(cnt + 4);
   UNGX_CUDA(ctx, ungx::launch_knn_rerank(rp, (uint32_t)plan.items.size(), s), "kNN rerank launch");
   UNGX_CUDA(ctx, cudaEventRecord(ctx->ev[2], s), "event");
   // the rejected rows, recomputed exactly with no host round trip: each group's rows
   // cut into tasks of a few rows, which share every staged column tile
   UNGX_CUDA(ctx,
             ungx::launch_knn_fallback_tasks(ctx->knn_fbc.as<uint32_t>(), num_groups, ctx->knn_fbt.as<uint32_t>(),
                                             (uint32_t)std::min<uint64_t>(rows_max, UINT32_MAX), cnt + 3, s),
             "kNN fallback task kernel");
   UNGX_CUDA(ctx, cudaEventRecord(ctx->ev[5], s), "event");
   UNGX_CUDA(ctx,
             ungx::launch_knn_fallback_rows(kp, ctx->knn_fb.as<uint32_t>(), ctx->knn_fbp.as<uint32_t>(),
                                            ctx->knn_pend.as<float2>(), ctx->knn_fbt.as<uint32_t>(), cnt + 3,
                                            ctx->num_sms, s),
             "kNN fallback kernel");
   launched = true;
   return UNGX_OK;
}

// After the tensor route's kernels are done: the prefilter's status, the rejected-row
// count and the phase times.
int finish_knn_tensor(ungx_context *ctx, uint64_t &rejected)
{
   uint32_t hc[8] = {};
   UNGX_CUDA(ctx, cudaMemcpy(hc, ctx->knn_cnt.p, sizeof(hc), cudaMemcpyDeviceToHost), "kNN counters");
   if (hc[2] != 0)
      return fail(ctx, (int)hc[2], "kNN tensor-core kernel reported status " + std::to_string((int)hc[2]));
   rejected = uint64_t(hc[6]) | (uint64_t(hc[7]) << 32);
   float a = 0.f, b = 0.f, c = 0.f, f = 0.f, g = 0.f;
   cudaEventElapsedTime(&a, ctx->ev[3], ctx->ev[4]);
   cudaEventElapsedTime(&b, ctx->ev[4], ctx->ev[2]);
   cudaEventElapsedTime(&c, ctx->ev[0], ctx->ev[3]);
   cudaEventElapsedTime(&f, ctx->ev[5], ctx->ev[1]);
   cudaEventElapsedTime(&g, ctx->ev[2], ctx->ev[5]);
   ctx->knn_phase_ms[0] = a;
   ctx->knn_phase_ms[1] = b;
   ctx->knn_phase_ms[2] = f;
   ctx->knn_phase_ms[4] = c;
   ctx->knn_phase_ms[5] = g;
   return UNGX_OK;
}
} // namespace

extern "C"
{

const char *ungx_status_string(int status)
{
   switch (status)
   {
   case UNGX_OK: return "ok";
   case UNGX_ERR_INVALID_ARG: return "invalid argument";
   case UNGX_ERR_OOM: return "out of memory";
   case UNGX_ERR_CUDA: return "CUDA error";
   case UNGX_ERR_TIMEOUT: return "timeout";
   case UNGX_ERR_ABORTED: return "aborted";
   case UNGX_ERR_NO_DEVICE: return "no usable device";
   case UNGX_ERR_STATE: return "invalid call order";
   default: return "unknown status";
   }
}

const char *ungx_last_error(const ungx_context *ctx) { return ctx ? ctx->err.c_str() : ungx::global_error(); }

int ungx_context_create(int device, ungx_context **out)
{
   if (!out)
      return fail(nullptr, UNGX_ERR_INVALID_ARG, "ungx_context_create: null output");
   *out = nullptr;
   int count = 0;
   cudaError_t e = cudaGetDeviceCount(&count);
   if (e != cudaSuccess || count == 0)
   {
      cudaGetLastError();
      return fail(nullptr, UNGX_ERR_NO_DEVICE, std::string("no CUDA device: ") + cudaGetErrorString(e));
   }
   if (device < 0 || device >= count)
      return fail(nullptr, UNGX_ERR_INVALID_ARG, "device index out of range");
   cudaDeviceProp prop{};
   if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess)
      return cuda_fail(nullptr, e, "cudaGetDeviceProperties");
   if (prop.major != 10 || prop.minor != 0)
      return fail(nullptr, UNGX_ERR_NO_DEVICE,
                  "device is sm_" + std::to_string(prop.major) + std::to_string(prop.minor) +
                      "; this build targets sm_100a (B200)");
   auto ctx = std::make_unique<ungx_context>();
   ctx->device = device;
   ctx->num_sms = prop.multiProcessorCount;
   if ((e = cudaSetDevice(device)) != cudaSuccess)
      return cuda_fail(nullptr, e, "cudaSetDevice");
   if ((e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking)) != cudaSuccess)
      return cuda_fail(nullptr, e, "stream");
   for (auto &ev : ctx->ev)
      if ((e = cudaEventCreate(&ev)) != cudaSuccess)
         return cuda_fail(nullptr, e, "event");
   for (auto &ev : ctx->dev_ev)
      if ((e = cudaEventCreate(&ev)) != cudaSuccess)
         return cuda_fail(nullptr, e, "event");
   if ((e = cudaHostAlloc(&ctx->h_counters, 64, cudaHostAllocDefault)) != cudaSuccess)
      return cuda_fail(nullptr, e, "pinned counters");
   void *fn = nullptr;
   cudaDriverEntryPointQueryResult q{};
   if ((e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q)) != cudaSuccess ||
       q != cudaDriverEntryPointSuccess || !fn)
      return fail(nullptr, UNGX_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
   ctx->encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
   *out = ctx.release();
   return UNGX_OK;
}

int ungx_context_destroy(ungx_context *ctx)
{
   if (!ctx)
      return UNGX_OK;
   cudaSetDevice(ctx->device);
   if (ctx->stream)
      cudaStreamSynchronize(ctx->stream);
   ungx_comm_destroy(ctx);
   ungx_release_base_vectors(ctx);
   for (DevBuf *b : {&ctx->items, &ctx->segs, &ctx->empties, &ctx->ranges, &ctx->gmax, &ctx->norm_chunks, &ctx->counters,
                     &ctx->fb_rows, &ctx->fb_items, &ctx->rows, &ctx->row_items, &ctx->out_ids, &ctx->out_dists,
                     &ctx->stage[0], &ctx->stage[1], &ctx->cand_key, &ctx->cand_col, &ctx->copy_ranges,
                     &ctx->compact, &ctx->g_ranges, &ctx->g_out_off, &ctx->g_out_ids, &ctx->group_of, &ctx->reach,
                     &ctx->add_items, &ctx->add_segs, &ctx->add_rows, &ctx->add_row_items, &ctx->add_pos,
                     &ctx->add_res, &ctx->add_off, &ctx->add_cols, &ctx->add_qoff, &ctx->add_loff, &ctx->add_from,
                     &ctx->add_to, &ctx->add_stats, &ctx->scan_scratch, &ctx->knn_ranges,
                     &ctx->knn_base, &ctx->knn_tasks, &ctx->knn_dist, &ctx->knn_dbase, &ctx->knn_tiles,
                     &ctx->knn_rows, &ctx->intra_off, &ctx->intra_cols, &ctx->graph_off, &ctx->graph_cols,
                     &ctx->own_runs, &ctx->all_runs, &ctx->recv, &ctx->pass_x, &ctx->pass_ids, &ctx->pass_dists,
                     &ctx->pass_ranges, &ctx->knn_items, &ctx->knn_segs, &ctx->knn_chunks, &ctx->knn_gmax,
                     &ctx->knn_fb, &ctx->knn_fbp, &ctx->knn_fbt, &ctx->knn_fbc, &ctx->knn_pend, &ctx->knn_cnt})
      b->release();
   ctx->host_stage.release();
   for (auto &ev : ctx->ev)
      if (ev)
         cudaEventDestroy(ev);
   for (auto &ev : ctx->dev_ev)
      if (ev)
         cudaEventDestroy(ev);
   if (ctx->h_counters)
      cudaFreeHost(ctx->h_counters);
   if (ctx->stream)
      cudaStreamDestroy(ctx->stream);
   delete ctx;
   return UNGX_OK;
}

int ungx_set_timeout_ms(ungx_context *ctx, uint32_t timeout_ms)
{
   if (!ctx || timeout_ms == 0)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "ungx_set_timeout_ms: bad argument");
   ctx->timeout_ms = timeout_ms;
   return UNGX_OK;
}

int ungx_set_device_wait_limit_ns(ungx_context *ctx, uint64_t limit_ns)
{
   if (!ctx || limit_ns == 0)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "ungx_set_device_wait_limit_ns: bad argument");
   ctx->device_wait_ns = limit_ns;
   return UNGX_OK;
}

uint64_t ungx_resident_bytes(uint32_t num_points, uint32_t dim, uint32_t topk)
{
   return uint64_t(num_points) * bytes_per_point(dim, topk) + (uint64_t(64) << 20);
}

int ungx_set_device_memory_limit(ungx_context *ctx, uint64_t bytes)
{
   if (!ctx)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "ungx_set_device_memory_limit: null context");
   ctx->mem_limit = bytes;
   return UNGX_OK;
}

int ungx_set_fault_injection(ungx_context *ctx, uint32_t flags)
{
   if (!ctx || flags > UNGX_INJECT_WITHHOLD_WORK)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "ungx_set_fault_injection: bad argument");
   ctx->inject = flags;
   return UNGX_OK;
}

int ungx_prepare_base_vectors(ungx_context *ctx, const float *vectors, uint32_t n, uint32_t d, int on_device)
{
   if (!ctx)
      return fail(nullptr, UNGX_ERR_INVALID_ARG, "null context");
   if (!vectors || n == 0 || d == 0)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "ungx_prepare_base_vectors: empty or null vectors");
   UNGX_CUDA(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
   // device buffers of an earlier preparation are reused when large enough
   ctx->have_vectors = false;
   ctx->X = nullptr;
   const auto t0 = std::chrono::steady_clock::now();
   const uint32_t dp = ungx::tc_operand_cols(d);
   const size_t xbytes = size_t(n) * d * sizeof(float);
   if (on_device)
      ctx->X = vectors;
   else
   {
      UNGX_CUDA(ctx, ctx->X_owned.ensure(xbytes), "vector allocation");
      int st = upload_vectors(ctx, ctx->X_owned.as<float>(), vectors, xbytes);
      if (st)
         return st;
      ctx->X = ctx->X_owned.as<float>();
   }
   UNGX_CUDA(ctx, ctx->Xh.ensure(size_t(n) * dp * sizeof(uint16_t)), "operand allocation");
   UNGX_CUDA(ctx, ctx->xnorm.ensure(size_t(n) * sizeof(float)), "norm allocation");
   UNGX_CUDA(ctx, ctx->mean.ensure(size_t(d) * sizeof(float)), "mean allocation");
   UNGX_CUDA(ctx, ctx->sums.ensure(size_t(d) * sizeof(double)), "mean allocation");
   UNGX_CUDA(ctx, ctx->range.ensure(size_t(d) * 2 * sizeof(uint32_t)), "range allocation");
   UNGX_CUDA(ctx, ctx->scale.ensure(sizeof(ungx::OperandScale)), "scale allocation");
   UNGX_CUDA(ctx, ctx->prep_flag.ensure(sizeof(uint32_t)), "flag allocation");
   UNGX_CUDA(ctx,
             ungx::launch_prepare_operand(ctx->X, n, d, dp, ctx->sums.as<double>(), ctx->range.as<uint32_t>(),
                                          ctx->mean.as<float>(), ctx->scale.as<ungx::OperandScale>(),
                                          ctx->Xh.as<uint16_t>(), ctx->xnorm.as<float>(), ctx->prep_flag.as<uint32_t>(),
                                          ctx->stream),
             "operand preparation kernels");
   // The preparation kernels run on while the caller goes on (a generate call plans on
   // the host meanwhile); work on the context's stream follows them in order, work on
   // another stream waits for this event, and a fault in them surfaces at that work's
   // wait.  Device vectors stay valid until ungx_release_base_vectors in any case.
   UNGX_CUDA(ctx, cudaEventRecord(ctx->ev[10], ctx->stream), "event");
   ctx->n = n;
   ctx->d = d;
   ctx->dp = dp;
   ctx->have_vectors = true;
   (void)t0;
   return UNGX_OK;
}

int ungx_release_base_vectors(ungx_context *ctx)
{
   if (!ctx)
      return UNGX_ERR_INVALID_ARG;
   cudaSetDevice(ctx->device);
   ctx->X_owned.release();
   ctx->Xh.release();
   ctx->xnorm.release();
   ctx->mean.release();
   ctx->sums.release();
   ctx->range.release();
   ctx->scale.release();
   ctx->X = nullptr;
   ctx->have_vectors = false;
   ctx->n = ctx->d = ctx->dp = 0;
   return UNGX_OK;
}

int ungx_cross_edges_generate_device(ungx_context *ctx, const ungx_cross_edge_problem *problem, uint32_t *d_ids,
                                     float *d_dists, void *stream, ungx_cross_edge_timing *timing)
{
   if (!ctx || !problem)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "null argument");
   if (!ctx->have_vectors)
      return fail(ctx, UNGX_ERR_STATE, "call ungx_prepare_base_vectors first");
   if (problem->num_points != ctx->n || problem->dim != ctx->d)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "problem n/d differ from the prepared base vectors");
   if (problem->num_points && !d_ids)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "null output");
   UNGX_CUDA(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
   const auto t0 = std::chrono::steady_clock::now();
   ungx_cross_edge_timing t{};
   Plan &plan = ctx->plan; // reused: its buffers keep their capacity across calls
   std::string err;
   bool reused = false;
   int st = ensure_plan(ctx, *problem, reused, err);
   if (st)
      return fail(ctx, st, "invalid problem: " + err);
   t.plan_ms = ms_since(t0);
   t.pairs = plan.pairs;
   cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
   st = run_generate(ctx, *problem, plan, d_ids, d_dists, s, t);
   t.generate_ms = ms_since(t0);
   if (timing)
      *timing = t;
   return st;
}

int ungx_cross_edges_generate(ungx_context *ctx, const ungx_cross_edge_problem *problem, uint32_t *out_ids,
                              float *out_dists, ungx_cross_edge_timing *timing)
{
   if (!ctx || !problem)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "null argument");
   if (!ctx->have_vectors)
      return fail(ctx, UNGX_ERR_STATE, "call ungx_prepare_base_vectors first");
   if (problem->num_points != ctx->n || problem->dim != ctx->d)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "problem n/d differ from the prepared base vectors");
   if (problem->num_points && !out_ids)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "null output");
   UNGX_CUDA(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
   const auto t0 = std::chrono::steady_clock::now();
   ungx_cross_edge_timing t{};
   Plan &plan = ctx->plan; // reused: its buffers keep their capacity across calls
   std::string err;
   int st;
   if (ctx->preplanned == problem)
   {
      st = ctx->preplan_status;
      err = ctx->preplan_err;
      t.plan_ms = ctx->preplan_ms;
      ctx->preplanned = nullptr;
   }
   else
   {
      bool reused = false;
      st = ensure_plan(ctx, *problem, reused, err);
      t.plan_ms = ms_since(t0);
   }
   if (st)
      return fail(ctx, st, "invalid problem: " + err);
   t.pairs = plan.pairs;
   const size_t nk = size_t(problem->num_points) * problem->topk;
   UNGX_CUDA(ctx, ctx->out_ids.ensure(nk * sizeof(uint32_t)), "output allocation");
   UNGX_CUDA(ctx, ctx->out_dists.ensure(nk * sizeof(float)), "output allocation");
   st = run_generate(ctx, *problem, plan, ctx->out_ids.as<uint32_t>(), ctx->out_dists.as<float>(), ctx->stream, t);
   if (st)
      return st;
   // device -> host: whole rows of this shard's work
   const uint32_t k = problem->topk;
   UNGX_CUDA(ctx, cudaEventRecord(ctx->ev[6], ctx->stream), "event");
   if (problem->shard_count <= 1)
   {
      UNGX_CUDA(ctx,
                cudaMemcpyAsync(out_ids, ctx->out_ids.as<uint32_t>(), nk * sizeof(uint32_t), cudaMemcpyDeviceToHost,
                                ctx->stream),
                "output copy");
      if (out_dists)
         UNGX_CUDA(ctx,
                   cudaMemcpyAsync(out_dists, ctx->out_dists.as<float>(), nk * sizeof(float), cudaMemcpyDeviceToHost,
                                   ctx->stream),
                   "output copy");
      UNGX_CUDA(ctx, cudaEventRecord(ctx->ev[7], ctx->stream), "event");
      if ((st = wait_event(ctx, ctx->ev[7], "output copy")))
         return st;
   }
   else
   {
      // a shard's rows are scattered over the id space (one range per work item):
      // gather them into a compact device buffer, copy it back in one piece and
      // scatter the ranges on the host
      std::vector<ungx::RowRange> rr;
      for (const auto &it : plan.items)
         rr.push_back({it.row_begin, it.row_count});
      rr.insert(rr.end(), plan.empty_rows.begin(), plan.empty_rows.end());
      std::sort(rr.begin(), rr.end(), [](const ungx::RowRange &a, const ungx::RowRange &b) { return a.begin < b.begin; });
      std::vector<ungx::CopyRange> cr;
      uint32_t rows = 0;
      for (size_t i = 0; i < rr.size();)
      {
         uint32_t b = rr[i].begin, e = rr[i].begin + rr[i].count;
         size_t j = i + 1;
         while (j < rr.size() && rr[j].begin == e)
            e += rr[j++].count;
         cr.push_back({b, rows, e - b, 0});
         rows += e - b;
         i = j;
      }
      const size_t cnk = size_t(rows) * k;
      const size_t id_bytes = cnk * sizeof(uint32_t), d_bytes = out_dists ? cnk * sizeof(float) : 0;
      UNGX_CUDA(ctx, ctx->copy_ranges.ensure(cr.size() * sizeof(ungx::CopyRange)), "copy-range allocation");
      UNGX_CUDA(ctx, ctx->compact.ensure(id_bytes + d_bytes), "compact output allocation");
      UNGX_CUDA(ctx, ctx->host_stage.ensure(id_bytes + d_bytes), "pinned output staging");
      UNGX_CUDA(ctx,
                cudaMemcpyAsync(ctx->copy_ranges.p, cr.data(), cr.size() * sizeof(ungx::CopyRange),
                                cudaMemcpyHostToDevice, ctx->stream),
                "copy-range upload");
      uint32_t *c_ids = ctx->compact.as<uint32_t>();
      float *c_d = out_dists ? reinterpret_cast<float *>(ctx->compact.as<char>() + id_bytes) : nullptr;
      UNGX_CUDA(ctx,
                ungx::launch_gather_rows(ctx->copy_ranges.as<ungx::CopyRange>(), (uint32_t)cr.size(), k,
                                         ctx->out_ids.as<uint32_t>(), out_dists ? ctx->out_dists.as<float>() : nullptr,
                                         c_ids, c_d, ctx->stream),
                "row gather kernel");
      t.gpu_launches += cr.empty() ? 0 : 1;
      UNGX_CUDA(ctx, cudaMemcpyAsync(ctx->host_stage.p, ctx->compact.p, id_bytes + d_bytes, cudaMemcpyDeviceToHost,
                                     ctx->stream),
                "output copy");
      UNGX_CUDA(ctx, cudaEventRecord(ctx->ev[7], ctx->stream), "event");
      if ((st = wait_event(ctx, ctx->ev[7], "output copy")))
         return st;
      const uint32_t *h_ids = static_cast<const uint32_t *>(ctx->host_stage.p);
      const float *h_d = reinterpret_cast<const float *>(static_cast<const char *>(ctx->host_stage.p) + id_bytes);
      ungx::parallel_for((int64_t)cr.size(), 0, 64, [&](int64_t i) {
         const ungx::CopyRange &c = cr[i];
         std::memcpy(out_ids + size_t(c.src_row) * k, h_ids + size_t(c.dst_row) * k, size_t(c.count) * k * 4);
         if (out_dists)
            std::memcpy(out_dists + size_t(c.src_row) * k, h_d + size_t(c.dst_row) * k, size_t(c.count) * k * 4);
      });
   }
   float d2h = 0;
   cudaEventElapsedTime(&d2h, ctx->ev[6], ctx->ev[7]);
   t.gpu_d2h_ms = d2h;
   t.generate_ms = ms_since(t0);
   if (timing)
      *timing = t;
   return UNGX_OK;
}

int ungx_cross_edges_build(ungx_context *ctx, const float *vectors, const ungx_cross_edge_problem *problem,
                           uint32_t *out_ids, float *out_dists, ungx_cross_edge_timing *timing)
{
   if (!ctx || !problem)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "null argument");
   const auto t0 = std::chrono::steady_clock::now();
   UNGX_CUDA(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
   // the capacity path when the resident footprint exceeds the device budget
   const ungx_cross_edge_problem &P = *problem;
   auto passes = [&](uint64_t budget) -> int {
      ungx_cross_edge_timing t{};
      std::string err;
      ungx::Plan probe; // validates the problem (sizes, ranges, group ids) before any pass
      int st = ungx::build_plan(P, probe, err);
      if (st)
         return fail(ctx, st, "invalid problem: " + err);
      if (!vectors || !out_ids)
         return fail(ctx, UNGX_ERR_INVALID_ARG, "null vectors or output");
      st = run_passes(ctx, vectors, P, budget, out_ids, out_dists, t);
      ctx->have_vectors = false;
      t.generate_ms = ms_since(t0);
      if (timing)
         *timing = t;
      return st;
   };
   if (P.shard_count <= 1 && P.num_points && P.dim && P.topk)
   {
      const uint64_t need = ungx_resident_bytes(P.num_points, P.dim, P.topk);
      const uint64_t budget = device_budget(ctx);
      if (need > budget)
         return passes(budget);
   }
   // the host plans while the vectors go to the device (planning reads only the problem)
   int pst = 0;
   std::string perr;
   double pms = 0;
   std::thread planner([&] {
      const auto a = std::chrono::steady_clock::now();
      bool reused = false;
      pst = ensure_plan(ctx, *problem, reused, perr);
      pms = ms_since(a);
   });
   int st = ungx_prepare_base_vectors(ctx, vectors, problem->num_points, problem->dim, 0);
   planner.join();
   auto retry_on_oom = [&]() -> int {
      // a resident attempt that ran out of device memory: free the context's large
      // buffers and take the capacity path with what is free now
      ctx->preplanned = nullptr;
      cudaStreamSynchronize(ctx->stream);
      cudaGetLastError();
      for (DevBuf *b : {&ctx->X_owned, &ctx->Xh, &ctx->xnorm, &ctx->cand_key, &ctx->cand_col, &ctx->out_ids,
                        &ctx->out_dists, &ctx->fb_rows, &ctx->fb_items})
         b->release();
      ctx->have_vectors = false;
      return passes(device_budget(ctx));
   };
   if (st == UNGX_ERR_OOM && P.shard_count <= 1)
      return retry_on_oom();
   if (st)
      return st;
   ctx->preplanned = problem;
   ctx->preplan_status = pst;
   ctx->preplan_err = perr;
   ctx->preplan_ms = pms;
   const double prep = ms_since(t0);
   ungx_cross_edge_timing t{};
   st = ungx_cross_edges_generate(ctx, problem, out_ids, out_dists, &t);
   if (st == UNGX_ERR_OOM && P.shard_count <= 1)
      return retry_on_oom();
   t.passes = 1;
   // the device buffers stay allocated in the context for the next build
   ctx->have_vectors = false;
   t.prepare_ms = prep;
   t.generate_ms = ms_since(t0);
   if (timing)
      *timing = t;
   return st;
}

int ungx_additional_edges_build(ungx_context *ctx, const ungx_cross_edge_problem *problem, const uint32_t *d_cross_ids,
                                void *stream, ungx_additional_stats *stats)
{
   if (!ctx || !problem)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "null argument");
   if (!ctx->have_vectors)
      return fail(ctx, UNGX_ERR_STATE, "call ungx_prepare_base_vectors first");
   const uint32_t n = problem->num_points, k = problem->topk, G = problem->num_groups;
   if (n != ctx->n || problem->dim != ctx->d)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "problem n/d differ from the prepared base vectors");
   if (n && !d_cross_ids)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "null cross-edge ids");
   if (k == 0 || k > ungx::kExactMaxK)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "k must be 1 .. " + std::to_string(ungx::kExactMaxK));
   if (G && (!problem->group_ranges || !problem->lng_out_offsets))
      return fail(ctx, UNGX_ERR_INVALID_ARG, "null group ranges or LNG offsets");
   const auto t0 = std::chrono::steady_clock::now();
   UNGX_CUDA(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
   const uint32_t *R = problem->group_ranges;
   const uint64_t *OO = problem->lng_out_offsets;
   const uint64_t nnz = G ? OO[G + 1] : 0;
   if (nnz && !problem->lng_out_ids)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "null LNG out ids");
   for (uint32_t g = 1; g <= G; ++g)
      if (R[2 * g] > R[2 * g + 1] || R[2 * g + 1] > n)
         return fail(ctx, UNGX_ERR_INVALID_ARG, "group range outside 0..num_points");
   for (uint64_t e = 0; e < nnz; ++e)
      if (problem->lng_out_ids[e] == 0 || problem->lng_out_ids[e] > G)
         return fail(ctx, UNGX_ERR_INVALID_ARG, "lng_out_ids holds a group id outside 1..G");
   // the caller's cross-edge output is complete before this context's stream reads it
   cudaStream_t us = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
   if (us != ctx->stream)
   {
      UNGX_CUDA(ctx, cudaEventRecord(ctx->ev[9], us), "event");
      UNGX_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, ctx->ev[9], 0), "stream wait");
   }
   cudaStream_t s = ctx->stream;
   // 1. which LNG edges do the cross edges reach
   auto up = [&](DevBuf &b, const void *src, size_t bytes, const char *what) -> int {
      UNGX_CUDA(ctx, b.ensure(std::max<size_t>(bytes, 8)), what);
      if (bytes)
         UNGX_CUDA(ctx, cudaMemcpyAsync(b.p, src, bytes, cudaMemcpyHostToDevice, s), what);
      return UNGX_OK;
   };
   int st;
   if ((st = up(ctx->g_ranges, R, 2 * (size_t(G) + 1) * sizeof(uint32_t), "group ranges")) ||
       (st = up(ctx->g_out_off, OO, (G ? size_t(G) + 2 : 0) * sizeof(uint64_t), "LNG upload")) ||
       (st = up(ctx->g_out_ids, problem->lng_out_ids, nnz * sizeof(uint32_t), "LNG upload")))
      return st;
   UNGX_CUDA(ctx, ctx->group_of.ensure(size_t(std::max(n, 1u)) * sizeof(uint32_t)), "group map");
   UNGX_CUDA(ctx, ctx->reach.ensure(std::max<uint64_t>(nnz, 1)), "edge flags");
   UNGX_CUDA(ctx, cudaMemsetAsync(ctx->reach.p, 0, std::max<uint64_t>(nnz, 1), s), "edge flags");
   UNGX_CUDA(ctx, ungx::launch_group_of(ctx->g_ranges.as<uint32_t>(), G, n, ctx->group_of.as<uint32_t>(), s),
             "group map kernel");
   if (G)
      UNGX_CUDA(ctx,
                ungx::launch_mark_reached(d_cross_ids, n, k, ctx->group_of.as<uint32_t>(), G,
                                          ctx->g_out_off.as<uint64_t>(), ctx->g_out_ids.as<uint32_t>(),
                                          ctx->reach.as<uint8_t>(), s),
                "edge marking kernel");
   // 2. the reference's loop over missing edges, as (vector, target) queries: each
   //    vector of f adds m = min(|f'|, k/2) edges, until k were added (|f| caps it);
   //    queries numbered in the reference's order by a scan over the edges
   const uint32_t kh = k / 2;
   UNGX_CUDA(ctx, ctx->add_qoff.ensure((nnz + 1) * sizeof(uint64_t)), "query offsets");
   UNGX_CUDA(ctx, ctx->add_stats.ensure(4 * sizeof(unsigned long long)), "counters");
   UNGX_CUDA(ctx, cudaMemsetAsync(ctx->add_qoff.p, 0, (nnz + 1) * sizeof(uint64_t), s), "query offsets");
   UNGX_CUDA(ctx, cudaMemsetAsync(ctx->add_stats.p, 0, 4 * sizeof(unsigned long long), s), "counters");
   UNGX_CUDA(ctx, ctx->scan_scratch.ensure(ungx::csr_scan_scratch_bytes((uint32_t)std::max<uint64_t>(nnz + 1, n + 1))),
             "scan scratch");
   uint64_t *qoff = ctx->add_qoff.as<uint64_t>();
   unsigned long long *cnt = ctx->add_stats.as<unsigned long long>();
   UNGX_CUDA(ctx,
             ungx::launch_add_edge_queries(ctx->g_ranges.as<uint32_t>(), G, ctx->g_out_off.as<uint64_t>(),
                                           ctx->g_out_ids.as<uint32_t>(), ctx->reach.as<uint8_t>(), k, qoff, cnt, s),
             "query count kernel");
   UNGX_CUDA(ctx, ungx::launch_exclusive_scan_u64(qoff, (uint32_t)(nnz + 1), ctx->scan_scratch.p, s), "query scan");
   UNGX_CUDA(ctx, cudaMemcpyAsync(cnt + 2, qoff + nnz, sizeof(uint64_t), cudaMemcpyDeviceToDevice, s), "query count");
   unsigned long long hc[3] = {0, 0, 0};
   UNGX_CUDA(ctx, cudaMemcpyAsync(hc, cnt, sizeof(hc), cudaMemcpyDeviceToHost, s), "query count");
   UNGX_CUDA(ctx, cudaEventRecord(ctx->ev[6], s), "event");
   if ((st = wait_event(ctx, ctx->ev[6], "query count")))
      return st;
   ungx_additional_stats sx{};
   sx.missing_group_edges = hc[0];
   sx.query_vectors = hc[1];
   if (hc[2] > UINT32_MAX)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "more than 2^32 additional-edge queries");
   const uint32_t nq = (uint32_t)hc[2];
   UNGX_CUDA(ctx, ctx->scan_scratch.ensure(ungx::csr_scan_scratch_bytes(std::max<uint32_t>(nq + 1u, n + 1u))),
             "scan scratch");
   // 3. exact top-(k/2) of every query, in the reference's distance and order
   UNGX_CUDA(ctx, ctx->add_items.ensure(std::max<uint64_t>(nnz, 1) * sizeof(ungx::WorkItem)), "query plan");
   UNGX_CUDA(ctx, ctx->add_segs.ensure(std::max<uint64_t>(nnz, 1) * sizeof(ungx::Segment)), "query plan");
   UNGX_CUDA(ctx, ctx->add_rows.ensure(size_t(std::max(nq, 1u)) * sizeof(uint32_t)), "query plan");
   UNGX_CUDA(ctx, ctx->add_row_items.ensure(size_t(std::max(nq, 1u)) * sizeof(uint32_t)), "query plan");
   UNGX_CUDA(ctx, ctx->add_pos.ensure(size_t(std::max(nq, 1u)) * sizeof(uint32_t)), "query plan");
   const size_t cap = size_t(std::max(nq, 1u)) * std::max(kh, 1u); // entries at most
   UNGX_CUDA(ctx, ctx->add_res.ensure(cap * sizeof(uint32_t)), "query results");
   UNGX_CUDA(ctx, ctx->add_loff.ensure((size_t(nq) + 1) * sizeof(uint64_t)), "edge offsets");
   UNGX_CUDA(ctx, ctx->add_from.ensure(cap * sizeof(uint32_t)), "edge list");
   UNGX_CUDA(ctx, ctx->add_to.ensure(cap * sizeof(uint32_t)), "edge list");
   UNGX_CUDA(ctx, ctx->add_off.ensure((size_t(n) + 1) * sizeof(uint64_t)), "edge offsets");
   UNGX_CUDA(ctx, ctx->add_cols.ensure(cap * sizeof(uint32_t)), "edge columns");
   UNGX_CUDA(ctx, cudaMemsetAsync(ctx->add_loff.p, 0, sizeof(uint64_t), s), "edge offsets");
   if (nq && kh)
   {
      UNGX_CUDA(ctx,
                ungx::launch_add_query_fill(ctx->g_ranges.as<uint32_t>(), G, ctx->g_out_off.as<uint64_t>(),
                                            ctx->g_out_ids.as<uint32_t>(), qoff, ctx->add_items.as<ungx::WorkItem>(),
                                            ctx->add_segs.as<ungx::Segment>(), ctx->add_rows.as<uint32_t>(),
                                            ctx->add_row_items.as<uint32_t>(), ctx->add_pos.as<uint32_t>(), s),
                "query fill kernel");
      ungx::ExactParams ep{};
      ep.items = ctx->add_items.as<ungx::WorkItem>();
      ep.segs = ctx->add_segs.as<ungx::Segment>();
      ep.X = ctx->X;
      ep.d = ctx->d;
      ep.k = kh;
      ep.rows = ctx->add_rows.as<uint32_t>();
      ep.row_items = ctx->add_row_items.as<uint32_t>();
      ep.count_host = nq;
      ep.out_ids = ctx->add_res.as<uint32_t>();
      ep.out_pos = ctx->add_pos.as<uint32_t>();
      ep.warp_per_row = 1; // a query scans one target group
      UNGX_CUDA(ctx, ungx::launch_exact(ep, (uint32_t)ctx->num_sms * 16, s), "additional-edge kernel");
      // 4. (from, to) in the reference's order, and the same edges per point
      UNGX_CUDA(ctx,
                ungx::launch_add_list(ctx->add_res.as<uint32_t>(), ctx->add_rows.as<uint32_t>(), nq, kh,
                                      ctx->add_loff.as<uint64_t>(), ctx->add_from.as<uint32_t>(),
                                      ctx->add_to.as<uint32_t>(), ctx->scan_scratch.p, s),
                "edge list kernel");
   }
   UNGX_CUDA(ctx,
             ungx::launch_add_points(ctx->g_ranges.as<uint32_t>(), nq && kh ? G : 0u, n, k,
                                     ctx->g_out_off.as<uint64_t>(), qoff, ctx->add_loff.as<uint64_t>(),
                                     ctx->add_to.as<uint32_t>(), ctx->add_off.as<uint64_t>(),
                                     ctx->add_cols.as<uint32_t>(), ctx->scan_scratch.p, s),
             "per-point edge kernel");
   uint64_t edges = 0;
   UNGX_CUDA(ctx, cudaMemcpyAsync(&edges, ctx->add_loff.as<uint64_t>() + nq, sizeof(uint64_t), cudaMemcpyDeviceToHost, s),
             "edge count");
   UNGX_CUDA(ctx, cudaEventRecord(ctx->ev[6], s), "event");
   if ((st = wait_event(ctx, ctx->ev[6], "additional edges")))
      return st;
   ctx->add_n = n;
   ctx->add_edges = edges;
   sx.edges = edges;
   sx.ms = ms_since(t0);
   if (stats)
      *stats = sx;
   return UNGX_OK;
}

int ungx_additional_edges_copy(const ungx_context *ctx, uint32_t *from_ids, uint32_t *to_ids, uint64_t *point_offsets,
                               uint32_t *point_cols)
{
   if (!ctx)
      return UNGX_ERR_INVALID_ARG;
   if (cudaSetDevice(ctx->device) != cudaSuccess)
      return UNGX_ERR_CUDA;
   const size_t m = ctx->add_edges;
   const struct
   {
      void *dst;
      const DevBuf *src;
      size_t bytes;
   } parts[4] = {{from_ids, &ctx->add_from, m * sizeof(uint32_t)},
                 {to_ids, &ctx->add_to, m * sizeof(uint32_t)},
                 {point_offsets, &ctx->add_off, ctx->add_n ? (size_t(ctx->add_n) + 1) * sizeof(uint64_t) : 0},
                 {point_cols, &ctx->add_cols, m * sizeof(uint32_t)}};
   for (const auto &pt : parts)
      if (pt.dst && pt.bytes && cudaMemcpy(pt.dst, pt.src->p, pt.bytes, cudaMemcpyDeviceToHost) != cudaSuccess)
      {
         ungx::set_global_error("ungx_additional_edges_copy: device to host copy failed");
         return UNGX_ERR_CUDA;
      }
   return UNGX_OK;
}

int ungx_graph_csr_device(ungx_context *ctx, uint32_t num_points, uint32_t topk, const uint64_t *d_intra_offsets,
                          const uint32_t *d_intra_cols, const uint32_t *d_cross_ids, int with_additional,
                          uint64_t *d_offsets, uint32_t *d_cols, uint64_t cols_capacity, uint64_t *num_cols,
                          void *stream)
{
   if (!ctx || !d_offsets || !num_cols)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "null argument");
   if (d_intra_offsets && !d_intra_cols)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "intra offsets without columns");
   if (d_cross_ids && topk == 0)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "cross edges with topk = 0");
   if (with_additional && ctx->add_n != num_points)
      return fail(ctx, UNGX_ERR_STATE, "no additional edges built for this num_points");
   UNGX_CUDA(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
   cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
   const uint64_t *add_off = with_additional ? ctx->add_off.as<uint64_t>() : nullptr;
   const uint32_t *add_cols = with_additional ? ctx->add_cols.as<uint32_t>() : nullptr;
   UNGX_CUDA(ctx, ctx->scan_scratch.ensure(ungx::csr_scan_scratch_bytes(num_points)), "scan scratch");
   UNGX_CUDA(ctx, ungx::launch_graph_degrees(num_points, topk, d_intra_offsets, d_cross_ids, add_off, d_offsets, s),
             "degree kernel");
   UNGX_CUDA(ctx, ungx::launch_exclusive_scan_u64(d_offsets, num_points + 1, ctx->scan_scratch.p, s), "scan kernels");
   uint64_t total = 0;
   UNGX_CUDA(ctx, cudaMemcpyAsync(ctx->h_counters, d_offsets + num_points, sizeof(uint64_t), cudaMemcpyDeviceToHost, s),
             "total");
   UNGX_CUDA(ctx, cudaEventRecord(ctx->ev[6], s), "event");
   int st;
   if ((st = wait_event(ctx, ctx->ev[6], "graph degrees")))
      return st;
   std::memcpy(&total, ctx->h_counters, sizeof(uint64_t));
   *num_cols = total;
   if (total > cols_capacity || (total && !d_cols))
      return fail(ctx, UNGX_ERR_INVALID_ARG,
                  "graph needs " + std::to_string(total) + " columns, capacity " + std::to_string(cols_capacity));
   UNGX_CUDA(ctx,
             ungx::launch_graph_fill(num_points, topk, d_intra_offsets, d_intra_cols, d_cross_ids, add_off, add_cols,
                                     d_offsets, d_cols, s),
             "fill kernel");
   UNGX_CUDA(ctx, cudaEventRecord(ctx->ev[6], s), "event");
   return wait_event(ctx, ctx->ev[6], "graph emission");
}

int ungx_comm_id_create(ungx_comm_id *id)
{
   static_assert(sizeof(ungx_comm_id) == sizeof(ncclUniqueId), "ungx_comm_id holds an ncclUniqueId");
   if (!id)
      return fail(nullptr, UNGX_ERR_INVALID_ARG, "ungx_comm_id_create: null id");
   std::string err;
   const ungx::NcclApi *api = ungx::nccl_api(err);
   if (!api)
      return fail(nullptr, UNGX_ERR_STATE, err);
   ncclUniqueId u;
   const ncclResult_t r = api->GetUniqueId(&u);
   if (r != ncclSuccess)
      return fail(nullptr, UNGX_ERR_CUDA, std::string("ncclGetUniqueId: ") + api->GetErrorString(r));
   std::memcpy(id, &u, sizeof(u));
   return UNGX_OK;
}

int ungx_comm_init(ungx_context *ctx, const ungx_comm_id *id, int world_size, int rank)
{
   if (!ctx || !id)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "ungx_comm_init: null argument");
   if (world_size < 1 || rank < 0 || rank >= world_size)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "ungx_comm_init: rank must be in 0 .. world_size-1");
   std::string err;
   const ungx::NcclApi *api = ungx::nccl_api(err);
   if (!api)
      return fail(ctx, UNGX_ERR_STATE, err);
   ungx_comm_destroy(ctx);
   UNGX_CUDA(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
   ncclUniqueId u;
   std::memcpy(&u, id, sizeof(u));
   ncclComm_t comm = nullptr;
   const ncclResult_t r = api->CommInitRank(&comm, world_size, u, rank);
   if (r != ncclSuccess)
      return fail(ctx, UNGX_ERR_CUDA, std::string("ncclCommInitRank: ") + api->GetErrorString(r));
   ctx->nccl = api;
   ctx->comm = comm;
   ctx->world = world_size;
   ctx->rank = rank;
   return UNGX_OK;
}

int ungx_comm_destroy(ungx_context *ctx)
{
   if (!ctx)
      return UNGX_ERR_INVALID_ARG;
   if (ctx->comm)
   {
      cudaSetDevice(ctx->device);
      ctx->nccl->CommDestroy(ctx->comm);
   }
   ctx->comm = nullptr;
   ctx->world = 1;
   ctx->rank = 0;
   return UNGX_OK;
}

int ungx_dist_slice(uint32_t num_points, uint32_t world_size, uint32_t rank, uint32_t *first, uint32_t *count)
{
   if (!first || !count || world_size == 0 || rank >= world_size)
      return fail(nullptr, UNGX_ERR_INVALID_ARG, "ungx_dist_slice: bad argument");
   const uint64_t per = (uint64_t(num_points) + world_size - 1) / world_size;
   const uint64_t a = std::min<uint64_t>(num_points, per * rank);
   *first = uint32_t(a);
   *count = uint32_t(std::min<uint64_t>(per, num_points - a));
   return UNGX_OK;
}

int ungx_cross_edges_build_distributed(ungx_context *ctx, const float *vectors, uint32_t flags,
                                       const ungx_cross_edge_problem *problem, uint32_t *out_ids, float *out_dists,
                                       ungx_dist_timing *timing)
{
   if (!ctx || !problem)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "null argument");
   if (flags & ~uint32_t(UNGX_DIST_DEVICE_VECTORS | UNGX_DIST_DEVICE_OUTPUT))
      return fail(ctx, UNGX_ERR_INVALID_ARG, "unknown flag");
   const int world = ctx->comm ? ctx->world : 1, rank = ctx->comm ? ctx->rank : 0;
   const uint32_t n = problem->num_points, d = problem->dim, k = problem->topk;
   if (n == 0 || d == 0 || k == 0)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "empty problem");
   uint32_t first = 0, cnt = 0;
   ungx_dist_slice(n, uint32_t(world), uint32_t(rank), &first, &cnt);
   if (!vectors && ((flags & UNGX_DIST_DEVICE_VECTORS) || cnt))
      return fail(ctx, UNGX_ERR_INVALID_ARG, "null vectors");
   if (rank == 0 && !out_ids)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "rank 0 needs out_ids");
   UNGX_CUDA(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
   const auto t0 = std::chrono::steady_clock::now();
   ungx_dist_timing T{};
   T.world_size = uint32_t(world);
   T.rank = uint32_t(rank);
   ungx_cross_edge_problem pr = *problem;
   pr.shard_rank = uint32_t(rank);
   pr.shard_count = uint32_t(world);
   cudaStream_t s = ctx->stream;
   cudaEvent_t *E = ctx->dev_ev;
   // plan on a host thread (or find the previous one reusable) while the vectors go up
   int pst = 0;
   bool reused = false;
   std::string perr;
   double pms = 0;
   std::thread planner([&] {
      const auto a = std::chrono::steady_clock::now();
      pst = ensure_plan(ctx, pr, reused, perr);
      pms = ms_since(a);
   });
   auto join_fail = [&](int code) {
      planner.join();
      return code;
   };
   const float *X = vectors;
   if (cudaEventRecord(E[0], s) != cudaSuccess)
      return join_fail(fail(ctx, UNGX_ERR_CUDA, "event"));
   if (!(flags & UNGX_DIST_DEVICE_VECTORS))
   {
      // this rank's slice into its place, then every slice to every rank over NVLink
      const size_t per = (size_t(n) + world - 1) / world;
      cudaError_t e = ctx->X_owned.ensure(per * world * d * sizeof(float));
      if (e != cudaSuccess)
         return join_fail(cuda_fail(ctx, e, "vector allocation"));
      float *Xo = ctx->X_owned.as<float>();
      if (cnt)
      {
         const int st = upload_vectors(ctx, Xo + size_t(first) * d, vectors, size_t(cnt) * d * sizeof(float));
         if (st)
            return join_fail(st);
      }
      cudaEventRecord(E[1], s);
      if (world > 1)
      {
         const ncclResult_t r = ctx->nccl->AllGather(Xo + size_t(rank) * per * d, Xo, per * d, ncclFloat32, ctx->comm, s);
         if (r != ncclSuccess)
            return join_fail(fail(ctx, UNGX_ERR_CUDA, std::string("ncclAllGather: ") + ctx->nccl->GetErrorString(r)));
      }
      X = Xo;
   }
   else
      cudaEventRecord(E[1], s);
   cudaEventRecord(E[2], s);
   int st = ungx_prepare_base_vectors(ctx, X, n, d, 1);
   if (st)
      return join_fail(st);
   cudaEventRecord(E[3], s);
   planner.join();
   if (pst)
      return fail(ctx, pst, "invalid problem: " + perr);
   T.plan_reused = reused ? 1u : 0u;
   T.cross.plan_ms = pms;
   T.cross.pairs = ctx->plan.pairs;
   // this rank's shard: straight into rank 0's device output when it has one
   const size_t nk = size_t(n) * k;
   const bool direct = rank == 0 && (flags & UNGX_DIST_DEVICE_OUTPUT);
   UNGX_CUDA(ctx, ctx->out_ids.ensure(nk * sizeof(uint32_t)), "output allocation");
   UNGX_CUDA(ctx, ctx->out_dists.ensure(nk * sizeof(float)), "output allocation");
   uint32_t *d_ids = direct ? out_ids : ctx->out_ids.as<uint32_t>();
   float *d_dists = direct && out_dists ? out_dists : ctx->out_dists.as<float>();
   if ((st = run_generate(ctx, pr, ctx->plan, d_ids, d_dists, s, T.cross)))
      return st;
   T.gpu_launches = T.cross.gpu_launches + 3; // + the operand kernels
   // every shard's rows to rank 0: [ids | dists] of a shard's rows in ascending row order
   UNGX_CUDA(ctx, cudaEventRecord(E[4], s), "event");
   if (!ctx->runs_valid)
   {
      ungx::shard_runs(pr, ctx->plan, ctx->runs, ctx->run_rows);
      std::vector<ungx::CopyRange> all;
      uint32_t base = 0;
      for (int r = 1; r < world; ++r)
      {
         for (ungx::CopyRange c : ctx->runs[r])
         {
            c.dst_row += base;
            all.push_back(c);
         }
         base += ctx->run_rows[r];
      }
      if ((st = upload(ctx, ctx->own_runs, ctx->runs[rank], "run upload")) || (st = upload(ctx, ctx->all_runs, all, "run upload")))
         return st;
      ctx->runs_valid = true;
   }
   T.shard_rows = ctx->run_rows[rank];
   T.shard_cost = ctx->plan.shard_load[rank];
   for (int r = 0; r < world; ++r)
   {
      T.shard_cost_max = std::max<uint64_t>(T.shard_cost_max, ctx->plan.shard_load[r]);
      T.shard_cost_total += ctx->plan.shard_load[r];
   }
   if (world > 1)
   {
      const ungx::NcclApi *api = ctx->nccl;
      ncclResult_t r = ncclSuccess;
      if (rank != 0)
      {
         const size_t rows = ctx->run_rows[rank];
         UNGX_CUDA(ctx, ctx->compact.ensure(std::max<size_t>(rows, 1) * k * 2 * sizeof(uint32_t)), "compact output");
         uint32_t *c_ids = ctx->compact.as<uint32_t>();
         float *c_d = reinterpret_cast<float *>(c_ids + rows * k);
         UNGX_CUDA(ctx,
                   ungx::launch_gather_rows(ctx->own_runs.as<ungx::CopyRange>(), uint32_t(ctx->runs[rank].size()), k,
                                            d_ids, d_dists, c_ids, c_d, s),
                   "row gather kernel");
         T.gpu_launches += ctx->runs[rank].empty() ? 0 : 1;
         if (rows)
         {
            r = api->GroupStart();
            if (r == ncclSuccess)
               r = api->Send(c_ids, rows * k, ncclUint32, 0, ctx->comm, s);
            if (r == ncclSuccess)
               r = api->Send(c_d, rows * k, ncclFloat32, 0, ctx->comm, s);
            const ncclResult_t r2 = api->GroupEnd();
            r = r == ncclSuccess ? r2 : r;
         }
      }
      else
      {
         size_t others = 0;
         for (int q = 1; q < world; ++q)
            others += ctx->run_rows[q];
         UNGX_CUDA(ctx, ctx->recv.ensure(std::max<size_t>(others, 1) * k * 2 * sizeof(uint32_t)), "receive buffer");
         uint32_t *r_ids = ctx->recv.as<uint32_t>();
         float *r_d = reinterpret_cast<float *>(r_ids + others * k);
         r = api->GroupStart();
         size_t base = 0;
         for (int q = 1; q < world && r == ncclSuccess; ++q)
         {
            const size_t rows = ctx->run_rows[q];
            if (rows)
            {
               r = api->Recv(r_ids + base * k, rows * k, ncclUint32, q, ctx->comm, s);
               if (r == ncclSuccess)
                  r = api->Recv(r_d + base * k, rows * k, ncclFloat32, q, ctx->comm, s);
            }
            base += rows;
         }
         const ncclResult_t r2 = api->GroupEnd();
         r = r == ncclSuccess ? r2 : r;
         if (r == ncclSuccess)
         {
            size_t nall = 0;
            for (int q = 1; q < world; ++q)
               nall += ctx->runs[q].size();
            UNGX_CUDA(ctx,
                      ungx::launch_scatter_rows(ctx->all_runs.as<ungx::CopyRange>(), uint32_t(nall), k, r_ids, r_d,
                                                d_ids, d_dists, s),
                      "row scatter kernel");
            T.gpu_launches += nall ? 1 : 0;
         }
      }
      if (r != ncclSuccess)
         return fail(ctx, UNGX_ERR_CUDA, std::string("NCCL gather: ") + api->GetErrorString(r));
   }
   UNGX_CUDA(ctx, cudaEventRecord(E[5], s), "event");
   if (rank == 0)
   {
      if (!(flags & UNGX_DIST_DEVICE_OUTPUT))
      {
         UNGX_CUDA(ctx, cudaMemcpyAsync(out_ids, d_ids, nk * sizeof(uint32_t), cudaMemcpyDeviceToHost, s), "output copy");
         if (out_dists)
            UNGX_CUDA(ctx, cudaMemcpyAsync(out_dists, d_dists, nk * sizeof(float), cudaMemcpyDeviceToHost, s),
                      "output copy");
      }
      else if (out_dists && d_dists != out_dists)
         UNGX_CUDA(ctx, cudaMemcpyAsync(out_dists, d_dists, nk * sizeof(float), cudaMemcpyDeviceToDevice, s),
                   "output copy");
   }
   UNGX_CUDA(ctx, cudaEventRecord(E[6], s), "event");
   if ((st = wait_event(ctx, E[6], "distributed build")))
   {
      if (st == UNGX_ERR_TIMEOUT && ctx->comm)
      {
         // a peer that never arrives: release this rank's NCCL kernels
         ctx->nccl->CommAbort(ctx->comm);
         ctx->comm = nullptr;
         ctx->world = 1;
         ctx->rank = 0;
      }
      return st;
   }
   float a = 0;
   cudaEventElapsedTime(&a, E[0], E[1]);
   T.upload_ms = a;
   cudaEventElapsedTime(&a, E[1], E[2]);
   T.replicate_ms = a;
   cudaEventElapsedTime(&a, E[2], E[3]);
   T.prepare_ms = a;
   cudaEventElapsedTime(&a, E[4], E[5]);
   T.gather_ms = a;
   cudaEventElapsedTime(&a, E[5], E[6]);
   T.d2h_ms = a;
   T.total_ms = ms_since(t0);
   T.cross.generate_ms = T.total_ms;
   if (timing)
      *timing = T;
   return UNGX_OK;
}

int ungx_build_cross_group_edges(ungx_context *ctx, const float *vectors, const ungx_cross_edge_problem *problem,
                                 const uint64_t *intra_offsets, const uint32_t *intra_cols, uint32_t flags,
                                 uint32_t *out_ids, float *out_dists, ungx_cross_group_stats *stats)
{
   if (!ctx || !problem || !vectors)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "null argument");
   if (flags & ~uint32_t(UNGX_BUILD_ADDITIONAL | UNGX_BUILD_INTRA_LOCAL_IDS | UNGX_BUILD_VECTORS_ON_DEVICE))
      return fail(ctx, UNGX_ERR_INVALID_ARG, "unknown build flag");
   if (problem->shard_count > 1)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "ungx_build_cross_group_edges builds the whole graph: shard_count must be 1");
   if (intra_offsets && !intra_cols)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "intra offsets without columns");
   const uint32_t n = problem->num_points, k = problem->topk, G = problem->num_groups;
   if (n == 0 || k == 0)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "empty problem");
   if (intra_offsets)
   {
      if (intra_offsets[0] != 0)
         return fail(ctx, UNGX_ERR_INVALID_ARG, "intra_offsets[0] must be 0");
      for (uint32_t v = 0; v < n; ++v)
         if (intra_offsets[v + 1] < intra_offsets[v])
            return fail(ctx, UNGX_ERR_INVALID_ARG, "intra_offsets must not decrease");
   }
   const auto t0 = std::chrono::steady_clock::now();
   ungx_cross_group_stats sx{};
   // 1. cross edges: plan on a host thread while the vectors are uploaded and prepared
   int pst = 0;
   std::string perr;
   double pms = 0;
   std::thread planner([&] {
      const auto a = std::chrono::steady_clock::now();
      bool reused = false;
      pst = ensure_plan(ctx, *problem, reused, perr);
      pms = ms_since(a);
   });
   int st = ungx_prepare_base_vectors(ctx, vectors, n, problem->dim, (flags & UNGX_BUILD_VECTORS_ON_DEVICE) ? 1 : 0);
   planner.join();
   if (st)
      return st;
   if (pst)
      return fail(ctx, pst, "invalid problem: " + perr);
   ungx_cross_edge_timing &t = sx.cross;
   t.plan_ms = pms;
   t.pairs = ctx->plan.pairs;
   const size_t nk = size_t(n) * k;
   UNGX_CUDA(ctx, ctx->out_ids.ensure(nk * sizeof(uint32_t)), "output allocation");
   UNGX_CUDA(ctx, ctx->out_dists.ensure(nk * sizeof(float)), "output allocation");
   uint32_t *d_ids = ctx->out_ids.as<uint32_t>();
   if ((st = run_generate(ctx, *problem, ctx->plan, d_ids, ctx->out_dists.as<float>(), ctx->stream, t)))
      return st;
   t.generate_ms = ms_since(t0);
   // 2. additional edges from the device cross edges
   if (flags & UNGX_BUILD_ADDITIONAL)
   {
      if ((st = ungx_additional_edges_build(ctx, problem, d_ids, nullptr, &sx.additional)))
         return st;
   }
   else
      ctx->add_n = 0;
   // 3 + 4. intra-group edges (offset to global ids), cross, additional: one CSR
   const auto tm = std::chrono::steady_clock::now();
   cudaStream_t s = ctx->stream;
   const uint64_t intra_nnz = intra_offsets ? intra_offsets[n] : 0;
   const uint64_t *d_ioff = nullptr;
   const uint32_t *d_icols = nullptr, *d_group_of = nullptr, *d_ranges = nullptr;
   if (intra_offsets)
   {
      UNGX_CUDA(ctx, ctx->intra_off.ensure((size_t(n) + 1) * sizeof(uint64_t)), "intra offsets");
      UNGX_CUDA(ctx, ctx->intra_cols.ensure(std::max<uint64_t>(intra_nnz, 1) * sizeof(uint32_t)), "intra columns");
      UNGX_CUDA(ctx, cudaMemcpyAsync(ctx->intra_off.p, intra_offsets, (size_t(n) + 1) * sizeof(uint64_t),
                                     cudaMemcpyHostToDevice, s),
                "intra upload");
      if (intra_nnz)
         UNGX_CUDA(ctx, cudaMemcpyAsync(ctx->intra_cols.p, intra_cols, intra_nnz * sizeof(uint32_t),
                                        cudaMemcpyHostToDevice, s),
                   "intra upload");
      d_ioff = ctx->intra_off.as<uint64_t>();
      d_icols = ctx->intra_cols.as<uint32_t>();
      if (flags & UNGX_BUILD_INTRA_LOCAL_IDS)
      {
         UNGX_CUDA(ctx, ctx->g_ranges.ensure(2 * (size_t(G) + 1) * sizeof(uint32_t)), "group ranges");
         if (G)
            UNGX_CUDA(ctx, cudaMemcpyAsync(ctx->g_ranges.p, problem->group_ranges, 2 * (size_t(G) + 1) * sizeof(uint32_t),
                                           cudaMemcpyHostToDevice, s),
                      "group ranges");
         UNGX_CUDA(ctx, ctx->group_of.ensure(size_t(n) * sizeof(uint32_t)), "group map");
         UNGX_CUDA(ctx, ungx::launch_group_of(ctx->g_ranges.as<uint32_t>(), G, n, ctx->group_of.as<uint32_t>(), s),
                   "group map kernel");
         d_group_of = ctx->group_of.as<uint32_t>();
         d_ranges = ctx->g_ranges.as<uint32_t>();
      }
   }
   const bool with_add = (flags & UNGX_BUILD_ADDITIONAL) != 0;
   const uint64_t *add_off = with_add ? ctx->add_off.as<uint64_t>() : nullptr;
   const uint32_t *add_cols = with_add ? ctx->add_cols.as<uint32_t>() : nullptr;
   UNGX_CUDA(ctx, ctx->graph_off.ensure((size_t(n) + 1) * sizeof(uint64_t)), "graph offsets");
   uint64_t *g_off = ctx->graph_off.as<uint64_t>();
   UNGX_CUDA(ctx, ctx->scan_scratch.ensure(ungx::csr_scan_scratch_bytes(n)), "scan scratch");
   UNGX_CUDA(ctx, ungx::launch_graph_degrees(n, k, d_ioff, d_ids, add_off, g_off, s), "degree kernel");
   UNGX_CUDA(ctx, ungx::launch_exclusive_scan_u64(g_off, n + 1, ctx->scan_scratch.p, s), "scan kernels");
   UNGX_CUDA(ctx, cudaMemcpyAsync(ctx->h_counters, g_off + n, sizeof(uint64_t), cudaMemcpyDeviceToHost, s), "total");
   UNGX_CUDA(ctx, cudaEventRecord(ctx->ev[6], s), "event");
   if ((st = wait_event(ctx, ctx->ev[6], "graph degrees")))
      return st;
   uint64_t total = 0;
   std::memcpy(&total, ctx->h_counters, sizeof(uint64_t));
   UNGX_CUDA(ctx, ctx->graph_cols.ensure(std::max<uint64_t>(total, 1) * sizeof(uint32_t)), "graph columns");
   UNGX_CUDA(ctx,
             ungx::launch_graph_fill(n, k, d_ioff, d_icols, d_ids, add_off, add_cols, g_off,
                                     ctx->graph_cols.as<uint32_t>(), s, d_group_of, d_ranges),
             "fill kernel");
   // the flat cross edges, when asked for
   if (out_ids)
      UNGX_CUDA(ctx, cudaMemcpyAsync(out_ids, d_ids, nk * sizeof(uint32_t), cudaMemcpyDeviceToHost, s), "output copy");
   if (out_dists)
      UNGX_CUDA(ctx, cudaMemcpyAsync(out_dists, ctx->out_dists.p, nk * sizeof(float), cudaMemcpyDeviceToHost, s),
                "output copy");
   UNGX_CUDA(ctx, cudaEventRecord(ctx->ev[6], s), "event");
   if ((st = wait_event(ctx, ctx->ev[6], "graph emission")))
      return st;
   ctx->graph_n = n;
   ctx->graph_nnz = total;
   sx.num_cols = total;
   sx.cross_edges = total - intra_nnz - (with_add ? sx.additional.edges : 0);
   sx.merge_ms = ms_since(tm);
   sx.total_ms = ms_since(t0);
   if (stats)
      *stats = sx;
   return UNGX_OK;
}

int ungx_graph_copy(const ungx_context *ctx, uint64_t *offsets, uint32_t *cols)
{
   if (!ctx)
      return fail(nullptr, UNGX_ERR_INVALID_ARG, "null context");
   if (ctx->graph_n == 0)
      return fail(nullptr, UNGX_ERR_STATE, "ungx_graph_copy: no merged graph built in this context");
   if (cudaSetDevice(ctx->device) != cudaSuccess)
      return fail(nullptr, UNGX_ERR_CUDA, "ungx_graph_copy: cudaSetDevice failed");
   if (offsets && cudaMemcpy(offsets, ctx->graph_off.p, (size_t(ctx->graph_n) + 1) * sizeof(uint64_t),
                             cudaMemcpyDeviceToHost) != cudaSuccess)
      return fail(nullptr, UNGX_ERR_CUDA, "ungx_graph_copy: device to host copy failed");
   if (cols && ctx->graph_nnz &&
       cudaMemcpy(cols, ctx->graph_cols.p, ctx->graph_nnz * sizeof(uint32_t), cudaMemcpyDeviceToHost) != cudaSuccess)
      return fail(nullptr, UNGX_ERR_CUDA, "ungx_graph_copy: device to host copy failed");
   return UNGX_OK;
}

void ungx_exact_knn_default_config(uint32_t candidate_k, uint32_t final_degree, ungx_exact_knn_config *cfg)
{
   if (!cfg)
      return;
   ungx_exact_knn_config c{};
   c.candidate_k = candidate_k <= final_degree ? final_degree + 1 : candidate_k;
   c.final_degree = final_degree;
   c.head_keep = final_degree > 8 ? final_degree - 8 : final_degree;
   c.anchor_tail = 1;
   c.anchor_slots = 0;
   c.bidir_anchor = 0;
   c.graph_stride = final_degree + 1;
   c.route = UNGX_ROUTE_AUTO;
   *cfg = c;
}

uint64_t ungx_exact_knn_rejected_rows(const ungx_context *ctx) { return ctx ? ctx->knn_rejected : 0; }

void ungx_exact_knn_phase_ms(const ungx_context *ctx, double out[6])
{
   if (!out)
      return;
   for (int i = 0; i < 6; ++i)
      out[i] = ctx ? ctx->knn_phase_ms[i] : 0.0;
}

int ungx_exact_knn_graph_device(ungx_context *ctx, uint32_t num_groups, const uint32_t *group_ranges,
                                const ungx_exact_knn_config *cfg, uint32_t *d_graph, uint32_t *d_entry_points,
                                void *stream, double *kernel_ms)
{
   if (!ctx || !cfg || (num_groups && (!group_ranges || !d_graph)))
      return fail(ctx, UNGX_ERR_INVALID_ARG, "null argument");
   if (!ctx->have_vectors)
      return fail(ctx, UNGX_ERR_STATE, "call ungx_prepare_base_vectors first");
   if (ctx->d > ungx::kKnnMaxDim)
      return fail(ctx, UNGX_ERR_INVALID_ARG,
                  "exact kNN seeding supports dim <= " + std::to_string(ungx::kKnnMaxDim));
   if (cfg->graph_stride < cfg->final_degree + 1)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "graph_stride must be at least final_degree + 1");
   if (cfg->route != UNGX_ROUTE_AUTO && cfg->route != UNGX_ROUTE_TENSOR && cfg->route != UNGX_ROUTE_EXACT)
      return fail(ctx, UNGX_ERR_INVALID_ARG, "unknown kNN route");
   std::vector<uint32_t> ranges(group_ranges, group_ranges + 2 * size_t(num_groups));
   std::vector<uint64_t> base(num_groups);
   uint64_t rows = 0;
   for (uint32_t g = 0; g < num_groups; ++g)
   {
      if (ranges[2 * g] > ranges[2 * g + 1] || ranges[2 * g + 1] > ctx->n)
         return fail(ctx, UNGX_ERR_INVALID_ARG, "group range outside the base vectors");
      base[g] = rows;
      rows += ranges[2 * g + 1] - ranges[2 * g];
   }
   UNGX_CUDA(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
   if (num_groups == 0)
      return UNGX_OK;
   int st;
   if ((st = upload(ctx, ctx->knn_ranges, ranges, "kNN upload")) || (st = upload(ctx, ctx->knn_base, base, "kNN upload")))
      return st;
   cudaStream_t us = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
   cudaStream_t s = ctx->stream;
   if (us != s)
   {
      UNGX_CUDA(ctx, cudaEventRecord(ctx->ev[9], us), "event");
      UNGX_CUDA(ctx, cudaStreamWaitEvent(s, ctx->ev[9], 0), "stream wait");
   }
   ungx::KnnParams kp{};
   kp.X = ctx->X;
   kp.d = ctx->d;
   kp.dpad = (ctx->d + 3) / 4 * 4;
   kp.ranges = ctx->knn_ranges.as<uint32_t>();
   kp.base = ctx->knn_base.as<uint64_t>();
   kp.candidate_k = cfg->candidate_k;
   kp.final_degree = cfg->final_degree;
   kp.head_keep = cfg->head_keep;
   kp.anchor_tail = cfg->anchor_tail;
   kp.anchor_slots = cfg->anchor_slots;
   kp.bidir_anchor = cfg->bidir_anchor;
   kp.graph_stride = cfg->graph_stride;
   kp.graph = d_graph;
   kp.entry_points = d_entry_points;
   uint32_t max_n = 0;
   for (uint32_t g = 0; g < num_groups; ++g)
      max_n = std::max(max_n, ranges[2 * g + 1] - ranges[2 * g]);
   // limits of the two-phase path; the environment may lower them (tests reach the
   // fused kernel and several batches with small groups that way)
   auto env_u64 = [](const char *name, uint64_t def) {
      const char *v = std::getenv(name);
      return v && *v ? std::strtoull(v, nullptr, 10) : def;
   };
   const uint64_t dist_max_n = env_u64("UNGX_KNN_DIST_MAX_N", ungx::kKnnDistMaxN);
   const uint64_t batch_entries = std::max<uint64_t>(1, env_u64("UNGX_KNN_BATCH_ENTRIES", ungx::kKnnDistBatch));
   UNGX_CUDA(ctx, cudaEventRecord(ctx->ev[0], s), "event");
   ctx->knn_rejected = 0;
   for (double &v : ctx->knn_phase_ms)
      v = 0.0;
   const uint32_t route = cfg->route == UNGX_ROUTE_AUTO ? uint32_t(UNGX_ROUTE_TENSOR) : cfg->route;
   bool tensor_launched = false;
   if (route == UNGX_ROUTE_TENSOR)
   {
      if ((st = run_knn_tensor(ctx, ranges, num_groups, kp, s, tensor_launched)))
         return st;
   }
   else if (max_n > std::min<uint64_t>(dist_max_n, ungx::kKnnDistMaxN))
   {
      // fused kernel: one block per 64 rows of a group, every candidate of the group
      const size_t ntask = ungx::knn_task_count(ranges.data(), num_groups);
      std::vector<uint32_t> tasks(2 * std::max<size_t>(ntask, 1));
      ungx::knn_tasks(ranges.data(), num_groups, tasks.data());
      if ((st = upload(ctx, ctx->knn_tasks, tasks, "kNN upload")))
         return st;
      UNGX_CUDA(ctx, ungx::launch_exact_knn(kp, ctx->knn_tasks.as<uint32_t>(), (uint32_t)ntask, s),
                "kNN kernel launch");
   }
   else
   {
      // two-phase path, groups in batches of at most kKnnDistBatch matrix entries (a
      // batch restarts the matrix offsets at 0): the tiles on and above each group's
      // diagonal, then its rows in pieces of 32
      std::vector<uint64_t> dbase(num_groups, 0);
      std::vector<uint32_t> batch_end;
      uint64_t dmax = 0;
      for (uint32_t g0 = 0; g0 < num_groups;)
      {
         uint64_t used = 0;
         uint32_t g1 = g0;
         for (; g1 < num_groups; ++g1)
         {
            const uint64_t n = ranges[2 * g1 + 1] - ranges[2 * g1];
            if (g1 > g0 && used + n * n > batch_entries)
               break;
            dbase[g1] = used;
            used += n * n;
         }
         dmax = std::max(dmax, used);
         batch_end.push_back(g1);
         g0 = g1;
      }
      UNGX_CUDA(ctx, ctx->knn_dist.ensure(std::max<uint64_t>(dmax, 1) * sizeof(float)), "kNN distance matrix");
      if ((st = upload(ctx, ctx->knn_dbase, dbase, "kNN upload")))
         return st;
      kp.dist = ctx->knn_dist.as<float>();
      kp.dbase = ctx->knn_dbase.as<uint64_t>();
      std::vector<uint32_t> tiles, rowt;
      uint32_t g0 = 0;
      for (const uint32_t g1 : batch_end)
      {
         tiles.clear();
         rowt.clear();
         for (uint32_t g = g0; g < g1; ++g)
         {
            const uint32_t n = ranges[2 * g + 1] - ranges[2 * g];
            const uint32_t T = (n + 63) / 64;
            for (uint32_t bi = 0; bi < T; ++bi)
               for (uint32_t bj = bi; bj < T; ++bj)
                  tiles.insert(tiles.end(), {g, bi, bj});
            for (uint32_t r = 0; r < n; r += 32)
               rowt.insert(rowt.end(), {g, r});
         }
         // the previous batch's kernels are done with the task lists and the matrix
         UNGX_CUDA(ctx, cudaStreamSynchronize(s), "kNN batch");
         if ((st = upload(ctx, ctx->knn_tiles, tiles, "kNN upload")) ||
             (st = upload(ctx, ctx->knn_rows, rowt, "kNN upload")))
            return st;
         UNGX_CUDA(ctx,
                   ungx::launch_knn_two_phase(kp, ctx->knn_tiles.as<uint32_t>(), (uint32_t)(tiles.size() / 3),
                                              ctx->knn_rows.as<uint32_t>(), (uint32_t)(rowt.size() / 2), s),
                   "kNN kernel launch");
         g0 = g1;
      }
   }
   UNGX_CUDA(ctx, cudaEventRecord(ctx->ev[1], s), "event");
   if ((st = wait_event(ctx, ctx->ev[1], "exact kNN seeding")))
      return st;
   float ms = 0;
   cudaEventElapsedTime(&ms, ctx->ev[0], ctx->ev[1]);
   if (tensor_launched && (st = finish_knn_tensor(ctx, ctx->knn_rejected)))
      return st;
   ctx->knn_phase_ms[3] = ms;
   if (kernel_ms)
      *kernel_ms = ms;
   return UNGX_OK;
}

} // extern "C"
