/*
 * ungx.h -- C ABI of the B200 UNG cross-group edge builder.
 *
 * Drop-in for the cross-edge generation step of UNG index construction in
 * panjd123/FilterVectorCode_refactor.  Plain pointers and sizes only; every
 * buffer passed in is owned by the caller and is never freed by the library.
 * All functions return an int status (UNGX_OK == 0, negative on error) and leave
 * a message retrievable with ungx_last_error().
 *
 * Id spaces follow the reference: vectors are addressed by their REORDERED id
 * (groups contiguous, group 1 first), exactly as UniNavGraph sees them after
 * prepare_group_storages_graphs (UNG/codes/src/uni_nav_graph.cpp:148-169).
 * Groups are numbered 1..G; index 0 of every per-group array is unused.
 */
#ifndef UNGX_H
#define UNGX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
enum
{
   UNGX_OK = 0,
   UNGX_ERR_INVALID_ARG = -1,  /* bad size, null pointer, unsupported shape */
   UNGX_ERR_OOM = -2,          /* device or host allocation failed */
   UNGX_ERR_CUDA = -3,         /* CUDA runtime / driver error */
   UNGX_ERR_TIMEOUT = -4,      /* a bounded device wait ran out */
   UNGX_ERR_ABORTED = -5,      /* a kernel reported an internal consistency error */
   UNGX_ERR_NO_DEVICE = -6,    /* no usable sm_100 device */
   UNGX_ERR_STATE = -7         /* call order violated (e.g. no base vectors prepared) */
};

/* Writeback modes of the reference, CrossEdgeGpuWritebackMode
 * (UNG/codes/include/ung_cross_edge_config.h:17-22).  The C ABI always emits the
 * flat layout; the C++ adapter (ungx_ung_adapter.hpp) materialises the others. */
enum
{
   UNGX_WRITEBACK_SEARCH_QUEUE = 0,
   UNGX_WRITEBACK_ID_VECTOR = 1,
   UNGX_WRITEBACK_FLAT_ID = 2
};

/* Route selection for ungx_cross_edges_generate. */
enum
{
   UNGX_ROUTE_AUTO = 0,        /* tensor-core prefilter + exact rerank when k allows, else exact */
   UNGX_ROUTE_TENSOR = 1,      /* tcgen05 fp16 prefilter + certified exact fp32 rerank */
   UNGX_ROUTE_EXACT = 2        /* CUDA-core exact scan in the reference's summation order */
};

typedef struct ungx_context ungx_context;
typedef struct ungx_label_graph ungx_label_graph;

/* Mirrors CrossEdgeBuildTiming (UNG/codes/include/ung_cross_edge_result.h:15-28)
 * for the fields this step owns, plus the breakdown of the device work. */
typedef struct
{
   double generate_ms;   /* whole call, host wall clock */
   double gpu_h2d_ms;    /* host -> device copies (vectors, plan) */
   double gpu_kernel_ms; /* device time of the generate kernels (CUDA events) */
   double gpu_d2h_ms;    /* device -> host copies of ids / dists */
   double plan_ms;       /* host work-item planning */
   double prepare_ms;    /* centring / rounding / norm kernels */
   double tc_kernel_ms;  /* tensor-core prefilter kernel alone */
   double rerank_ms;     /* exact rerank + certificate of the candidates */
   double fallback_ms;   /* exact rescan of rows the certificate rejected */
   uint64_t pairs;       /* sum over LNG edges f->f' of |f|*|f'| (the reference's dim_ops / dim) */
   uint64_t rows_certified;
   uint64_t rows_fallback;
   uint32_t route_used;  /* UNGX_ROUTE_TENSOR or UNGX_ROUTE_EXACT */
   uint32_t gpu_launches;/* kernels this call launched */
   uint32_t passes;      /* 1: the whole problem resident; more: the capacity path's passes */
   uint32_t reserved;
} ungx_cross_edge_timing;

/* The inputs UniNavGraph::build_cross_edges_generate_gpu_optimized reads
 * (UNG/codes/include/uni_nav_graph.h:403-407, UNG/codes/src/uni_nav_graph_cross_edges.cpp:334-440). */
typedef struct
{
   uint32_t num_points;        /* n */
   uint32_t dim;               /* d */
   uint32_t topk;              /* k = _num_cross_edges */
   uint32_t num_groups;        /* G */
   const uint32_t *group_ranges;   /* [2*(G+1)]: group g owns rows [ranges[2g], ranges[2g+1]);
                                      the memory layout of std::vector<std::pair<IdxType,IdxType>>
                                      _group_id_to_range */
   const uint64_t *lng_out_offsets;/* [G+2]: out-neighbours (minimal supersets) of g are */
   const uint32_t *lng_out_ids;    /*        lng_out_ids[off[g] .. off[g+1]) */
   const uint8_t *skip_source_group;/* optional [G+1]: non-zero = do not emit cross edges for
                                      the group's vectors (special-block trivial roots,
                                      UNG/codes/src/gpu_gemm_topk.cu:399-412); may be NULL */
   uint32_t route;             /* UNGX_ROUTE_* */
   uint32_t shard_rank;        /* work-item shard this call computes (0 for one GPU) */
   uint32_t shard_count;       /* number of shards (1 for one GPU) */
} ungx_cross_edge_problem;

/* ---------------------------------------------------------------- context */
int ungx_context_create(int device, ungx_context **out);
int ungx_context_destroy(ungx_context *ctx);
const char *ungx_last_error(const ungx_context *ctx);
const char *ungx_status_string(int status);
/* Bounded-wait limit (milliseconds) for every host wait on device work. */
int ungx_set_timeout_ms(ungx_context *ctx, uint32_t timeout_ms);
/* Limit (nanoseconds, default 4e9) of each spin wait inside the tensor-core kernel
 * (pipeline barriers between its producer, MMA and epilogue warps).  A wait that
 * runs out makes the kernel stop issuing work, drain what is in flight, free its
 * tensor memory and report UNGX_ERR_TIMEOUT; the context stays usable. */
int ungx_set_device_wait_limit_ns(ungx_context *ctx, uint64_t limit_ns);
/* Device memory budget (bytes) of ungx_cross_edges_build; 0 (the default) = the free
 * device memory at the time of the call.  A problem above it takes the capacity path. */
int ungx_set_device_memory_limit(ungx_context *ctx, uint64_t bytes);
/* Device bytes ungx_cross_edges_build needs to hold a problem of n points resident
 * (the estimate it compares with the budget); the capacity path needs about
 * n*k*8 + 64 MiB plus two slices of this per-point size. */
uint64_t ungx_resident_bytes(uint32_t num_points, uint32_t dim, uint32_t topk);

/* Failure-detection test hook.  UNGX_INJECT_WITHHOLD_WORK makes the tensor-core
 * kernel's producer warp publish no work item, as if it had been lost: the MMA
 * and epilogue warps' bounded waits run out and the call returns
 * UNGX_ERR_TIMEOUT without faulting the device.  0 restores normal operation. */
enum
{
   UNGX_INJECT_NONE = 0,
   UNGX_INJECT_WITHHOLD_WORK = 1
};
int ungx_set_fault_injection(ungx_context *ctx, uint32_t flags);

/* ------------------------------------------ a4: resident base vectors + norms
 * Replaces gpu_prepare_all_vectors_on_device
 * (UNG/codes/src/gpu_cross_edge_resident_vectors.cuh:10-215): one upload of the
 * reordered n x d fp32 matrix, then the device builds the tensor-core operand
 * (centred, scaled by a power of two, rounded to fp16, zero-padded to a multiple of
 * 16 columns) and the row norms.  `vectors_on_device` != 0 means `vectors` is a device pointer that stays
 * valid until ungx_release_base_vectors (no copy is made of it). */
int ungx_prepare_base_vectors(ungx_context *ctx, const float *vectors, uint32_t num_points, uint32_t dim,
                              int vectors_on_device);
/* Replaces gpu_release_all_vectors_on_device. */
int ungx_release_base_vectors(ungx_context *ctx);

/* ------------------------------------- a6-a11: the cross-edge generate step
 * Replaces build_cross_edges_generate_gpu_optimized's device work
 * (UNG/codes/src/uni_nav_graph_cross_edges.cpp:334-440 and the GPU routes under it,
 * UNG/codes/src/gpu_gemm_topk.cu:377-970).  For every vector v of every group f
 * with out(f) non-empty, row v of the output receives the k nearest vectors (squared
 * L2, the reference's fp32 summation order) over the union of the groups in
 * out(f), sorted by (distance, id) ascending -- the content of the reference's
 * SearchQueue after the exact scan.  Slots past the number of candidates, and every
 * slot of a row whose group has no out-neighbour, hold id UINT32_MAX and distance
 * +inf (the FlatId writeback sentinel of UNG/codes/src/ung_cross_edge_output_writer.cpp:78-88).
 *
 * `out_ids` [n*k] and `out_dists` [n*k] (may be NULL) are HOST buffers.  With
 * shard_count > 1 only the rows of this shard's work items are written; the other
 * rows are left untouched. */
int ungx_cross_edges_generate(ungx_context *ctx, const ungx_cross_edge_problem *problem, uint32_t *out_ids,
                              float *out_dists, ungx_cross_edge_timing *timing);

/* Same, with DEVICE output buffers on the context's device.  `stream` is a
 * cudaStream_t (NULL = the context's own stream); the call returns after the
 * work completed (bounded wait). */
int ungx_cross_edges_generate_device(ungx_context *ctx, const ungx_cross_edge_problem *problem,
                                     uint32_t *d_out_ids, float *d_out_dists, void *stream,
                                     ungx_cross_edge_timing *timing);

/* One call = prepare + generate with host buffers: the whole step as the
 * reference's UniNavGraph calls it.  The device buffers stay allocated in the
 * context and are reused by the next call; ungx_release_base_vectors or
 * ungx_context_destroy frees them.
 *
 * Capacity path (the reference's X-side streaming, UNG/codes/src/uni_nav_graph_cross_edges.cpp:402-418,
 * UNG/codes/src/gpu_cross_edge_x_streaming.cuh:12-404): when the resident footprint
 * (base vectors, tensor-core operand, norms, candidate lists, outputs) exceeds the
 * context's device memory limit, or a resident attempt runs out of device memory, the
 * rows are cut into slices and the call runs one pass per (source slice, target slice)
 * holding two slices on the device; each pass's exact per-row top-k is merged into the
 * running top-k by (distance, id), so the rows equal the resident result.
 * timing->passes reports the number of passes (1 = resident). */
int ungx_cross_edges_build(ungx_context *ctx, const float *vectors, const ungx_cross_edge_problem *problem,
                           uint32_t *out_ids, float *out_dists, ungx_cross_edge_timing *timing);

/* The exact route without any device allocation.  No counterpart in the reference.
 * For callers that cannot call cudaMalloc when they need the cross edges: code
 * whose device memory belongs to another allocator (a framework's caching
 * allocator, a pool with a hard budget, where a foreign cudaMalloc would be
 * invisible to that allocator's accounting or could fail against its limit), or a
 * service that must not grow its device footprint once it is serving.  The caller
 * passes the reordered base vectors (`d_vectors`, device, n x d fp32) and the
 * device outputs (`d_out_ids` [n*k], `d_out_dists` [n*k] or NULL); the rows'
 * results are those of ungx_cross_edges_generate with UNGX_ROUTE_EXACT.  The work
 * plan lives in one 64 MiB __device__ array of the library, so the plan must fit:
 * about 8 bytes per source row plus 16 per work item and target segment; larger
 * problems return UNGX_ERR_INVALID_ARG naming the size.  The array is part of the
 * library's device module, which the CUDA runtime loads on a device at the first
 * use of the library there (with lazy module loading, at the first call of this
 * entry point or of any kernel of the library); from then on that device holds it
 * until the process exits.  A caller that needs a fixed footprint makes one call
 * (any small problem) at start-up on every device it will use.  That first call on
 * a device also fetches the array's device address (cudaGetSymbolAddress, with
 * the device current).  Runs on the current device and on `stream` (a
 * cudaStream_t, NULL = the legacy stream); returns after the work finished
 * (bounded wait of 10 minutes).  All calls share the array: calls that overlap on
 * the GPU race.  After UNGX_ERR_TIMEOUT the copies and kernels of that call may
 * still be using the array: synchronise `stream` before the next call.  Errors are
 * reported through ungx_last_error(NULL). */
int ungx_cross_edges_exact_noalloc(const ungx_cross_edge_problem *problem, const float *d_vectors,
                                   uint32_t *d_out_ids, float *d_out_dists, void *stream);

/* Rows (reordered vector ids) this shard owns, ascending; `*count` receives the
 * number.  `rows` may be NULL to query the count only. */
int ungx_shard_rows(const ungx_cross_edge_problem *problem, uint32_t *rows, uint64_t *count);

/* ---------------------------------------------- multi-GPU: one process per GPU
 * No counterpart in the reference, which builds on one GPU.  The LNG group pairs are
 * sharded across the GPUs of one box (each rank computes the work items of its shard,
 * longest first, over the whole problem), the base vectors are replicated over
 * NVLink, and rank 0 gathers every shard's rows with NCCL send / receive.  NCCL is
 * loaded at the first of these calls: $UNGX_NCCL_LIBRARY when set, else the
 * libnccl.so.2 already in the process, else libnccl.so.2 from the loader's path.  One
 * libnccl.so.2 lives in a process, so a framework that brings its own NCCL (PyTorch,
 * say) is loaded before that first call.
 *
 * Rank 0 makes an id with ungx_comm_id_create and hands its bytes to every rank by its
 * own means (a file, a socket, MPI, a framework's store); every rank then calls
 * ungx_comm_init on a context of its own GPU.  A context without a communicator runs
 * ungx_cross_edges_build_distributed as a world of one. */
typedef struct ungx_comm_id
{
   char internal[128];
} ungx_comm_id;

int ungx_comm_id_create(ungx_comm_id *id);
int ungx_comm_init(ungx_context *ctx, const ungx_comm_id *id, int world_size, int rank);
int ungx_comm_destroy(ungx_context *ctx);

/* The rows of the reordered base matrix that rank `rank` passes from host memory:
 * [*first, *first + *count), a balanced split of n rows over world_size ranks. */
int ungx_dist_slice(uint32_t num_points, uint32_t world_size, uint32_t rank, uint32_t *first, uint32_t *count);

enum
{
   UNGX_DIST_DEVICE_VECTORS = 1, /* `vectors`: the whole n x d matrix in this rank's device memory */
   UNGX_DIST_DEVICE_OUTPUT = 2   /* rank 0's out_ids / out_dists are device pointers on its GPU */
};

typedef struct ungx_dist_timing
{
   ungx_cross_edge_timing cross; /* this rank's generate step (plan_ms: planning or its reuse check) */
   double upload_ms;             /* host -> device copy of this rank's slice (device time) */
   double replicate_ms;          /* NCCL all-gather of the slices over NVLink */
   double prepare_ms;            /* the tensor-core operand and norms */
   double gather_ms;             /* compaction, NCCL send / receive, scatter on rank 0 */
   double d2h_ms;                /* rank 0: the whole output to host memory */
   double total_ms;              /* the whole call (wall) */
   uint64_t shard_rows;          /* rows this rank computed */
   uint64_t shard_cost;          /* its shard's cost (the planner's padded target columns) */
   uint64_t shard_cost_max;      /* the largest shard cost over all ranks */
   uint64_t shard_cost_total;    /* the sum over ranks */
   uint32_t world_size, rank;
   uint32_t plan_reused;         /* 1: the plan of the previous call was reused (same problem arrays) */
   uint32_t gpu_launches;        /* kernels this call launched on this rank */
} ungx_dist_timing;

/* The cross-edge build over every rank of the context's communicator; every rank calls
 * it with the same problem (its shard fields are ignored).  `vectors`: this rank's
 * slice of the reordered rows (ungx_dist_slice) in host memory, or with
 * UNGX_DIST_DEVICE_VECTORS the whole matrix in device memory.  Rank 0 receives the
 * whole output in out_ids [n*k] (required) and out_dists [n*k] (may be NULL) -- host
 * buffers, or device buffers with UNGX_DIST_DEVICE_OUTPUT; the other ranks' outputs
 * are ignored.  The plan is reused across calls while the problem's arrays stay the
 * same.  A device wait that runs out aborts the communicator (UNGX_ERR_TIMEOUT); a
 * new ungx_comm_init is then needed. */
int ungx_cross_edges_build_distributed(ungx_context *ctx, const float *vectors, uint32_t flags,
                                       const ungx_cross_edge_problem *problem, uint32_t *out_ids, float *out_dists,
                                       ungx_dist_timing *timing);

/* ---------------------------------------------- a16: grouping + reorder + LNG
 * build_trie_and_divide_groups (UNG/codes/src/uni_nav_graph_label_graph.cpp:21-43),
 * the reorder of prepare_group_storages_graphs (UNG/codes/src/uni_nav_graph.cpp:148-169)
 * and the minimal-superset label navigating graph
 * (UNG/codes/src/uni_nav_graph_label_graph.cpp:103-206, 851-911).
 * Labels are CSR: vector i (original id) carries labels[label_offsets[i] .. label_offsets[i+1]),
 * in any order (they are sorted, as Storage::load_from_file does).  Group ids follow
 * the first appearance of each exact sorted label sequence. */
int ungx_label_graph_build(uint32_t num_points, const uint64_t *label_offsets, const uint32_t *labels,
                           int num_threads, ungx_label_graph **out);
int ungx_label_graph_destroy(ungx_label_graph *lg);
uint32_t ungx_label_graph_num_groups(const ungx_label_graph *lg);
uint64_t ungx_label_graph_num_edges(const ungx_label_graph *lg);
/* new_to_old [n]; group_ranges [2*(G+1)] as in ungx_cross_edge_problem. */
int ungx_label_graph_copy_groups(const ungx_label_graph *lg, uint32_t *new_to_old, uint32_t *group_ranges);
/* out-neighbours (ascending group id within a group): offsets [G+2], ids [num_edges]. */
int ungx_label_graph_copy_out_neighbors(const ungx_label_graph *lg, uint64_t *offsets, uint32_t *ids);
/* in-neighbours, ascending source id (uni_nav_graph_label_graph.cpp:889-906). */
int ungx_label_graph_copy_in_neighbors(const ungx_label_graph *lg, uint64_t *offsets, uint32_t *ids);
/* label set of each group as CSR: offsets [G+2], labels [offsets[G+1]]. */
uint64_t ungx_label_graph_num_set_labels(const ungx_label_graph *lg);
int ungx_label_graph_copy_label_sets(const ungx_label_graph *lg, uint64_t *offsets, uint32_t *labels);

/* ------------------------------------------- a14: CSR of the cross edges
 * CrossEdgeGraphMaterializationWriter::build_csr_adjacency
 * (UNG/codes/src/ung_cross_edge_output_writer.cpp:44-66) from the flat output:
 * row_offsets [n+1], col_indices [row_offsets[n]] (skip UINT32_MAX slots). */
int ungx_flat_to_csr(const uint32_t *flat_ids, uint32_t num_points, uint32_t topk, uint64_t *row_offsets,
                     uint32_t *col_indices);

/* ------------------------------------------- the graph in the reference's text format
 * ANNS::Graph::save (UNG/codes/include/graph.h:207-216), the <prefix>graph file of
 * UniNavGraph::save (UNG/codes/src/uni_nav_graph_io.cpp:383-386), from a host CSR:
 * for each point v, "v " then "c " for each column of row v in order, then '\n'.
 * Returns UNGX_ERR_INVALID_ARG for a null or non-monotone argument or a file error. */
int ungx_graph_save_text(const char *path, uint32_t num_points, const uint64_t *offsets, const uint32_t *cols);

/* ------------------------------------------- additional edges (exact variant)
 * Replaces UniNavGraph::build_cross_edges_generate_additional with
 * UngAdditionalEdgesImpl::CpuExactScan (UNG/codes/src/uni_nav_graph_cross_edges.cpp:442-596).
 * From a finished cross-edge output `d_cross_ids` (device, [n x k], UINT32_MAX = empty):
 * every LNG edge f -> f' that no cross edge of f's vectors reaches gets, from f's
 * vectors in ascending order, the first k/2 entries of each vector's exact top-k over
 * f' (reference distance, (distance, id) order) until k edges were added for that f'.
 * Uses the base vectors of ungx_prepare_base_vectors.  The edges stay in the context
 * (copy them with ungx_additional_edges_copy, or emit them with ungx_graph_csr_device). */
typedef struct ungx_additional_stats
{
   uint64_t missing_group_edges; /* LNG edges no cross edge realises */
   uint64_t query_vectors;       /* source vectors scanned for them (the reference's count) */
   uint64_t edges;               /* additional edges */
   double ms;                    /* wall time of the call */
} ungx_additional_stats;

int ungx_additional_edges_build(ungx_context *ctx, const ungx_cross_edge_problem *problem, const uint32_t *d_cross_ids,
                                void *stream, ungx_additional_stats *stats);

/* The last build's edges, host buffers, any of them NULL to skip:
 *   from_ids / to_ids [edges]: (from, to) pairs in the reference's materialised order
 *     (source group ascending; per group its LNG out-groups in order, vectors
 *     ascending, queue rank), the list append_materialized_additional_edges
 *     (UNG/codes/src/ung_cross_edge_output_writer.cpp:30-42) appends;
 *   point_offsets [n+1] / point_cols [edges]: the same edges per source point. */
int ungx_additional_edges_copy(const ungx_context *ctx, uint32_t *from_ids, uint32_t *to_ids, uint64_t *point_offsets,
                               uint32_t *point_cols);

/* ------------------------------------------- device emission of the whole graph
 * No single reference counterpart: the per-point adjacency the reference assembles on
 * the host (intra-group edges offset to global ids, UNG/codes/src/uni_nav_graph.cpp:285-297;
 * then cross edges in queue order and additional edges,
 * UNG/codes/src/ung_cross_edge_output_writer.cpp:17-42), emitted as CSR in device memory
 * for NeighborList64 / CSR consumers (UNG/include/graph.h:18-250).
 * Inputs, all device pointers, NULL to leave a part out: d_intra_offsets [n+1] +
 * d_intra_cols (global ids); d_cross_ids [n x k]; with_additional != 0 appends the
 * context's last additional edges.  Outputs: d_offsets [n+1]; d_cols with room for
 * cols_capacity ids.  *num_cols receives the total; when it exceeds cols_capacity the
 * call returns UNGX_ERR_INVALID_ARG and writes no column. */
int ungx_graph_csr_device(ungx_context *ctx, uint32_t num_points, uint32_t topk, const uint64_t *d_intra_offsets,
                          const uint32_t *d_intra_cols, const uint32_t *d_cross_ids, int with_additional,
                          uint64_t *d_offsets, uint32_t *d_cols, uint64_t cols_capacity, uint64_t *num_cols,
                          void *stream);

/* ------------------------------------------- a1: the whole cross-group edge step
 * UniNavGraph::build_cross_group_edges (UNG/codes/src/uni_nav_graph_cross_edges.cpp:613-913)
 * with the GPU generate route, the exact additional edges and the merge, in one call
 * whose intermediates stay in device memory:
 *   1. the cross edges (as ungx_cross_edges_build);
 *   2. with UNGX_BUILD_ADDITIONAL, the additional edges (as ungx_additional_edges_build,
 *      build_cross_edges_generate_additional with CpuExactScan, :442-596);
 *   3. add_offset_for_uni_nav_graph (UNG/codes/src/uni_nav_graph.cpp:285-297): with
 *      UNGX_BUILD_INTRA_LOCAL_IDS the intra-group columns are group-local ids and get the
 *      first row of the point's group added;
 *   4. merge_cross_edges_to_graph + merge_additional_edges_to_graph (:598-611,
 *      UNG/codes/src/ung_cross_edge_output_writer.cpp:17-42): per point, its intra-group
 *      edges, its cross edges nearest first, then its additional edges, as CSR.
 * `vectors`: the reordered n x d fp32 rows, host memory (device memory with
 * UNGX_BUILD_VECTORS_ON_DEVICE).  `intra_offsets` [n+1] / `intra_cols` (host, NULL = no
 * intra-group edges): the graph of each group.  `out_ids` / `out_dists` (host [n*k], each
 * may be NULL): the flat cross edges as ungx_cross_edges_generate writes them.  The
 * merged adjacency stays in the context: *num_cols in `stats` gives its size, and
 * ungx_graph_copy copies it out.  The base vectors stay prepared afterwards (for
 * ungx_exact_knn_graph_device, say) until ungx_release_base_vectors. */
enum
{
   UNGX_BUILD_ADDITIONAL = 1,
   UNGX_BUILD_INTRA_LOCAL_IDS = 2,
   UNGX_BUILD_VECTORS_ON_DEVICE = 4
};

typedef struct ungx_cross_group_stats
{
   ungx_cross_edge_timing cross;     /* the generate step */
   ungx_additional_stats additional; /* zero without UNGX_BUILD_ADDITIONAL */
   uint64_t cross_edges;             /* non-empty cross-edge slots */
   uint64_t num_cols;                /* columns of the merged adjacency */
   double merge_ms;                  /* intra upload + offset + CSR emission (wall) */
   double total_ms;                  /* the whole call (wall) */
} ungx_cross_group_stats;

int ungx_build_cross_group_edges(ungx_context *ctx, const float *vectors, const ungx_cross_edge_problem *problem,
                                 const uint64_t *intra_offsets, const uint32_t *intra_cols, uint32_t flags,
                                 uint32_t *out_ids, float *out_dists, ungx_cross_group_stats *stats);

/* The merged adjacency of the last ungx_build_cross_group_edges call, host buffers:
 * offsets [n+1], cols [num_cols]; either may be NULL. */
int ungx_graph_copy(const ungx_context *ctx, uint64_t *offsets, uint32_t *cols);

/* ------------------------------------------- a15: large-group exact kNN seeding
 * batched_exact_knn_graph_kernel with the defaults of make_fast_exact_batch_config
 * (UNG/codes/src/tagore_graph_builder.cu:650-795, UNG/codes/src/tagore_cuda_config.cpp:23-45),
 * the intra-group graph seed of the groups below UNG_FAST_GRNND_BATCH_EXACT_NX.
 * Each point of a group keeps its min(64, K - 1, n - 1) nearest other points of the
 * group (the reference's fp32 distance of its 128-thread kernel built with
 * --use_fast_math, strict-< insertion in ascending local id), then writes one row of
 * graph_stride uint32: [degree, local ids in head / ring-anchor / tail order, padding
 * with its own local id]. */
typedef struct ungx_exact_knn_config
{
   uint32_t candidate_k;  /* K (UNG_TAGORE_K, 64); raised to final_degree + 1 when not above it */
   uint32_t final_degree; /* degree of a row (the graph's max degree) */
   uint32_t head_keep;    /* nearest entries kept first */
   uint32_t anchor_tail;  /* 1: ring anchors fill the remaining slots */
   uint32_t anchor_slots; /* 0: all remaining slots */
   uint32_t bidir_anchor; /* 1: every second anchor walks backwards */
   uint32_t graph_stride; /* row length in uint32, at least final_degree + 1 */
   uint32_t route;        /* UNGX_ROUTE_TENSOR (AUTO): tcgen05 fp16 prefilter of each group's
                             self-join keeping 96 candidates per point, the reference's
                             distance for those, a certificate that no other point could
                             enter, the exact kernel (a warp per row) for the rows it
                             rejects;
                             UNGX_ROUTE_EXACT: the reference's distance for every pair */
} ungx_exact_knn_config;

/* The reference's defaults for K and a degree (environment overrides not read);
 * route UNGX_ROUTE_AUTO. */
void ungx_exact_knn_default_config(uint32_t candidate_k, uint32_t final_degree, ungx_exact_knn_config *cfg);
/* Rows of the last ungx_exact_knn_graph_device call (tensor route) whose certificate
 * failed, rewritten by the exact kernel. */
uint64_t ungx_exact_knn_rejected_rows(const ungx_context *ctx);
/* Device time (CUDA events, ms) of the last ungx_exact_knn_graph_device call: out[0] the
 * tensor route's prefilter kernel, out[1] its rerank and certificate, out[2] the exact
 * kernel for the rejected rows (all 0 on the exact route), out[3] the whole call,
 * out[4] from the call's start to the prefilter (plan, uploads, group norms), out[5]
 * from the rerank's end to the fallback's start (the rejected rows' task list). */
void ungx_exact_knn_phase_ms(const ungx_context *ctx, double out[6]);

/* Groups g = 0 .. num_groups-1 are rows [group_ranges[2g], group_ranges[2g+1]) of the
 * base vectors of ungx_prepare_base_vectors (any dim up to 352).  d_graph (device):
 * one row per point, groups in the given order; d_entry_points (device, may be NULL):
 * 0 per group, as the reference writes.  *kernel_ms (may be NULL): device time. */
int ungx_exact_knn_graph_device(ungx_context *ctx, uint32_t num_groups, const uint32_t *group_ranges,
                                const ungx_exact_knn_config *cfg, uint32_t *d_graph, uint32_t *d_entry_points,
                                void *stream, double *kernel_ms);

#ifdef __cplusplus
}
#endif

#endif /* UNGX_H */
