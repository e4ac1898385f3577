// Device kernels of libungx and their host-side launch wrappers.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "ungx_internal.h"

namespace ungx
{

// fp16 operand rows (n x dp, dp a multiple of 16), 128-byte swizzled boxes of 64
// columns: A = 128 rows, B[i] = 16 (i + 1) rows (the narrowest box covering a tile).
constexpr uint32_t kTcBoxes = 12;
struct TcMaps
{
   CUtensorMap a;
   CUtensorMap b[kTcBoxes];
};

// Scale of the fp16 operand: it holds fp16(s * fl(x - mean)) with s = 2^e, chosen
// from the column ranges so that no element exceeds 2^15 in magnitude.
struct OperandScale
{
   float s;            // 2^e
   float neg2_inv_s2;  // -2 / s^2 (exact)
   float inv_s;        // 1 / s
   int exact_only;     // 1: the data range does not fit the fp16 operand; certify nothing
};

// Candidate lists per row: one per column third of a tile (three epilogue warps share
// a TMEM lane quarter).
constexpr uint32_t kTcLists = 3;

// Depth of each list for a merged candidate list of kp entries.  The rerank certifies
// against min(merged kp-th key, every list's last key), so a list may be shallower
// than kp: three lists of 12 lose nothing against three of 16 unless 12 of a row's
// nearest keys fall in one column third.  Shallower lists take fewer insertions, each
// cheaper, in the prefilter's epilogue (its bottleneck).  kp = 32 keeps full lists.
__host__ __device__ constexpr int tc_list_depth(int kp) { return kp == 16 ? 12 : kp; }

// Tensor-core prefilter: per source row, the tc_list_depth(KP) smallest keys
// ||x||^2 - 2 q.x of each column third, written to cand_key / cand_col
// [row][kTcLists][tc_list_depth(KP)].
struct TcParams
{
   const WorkItem *items;
   const Segment *segs;
   uint32_t num_items;
   uint32_t *item_counter;   // zeroed before launch
   const float *xnorm;       // ||fl(x - mean)||^2, fp32
   const OperandScale *scale;
   uint32_t dp;
   float *cand_key;
   uint32_t *cand_col;
   int *status;              // 0 or a UNGX_ERR_* code
   unsigned long long timeout_ns;
   uint32_t inject;          // UNGX_INJECT_* test hook
   uint32_t exclude_self;    // 1: a row never takes its own column (self-join of a group)
};

// Exact rerank + certificate of the candidates.
struct RerankParams
{
   const WorkItem *items;
   const Segment *segs;
   uint32_t item_offset;
   const float *X;           // original reordered vectors [n x d]
   const float *xnorm;
   const float *group_maxn2; // [G+1] max xnorm per group
   uint32_t n, d, k;
   const int *status;        // the prefilter's status word: non-zero = nothing to rerank
   const float *cand_key;
   const uint32_t *cand_col;
   uint32_t *out_ids;
   float *out_dists;
   uint32_t *fb_rows;        // rows the certificate rejected
   uint32_t *fb_items;
   uint32_t *fb_count;       // zeroed before launch
   unsigned long long *counters; // [0] certified rows, [1] rejected rows
   const OperandScale *scale;
   double c1, c2, c3, c4, gd, gref; // certificate constants, see tc_certificate_constants
};

struct ExactParams
{
   const WorkItem *items;
   const Segment *segs;
   const float *X;
   uint32_t d, k;
   const uint32_t *rows;      // rows to compute
   const uint32_t *row_items; // work item of each row
   const uint32_t *count_dev; // number of rows (device word) or NULL
   uint32_t count_host;       // number of rows when count_dev is NULL
   uint32_t *out_ids;
   float *out_dists;
   const uint32_t *out_pos;   // output row of each listed row, or NULL for the row itself
   uint32_t warp_per_row;     // 1: a warp per row (short target lists, k <= 16), else a block
};

// Largest k the tensor-core route supports (candidate list of 32 per row).
constexpr uint32_t kTcMaxK = 24;
// Largest k the exact route supports (per-lane list of 128).
constexpr uint32_t kExactMaxK = 128;

int tc_candidates_for_k(uint32_t k);              // 16 or 32; 0 = unsupported
uint32_t tc_operand_cols(uint32_t d);             // dp: d rounded up to 16, at least 64
bool tc_a_resident(uint32_t dp);                  // A operand kept in TMEM per item
size_t tc_smem_bytes(uint32_t dp, uint32_t k);
void tc_certificate_constants(uint32_t d, uint32_t dp, RerankParams &p);

// The fp16 operand Xh [n x dp] (centred, scaled by a power of two) and the fp32 norms
// of the centred rows.  The mean and the scale come from every row when n <= 2^18, else
// from the rows i * operand_sample_stride(n), with two bits of headroom in the scale;
// an element beyond the fp16 range then sets *flag, and gated kernels redo the
// statistics and the operand from every row (the result is then the same as the full
// pass's).  No host synchronisation.
uint32_t operand_sample_stride(uint32_t n);
cudaError_t launch_prepare_operand(const float *X, uint32_t n, uint32_t d, uint32_t dp, double *sums, uint32_t *range,
                                   float *mean, OperandScale *scale, uint16_t *Xh, float *xnorm, uint32_t *flag,
                                   cudaStream_t s);
cudaError_t launch_group_maxnorm(const float *xnorm, const uint32_t *chunks, uint32_t nchunks, uint32_t G, float *out,
                                 cudaStream_t s);
cudaError_t launch_fill_empty(const RowRange *ranges, uint32_t nranges, uint32_t k, uint32_t *ids, float *dists,
                              cudaStream_t s);

// CopyRange (ungx_internal.h): a shard's rows into a compact buffer, and back.
cudaError_t launch_gather_rows(const CopyRange *ranges, uint32_t nranges, uint32_t k, const uint32_t *ids,
                               const float *dists, uint32_t *out_ids, float *out_dists, cudaStream_t s);
// The reverse of launch_gather_rows: compact rows [dst_row, +count) of (ids, dists) go back
// to rows [src_row, +count) of the n x k output.
cudaError_t launch_scatter_rows(const CopyRange *ranges, uint32_t nranges, uint32_t k, const uint32_t *ids,
                                const float *dists, uint32_t *out_ids, float *out_dists, cudaStream_t s);
// Capacity path: merge a pass's per-row top-k (ids = rows of the pass buffer: [0, split)
// are global rows base_src.., the rest base_tgt..) into the running global top-k of rows
// base_src .. base_src + rows.  k <= kMergeMaxK.
constexpr uint32_t kMergeMaxK = 128;
cudaError_t launch_merge_pass(const uint32_t *pass_ids, const float *pass_dists, uint32_t rows, uint32_t k,
                              uint32_t base_src, uint32_t split, uint32_t base_tgt, uint32_t *ids, float *dists,
                              cudaStream_t s);
cudaError_t launch_exact(const ExactParams &p, uint32_t grid_hint, cudaStream_t s);

// ---- exact kNN graph seeding (knn.cu)
struct KnnParams
{
   const float *X;             // base vectors [* x d]
   uint32_t d, dpad;           // dpad = d rounded up to 4
   const uint32_t *ranges;     // [2 * groups]: rows [first, end) of each group
   const uint64_t *base;       // [groups]: output row of each group's first point
   uint32_t candidate_k, final_degree, head_keep, anchor_tail, anchor_slots, bidir_anchor, graph_stride;
   uint32_t *graph;            // [points x graph_stride]
   uint32_t *entry_points;     // [groups] or NULL
   float *dist;                // two-phase path: the groups' distance matrices, [n_g x n_g] each
   const uint64_t *dbase;      // [groups]: offset of group g's matrix in dist
};
constexpr uint32_t kKnnMaxDim = 352; // both 64-row tiles hold every dimension in shared memory
// Groups of at most kKnnDistMaxN points take the two-phase path (symmetric distance
// matrix, then a warp per row), in batches of at most kKnnDistBatch matrix entries;
// a call with a larger group takes the fused kernel (one block per 64 rows).
constexpr uint32_t kKnnDistMaxN = 8192;
constexpr uint64_t kKnnDistBatch = 1ull << 30;
size_t knn_smem_bytes(uint32_t d);
size_t knn_task_count(const uint32_t *ranges, uint32_t num_groups);
void knn_tasks(const uint32_t *ranges, uint32_t num_groups, uint32_t *tasks); // [2 * count]: (group, first row)
cudaError_t launch_exact_knn(const KnnParams &p, const uint32_t *d_tasks, uint32_t num_tasks, cudaStream_t s);
// Two-phase path: tiles [3 * num_tiles] = (group, row tile, column tile >= row tile) of
// 64 x 64; rows [2 * num_rows] = (group, first row) of 32-row pieces.
cudaError_t launch_knn_two_phase(const KnnParams &p, const uint32_t *d_tiles, uint32_t num_tiles,
                                 const uint32_t *d_rows, uint32_t num_rows, cudaStream_t s);

// Tensor-core route of the seeding: tc_kernel (lists of 32 per column third, the
// diagonal excluded) over a plan whose items are 128-row blocks of each group with the
// group itself as the only target; then this rerank, a block per item: each row's 96
// list entries get the reference's distance, the cand smallest by (distance, local id)
// are laid out, and the certificate decides whether a column outside the lists could
// have entered (then the row is queued in fb_rows for the exact kernel).
struct KnnRerankParams
{
   KnnParams p;              // layout, output rows, group ranges (groups 0-based)
   const WorkItem *items;    // the tensor-core plan's items; segment group id = group + 1
   const Segment *segs;
   const float *cand_key;    // [row][3][32] (global rows of X)
   const uint32_t *cand_col;
   const float *xnorm;
   const float *group_maxn2; // [groups + 1], index = group + 1
   const OperandScale *scale;
   const int *status;        // the prefilter's status word: non-zero = nothing to do
   double c1, c2, c3, c4, gd, gref, abs_err;
   // Rows the certificate rejected, in four buckets per group: bucket h < 3 holds rows
   // whose lists all passed but list h (only list h's columns are rescanned), bucket 3
   // the rows rescanned in full.  Local row at 4 base[group] + h n_group + slot.
   uint32_t *fb_rows;
   uint32_t *fb_pend_idx;       // same index: the row's pending entries (bucket h < 3)
   uint32_t *fb_group_count;    // [4 groups], zeroed before launch: the slots taken per bucket
   float2 *fb_pend;             // [fb_pend_cap][96]: the passing lists' (distance, id) by rank
   uint32_t *fb_pend_count;     // zeroed before launch
   uint32_t fb_pend_cap;
   unsigned long long *counters; // [0] certified rows, [1] rejected rows
};
cudaError_t launch_knn_rerank(const KnnRerankParams &p, uint32_t num_items, cudaStream_t s);
// The exact seeding of the rows the rerank's certificate rejected, with no host round
// trip: launch_knn_fallback_tasks cuts each bucket (group, h) of rejected rows into
// tasks of up to 8 rows, d_tasks [4 x max_tasks] = (group, bucket, first slot, rows) and
// *d_num_tasks (one block); launch_knn_fallback_rows then runs them on a persistent grid
// (num_sms x a few blocks) that reads *d_num_tasks.  max_tasks bounds the task list
// (the number of points of the call suffices).
cudaError_t launch_knn_fallback_tasks(const uint32_t *d_group_count, uint32_t num_groups, uint32_t *d_tasks,
                                      uint32_t max_tasks, uint32_t *d_num_tasks, cudaStream_t s);
cudaError_t launch_knn_fallback_rows(const KnnParams &p, const uint32_t *d_fb_rows, const uint32_t *d_pend_idx,
                                     const float2 *d_pend, const uint32_t *d_tasks, const uint32_t *d_num_tasks,
                                     uint32_t num_sms, cudaStream_t s);

// ---- graph assembly (graph.cu)
// group_of[v] = group of row v (1..G), G + 1 for rows outside every group.
cudaError_t launch_group_of(const uint32_t *ranges, uint32_t G, uint32_t n, uint32_t *group_of, cudaStream_t s);
// flags[e] = 1 for every LNG edge f -> g (e in f's out list) that some row of f
// reaches through its cross edges; flags zeroed by the caller.
cudaError_t launch_mark_reached(const uint32_t *cross_ids, uint32_t n, uint32_t k, const uint32_t *group_of,
                                uint32_t G, const uint64_t *out_offsets, const uint32_t *out_ids, uint8_t *flags,
                                cudaStream_t s);
// Per point: intra-group edges (optional CSR), then its cross edges up to the first
// sentinel, then its additional edges (optional CSR): degree, exclusive scan into
// offsets[n + 1], then the columns.  scratch: >= csr_scan_scratch_bytes(n) bytes.
size_t csr_scan_scratch_bytes(uint32_t n);
cudaError_t launch_graph_degrees(uint32_t n, uint32_t k, const uint64_t *intra_off, const uint32_t *cross_ids,
                                 const uint64_t *add_off, uint64_t *offsets, cudaStream_t s);
cudaError_t launch_exclusive_scan_u64(uint64_t *data, uint32_t count, void *scratch, cudaStream_t s);
// Additional edges (the reference's rule for unreached LNG edges), device passes:
// per edge its query count into qcnt[nnz] and the counters stats[0] (missing edges),
// stats[1] (vectors the reference scans); after an exclusive scan of qcnt into qoff,
// the work items / segments (indexed by edge) and per query its row, item and slot;
// after the exact top-(k/2), the (from, to) list at loff (nq + 1 entries, scanned
// here); the same edges per point: off[n + 1] and cols.
cudaError_t launch_add_edge_queries(const uint32_t *ranges, uint32_t G, const uint64_t *out_off, const uint32_t *out_ids,
                                    const uint8_t *reached, uint32_t k, uint64_t *qcnt, unsigned long long *stats,
                                    cudaStream_t s);
cudaError_t launch_add_query_fill(const uint32_t *ranges, uint32_t G, const uint64_t *out_off, const uint32_t *out_ids,
                                  const uint64_t *qoff, WorkItem *items, Segment *segs, uint32_t *rows,
                                  uint32_t *row_items, uint32_t *pos, cudaStream_t s);
cudaError_t launch_add_list(const uint32_t *res, const uint32_t *rows, uint32_t nq, uint32_t kh, uint64_t *loff,
                            uint32_t *from, uint32_t *to, void *scratch, cudaStream_t s);
cudaError_t launch_add_points(const uint32_t *ranges, uint32_t G, uint32_t n, uint32_t k, const uint64_t *out_off,
                              const uint64_t *qoff, const uint64_t *loff, const uint32_t *to, uint64_t *off,
                              uint32_t *cols, void *scratch, cudaStream_t s);
// group_of / ranges (optional): intra columns are group-local; row v's get ranges[2 group_of[v]] added.
cudaError_t launch_graph_fill(uint32_t n, uint32_t k, const uint64_t *intra_off, const uint32_t *intra_cols,
                              const uint32_t *cross_ids, const uint64_t *add_off, const uint32_t *add_cols,
                              const uint64_t *offsets, uint32_t *cols, cudaStream_t s,
                              const uint32_t *group_of = nullptr, const uint32_t *ranges = nullptr);
cudaError_t launch_tc(const TcMaps &maps, const TcParams &p, uint32_t kp, uint32_t grid, cudaStream_t s);
cudaError_t launch_rerank(const RerankParams &p, uint32_t kp, uint32_t num_items, cudaStream_t s);

} // namespace ungx
