// Internal declarations shared by the host (.cpp) and device (.cu) halves of libungx.
#pragma once

#include <cstdint>
#include <string>
#include <thread>
#include <vector>

#include "../../include/ungx.h"

namespace ungx
{

// Thread-local message for calls that have no context (label graph, planning).
void set_global_error(const std::string &msg);
const char *global_error();

// Run body(i) for i in [0, count) on up to `threads` std::threads, dynamic chunks.
template <class F>
void parallel_for(int64_t count, int threads, int64_t chunk, F &&body);

// ------------------------------------------------------------------ planning
// One unit of device work: <=128 consecutive rows of one source group f, paired
// with every target group of out(f).  Source-centric, so a row's final top-k is
// produced by exactly one CTA and written once (no merge, no locks).
struct WorkItem
{
   uint32_t row_begin;
   uint32_t row_count;  // 1..128
   uint32_t seg_begin;  // into Plan::segs
   uint32_t seg_count;
};

// A target group's contiguous row range (one LNG edge f -> f').
struct Segment
{
   uint32_t x_begin;
   uint32_t x_count;
   uint32_t group_id;
   uint32_t pad;
};

struct RowRange
{
   uint32_t begin, count;
};

// Rows [src_row, src_row+count) of a row-major n x k output go to rows
// [dst_row, dst_row+count) of a compact buffer (a shard's rows, copied at once).
struct CopyRange
{
   uint32_t src_row, dst_row, count, pad;
};

struct Plan
{
   std::vector<WorkItem> items;       // this shard's items, longest first
   std::vector<Segment> segs;
   std::vector<RowRange> empty_rows;  // this shard's rows that get no candidates
   uint64_t pairs = 0;                // sum |f|*|f'| over this shard's rows
   uint64_t padded_cols = 0;          // sum over items of sum roundup16(|f'|)
   uint32_t max_item_cols = 0;
   // working storage of build_plan, kept so that a reused Plan allocates nothing
   std::vector<uint64_t> g_cols, g_cost;            // per group: target columns, cost
   std::vector<uint32_t> g_nseg, g_seg0, g_item0;   // per group: segments, offsets
   std::vector<WorkItem> all;                       // every shard's items, group order
   std::vector<uint64_t> key, item_pairs;           // per item: cost (sort key), pairs
   std::vector<uint32_t> order, order2;             // item permutation
   std::vector<uint32_t> norm_chunks;               // (group, first row, rows <= 4096) of every group
   std::vector<uint32_t> item_shard;                // per item of `all`: its shard
   std::vector<uint64_t> shard_load;                // per shard: its LPT cost
};

constexpr uint32_t kRowsPerItem = 128;

// Validates the problem and builds this shard's plan.  Returns UNGX_OK or an error
// status with a message in `err`.
int build_plan(const ungx_cross_edge_problem &p, Plan &plan, std::string &err);

// Every shard's rows (work items and rows without targets) in ascending row order, as
// runs of consecutive rows: runs[s][i].src_row is the run's first row, dst_row its
// position in shard s's compact order; rows[s] is the shard's row count.  `plan` is
// build_plan's result for any shard of p.shard_count.
void shard_runs(const ungx_cross_edge_problem &p, const Plan &plan, std::vector<std::vector<CopyRange>> &runs,
                std::vector<uint32_t> &rows);

} // namespace ungx

#include "ungx_parallel.inl"
