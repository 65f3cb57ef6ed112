// Shared definitions of libaspire_b200: plan layout, work items, helpers.
#pragma once

#include <cstdint>
#include <cstddef>

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "../../include/aspire_b200.h"

namespace aspire {

constexpr int kHeadDim = 128;
constexpr int kPageSize = 16;

// The int workspace starts with a 256-byte control block (status word at
// offset 0); the uploaded plan follows it.
constexpr size_t kStatusBytes = 256;

// Plan header (int32 words at the start of the plan).
enum PlanHeader : int {
  kHdrMagic = 0,
  kHdrNumItems = 1,
  kHdrNumGatherCtas = 2,     // grid of the gather kernel the list was built for
  kHdrOffGatherIndptr = 3,   // int32 index of gather CTA indptr [num_ctas + 1]
  kHdrTcFirst = 4,           // index of the first tcgen05 decode item; they run to kHdrPfFirst
  kHdrOffItems = 5,          // int32 index of the item array
  kHdrOffMerge = 6,          // int32 index of the merge descriptors [num_merge]
  kHdrNumMerge = 7,
  kHdrPartialLseLo = 8,      // float index of the partial LSE array (lo/hi words)
  kHdrPartialLseHi = 9,
  kHdrCausal = 10,
  kHdrNumTcCtas = 11,        // grid of the tcgen05 kernel the list was built for
  kHdrOffMergeUnits = 12,    // int32 index of the merge units [num_merge_units]
  kHdrNumMergeUnits = 13,    // (merge group, packed row) pairs, one warp each
  kHdrTcClaim = 14,          // tcgen05 items claimed so far (0 at upload; the merge kernel resets it)
  kHdrPfFirst = 15,          // index of the first prefill item; they run to kHdrNumItems
  kHdrPfClaim = 16,          // prefill items claimed so far (same rule as kHdrTcClaim)
  kHdrChunkTokens = 17,      // the plan's common split-KV chunk length (tokens)
  kHdrWords = 32,
};
constexpr int32_t kPlanMagic = 0x41535042;  // "ASPB"

// One unit of work: a KV chunk of one (request row, KV head, packed-query tile).
struct WorkItem {
  int32_t row;           // request index (also the dump batch index)
  int32_t kv_head;
  int32_t q_start;       // first query token of the request
  int32_t q_len;         // query tokens of the request
  int32_t kv_page_base;  // offset of the request's page list in kv_indices
  int32_t kv_len;        // KV tokens attended by the request
  int32_t tok_begin;     // KV token range of this chunk
  int32_t tok_end;
  int32_t pq_begin;      // packed query rows [pq_begin, pq_end); packed = q_idx*group + g
  int32_t pq_end;
  int32_t chunk;         // chunk index within the merge group
  int32_t n_chunks;
  int32_t partial_base;  // partial row of chunk 0 of the merge group
  int32_t merge_id;      // merge descriptor index, -1 when n_chunks == 1
  int32_t kind;          // 0 = CUDA-core gather kernel, 1 = tcgen05 decode kernel, 2 = prefill kernel
  int32_t cols;          // tcgen05 decode items: product columns, 0 = packed rows rounded up to 16
};
static_assert(sizeof(WorkItem) == 64, "WorkItem must stay 64 bytes");

constexpr int kItemWords = sizeof(WorkItem) / 4;

// A (row, KV head, packed-query tile) whose KV range was split into chunks:
// the merge kernel combines its chunk partials (chunk c of packed row j at
// partial row partial_base + c * nrows + j).
struct MergeDesc {
  int32_t q_start;
  int32_t pq_begin;
  int32_t nrows;
  int32_t kv_head;
  int32_t partial_base;
  int32_t n_chunks;
  int32_t reserved0;
  int32_t reserved1;
};
static_assert(sizeof(MergeDesc) == 32, "MergeDesc must stay 32 bytes");
constexpr int kMergeWords = sizeof(MergeDesc) / 4;

// Split-KV chunk length = total KV tokens / (SMs x items per CTA), at least
// 512, rounded up to 128 (both planners).  Batches whose (row, KV head,
// query-tile) groups differ in span by more than 2x (long verify rows beside
// short draft rows, or the query tiles of a causal prefill chunk) take about
// kItemsPerCtaMixed items per CTA: every item boundary costs a few
// microseconds, and the spread of item sizes balances the CTAs.  Groups of
// similar span (a full-context refresh layer) are cut into about
// kItemsPerCtaUniform per CTA, since fewer equal items balance poorly.
constexpr int kItemsPerCtaMixed = 2;
constexpr int kItemsPerCtaUniform = 4;
__host__ __device__ inline int64_t chunk_for(int64_t total_tokens, int64_t num_sms, int64_t per_cta) {
  const int64_t target = num_sms * per_cta;
  int64_t chunk = (total_tokens + target - 1) / (target > 0 ? target : 1);
  chunk = chunk < 512 ? 512 : chunk;
  return (chunk + 127) / 128 * 128;
}

// Whole (row, KV head, query-tile) groups instead of split-KV chunks, when
// they would fill the grid about as evenly: a medium draft-only batch (16 to
// 64 rows over a 64-512 page budget) otherwise pays item boundaries and the
// merge for balance it does not need.  Both planners compare two makespan
// estimates in tenths of a 128-token tile (1.5-1.8 us on B200 at any load):
//   whole = ceil(groups / SMs) x (longest span + item)
//   split = max(tokens / SMs, chunk) + ceil(chunk items / SMs) x item
//           + merge (when any group splits)
// with an item boundary at 2.3 tiles and the merge (its launch and the extra
// kernel boundary) at 2.5, fitted to timed draft-only batches: 16 rows over
// 64 pages ran 22.0 us whole against 28.1 us split, one row 19.1 us whole
// against 15.5 us split (its few SMs gain more from halving the span).
constexpr int64_t kItemCost10 = 23;
constexpr int64_t kMergeCost10 = 25;
__host__ __device__ inline bool whole_groups_cheaper(int64_t n_groups, int64_t max_span, int64_t total_tokens,
                                                     int64_t chunk, int64_t n_chunk_items, int64_t num_sms) {
  if (n_groups <= 0 || num_sms <= 0) return false;
  const int64_t whole = (n_groups + num_sms - 1) / num_sms * ((max_span + 127) / 128 * 10 + kItemCost10);
  const int64_t avg10 = (total_tokens * 10 + 128 * num_sms - 1) / (128 * num_sms);
  const int64_t chunk10 = chunk / 128 * 10;
  const int64_t split = (avg10 > chunk10 ? avg10 : chunk10) + (n_chunk_items + num_sms - 1) / num_sms * kItemCost10 +
                        (n_chunk_items > n_groups ? kMergeCost10 : 0);
  return whole <= split;
}
// Mixed batches (long verify groups beside short draft groups) whose long
// groups are few enough: cutting each long group (span > max_span / 2) into
// k = SMs / n_long equal pieces gives every piece its own SM, and the short
// groups fill the SMs left over.  The common rule's two items per SM leave a
// partly filled second round there instead (a TP-8 share of the bench: 288
// verify chunks + 32 draft items on 148 SMs).  Returns that chunk length when
// the short groups' work (tenths of a tile, each group whole) fits into the
// spare SMs' time, else 0.  Both planners use it.  Measured on the bench's
// mixed layer-call: TP-8 share 0.108 -> 0.101 ms (chunk 3840 -> 8192), TP-4
// 0.188 -> 0.181 ms (7552 -> 16384); TP 1 has more long groups than SMs.
__host__ __device__ inline int64_t long_group_chunk(int64_t n_long, int64_t max_span, int64_t short_work10,
                                                    int64_t num_sms) {
  if (n_long <= 0 || num_sms <= 0) return 0;
  const int64_t k = num_sms / n_long;
  if (k < 1) return 0;
  int64_t chunk = ((max_span + k - 1) / k + 127) / 128 * 128;
  chunk = chunk < 512 ? 512 : chunk;
  const int64_t pieces = n_long * ((max_span + chunk - 1) / chunk);
  const int64_t spare = num_sms - pieces;
  if (spare < 0 || short_work10 > spare * (chunk / 128 * 10 + kItemCost10)) return 0;
  return chunk;
}
// A group counts as long for long_group_chunk when its span exceeds half the
// longest; a short group's work is its tiles plus one item boundary.
__host__ __device__ inline bool long_group(int64_t span, int64_t max_span) { return 2 * span > max_span; }
__host__ __device__ inline int64_t short_group_work10(int64_t span) {
  return (span + 127) / 128 * 10 + kItemCost10;
}

// Split plans at the 512-token minimum that keep at most a quarter of the
// SMs busy (a drafting row over 64 pages: 8 groups of 1024 tokens, 16
// items) take 256-token chunks: such a call is bound by the latency of its
// first tiles, not by HBM, and each item's share of it halves.  Measured on
// the config-5 sweep: one drafting row over 64 pages 13.9 -> 12.9-13.0 us at
// every context.  Plans of 64 items doubled to 128 were 4-8.5 % slower (one
// row of 4k context: the extra merge work and item boundaries outweigh the
// shorter items) and four drafting rows only 1-2 % faster, so the rule stops
// at a quarter; a 256-token minimum for every plan slowed the calls whose
// items then outnumber the SMs (one row of 16k context: 32 -> 47 us).  Both
// planners use it.
__host__ __device__ inline int64_t small_plan_chunk(int64_t chunk, int64_t n_groups, int64_t n_items,
                                                    int64_t num_sms) {
  return chunk == 512 && n_items > n_groups && 4 * n_items <= num_sms ? 256 : chunk;
}

// The chunk length that keeps every group whole.
__host__ __device__ inline int64_t whole_group_chunk(int64_t max_span) {
  const int64_t c = (max_span + 127) / 128 * 128;
  return c < 512 ? 512 : c;
}

// Resident CTAs per SM of each kernel class (sets the persistent grids).
constexpr int kGatherCtasPerSm = 4;
constexpr int kTcCtasPerSm = 1;

// Product columns of the tcgen05 decode items.  Each item's products take
// its packed rows rounded up to 16 columns, except that when the decode list
// holds at most kPadMaxItemsPerCta items per CTA, the long groups' items
// (long_group) all take the widest of their widths.  Then most CTAs run one
// long item and nothing else, and the launch ends when the slowest of them
// does; long items of different widths (verify rows with 3 to 9 queries: 16,
// 32 and 48 columns) stream at different rates, and the fast CTAs idle.  At
// one width they finish together.  Measured per mixed layer-call on the
// bench's batch (B=64, 32k, verify q_len 3-9): TP-8 share 0.101 -> 0.097 ms,
// TP-4 0.181 -> 0.175 ms; with one q_len for every verify row, or with more
// items per CTA (TP 1), padding gains nothing, and padding the short
// (draft) items too, as a launch-wide single width did, cost up to 15 %
// (one draft row: 13.9 -> 16.3 us).  Both planners use it.
constexpr int kPadMaxItemsPerCta = 2;
__host__ __device__ inline int32_t tc_columns(int32_t rows) { return (rows + 15) / 16 * 16; }
__host__ __device__ inline bool pad_long_items(int64_t n_decode_items, int64_t num_sms) {
  return n_decode_items > 0 && n_decode_items <= int64_t(kPadMaxItemsPerCta) * num_sms * kTcCtasPerSm;
}

// Packed query rows handled by one gather-kernel item.
constexpr int kGatherQTile = 4;
// Packed query rows handled by one tcgen05 item (N of the MMA after padding).
constexpr int kTcQTile = 48;
// Prefill items: two halves of up to kPfQTile packed query rows (the M of
// the MMA), whole query positions per half, sharing every K/V tile.  Rows
// with at least kPfMinRows packed query rows (long queries: prefill chunks)
// go to the prefill phase of the tcgen05 kernel.
constexpr int kPfQTile = 128;
constexpr int kPfMinRows = 128;
constexpr int kPfMaxRows = 2 * kPfQTile;
__host__ __device__ constexpr int pf_half_rows(int group) { return (kPfQTile / group) * group; }
__host__ __device__ constexpr int pf_item_rows(int group) { return 2 * pf_half_rows(group); }

}  // namespace aspire
