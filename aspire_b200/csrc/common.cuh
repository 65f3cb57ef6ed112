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
  int32_t reserved;
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

// Resident CTAs per SM of each kernel class (sets the persistent grids).
constexpr int kGatherCtasPerSm = 4;
constexpr int kTcCtasPerSm = 1;

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
