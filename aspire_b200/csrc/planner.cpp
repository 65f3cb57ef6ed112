// Host work-list planner for the mixed paged attention.
//
// Stands in for FlashInfer's TwoStageHolisticPlan as called from
// HolisticAttentionWrapper.plan / plan_host (aspire/attention/
// holistic_wrapper.py:253-265, :323-335).  The planner is a different
// design: every (request row, KV head, packed-query tile) is cut into
// split-KV chunks of a common length (common.cuh: about two or four items
// per CTA, one piece per SM for few long groups, or every group whole), and
// items are placed on CTAs longest-first onto the least-loaded CTA (LPT).  By default every row goes to the
// tcgen05 kernel (decode items, or prefill items for rows of at least 128
// packed query rows); the CUDA-core gather kernel takes narrow rows only when
// the routing thresholds (ASPIRE_B200_TC_MIN_ROWS / ASPIRE_B200_TC_MIN_KV)
// send them there.
#include <algorithm>
#include <cstring>
#include <numeric>
#include <queue>
#include <string>
#include <vector>

#include "common.cuh"
#include "errors.h"

namespace aspire {

namespace {

struct GroupDesc {
  int32_t row, kv_head, q_start, q_len, kv_page_base, kv_len, pq_begin, pq_end, kind;
  int32_t span;  // KV tokens the tile can see: kv_len, or under the causal mask up to its last query
};

// Under the bottom-right causal mask the tile's last query (packed row
// pq_end - 1) sees keys [0, kv_len - q_len + q_idx + 1); later keys are
// masked for every query of the tile, so the tile's work stops there.  For a
// decode row (one tile holding all queries) this is kv_len itself; for
// long-query rows (prefill chunks) it skips the fully masked tiles.  Tiles
// holding any row of query 0 (more than one when the group is wider than the
// tile) keep the whole range: the first/last logit dump records query 0's raw
// logits at every key, masked or not.
inline int32_t visible_span(int32_t kv_len, int32_t q_len, int32_t pq_begin, int32_t pq_end, int group,
                            bool causal) {
  if (!causal || pq_begin < group) return kv_len;
  const int64_t q_last = (pq_end - 1) / group;
  const int64_t lim = int64_t(kv_len) - q_len + q_last + 1;
  return static_cast<int32_t>(std::max<int64_t>(0, std::min<int64_t>(kv_len, lim)));
}

// Item cost in "tokens": the KV tokens streamed plus a fixed per-item
// overhead covering setup, the first tile's reduction and the epilogue.
inline int64_t item_cost(const WorkItem& it) {
  return int64_t(it.tok_end - it.tok_begin) + 512;
}

// Longest first: the order in which the tcgen05 CTAs claim items at run time.
void order_by_cost(std::vector<WorkItem>& items) {
  std::stable_sort(items.begin(), items.end(), [](const WorkItem& a, const WorkItem& b) {
    return item_cost(a) > item_cost(b);
  });
}

void assign_lpt(std::vector<WorkItem>& items, int num_ctas, std::vector<int32_t>& indptr,
                std::vector<WorkItem>& ordered) {
  indptr.assign(num_ctas + 1, 0);
  ordered.clear();
  if (items.empty()) return;
  std::vector<int> order(items.size());
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) {
    return item_cost(items[a]) > item_cost(items[b]);
  });
  using Load = std::pair<int64_t, int>;  // (load, cta)
  std::priority_queue<Load, std::vector<Load>, std::greater<Load>> heap;
  for (int c = 0; c < num_ctas; ++c) heap.push({0, c});
  std::vector<std::vector<int>> per_cta(num_ctas);
  for (int idx : order) {
    Load top = heap.top();
    heap.pop();
    per_cta[top.second].push_back(idx);
    top.first += item_cost(items[idx]);
    heap.push(top);
  }
  ordered.reserve(items.size());
  for (int c = 0; c < num_ctas; ++c) {
    indptr[c] = static_cast<int32_t>(ordered.size());
    for (int idx : per_cta[c]) ordered.push_back(items[idx]);
  }
  indptr[num_ctas] = static_cast<int32_t>(ordered.size());
}

}  // namespace

int plan_impl(const int32_t* qo_indptr, const int32_t* kv_indptr, const int32_t* kv_len,
              int32_t batch_size, int32_t num_qo_heads, int32_t num_kv_heads, int32_t head_dim,
              int32_t page_size, int32_t causal, int32_t num_sms, bool tc_enabled, int32_t tc_min_rows,
              int32_t tc_min_kv, void* host_buf, size_t host_buf_bytes, size_t float_ws_bytes,
              AspirePlanInfo* info) {
  if (!qo_indptr || !kv_indptr || !kv_len || !host_buf || !info)
    return set_error(ASPIRE_ERR_INVALID, "aspire_plan: null pointer argument");
  if (batch_size < 0) return set_error(ASPIRE_ERR_INVALID, "aspire_plan: batch_size < 0");
  if (head_dim != kHeadDim)
    return set_error(ASPIRE_ERR_INVALID, "aspire_plan: head_dim must be 128, got " +
                                             std::to_string(head_dim));
  if (page_size != kPageSize)
    return set_error(ASPIRE_ERR_INVALID, "aspire_plan: page_size must be 16, got " +
                                             std::to_string(page_size));
  if (num_kv_heads <= 0 || num_qo_heads <= 0 || num_qo_heads % num_kv_heads != 0)
    return set_error(ASPIRE_ERR_INVALID,
                     "aspire_plan: num_qo_heads must be a positive multiple of num_kv_heads");
  if (num_sms <= 0) return set_error(ASPIRE_ERR_INVALID, "aspire_plan: num_sms must be > 0");
  const int gather_ctas = num_sms * kGatherCtasPerSm;
  const int tc_ctas = num_sms * kTcCtasPerSm;
  const int group = num_qo_heads / num_kv_heads;

  // Rows -> (row, head, q-tile) groups.
  std::vector<GroupDesc> groups;
  int64_t total_tokens = 0;
  int32_t max_q_len = 0;
  for (int b = 0; b < batch_size; ++b) {
    const int32_t q0 = qo_indptr[b], q1 = qo_indptr[b + 1];
    const int32_t ql = q1 - q0;
    if (ql < 0) return set_error(ASPIRE_ERR_INVALID, "aspire_plan: qo_indptr not monotonic");
    if (ql == 0) continue;
    const int32_t kl = kv_len[b];
    if (kl < 0) return set_error(ASPIRE_ERR_INVALID, "aspire_plan: negative kv_len");
    const int64_t pages_avail = int64_t(kv_indptr[b + 1]) - kv_indptr[b];
    if (int64_t(kl) > pages_avail * kPageSize && kl > 0) {
      // The page list must cover kv_len tokens.  (The dump program of the
      // reference passes a constant-stride indptr that over-covers; that is
      // fine.  Under-coverage would read foreign pages.)
      return set_error(ASPIRE_ERR_INVALID,
                       "aspire_plan: row " + std::to_string(b) + " kv_len " + std::to_string(kl) +
                           " exceeds its page list (" + std::to_string(pages_avail) + " pages)");
    }
    max_q_len = std::max(max_q_len, ql);
    const int32_t nq = ql * group;
    // tcgen05 for wide query tiles, and for narrow rows with long contexts
    // (the tensor-core tile streams K/V better than the CUDA-core gather).
    // A tcgen05 q-tile holds whole query positions (all `group` heads of each),
    // so that one TMA box loads it.
    const bool wide = tc_enabled && group <= kTcQTile &&
                      (nq > kGatherQTile || nq >= tc_min_rows || kl >= tc_min_kv);
    // Long queries (prefill chunks) go to the prefill phase: items of two
    // 128-row halves (whole query positions each) that share every K/V tile.
    const bool prefill = wide && nq >= kPfMinRows;
    const int tile = prefill ? pf_item_rows(group) : wide ? (kTcQTile / group) * group : kGatherQTile;
    const int kind = prefill ? 2 : (wide ? 1 : 0);
    for (int h = 0; h < num_kv_heads; ++h) {
      for (int p0 = 0; p0 < nq; p0 += tile) {
        const int32_t p1 = std::min(nq, p0 + tile);
        GroupDesc g{b, h, q0, ql, kv_indptr[b], kl, p0, p1, kind,
                    visible_span(kl, ql, p0, p1, group, causal != 0)};
        groups.push_back(g);
        total_tokens += std::max<int32_t>(g.span, 1);
      }
    }
  }

  // Common chunk length (chunk_for): a multiple of 128 tokens (one tcgen05 KV
  // tile = 8 pages), at least 512 (256 for small split plans); two or four
  // items per CTA by the spread of the groups' spans, then the rules below.
  int32_t max_span = 0, min_span = INT32_MAX;
  for (const GroupDesc& g : groups) {
    max_span = std::max(max_span, g.span);
    min_span = std::min(min_span, g.span);
  }
  const bool similar = 2 * int64_t(min_span) >= max_span;
  int64_t chunk = chunk_for(total_tokens, num_sms, similar ? kItemsPerCtaUniform : kItemsPerCtaMixed);
  if (!similar) {
    int64_t n_long = 0, short_work10 = 0;
    for (const GroupDesc& g : groups) {
      if (long_group(g.span, max_span))
        ++n_long;
      else
        short_work10 += short_group_work10(g.span);
    }
    const int64_t c = long_group_chunk(n_long, max_span, short_work10, num_sms);
    if (c > 0) chunk = c;
  }
  {
    int64_t n_chunk_items = 0;
    for (const GroupDesc& g : groups) n_chunk_items += g.span > 0 ? (g.span + chunk - 1) / chunk : 1;
    if (whole_groups_cheaper(int64_t(groups.size()), max_span, total_tokens, chunk, n_chunk_items, num_sms))
      chunk = whole_group_chunk(max_span);
    else
      chunk = small_plan_chunk(chunk, int64_t(groups.size()), n_chunk_items, num_sms);
  }

  // Few decode items per CTA: the long groups' items take one width (pad_long_items).
  int32_t pad_cols = 0;
  {
    int64_t n_tc = 0;
    for (const GroupDesc& g : groups) {
      if (g.kind != 1) continue;
      n_tc += g.span > 0 ? (g.span + chunk - 1) / chunk : 1;
      if (long_group(g.span, max_span)) pad_cols = std::max(pad_cols, tc_columns(g.pq_end - g.pq_begin));
    }
    if (!pad_long_items(n_tc, num_sms)) pad_cols = 0;
  }

  std::vector<WorkItem> gather_items, tc_items, pf_items;
  std::vector<MergeDesc> merges;
  std::vector<int32_t> merge_units;  // (merge index << 8) | packed row within the tile
  int32_t num_merge = 0;
  int64_t partial_rows = 0;
  for (const GroupDesc& g : groups) {
    const int32_t n_chunks =
        g.span > 0 ? static_cast<int32_t>((g.span + chunk - 1) / chunk) : 1;
    const int32_t rows = g.pq_end - g.pq_begin;
    int32_t merge_id = -1, partial_base = 0;
    if (n_chunks > 1) {
      merge_id = num_merge++;
      if (partial_rows + int64_t(n_chunks) * rows > INT32_MAX)
        return set_error(ASPIRE_ERR_CAPACITY, "aspire_plan: too many partial rows");
      partial_base = static_cast<int32_t>(partial_rows);
      partial_rows += int64_t(n_chunks) * rows;
      MergeDesc md{};
      md.q_start = g.q_start;
      md.pq_begin = g.pq_begin;
      md.nrows = rows;
      md.kv_head = g.kv_head;
      md.partial_base = partial_base;
      md.n_chunks = n_chunks;
      merges.push_back(md);
      for (int32_t j = 0; j < rows; ++j) merge_units.push_back((merge_id << 8) | j);
    }
    for (int32_t c = 0; c < n_chunks; ++c) {
      WorkItem it{};
      it.row = g.row;
      it.kv_head = g.kv_head;
      it.q_start = g.q_start;
      it.q_len = g.q_len;
      it.kv_page_base = g.kv_page_base;
      it.kv_len = g.kv_len;
      it.tok_begin = static_cast<int32_t>(std::min<int64_t>(int64_t(c) * chunk, g.span));
      it.tok_end = static_cast<int32_t>(std::min<int64_t>(int64_t(c + 1) * chunk, g.span));
      it.pq_begin = g.pq_begin;
      it.pq_end = g.pq_end;
      it.chunk = c;
      it.n_chunks = n_chunks;
      it.partial_base = partial_base;
      it.merge_id = merge_id;
      it.kind = g.kind;
      it.cols = g.kind == 1 && long_group(g.span, max_span) ? pad_cols : 0;
      (g.kind == 2 ? pf_items : g.kind == 1 ? tc_items : gather_items).push_back(it);
    }
  }

  // CUDA-core items are placed on CTAs ahead of time (LPT); tcgen05 items are
  // claimed by the persistent CTAs at run time, longest first.
  std::vector<int32_t> gather_indptr;
  std::vector<WorkItem> gather_ordered;
  assign_lpt(gather_items, gather_ctas, gather_indptr, gather_ordered);
  order_by_cost(tc_items);
  order_by_cost(pf_items);
  std::vector<WorkItem> tc_ordered = tc_items;
  tc_ordered.insert(tc_ordered.end(), pf_items.begin(), pf_items.end());
  // One item array: gather list | tcgen05 decode list | prefill list.
  const int32_t n_gather = static_cast<int32_t>(gather_ordered.size());
  const int32_t n_decode_tc = static_cast<int32_t>(tc_items.size());
  const int32_t num_items = n_gather + static_cast<int32_t>(tc_ordered.size());

  // Layout (int32 words): header | gather indptr | items | merges | merge units.
  const int64_t off_gather = kHdrWords;
  int64_t off_items = off_gather + gather_ctas + 1;
  off_items = (off_items + 15) / 16 * 16;  // 64-byte aligned items
  const int64_t off_merge = off_items + int64_t(num_items) * kItemWords;
  const int64_t off_units = off_merge + int64_t(num_merge) * kMergeWords;
  const int32_t num_units = static_cast<int32_t>(merge_units.size());
  const int64_t total_words = off_units + num_units;
  const int64_t int_bytes = total_words * 4;
  if (size_t(int_bytes) > host_buf_bytes)
    return set_error(ASPIRE_ERR_CAPACITY, "aspire_plan: plan needs " + std::to_string(int_bytes) +
                                              " bytes, host buffer has " +
                                              std::to_string(host_buf_bytes));
  const int64_t float_bytes = partial_rows * (kHeadDim + 1) * 4;
  if (size_t(float_bytes) > float_ws_bytes)
    return set_error(ASPIRE_ERR_CAPACITY,
                     "aspire_plan: split-KV partials need " + std::to_string(float_bytes) +
                         " bytes of float workspace, have " + std::to_string(float_ws_bytes));

  int32_t* w = static_cast<int32_t*>(host_buf);
  std::memset(w, 0, kHdrWords * 4);
  w[kHdrMagic] = kPlanMagic;
  w[kHdrNumItems] = num_items;
  w[kHdrNumGatherCtas] = gather_ctas;
  w[kHdrNumTcCtas] = tc_ctas;
  w[kHdrCausal] = causal ? 1 : 0;
  w[kHdrOffGatherIndptr] = static_cast<int32_t>(off_gather);
  w[kHdrTcFirst] = n_gather;
  w[kHdrTcClaim] = 0;
  w[kHdrPfFirst] = n_gather + n_decode_tc;
  w[kHdrPfClaim] = 0;
  w[kHdrChunkTokens] = static_cast<int32_t>(chunk);
  w[kHdrOffItems] = static_cast<int32_t>(off_items);
  w[kHdrOffMerge] = static_cast<int32_t>(off_merge);
  w[kHdrNumMerge] = num_merge;
  w[kHdrOffMergeUnits] = static_cast<int32_t>(off_units);
  w[kHdrNumMergeUnits] = num_units;
  const int64_t lse_off = partial_rows * kHeadDim;
  w[kHdrPartialLseLo] = static_cast<int32_t>(lse_off & 0xffffffff);
  w[kHdrPartialLseHi] = static_cast<int32_t>(lse_off >> 32);
  std::memcpy(w + off_gather, gather_indptr.data(), size_t(gather_ctas + 1) * 4);
  for (int64_t i = off_gather + gather_ctas + 1; i < off_items; ++i) w[i] = 0;
  if (n_gather) std::memcpy(w + off_items, gather_ordered.data(), size_t(n_gather) * sizeof(WorkItem));
  if (!tc_ordered.empty())
    std::memcpy(w + off_items + int64_t(n_gather) * kItemWords, tc_ordered.data(),
                tc_ordered.size() * sizeof(WorkItem));
  if (num_merge) std::memcpy(w + off_merge, merges.data(), merges.size() * sizeof(MergeDesc));
  if (num_units) std::memcpy(w + off_units, merge_units.data(), merge_units.size() * 4);

  std::memset(info, 0, sizeof(*info));
  info->num_items = num_items;
  info->num_items_gather = n_gather;
  info->num_items_tc = n_decode_tc;
  info->num_items_prefill = static_cast<int32_t>(pf_items.size());
  info->num_ctas = num_sms;
  info->num_merge = num_merge;
  info->chunk_tokens = static_cast<int32_t>(chunk);
  info->partial_rows = partial_rows;
  info->int_bytes = int_bytes;
  info->float_bytes = float_bytes;
  info->num_qo_heads = num_qo_heads;
  info->num_kv_heads = num_kv_heads;
  info->causal = causal ? 1 : 0;
  info->batch_size = batch_size;
  info->max_q_len = max_q_len;
  info->tc_enabled = tc_enabled ? 1 : 0;
  return ASPIRE_OK;
}

}  // namespace aspire
