// Device-side planner: renders the work list of the mixed attention from
// device arrays, with no host round trip, so planning can live inside a CUDA
// graph (the reference plans on the host every step: HolisticAttentionWrapper.
// plan / plan_host, aspire/attention/holistic_wrapper.py:200-342, fed by
// HostPlanState, aspire/backends/host_plan.py:154-306).
//
// It produces the same items as the host planner (planner.cpp): every
// (row, KV head, packed-query tile) is cut into chunks of one common length
// (a multiple of 128 tokens, at least 512, or 256 for small split plans:
// about two or four items per SM by the spread of the groups' spans, one
// piece per SM for few long groups, or every group whole; common.cuh), with merge descriptors for the split
// groups, and the long groups' items take one product width when there are
// few items per CTA (pad_long_items).  Rows go to the tcgen05 decode
// kernel, or to the prefill kernel when their packed queries reach
// kPfMinRows (the default routing); each list is stored longest first through
// a counting sort on item length in 128-token tiles, the order in which the
// persistent CTAs claim them.  One CTA of 1024 threads; each thread owns a contiguous run
// of rows.  An invalid input row or a plan larger than the workspaces sets
// ASPIRE_STATUS_BAD_PLAN and leaves a plan with no magic, which every kernel
// skips.
#include "kernels.cuh"

namespace aspire {

namespace {

constexpr int kCostBuckets = 1024;

// Exclusive block scan of one int64 per thread; returns the thread's offset
// and writes the total to *total.
__device__ int64_t block_exclusive_scan(int64_t v, int64_t* warp_sums, int64_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  int64_t x = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int64_t y = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int64_t w = lane < nwarps ? warp_sums[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += y;
    }
    if (lane < nwarps) warp_sums[lane] = w;  // inclusive
  }
  __syncthreads();
  const int64_t before = (warp > 0 ? warp_sums[warp - 1] : 0) + x - v;
  *total = warp_sums[nwarps - 1];
  __syncthreads();
  return before;
}

struct RowShape {
  int32_t ql, kl, nq, ntq, tile, kind;  // kind 1: tcgen05 decode kernel, 2: prefill kernel
  bool valid;
};

// KV tokens a query tile [pq_begin, pq_end) can see (the host planner's
// visible_span): all of kv_len, or under the causal mask up to the tile's last
// query, except for the tiles holding rows of query 0 (the dump needs all its
// logits).
__device__ __forceinline__ int32_t tile_span(const DevPlanParams& p, const RowShape& s, int32_t pq_begin,
                                             int32_t pq_end) {
  if (!p.causal || pq_begin < p.group) return s.kl;
  const int64_t q_last = (pq_end - 1) / p.group;
  const int64_t lim = int64_t(s.kl) - s.ql + q_last + 1;
  return int32_t(max(int64_t(0), min(int64_t(s.kl), lim)));
}

__device__ __forceinline__ int32_t span_chunks(int32_t span, int64_t chunk) {
  return span > 0 ? int32_t((span + chunk - 1) / chunk) : 1;
}

__device__ __forceinline__ RowShape row_shape(const DevPlanParams& p, int b) {
  RowShape r{};
  const int32_t ql = p.qo_indptr[b + 1] - p.qo_indptr[b];
  const int32_t pages = p.kv_indptr[b + 1] - p.kv_indptr[b];
  const int32_t last = p.last_page_len[b];
  const int32_t kl = (pages > 1 ? pages - 1 : 0) * kPageSize + last;
  r.valid = ql >= 0 && pages >= 0 && last >= 0 && !(kl > 0 && int64_t(kl) > int64_t(pages) * kPageSize);
  r.ql = r.valid ? ql : 0;
  r.kl = r.valid ? kl : 0;
  r.nq = r.ql * p.group;
  r.kind = r.nq >= kPfMinRows ? 2 : 1;
  r.tile = r.kind == 2 ? pf_item_rows(p.group) : (kTcQTile / p.group) * p.group;
  r.ntq = (r.nq + r.tile - 1) / r.tile;
  return r;
}

__device__ __forceinline__ int cost_bucket(int64_t tokens) {
  const int64_t tiles = (tokens + 127) / 128;
  return int(tiles < kCostBuckets - 1 ? tiles : kCostBuckets - 1);
}

}  // namespace

__global__ void __launch_bounds__(kDevPlanThreads) aspire_plan_device_kernel(DevPlanParams p) {
  pdl_begin();
  __shared__ int64_t warp_sums[32];
  __shared__ int32_t bucket[2][kCostBuckets];  // per kernel list: decode (1), prefill (2)
  __shared__ int bad, max_span, min_span, long_cols;
  const int tid = threadIdx.x, nthreads = blockDim.x;
  if (tid == 0) {
    bad = 0;
    max_span = 0;
    min_span = INT_MAX;
    long_cols = 0;
  }
  for (int i = tid; i < 2 * kCostBuckets; i += nthreads) bucket[i / kCostBuckets][i % kCostBuckets] = 0;
  __syncthreads();
  const int rpt = (p.batch + nthreads - 1) / nthreads;  // rows per thread
  const int r0 = min(tid * rpt, p.batch), r1 = min(r0 + rpt, p.batch);

  // Total tokens over (row, head, q-tile) groups and the longest group span
  // -> the common chunk length.
  int64_t tokens = 0;
  int my_max_span = 0, my_min_span = INT_MAX;
  for (int b = r0; b < r1; ++b) {
    const RowShape s = row_shape(p, b);
    if (!s.valid) bad = 1;
    if (s.ql <= 0) continue;
    for (int qt = 0; qt < s.ntq; ++qt) {
      const int32_t span = tile_span(p, s, qt * s.tile, min(s.nq, (qt + 1) * s.tile));
      tokens += int64_t(p.num_kv_heads) * (span > 1 ? span : 1);
      my_max_span = max(my_max_span, int(span));
      my_min_span = min(my_min_span, int(span));
    }
  }
  atomicMax(&max_span, my_max_span);
  atomicMin(&min_span, my_min_span);
  int64_t total_tokens;
  block_exclusive_scan(tokens, warp_sums, &total_tokens);  // (its barriers publish max_span)
  const bool similar = 2 * int64_t(min_span) >= max_span;
  int64_t chunk = chunk_for(total_tokens, p.num_sms, similar ? kItemsPerCtaUniform : kItemsPerCtaMixed);
  if (!similar) {
    // Long groups cut into one piece per SM when that packs the grid (long_group_chunk).
    int64_t my_long = 0, my_short = 0;
    for (int b = r0; b < r1; ++b) {
      const RowShape s = row_shape(p, b);
      if (s.ql <= 0) continue;
      for (int qt = 0; qt < s.ntq; ++qt) {
        const int32_t span = tile_span(p, s, qt * s.tile, min(s.nq, (qt + 1) * s.tile));
        if (long_group(span, max_span))
          my_long += p.num_kv_heads;
        else
          my_short += int64_t(p.num_kv_heads) * short_group_work10(span);
      }
    }
    int64_t n_long, short_work10;
    block_exclusive_scan(my_long, warp_sums, &n_long);
    block_exclusive_scan(my_short, warp_sums, &short_work10);
    const int64_t c = long_group_chunk(n_long, max_span, short_work10, p.num_sms);
    if (c > 0) chunk = c;
  }
  {
    // Whole groups when they balance about as well (whole_groups_cheaper),
    // else 256-token chunks for small split plans (small_plan_chunk).
    int64_t my_groups = 0, my_chunk_items = 0;
    for (int b = r0; b < r1; ++b) {
      const RowShape s = row_shape(p, b);
      if (s.ql <= 0) continue;
      for (int qt = 0; qt < s.ntq; ++qt) {
        const int32_t span = tile_span(p, s, qt * s.tile, min(s.nq, (qt + 1) * s.tile));
        my_groups += p.num_kv_heads;
        my_chunk_items += int64_t(p.num_kv_heads) * span_chunks(span, chunk);
      }
    }
    int64_t n_groups, n_chunk_items;
    block_exclusive_scan(my_groups, warp_sums, &n_groups);
    block_exclusive_scan(my_chunk_items, warp_sums, &n_chunk_items);
    if (whole_groups_cheaper(n_groups, max_span, total_tokens, chunk, n_chunk_items, p.num_sms))
      chunk = whole_group_chunk(max_span);
    else
      chunk = small_plan_chunk(chunk, n_groups, n_chunk_items, p.num_sms);
  }

  // Per-thread counts; item lengths into the cost histogram; the widest long
  // decode group (pad_long_items).
  int64_t n_items = 0, n_merge = 0, n_prow = 0, n_units = 0;
  int my_long_cols = 0;
  for (int b = r0; b < r1; ++b) {
    const RowShape s = row_shape(p, b);
    if (s.ql <= 0) continue;
    int32_t* hist = bucket[s.kind - 1];
    for (int qt = 0; qt < s.ntq; ++qt) {
      const int32_t pq1 = min(s.nq, (qt + 1) * s.tile), rows = pq1 - qt * s.tile;
      const int32_t span = tile_span(p, s, qt * s.tile, pq1);
      const int32_t nch = span_chunks(span, chunk);
      const int32_t heads = p.num_kv_heads;
      n_items += int64_t(heads) * nch;
      if (nch > 1) {
        n_merge += heads;
        n_prow += int64_t(heads) * rows * nch;
        n_units += int64_t(heads) * rows;
        atomicAdd(&hist[cost_bucket(chunk)], heads * (nch - 1));
      }
      const int64_t last_len = span - int64_t(nch - 1) * chunk;
      atomicAdd(&hist[cost_bucket(last_len)], heads);
      if (s.kind == 1 && long_group(span, max_span)) my_long_cols = max(my_long_cols, int(tc_columns(rows)));
    }
  }
  if (my_long_cols > 0) atomicMax(&long_cols, my_long_cols);
  int64_t tot_items, tot_merge, tot_prow, tot_units;
  int64_t off_item = block_exclusive_scan(n_items, warp_sums, &tot_items);
  (void)off_item;
  int64_t off_merge = block_exclusive_scan(n_merge, warp_sums, &tot_merge);
  int64_t off_prow = block_exclusive_scan(n_prow, warp_sums, &tot_prow);
  int64_t off_unit = block_exclusive_scan(n_units, warp_sums, &tot_units);
  // Bucket starts, longest first within each list; the decode list comes
  // first, the prefill list after it: start[k] = items in buckets above k.
  int64_t n_decode = 0;
  for (int list = 0; list < 2; ++list) {
    int64_t mine = 0, tot;
    const int k = kCostBuckets - 1 - tid;
    if (tid < kCostBuckets) mine = bucket[list][k];
    __syncthreads();
    const int64_t start = block_exclusive_scan(mine, warp_sums, &tot);
    if (tid < kCostBuckets) bucket[list][k] = int32_t(start + (list == 1 ? n_decode : 0));
    if (list == 0) n_decode = tot;
    __syncthreads();
  }

  // Layout (int32 words): header | gather indptr | items | merges | merge units.
  const int gather_ctas = p.num_sms * kGatherCtasPerSm;
  const int64_t off_gather = kHdrWords;
  const int64_t off_items = (off_gather + gather_ctas + 1 + 15) / 16 * 16;
  const int64_t off_merges = off_items + tot_items * kItemWords;
  const int64_t off_units = off_merges + tot_merge * kMergeWords;
  const int64_t words = off_units + tot_units;
  if (tid == 0 && (words > p.plan_words || tot_prow * (kHeadDim + 1) * 4 > p.float_ws_bytes ||
                   tot_items > INT32_MAX || tot_merge >= (int64_t(1) << 23)))
    bad = 1;
  __syncthreads();
  int32_t* w = p.plan;
  if (bad) {
    if (tid == 0) {
      w[kHdrMagic] = 0;
      if (p.status) atomicOr(p.status, ASPIRE_STATUS_BAD_PLAN);
    }
    return;
  }

  const int32_t pad_cols = pad_long_items(n_decode, p.num_sms) ? long_cols : 0;
  WorkItem* items = reinterpret_cast<WorkItem*>(w + off_items);
  MergeDesc* merges = reinterpret_cast<MergeDesc*>(w + off_merges);
  int32_t* units = w + off_units;
  for (int b = r0; b < r1; ++b) {
    const RowShape s = row_shape(p, b);
    if (s.ql <= 0) continue;
    int32_t* slots = bucket[s.kind - 1];
    for (int h = 0; h < p.num_kv_heads; ++h) {
      for (int qt = 0; qt < s.ntq; ++qt) {
        const int32_t pq0 = qt * s.tile, pq1 = min(s.nq, pq0 + s.tile), rows = pq1 - pq0;
        const int32_t span = tile_span(p, s, pq0, pq1);
        const int32_t nch = span_chunks(span, chunk);
        int32_t merge_id = -1, pbase = 0;
        if (nch > 1) {
          merge_id = int32_t(off_merge++);
          pbase = int32_t(off_prow);
          off_prow += int64_t(nch) * rows;
          MergeDesc md{};
          md.q_start = p.qo_indptr[b];
          md.pq_begin = pq0;
          md.nrows = rows;
          md.kv_head = h;
          md.partial_base = pbase;
          md.n_chunks = nch;
          merges[merge_id] = md;
          for (int j = 0; j < rows; ++j) units[off_unit++] = (merge_id << 8) | j;
        }
        for (int c = 0; c < nch; ++c) {
          WorkItem it{};
          it.row = b;
          it.kv_head = h;
          it.q_start = p.qo_indptr[b];
          it.q_len = s.ql;
          it.kv_page_base = p.kv_indptr[b];
          it.kv_len = s.kl;
          it.tok_begin = int32_t(min(int64_t(c) * chunk, int64_t(span)));
          it.tok_end = int32_t(min(int64_t(c + 1) * chunk, int64_t(span)));
          it.pq_begin = pq0;
          it.pq_end = pq1;
          it.chunk = c;
          it.n_chunks = nch;
          it.partial_base = pbase;
          it.merge_id = merge_id;
          it.kind = s.kind;
          it.cols = s.kind == 1 && long_group(span, max_span) ? pad_cols : 0;
          const int slot = atomicAdd(&slots[cost_bucket(it.tok_end - it.tok_begin)], 1);
          items[slot] = it;
        }
      }
    }
  }
  for (int64_t i = off_gather + tid; i < off_items; i += nthreads) w[i] = 0;  // empty CUDA-core list
  if (tid == 0) {
    for (int i = 0; i < kHdrWords; ++i) w[i] = 0;
    w[kHdrNumItems] = int32_t(tot_items);
    w[kHdrNumGatherCtas] = gather_ctas;
    w[kHdrNumTcCtas] = p.num_sms * kTcCtasPerSm;
    w[kHdrCausal] = p.causal ? 1 : 0;
    w[kHdrOffGatherIndptr] = int32_t(off_gather);
    w[kHdrTcFirst] = 0;
    w[kHdrOffItems] = int32_t(off_items);
    w[kHdrOffMerge] = int32_t(off_merges);
    w[kHdrNumMerge] = int32_t(tot_merge);
    w[kHdrOffMergeUnits] = int32_t(off_units);
    w[kHdrNumMergeUnits] = int32_t(tot_units);
    const int64_t lse_off = tot_prow * kHeadDim;
    w[kHdrPartialLseLo] = int32_t(lse_off & 0xffffffff);
    w[kHdrPartialLseHi] = int32_t(lse_off >> 32);
    w[kHdrTcClaim] = 0;
    w[kHdrPfFirst] = int32_t(n_decode);
    w[kHdrPfClaim] = 0;
    w[kHdrChunkTokens] = int32_t(chunk);
    w[kHdrMagic] = kPlanMagic;
  }
}

}  // namespace aspire
