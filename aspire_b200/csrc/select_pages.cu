// Refresh-layer page scoring + block radix top-k page re-selection.
//
// Phase 1 (its own launch over rows x page splits) turns the first/last logit
// dump of the refresh layer into fp32 page scores, restating
// PageSelectorFirstLastAvg._select_first_last_impl
// (aspire/backends/page_selector.py:163-181):
//   norm  = float(half(float(logit) * sm_scale*log2e)) - lse      (NaN -> -inf)
//   tok   = max_h exp2(norm[slot 0]) + max_h exp2(norm[slot 1])
//   score = sum of the 16 token scores of the page + (-page * 1e-7)
// with tokens past max_seq_len counting as zero.  One CTA per request row
// then runs phase 2, which restates
// _finalize_scores (page_selector.py:79-108) and compute_valid_counts
// (:52-62): the last L valid pages are forced to +inf, pages past num_pages
// to -inf, and the top `valid` pages are taken with ties broken by the lower
// page index (an MSB-first 8-bit radix select over order-preserving keys,
// then an index-ordered pick among the threshold ties).  The selected
// block-table ids are sorted ascending and written in place with a zero tail,
// as LMBackendBase._store_draft_rows (aspire/backends/base.py:1421-1471)
// leaves the draft table.  With order_by_page (given scores only) the last L
// pages are not forced and the pages are listed in page order: with page-index
// scores that is the recent-page seeding of
// LMBackendBase._build_recent_draft_rows (base.py:1522-1537).
#include "kernels.cuh"

namespace aspire {



__device__ __forceinline__ uint32_t order_key(float f) {
  uint32_t u = __float_as_uint(f);
  if (u == 0x80000000u) u = 0;  // -0 ranks with +0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ int valid_count(const SelectParams& p, int np) {
  const int k = p.subset_cache_size;
  const int hi = min(np, k);
  if (p.draft_percent < 0.f) {
    if (p.min_draft_pages >= 0) return min(np, p.min_draft_pages);
    return hi;
  }
  const int floor_pages = p.min_draft_pages >= 0 ? p.min_draft_pages : p.L;
  const int lo = min(np, floor_pages);
  // fp32 arithmetic as the reference: (float(num_pages) * pct) / 100, ceil.
  const float prod = __fmul_rn(float(np), p.draft_percent);
  const int target = static_cast<int>(ceilf(__fdiv_rn(prod, 100.0f)));
  return min(max(target, lo), hi);
}

// Phase 1 on its own grid (rows x page splits), one page per thread: the
// scores go to p.scores_out, which the selection launch then reads as its
// scores_in.  exp2 is monotonic, so the max over heads is taken on the
// normalised logits and exponentiated once per (token, slot).
__global__ void __launch_bounds__(kScoreThreads) aspire_page_scores_kernel(SelectParams p) {
  pdl_begin();
  __shared__ float lse_s[2][kMaxSelHeads];
  const int b = blockIdx.x;
  const int src_row = p.row_ids ? p.row_ids[b] : b;
  const int tid = threadIdx.x;
  const int pps = p.pages_per_slot;
  const int64_t max_q = p.lse_rows > 0 ? p.lse_rows - 1 : 0;
  int64_t q_first = p.qo_indptr[src_row];
  int64_t q_last = int64_t(p.qo_indptr[src_row + 1]) - 1;
  q_first = q_first < 0 ? 0 : (q_first > max_q ? max_q : q_first);
  q_last = q_last < 0 ? 0 : (q_last > max_q ? max_q : q_last);
  for (int h = tid; h < p.num_heads; h += blockDim.x) {
    lse_s[0][h] = p.lse[q_first * p.num_heads + h];
    lse_s[1][h] = p.lse[q_last * p.num_heads + h];
  }
  __syncthreads();
  const int pg = blockIdx.y * blockDim.x + tid;
  if (pg >= pps) return;
  float tok[kPageSize];
#pragma unroll
  for (int i = 0; i < kPageSize; ++i) tok[i] = 0.f;
  const int64_t t0 = int64_t(pg) * kPageSize;
  if (t0 < p.max_seq_len) {
    float mx[2][kPageSize];
#pragma unroll
    for (int s = 0; s < 2; ++s)
#pragma unroll
      for (int i = 0; i < kPageSize; ++i) mx[s][i] = -INFINITY;
    const bool full = t0 + kPageSize <= p.max_seq_len;
    const __half* row = p.dump + int64_t(src_row) * p.num_heads * 2 * p.kv_stride + t0;
    const bool vec = full && ((reinterpret_cast<uintptr_t>(row) | uintptr_t(p.kv_stride * 2)) & 15) == 0;
    for (int h = 0; h < p.num_heads; ++h) {
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const __half* src = row + (int64_t(h) * 2 + s) * p.kv_stride;
        const float ls = lse_s[s][h];
        __half2 vals[kPageSize / 2];
        if (vec) {
          *reinterpret_cast<uint4*>(vals) = __ldcs(reinterpret_cast<const uint4*>(src));
          *reinterpret_cast<uint4*>(vals + 4) = __ldcs(reinterpret_cast<const uint4*>(src) + 1);
        } else {
#pragma unroll
          for (int i = 0; i < kPageSize / 2; ++i) {
            const __half lo = (t0 + 2 * i < p.max_seq_len) ? src[2 * i] : __float2half_rn(-INFINITY);
            const __half hi = (t0 + 2 * i + 1 < p.max_seq_len) ? src[2 * i + 1] : __float2half_rn(-INFINITY);
            vals[i] = __halves2half2(lo, hi);
          }
        }
#pragma unroll
        for (int i = 0; i < kPageSize / 2; ++i) {
          // fp16 * scalar is computed in fp32 and rounded back to fp16.
          const float2 f = __half22float2(vals[i]);
          const float2 r = __half22float2(__floats2half2_rn(f.x * p.scale_log2, f.y * p.scale_log2));
          float n0 = r.x - ls, n1 = r.y - ls;
          if (isnan(n0)) n0 = -INFINITY;
          if (isnan(n1)) n1 = -INFINITY;
          mx[s][2 * i] = fmaxf(mx[s][2 * i], n0);
          mx[s][2 * i + 1] = fmaxf(mx[s][2 * i + 1], n1);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < kPageSize; ++i)
      tok[i] = (t0 + i < p.max_seq_len) ? (exp2f(mx[0][i]) + exp2f(mx[1][i])) : 0.f;
  }
  // Pairwise sum of the 16 token scores.
#pragma unroll
  for (int w = kPageSize / 2; w >= 1; w >>= 1)
#pragma unroll
    for (int i = 0; i < w; ++i) tok[i] = tok[i] + tok[i + w];
  p.scores_out[int64_t(b) * pps + pg] = tok[0] + (-(float(pg) * 1e-7f));
}

__global__ void __launch_bounds__(kSelThreads) aspire_select_pages_kernel(SelectParams p) {
  pdl_begin();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int pps = p.pages_per_slot;
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem_raw);         // [pps]
  int32_t* sortbuf = reinterpret_cast<int32_t*>(keys + pps);      // [sort_cap]
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sh_prefix, sh_remaining;
  __shared__ int sh_count;
  __shared__ int scan_buf[kSelThreads];

  const int b = blockIdx.x;  // output row
  const int tid = threadIdx.x;
  const int np = p.num_pages[b];

  // ---------------- Phase 1: the row's page scores (from aspire_page_scores_kernel
  // or the caller), forced and turned into order-preserving keys ----------------
  // Recent-page seeding (order_by_page) ranks pages by the given scores
  // alone: no forced trailing pages.
  const int last_start = p.order_by_page ? np : max(np - p.L, 0);
  for (int pg = tid; pg < pps; pg += blockDim.x) {
    float score = p.scores_in[int64_t(b) * pps + pg];
    if (p.scores_out) p.scores_out[int64_t(b) * pps + pg] = score;
    if (pg >= last_start && pg < np) score = INFINITY;
    if (pg >= np) score = -INFINITY;
    keys[pg] = order_key(score);
  }
  __syncthreads();

  // ---------------- Phase 2: radix select of the top `valid` keys ----------------
  // The reference keeps min(valid, k) of its top-k columns and reports
  // `valid` itself as the row's count (which may exceed k).
  const int reported = valid_count(p, np);
  const int valid = min(min(reported, p.subset_cache_size), pps);
  if (tid == 0) {
    sh_prefix = 0;
    sh_remaining = static_cast<uint32_t>(valid);
  }
  __syncthreads();
  for (int pass = 0; pass < 4 && valid > 0; ++pass) {
    const int shift = 24 - 8 * pass;
    const uint32_t hi_mask = pass == 0 ? 0u : (0xffffffffu << (32 - 8 * pass));
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = sh_prefix;
    for (int pg = tid; pg < pps; pg += blockDim.x) {
      const uint32_t k = keys[pg];
      if ((k & hi_mask) == prefix) atomicAdd(&hist[(k >> shift) & 0xff], 1u);
    }
    __syncthreads();
    if (tid < 32) {
      // Suffix sums from digit 255 downwards, 8 bins per lane.
      uint32_t local[8];
      uint32_t lane_sum = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        local[i] = hist[255 - (tid * 8 + i)];
        lane_sum += local[i];
      }
      uint32_t incl = lane_sum;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, incl, off);
        if (tid >= off) incl += v;
      }
      uint32_t run = incl - lane_sum;  // count of keys with larger digit than this lane's bins
      const uint32_t rem = sh_remaining;
      int found = -1;
      uint32_t above = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (found < 0 && run < rem && run + local[i] >= rem) {
          found = 255 - (tid * 8 + i);
          above = run;
        }
        run += local[i];
      }
      const unsigned ballot = __ballot_sync(0xffffffffu, found >= 0);
      const int src = ballot ? __ffs(ballot) - 1 : 0;
      const int digit = __shfl_sync(0xffffffffu, found, src);
      const uint32_t ab = __shfl_sync(0xffffffffu, above, src);
      if (tid == 0) {
        sh_prefix = prefix | (uint32_t(digit) << shift);
        sh_remaining = rem - ab;
      }
    }
    __syncthreads();
  }
  // Threshold key T = sh_prefix; `need` = sh_remaining keys equal to T are taken
  // in ascending page order, every key > T is taken.
  const uint32_t T = sh_prefix;
  const uint32_t need = sh_remaining;

  // Index-ordered pick: thread t scans a contiguous index range.
  const int per = (pps + blockDim.x - 1) / blockDim.x;
  const int i0 = min(tid * per, pps), i1 = min(i0 + per, pps);
  int eq_local = 0;
  if (valid > 0)
    for (int i = i0; i < i1; ++i) eq_local += (keys[i] == T);
  scan_buf[tid] = eq_local;
  if (tid == 0) sh_count = 0;
  __syncthreads();
  // Exclusive scan of eq counts (Hillis-Steele over kSelThreads entries).
  for (int off = 1; off < kSelThreads; off <<= 1) {
    const int v = (tid >= off) ? scan_buf[tid - off] : 0;
    __syncthreads();
    scan_buf[tid] += v;
    __syncthreads();
  }
  int eq_before = scan_buf[tid] - eq_local;
  const int32_t* bt = p.block_table + int64_t(b) * p.block_table_stride;
  if (valid > 0) {
    for (int i = i0; i < i1; ++i) {
      const uint32_t k = keys[i];
      bool take = k > T;
      if (k == T) {
        take = uint32_t(eq_before) < need;
        ++eq_before;
      }
      if (take) {
        const int slot = atomicAdd(&sh_count, 1);
        if (slot < p.sort_cap) sortbuf[slot] = p.order_by_page ? i : bt[min(i, p.block_table_cols - 1)];
      }
    }
  }
  __syncthreads();
  const int count = min(sh_count, valid);
  if (tid == 0 && sh_count != valid && p.status) atomicOr(p.status, ASPIRE_STATUS_BAD_ROW);

  // ---------------- Phase 3: ascending sort of the selected ids ----------------
  int n2 = 1;
  while (n2 < count) n2 <<= 1;
  for (int i = count + tid; i < n2; i += blockDim.x) sortbuf[i] = INT32_MAX;
  __syncthreads();
  for (int size = 2; size <= n2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < n2; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;
          const int a = sortbuf[i], c = sortbuf[j];
          if ((a > c) == up) {
            sortbuf[i] = c;
            sortbuf[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  int32_t* row_out = p.table_out + int64_t(b) * p.table_stride;
  for (int c = tid; c < p.table_width; c += blockDim.x) {
    int32_t v = 0;
    if (c < count && c < p.subset_cache_size)
      v = p.order_by_page ? bt[min(sortbuf[c], p.block_table_cols - 1)] : sortbuf[c];
    row_out[c] = v;
  }
  if (tid == 0) p.counts_out[b] = reported;
}

size_t select_smem_bytes(int pages_per_slot, int sort_cap) {
  return size_t(pages_per_slot) * 4 + size_t(sort_cap) * 4;
}

}  // namespace aspire
