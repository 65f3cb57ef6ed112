// Refresh-layer page scoring + block radix top-k page re-selection.
//
// Phase 1 (its own launch over rows x page splits) turns the logit dump of
// the refresh layer into fp32 page scores, restating
// PageSelectorFirstLastAvg._select_first_last_impl
// (aspire/backends/page_selector.py:163-181) for a first/last dump:
//   norm  = float(half(float(logit) * sm_scale*log2e)) - lse      (NaN -> -inf)
//   tok   = max_h exp2(norm[slot 0]) + max_h exp2(norm[slot 1])
//   score = sum of the 16 token scores of the page + (-page * 1e-7)
// and PageSelector._select_impl (:110-130, select :140-146) for a last-token
// dump (one slot, normalised by the last query's LSE: tok = max_h
// exp2(norm)); with an fp32 dump the product stays fp32.  Tokens past
// max_seq_len count as zero.  One CTA per request row
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

// The 16 raw logits of one page of one (head, slot) dump row, as fp32;
// positions at or past max_seq_len read -inf.
__device__ __forceinline__ void load_page_logits(const __half* src, bool vec, int64_t t0, int64_t max_seq_len,
                                                 float* v) {
  __half2 h[kPageSize / 2];
  if (vec) {
    *reinterpret_cast<uint4*>(h) = __ldcs(reinterpret_cast<const uint4*>(src));
    *reinterpret_cast<uint4*>(h + 4) = __ldcs(reinterpret_cast<const uint4*>(src) + 1);
  } else {
#pragma unroll
    for (int i = 0; i < kPageSize / 2; ++i) {
      const __half lo = (t0 + 2 * i < max_seq_len) ? src[2 * i] : __float2half_rn(-INFINITY);
      const __half hi = (t0 + 2 * i + 1 < max_seq_len) ? src[2 * i + 1] : __float2half_rn(-INFINITY);
      h[i] = __halves2half2(lo, hi);
    }
  }
#pragma unroll
  for (int i = 0; i < kPageSize / 2; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load_page_logits(const float* src, bool vec, int64_t t0, int64_t max_seq_len,
                                                 float* v) {
  if (vec) {
#pragma unroll
    for (int i = 0; i < kPageSize / 4; ++i) *reinterpret_cast<float4*>(v + 4 * i) = __ldcs(reinterpret_cast<const float4*>(src) + i);
  } else {
#pragma unroll
    for (int i = 0; i < kPageSize; ++i) v[i] = (t0 + i < max_seq_len) ? src[i] : -INFINITY;
  }
}
// logit * sm_scale*log2(e) in the dump's own type, two at a time: an fp16
// tensor times a scalar is computed in fp32 and rounded back to fp16; an fp32
// one stays fp32.
__device__ __forceinline__ float2 scaled_logits(float a, float b, float scale, const __half*) {
  return __half22float2(__floats2half2_rn(a * scale, b * scale));
}
__device__ __forceinline__ float2 scaled_logits(float a, float b, float scale, const float*) {
  return make_float2(a * scale, b * scale);
}

// Token scores of page pg of one row: tok[t] = sum over the dump's slots of
// max_h exp2(norm), norm = scaled_logit - lse (NaN -> -inf); zero past
// max_seq_len.  exp2 is monotonic, so the max over heads is taken on the
// normalised logits and exponentiated once per (token, slot).
template <typename T, int kSlots>
__device__ __forceinline__ void page_token_scores(const SelectParams& p, const float (*lse_s)[kMaxSelHeads],
                                                  int src_row, int pg, float* tok) {
#pragma unroll
  for (int i = 0; i < kPageSize; ++i) tok[i] = 0.f;
  const int64_t t0 = int64_t(pg) * kPageSize;
  if (t0 >= p.max_seq_len) return;
  float mx[kSlots][kPageSize];
#pragma unroll
  for (int s = 0; s < kSlots; ++s)
#pragma unroll
    for (int i = 0; i < kPageSize; ++i) mx[s][i] = -INFINITY;
  const bool full = t0 + kPageSize <= p.max_seq_len;
  const T* row = static_cast<const T*>(p.dump) + int64_t(src_row) * p.num_heads * kSlots * p.kv_stride + t0;
  const bool vec =
      full && ((reinterpret_cast<uintptr_t>(row) | uintptr_t(p.kv_stride * int64_t(sizeof(T)))) & 15) == 0;
  for (int h = 0; h < p.num_heads; ++h) {
#pragma unroll
    for (int s = 0; s < kSlots; ++s) {
      const T* src = row + (int64_t(h) * kSlots + s) * p.kv_stride;
      // Slot 0 of a first/last dump is normalised by the first query's LSE;
      // the last-query slot by the last query's.
      const float ls = lse_s[kSlots == 2 ? s : 1][h];
      float v[kPageSize];
      load_page_logits(src, vec, t0, p.max_seq_len, v);
      // NaN (a -inf logit under a -inf LSE) counts as -inf: fmaxf returns
      // its other operand for a NaN, and every maximum starts at -inf.
#pragma unroll
      for (int i = 0; i < kPageSize; i += 2) {
        const float2 r = scaled_logits(v[i], v[i + 1], p.scale_log2, src);
        mx[s][i] = fmaxf(mx[s][i], r.x - ls);
        mx[s][i + 1] = fmaxf(mx[s][i + 1], r.y - ls);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kPageSize; ++i) {
    float t = 0.f;
#pragma unroll
    for (int s = 0; s < kSlots; ++s) t = (s == 0) ? exp2f(mx[0][i]) : t + exp2f(mx[s][i]);
    tok[i] = (t0 + i < p.max_seq_len) ? t : 0.f;
  }
}

// Phase 1 on its own grid (rows x page splits), one page per thread: the
// scores go to p.scores_out, which the selection launch then reads as its
// scores_in.
__global__ void __launch_bounds__(kScoreThreads, 8) aspire_page_scores_kernel(SelectParams p) {
  // The selection launch that follows is released only after this CTA's
  // scores are stored (or it has no page): released at the start, its
  // waiting CTAs took SM slots from the scoring CTAs.
  pdl_wait();
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
  if (p.dump_f32) {
    if (p.dump_slots == 1)
      page_token_scores<float, 1>(p, lse_s, src_row, pg, tok);
    else
      page_token_scores<float, 2>(p, lse_s, src_row, pg, tok);
  } else {
    if (p.dump_slots == 1)
      page_token_scores<__half, 1>(p, lse_s, src_row, pg, tok);
    else
      page_token_scores<__half, 2>(p, lse_s, src_row, pg, tok);
  }
  // Pairwise sum of the 16 token scores.
#pragma unroll
  for (int w = kPageSize / 2; w >= 1; w >>= 1)
#pragma unroll
    for (int i = 0; i < w; ++i) tok[i] = tok[i] + tok[i + w];
  p.scores_out[int64_t(b) * pps + pg] = tok[0] + (-(float(pg) * 1e-7f));
  pdl_launch_dependents();
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
  __shared__ int scan_buf[kSelThreads / 32];

  const int b = blockIdx.x;  // output row
  const int tid = threadIdx.x;
  const int np = p.num_pages[b];

  // ---------------- Phase 1: the row's page scores (from aspire_page_scores_kernel
  // or the caller), forced and turned into order-preserving keys ----------------
  // Recent-page seeding (order_by_page) ranks pages by the given scores
  // alone: no forced trailing pages.
  const int last_start = p.order_by_page ? np : max(np - p.L, 0);
  // Four scores per thread in flight at a time (one round trip instead of four).
  constexpr int kLoadBatch = 4;
  for (int pg0 = tid; pg0 < pps; pg0 += kLoadBatch * blockDim.x) {
    float sc[kLoadBatch];
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int pg = pg0 + u * blockDim.x;
      sc[u] = pg < pps ? p.scores_in[int64_t(b) * pps + pg] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int pg = pg0 + u * blockDim.x;
      if (pg >= pps) break;
      float score = sc[u];
      if (p.scores_out) p.scores_out[int64_t(b) * pps + pg] = score;
      if (pg >= last_start && pg < np) score = INFINITY;
      if (pg >= np) score = -INFINITY;
      keys[pg] = order_key(score);
    }
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
  if (tid == 0) sh_count = 0;
  // Exclusive scan of eq counts: within each warp by shuffles, then over the
  // warp totals.
  const int lane = tid & 31, warp = tid >> 5;
  int incl = eq_local;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += v;
  }
  if (lane == 31) scan_buf[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    constexpr int kWarps = kSelThreads / 32;
    int w = lane < kWarps ? scan_buf[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += v;
    }
    if (lane < kWarps) scan_buf[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  int eq_before = (warp > 0 ? scan_buf[warp - 1] : 0) + incl - eq_local;
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

  // ---------------- Phase 3: ascending order of the selected ids ----------------
  // Each selected id goes straight to its rank (the ids below it plus the
  // equal ids picked before it): one pass over at most k ids per id, no
  // sorting network.  The tail of the row is zero.
  int32_t* row_out = p.table_out + int64_t(b) * p.table_stride;
  const int width = min(p.table_width, p.subset_cache_size);
  for (int j = tid; j < count; j += blockDim.x) {
    const int x = sortbuf[j];
    int r = 0;
    for (int i = 0; i < count; ++i) {
      const int y = sortbuf[i];
      r += (y < x) || (y == x && i < j);
    }
    if (r < width) row_out[r] = p.order_by_page ? bt[min(x, p.block_table_cols - 1)] : x;
  }
  for (int c = count + tid; c < p.table_width; c += blockDim.x) row_out[c] = 0;
  if (tid == 0) p.counts_out[b] = reported;
}

size_t select_smem_bytes(int pages_per_slot, int sort_cap) {
  return size_t(pages_per_slot) * 4 + size_t(sort_cap) * 4;
}

}  // namespace aspire
