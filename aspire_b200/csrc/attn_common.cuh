// Device helpers shared by the two attention kernels: parameters, plan
// access, fast exp2/log2, bf16 unpacking and the split-KV merge.
#pragma once

#include "common.cuh"

namespace aspire {

struct AttnParams {
  const __nv_bfloat16* q;
  int64_t q_stride_n, q_stride_h;
  const __nv_bfloat16* kv;
  int64_t num_pages_total;
  const int32_t* kv_indices;  // flat page list, or NULL for the page tables below
  const int32_t* mode_flags;  // page tables: draft rows (mode 0) read draft_table,
  const int32_t* draft_table; // the others block_table
  int64_t draft_stride;
  const int32_t* block_table;
  int64_t block_table_stride;
  __nv_bfloat16* out;
  int64_t o_stride_n, o_stride_h;
  float* lse;                // optional
  void* dump;                // optional logit dump (dump_kind, dump_f32)
  int64_t dump_num_heads, dump_kv_stride;
  int32_t dump_kind;         // ASPIRE_DUMP_FIRST_LAST or ASPIRE_DUMP_LAST_TOKEN
  int32_t dump_f32;          // 1: fp32 elements holding the fp16-rounded logit
  const int32_t* dump_flags; // optional per-row enable (row dumps iff flag != 0)
  float scale_log2;          // sm_scale * log2(e)
  int32_t num_qo_heads, num_kv_heads, group;
  int32_t q_box_tokens;      // tokens per query-tile TMA box (tcgen05 kernel, decode phase)
  int32_t pf_box_tokens;     // the same for the prefill phase
  int64_t q_rows;            // rows of q and out: plan rows past them are skipped (BAD_ROW)
  const int32_t* plan;       // int workspace + kStatusBytes
  uint32_t* status;          // int workspace (first word)
  float* partial_o;          // float workspace
  uint64_t wait_ns;          // bound of one pipeline wait of the tcgen05 kernel (ns)
  // Optional fused KV append (decode items of the tcgen05 kernel): the rows'
  // new K / V tokens, bf16 [tokens, num_kv_heads, 128] with these strides.
  const __nv_bfloat16* k_new;
  const __nv_bfloat16* v_new;
  int64_t k_new_stride_n, k_new_stride_h, v_new_stride_n, v_new_stride_h;
};

// Page id of logical page lp of a row: from the flat page list at the row's
// base, or from the row's draft / block table by its mode flag.
__device__ __forceinline__ int32_t row_page(const int32_t* kv_indices, int64_t page_base, const int32_t* mode_flags,
                                            const int32_t* draft_table, int64_t draft_stride,
                                            const int32_t* block_table, int64_t block_table_stride, int row,
                                            int64_t lp) {
  if (kv_indices) return __ldg(kv_indices + page_base + lp);
  return __ldg(mode_flags + row) == 0 ? __ldg(draft_table + row * draft_stride + lp)
                                      : __ldg(block_table + row * block_table_stride + lp);
}

// Logit dump of the chosen queries (raw q.k before scale and mask, rounded to
// fp16), the LogitsTransform bodies of aspire/backends/jit_kernels.py:180-203:
// first/last writes query 0 to slot 0 and query q_len-1 (q_len > 1) to slot 1
// of [batch, heads, 2, stride]; last-token writes query q_len-1 (q_len >= 1)
// to [batch, heads, stride].  With dump_flags a row writes only when its flag
// is set.
__device__ __forceinline__ bool dump_row_on(const AttnParams& p, int row) {
  return p.dump != nullptr && (p.dump_flags == nullptr || p.dump_flags[row] != 0);
}
__device__ __forceinline__ bool dump_has_first(const AttnParams& p) { return p.dump_kind == ASPIRE_DUMP_FIRST_LAST; }
__device__ __forceinline__ bool dump_has_last(const AttnParams& p, int q_len) {
  return p.dump_kind == ASPIRE_DUMP_LAST_TOKEN || q_len > 1;
}
// Elements between consecutive heads of the dump.
__device__ __forceinline__ int64_t dump_head_stride(const AttnParams& p) {
  return p.dump_kind == ASPIRE_DUMP_LAST_TOKEN ? p.dump_kv_stride : 2 * p.dump_kv_stride;
}
// Element index of token 0 of (row, head) for the first (last = false) or the
// last query.
__device__ __forceinline__ int64_t dump_index(const AttnParams& p, int row, int64_t head, bool last) {
  return (int64_t(row) * p.dump_num_heads + head) * dump_head_stride(p) +
         (last && p.dump_kind == ASPIRE_DUMP_FIRST_LAST ? p.dump_kv_stride : 0);
}
__device__ __forceinline__ void dump_store(const AttnParams& p, int64_t idx, float logit) {
  const __half h = __float2half_rn(logit);
  if (p.dump_f32)
    static_cast<float*>(p.dump)[idx] = __half2float(h);
  else
    static_cast<__half*>(p.dump)[idx] = h;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4 u, float* f) {
  f[0] = __uint_as_float(u.x << 16);
  f[1] = __uint_as_float(u.x & 0xffff0000u);
  f[2] = __uint_as_float(u.y << 16);
  f[3] = __uint_as_float(u.y & 0xffff0000u);
  f[4] = __uint_as_float(u.z << 16);
  f[5] = __uint_as_float(u.z & 0xffff0000u);
  f[6] = __uint_as_float(u.w << 16);
  f[7] = __uint_as_float(u.w & 0xffff0000u);
}

__device__ __forceinline__ WorkItem load_item(const int32_t* plan, int idx) {
  const int4* src = reinterpret_cast<const int4*>(plan + plan[kHdrOffItems]) + idx * 4;
  WorkItem it;
  int4* dst = reinterpret_cast<int4*>(&it);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = src[i];
  return it;
}

__device__ __forceinline__ float* partial_lse_ptr(const AttnParams& p) {
  const int64_t off = (int64_t(uint32_t(p.plan[kHdrPartialLseLo]))) |
                      (int64_t(p.plan[kHdrPartialLseHi]) << 32);
  return p.partial_o + off;
}

__device__ __forceinline__ void record_status(uint32_t* status, uint32_t bits) {
  if (status) atomicOr(status, bits);
}

// Location of packed query row `pq` of an item: token row and query head.
__device__ __forceinline__ void packed_row(const AttnParams& p, const WorkItem& it, int pq,
                                           int& q_idx, int& head) {
  q_idx = pq / p.group;
  head = it.kv_head * p.group + (pq - q_idx * p.group);
}

// Writes one finished (normalised) output row element and its LSE.
__device__ __forceinline__ void store_final(const AttnParams& p, const WorkItem& it, int pq, int d,
                                            float o, float lse) {
  int q_idx, head;
  packed_row(p, it, pq, q_idx, head);
  const int64_t tok = int64_t(it.q_start) + q_idx;
  if (tok >= p.q_rows) {
    if (d == 0) record_status(p.status, ASPIRE_STATUS_BAD_ROW);
    return;
  }
  p.out[tok * p.o_stride_n + int64_t(head) * p.o_stride_h + d] = __float2bfloat16_rn(o);
  if (d == 0 && p.lse) p.lse[tok * p.num_qo_heads + head] = lse;
}

// Epilogue of one item, run by all `nthreads` threads of the CTA once the
// normalised rows (get_o(r, d), get_lse(r)) of this chunk are available.
// Items that own their whole KV range write through; chunked items write an
// fp32 partial (normalised O and LSE), combined later by the merge kernel.
template <typename GetO, typename GetLse>
__device__ __forceinline__ void finish_item(const AttnParams& p, const WorkItem& it, int tid,
                                            int nthreads, GetO get_o, GetLse get_lse) {
  const int nrows = it.pq_end - it.pq_begin;
  if (it.n_chunks <= 1) {
    for (int e = tid; e < nrows * kHeadDim; e += nthreads) {
      const int r = e / kHeadDim, d = e - r * kHeadDim;
      store_final(p, it, it.pq_begin + r, d, get_o(r, d), get_lse(r));
    }
    return;
  }
  float* plse = partial_lse_ptr(p);
  const int64_t base = int64_t(it.partial_base) + int64_t(it.chunk) * nrows;
  for (int e = tid; e < nrows * kHeadDim; e += nthreads) {
    const int r = e / kHeadDim, d = e - r * kHeadDim;
    p.partial_o[(base + r) * kHeadDim + d] = get_o(r, d);
    if (d == 0) plse[base + r] = get_lse(r);
  }
}

}  // namespace aspire
