// Fused attention prologue of one layer: q/k RMSNorm (per head), the
// HF-to-interleaved permutation, interleaved RoPE, and the paged append of
// the rotated K and of V — one launch instead of the reference's three ops:
//
//   q = q_norm(q); k = k_norm(k); q, k = _permute_for_rope(q), _permute_for_rope(k)
//       (aspire/models/sparse_draft_transformer.py:150-158, transformer.py:360-364,505-515)
//   rope(q, k, kv_append_indptr, offsets)      FlashInfer apply_rope_inplace /
//       apply_llama31_rope_inplace with interleave=True (mixed_transformer.py:159-197)
//   update_kv_padded(k, v, ...)                 (kv_ops.py:127-187, as in append_kv.cu)
//
// RMSNorm follows the reference module: x * rsqrt(mean(x^2) + eps) in fp32,
// rounded to bf16, then times the bf16 weight (rounded to bf16).  The
// permutation sends element i of the first half to 2i and element 64+i to
// 2i+1.  RoPE rotates the pair (2p, 2p+1) by pos * freq_p with
// freq_p = theta^(-2p/128) (scaled, with the Llama-3.1 smoothing when set),
// pos = offsets[b] + (t - append_indptr[b]), using the fast powf / sincosf
// intrinsics as FlashInfer's kernel does.  Tokens after the last row (bucket
// padding) get the norm and permutation but no rotation and no append, as in
// the reference, where the norm runs over the whole tensor and the RoPE and
// the append over the rows.
//
// Grid (rows + 1, y): CTA (b, y) handles row b's (token, head slot) units
// y, y + Y, ... in its 8 warps; head slots are the Hq query heads, then the
// Hkv key heads, then the Hkv value heads.  Lane l owns dims 2l, 2l+1,
// 64+2l, 64+2l+1 of the input row, i.e. output dims 4l..4l+3 after the
// permutation, so loads and stores stay coalesced.
#include "kernels.cuh"

namespace aspire {

namespace {

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ float rope_freq(const PrologueParams& p, int pair) {
  float f = __powf(p.rcp_theta, float(2 * pair) / float(kHeadDim));
  float smooth = f * p.smooth_a + p.smooth_b;
  smooth = fmaxf(0.0f, fminf(1.0f, smooth));
  return (1 - smooth) * (f * p.rcp_scale) + smooth * f;
}

// Loads one head row (lane l: the dims it owns), applies the optional norm +
// permutation and the optional rotation; returns output dims 4l..4l+3.
__device__ __forceinline__ void transform_row(const PrologueParams& p, const __nv_bfloat16* src,
                                              const __nv_bfloat16* weight, bool rotate, int64_t pos, int lane,
                                              float out[4]) {
  float a0, a1, b0, b1;  // output pairs (a0, b0) -> dims 4l, 4l+1 and (a1, b1) -> 4l+2, 4l+3
  if (weight != nullptr) {
    const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(src + 2 * lane);
    const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(src + 64 + 2 * lane);
    const float x0 = __low2float(lo), x1 = __high2float(lo), x2 = __low2float(hi), x3 = __high2float(hi);
    float ss = x0 * x0 + x1 * x1 + x2 * x2 + x3 * x3;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float rms = rsqrtf(ss / float(kHeadDim) + p.eps);
    const __nv_bfloat162 wlo = *reinterpret_cast<const __nv_bfloat162*>(weight + 2 * lane);
    const __nv_bfloat162 whi = *reinterpret_cast<const __nv_bfloat162*>(weight + 64 + 2 * lane);
    a0 = bf16r(bf16r(x0 * rms) * __low2float(wlo));
    a1 = bf16r(bf16r(x1 * rms) * __high2float(wlo));
    b0 = bf16r(bf16r(x2 * rms) * __low2float(whi));
    b1 = bf16r(bf16r(x3 * rms) * __high2float(whi));
  } else {
    const uint2 raw = *reinterpret_cast<const uint2*>(src + 4 * lane);
    const __nv_bfloat162 u = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
    const __nv_bfloat162 w = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
    a0 = __low2float(u);
    b0 = __high2float(u);
    a1 = __low2float(w);
    b1 = __high2float(w);
  }
  if (rotate) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int pair = 2 * lane + k;
      const float embed = float(pos) * rope_freq(p, pair);
      float s, c;
      __sincosf(embed, &s, &c);
      float& e = k == 0 ? a0 : a1;
      float& o = k == 0 ? b0 : b1;
      const float ev = e, ov = o;
      e = ev * c + (-ov) * s;
      o = ov * c + ev * s;
    }
  }
  out[0] = a0;
  out[1] = b0;
  out[2] = a1;
  out[3] = b1;
}

__device__ __forceinline__ void store4(__nv_bfloat16* dst, const float v[4]) {
  __nv_bfloat162 x = __floats2bfloat162_rn(v[0], v[1]);
  __nv_bfloat162 y = __floats2bfloat162_rn(v[2], v[3]);
  uint2 raw;
  raw.x = *reinterpret_cast<uint32_t*>(&x);
  raw.y = *reinterpret_cast<uint32_t*>(&y);
  *reinterpret_cast<uint2*>(dst) = raw;
}

}  // namespace

__global__ void __launch_bounds__(256) aspire_qkv_prologue_kernel(PrologueParams p) {
  pdl_begin();
  const AppendParams& ap = p.ap;
  const int b = blockIdx.x;
  const bool tail = b == ap.num_rows;  // tokens after the last row: norm only
  const int32_t start = ap.append_indptr[b];
  const int32_t end = tail ? static_cast<int32_t>(ap.num_tokens) : ap.append_indptr[b + 1];
  const int32_t n = end - start;
  if (n <= 0) return;
  int32_t page_begin = 0, page_count = 0, seq_len = 0, rope_base = 0;
  if (!tail) {
    page_begin = ap.page_indptr[b];
    page_count = ap.page_indptr[b + 1] - page_begin;
    seq_len = page_count > 0 ? (page_count - 1) * kPageSize + ap.last_page_len[b] : 0;
    rope_base = p.rope_offsets[b];
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hq = p.num_qo_heads, hkv = ap.num_kv_heads;
  const int slots = tail ? hq : hq + 2 * hkv;
  const int64_t units = int64_t(n) * slots;
  const int64_t step = int64_t(gridDim.y) * (blockDim.x >> 5);
  for (int64_t e = int64_t(blockIdx.y) * (blockDim.x >> 5) + warp; e < units; e += step) {
    const int32_t i = static_cast<int32_t>(e / slots);
    const int s = static_cast<int>(e - int64_t(i) * slots);
    const int64_t t = int64_t(start) + i;
    if (t >= ap.num_tokens) break;
    const int64_t rope_pos = int64_t(rope_base) + i;
    if (s < hq) {
      float v[4];
      transform_row(p, p.q + t * p.q_stride_n + int64_t(s) * p.q_stride_h, p.q_norm_w, !tail, rope_pos, lane, v);
      store4(p.q_out + t * p.qo_stride_n + int64_t(s) * p.qo_stride_h + 4 * lane, v);
      continue;
    }
    // K or V row of head h: only tokens whose cache position exists are written.
    const bool is_k = s < hq + hkv;
    const int h = is_k ? s - hq : s - hq - hkv;
    if (page_count <= 0) continue;
    const int64_t pos = int64_t(i) + seq_len - n;
    if (pos < 0 || pos >= seq_len) continue;
    const int32_t page = row_page(ap.page_indices, page_begin, ap.mode_flags, ap.draft_table, ap.draft_stride,
                                  ap.block_table, ap.block_table_stride, b, pos / kPageSize);
    if (page < 0 || int64_t(page) >= ap.num_pages_total) {
      if (lane == 0 && ap.status) atomicOr(ap.status, ASPIRE_STATUS_BAD_PAGE);
      continue;
    }
    __nv_bfloat16* dst = ap.kv + ((int64_t(page) * 2 + (is_k ? 0 : 1)) * kPageSize + (pos % kPageSize)) *
                                     int64_t(hkv) * kHeadDim +
                         int64_t(h) * kHeadDim;
    if (is_k) {
      float v[4];
      transform_row(p, ap.k + t * ap.k_stride_n + int64_t(h) * ap.k_stride_h, p.k_norm_w, true, rope_pos, lane, v);
      store4(dst + 4 * lane, v);
    } else {
      const uint2 raw = *reinterpret_cast<const uint2*>(ap.v + t * ap.v_stride_n + int64_t(h) * ap.v_stride_h + 4 * lane);
      *reinterpret_cast<uint2*>(dst + 4 * lane) = raw;
    }
  }
}

}  // namespace aspire
