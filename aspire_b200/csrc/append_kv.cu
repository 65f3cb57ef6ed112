// Paged KV append: writes each new token's K and V rows into its page.
//
// Same addressing as the reference's mylib::update_kv_padded
// (aspire/attention/kv_ops.py:63-187) with FlashInfer's
// get_batch_indices_positions (flashinfer/triton/page.py) and get_seq_lens
// (flashinfer/page.py): token t of row b (append_indptr[b] <= t <
// append_indptr[b+1]) goes to position seq_len[b] - append_len[b] + i,
// where seq_len[b] = max(pages[b]-1, 0)*16 + last_page_len[b]; tokens with
// a negative position, rows without pages and positions past the row's
// length are skipped (bucket padding).  One warp moves one (token, KV head)
// at a time: lanes 0-15 copy the 256-byte K row, lanes 16-31 the V row, 16
// bytes each.
#include "kernels.cuh"

namespace aspire {


// Grid (rows, y): CTA (b, y) handles row b's (token, head) pairs y, y + Y, ...
// in its 8 warps, so the row's offsets and lengths are read once and nothing
// searches for a token's row (the reference's helper grids over rows too).
__global__ void __launch_bounds__(256) aspire_append_kv_kernel(AppendParams p) {
  pdl_begin();
  const int b = blockIdx.x;
  const int32_t start = p.append_indptr[b], end = p.append_indptr[b + 1];
  const int32_t page_begin = p.page_indptr[b];
  const int32_t page_count = p.page_indptr[b + 1] - page_begin;
  const int32_t last = p.last_page_len[b];
  const int32_t n = end - start;
  if (n <= 0 || page_count <= 0) return;
  const int32_t seq_len = (page_count - 1) * kPageSize + last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = p.num_kv_heads;
  const int which = lane >> 4;  // 0 = K, 1 = V
  const int col = (lane & 15) * 8;
  const int64_t pairs = int64_t(n) * heads;
  const int64_t step = int64_t(gridDim.y) * (blockDim.x >> 5);
  for (int64_t e = int64_t(blockIdx.y) * (blockDim.x >> 5) + warp; e < pairs; e += step) {
    const int32_t i = static_cast<int32_t>(e / heads);
    const int h = static_cast<int>(e - int64_t(i) * heads);
    const int64_t t = int64_t(start) + i;
    if (t >= p.num_tokens) break;
    const int64_t pos = int64_t(i) + seq_len - n;  // = t + seq_len - append_indptr[b + 1]
    if (pos < 0 || pos >= seq_len) continue;
    const int32_t page = row_page(p.page_indices, page_begin, p.mode_flags, p.draft_table, p.draft_stride,
                                  p.block_table, p.block_table_stride, b, pos / kPageSize);
    if (page < 0 || int64_t(page) >= p.num_pages_total) {
      if (lane == 0 && p.status) atomicOr(p.status, ASPIRE_STATUS_BAD_PAGE);
      continue;
    }
    const __nv_bfloat16* src = which == 0 ? p.k + t * p.k_stride_n + int64_t(h) * p.k_stride_h
                                          : p.v + t * p.v_stride_n + int64_t(h) * p.v_stride_h;
    const int64_t dst_off =
        ((int64_t(page) * 2 + which) * kPageSize + (pos % kPageSize)) * int64_t(heads) * kHeadDim +
        int64_t(h) * kHeadDim + col;
    *reinterpret_cast<uint4*>(p.kv + dst_off) = *reinterpret_cast<const uint4*>(src + col);
  }
}

}  // namespace aspire
