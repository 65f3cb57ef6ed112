// Paged KV append: writes each new token's K and V rows into its page.
//
// Same addressing as the reference's mylib::update_kv_padded
// (aspire/attention/kv_ops.py:63-187) with FlashInfer's
// get_batch_indices_positions (flashinfer/triton/page.py) and get_seq_lens
// (flashinfer/page.py): token t of row b (append_indptr[b] <= t <
// append_indptr[b+1]) goes to position seq_len[b] - append_len[b] + i,
// where seq_len[b] = max(pages[b]-1, 0)*16 + last_page_len[b]; tokens with
// a negative position, rows without pages and positions past the row's
// length are skipped (bucket padding).  One warp moves one (token, KV head):
// lanes 0-15 copy the 256-byte K row, lanes 16-31 the V row, 16 bytes each.
#include "kernels.cuh"

namespace aspire {


__global__ void __launch_bounds__(256) aspire_append_kv_kernel(AppendParams p) {
  const int64_t warp_id = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_id >= p.num_tokens * p.num_kv_heads) return;
  const int64_t t = warp_id / p.num_kv_heads;
  const int h = static_cast<int>(warp_id - t * p.num_kv_heads);

  // Last row b with append_indptr[b] <= t.
  int lo = 0, hi = p.num_rows - 1, b = -1;
  while (lo <= hi) {
    const int mid = (lo + hi) >> 1;
    if (int64_t(p.append_indptr[mid]) <= t) {
      b = mid;
      lo = mid + 1;
    } else {
      hi = mid - 1;
    }
  }
  if (b < 0) return;
  const int32_t end = p.append_indptr[b + 1];
  if (t >= end) return;
  const int32_t page_begin = p.page_indptr[b];
  const int32_t page_count = p.page_indptr[b + 1] - page_begin;
  if (page_count <= 0) return;
  const int32_t seq_len = (page_count - 1) * kPageSize + p.last_page_len[b];
  const int64_t pos = t + seq_len - end;
  if (pos < 0 || pos >= seq_len) return;
  const int32_t page = p.page_indices[page_begin + pos / kPageSize];
  if (page < 0 || int64_t(page) >= p.num_pages_total) {
    if (lane == 0 && p.status) atomicOr(p.status, ASPIRE_STATUS_BAD_PAGE);
    return;
  }
  const int which = lane >> 4;  // 0 = K, 1 = V
  const int col = (lane & 15) * 8;
  const __nv_bfloat16* src = which == 0 ? p.k + t * p.k_stride_n + int64_t(h) * p.k_stride_h
                                        : p.v + t * p.v_stride_n + int64_t(h) * p.v_stride_h;
  const int64_t dst_off =
      ((int64_t(page) * 2 + which) * kPageSize + (pos % kPageSize)) * int64_t(p.num_kv_heads) * kHeadDim +
      int64_t(h) * kHeadDim + col;
  *reinterpret_cast<uint4*>(p.kv + dst_off) = *reinterpret_cast<const uint4*>(src + col);
}

}  // namespace aspire
