// Mixed page-list build: each request row's attended pages are copied into one
// flat list, from the row's draft table (draft rows) or its block-table prefix
// (verify rows), with the list offsets as an exclusive prefix sum.
//
// Same result as the reference's build_unified_indices
// (aspire/models/sparse_draft_runner.py:126-153: indptr = cumsum of
// where(mode == DRAFT_MODE, draft_num_pages, verify_num_pages), then the
// Triton _copy_indices_kernel, :93-123).  One CTA per row: it sums the page
// counts of the rows before it (B is at most a few hundred), writes its own
// offset and copies its pages with 16-byte vector accesses when aligned; no
// second launch is needed for the prefix sum.
#include "kernels.cuh"

namespace aspire {

__global__ void __launch_bounds__(kIndicesThreads) aspire_build_indices_kernel(IndicesParams p) {
  pdl_begin();
  const int b = blockIdx.x;
  const int tid = threadIdx.x;
  __shared__ int64_t partial[kIndicesThreads];
  // A negative count (a malformed row) counts as 0.
  auto count_of = [&](int r) -> int64_t {
    const int32_t c = p.mode_flags[r] == 0 ? p.draft_num_pages[r] : p.verify_num_pages[r];
    return c > 0 ? c : 0;
  };
  int64_t acc = 0;
  for (int r = tid; r < b; r += blockDim.x) acc += count_of(r);
  partial[tid] = acc;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if (tid < s) partial[tid] += partial[tid + s];
    __syncthreads();
  }
  const int64_t start = partial[0];
  const int64_t n = count_of(b);
  if (tid == 0) {
    if (b == 0) p.indptr_out[0] = 0;
    p.indptr_out[b + 1] = static_cast<int32_t>(start + n);
    const int32_t raw = p.mode_flags[b] == 0 ? p.draft_num_pages[b] : p.verify_num_pages[b];
    if (raw < 0 && p.status) atomicOr(p.status, ASPIRE_STATUS_BAD_ROW);
  }
  if (n <= 0) return;
  const bool draft = p.mode_flags[b] == 0;
  const int32_t* src = draft ? p.draft_indices + int64_t(b) * p.draft_stride
                             : p.verify_indices + int64_t(b) * p.verify_stride;
  const int64_t cap = draft ? p.draft_cols : p.verify_cols;
  // A count past the table width copies the table; pages past the output's
  // capacity are not written.
  const int64_t room = p.indices_capacity - start;
  int64_t m = n < cap ? n : cap;
  m = m < room ? m : (room > 0 ? room : 0);
  if (m < n && tid == 0 && p.status) atomicOr(p.status, ASPIRE_STATUS_BAD_ROW);
  if (m <= 0) return;
  int32_t* dst = p.indices_out + start;
  const bool vec = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0;
  const int mi = static_cast<int>(m);
  if (vec) {
    const int nv = mi / 4;
    for (int i = tid; i < nv; i += blockDim.x)
      reinterpret_cast<int4*>(dst)[i] = __ldg(reinterpret_cast<const int4*>(src) + i);
    for (int i = nv * 4 + tid; i < mi; i += blockDim.x) dst[i] = __ldg(src + i);
  } else {
    for (int i = tid; i < mi; i += blockDim.x) dst[i] = __ldg(src + i);
  }
}

}  // namespace aspire
