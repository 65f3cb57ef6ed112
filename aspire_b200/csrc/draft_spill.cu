// Draft-page spill insert: one thread per request row.
//
// A draft step appends its token through the row's sparse draft table, whose
// last listed page must therefore be the page that holds the token.  When the
// token is the first of a new page, that page is appended to the table
// (LMBackendBase.prepare_forward_inputs, aspire/backends/base.py:1222-1236,
// and _handle_draft_page_spill, :718-742).  The reference computes the mask
// with several torch operations and synchronises the host on need_spill.any()
// before the insert; here the check and the insert are one launch.
#include "kernels.cuh"
#include "errors.h"

namespace aspire {

__global__ void aspire_draft_spill_kernel(SpillParams p) {
  pdl_begin();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= p.batch) return;
  if (p.mode_flags[b] != 0 || p.dec_lens[b] <= 0) return;  // verify or finished row
  const int32_t len = p.draft_cachelens[b];
  if (len <= 0 || (len - 1) % kPageSize != 0) return;       // the token did not open a page
  const int32_t needed = (len + kPageSize - 1) / kPageSize;
  const int32_t new_col = needed - 1;
  if (new_col >= p.block_table_cols) {
    record_status(p.status, ASPIRE_STATUS_BAD_ROW);
    return;
  }
  const int32_t new_page = p.block_table[int64_t(b) * p.block_table_stride + new_col];
  int32_t* row = p.draft_indices + int64_t(b) * p.draft_stride;
  const int32_t count = p.draft_num_pages[b];
  const int32_t tail_col = count > 0 ? count - 1 : 0;
  if (tail_col < p.draft_cols && row[tail_col] == new_page) return;  // already listed last
  if (count < 0 || count >= p.draft_cols) return;                      // no free column
  row[count] = new_page;
  p.draft_num_pages[b] = count + 1;
}

}  // namespace aspire

using namespace aspire;

extern "C" int aspire_draft_page_spill(const AspireSpillArgs* a, void* stream) {
  clear_error();
  if (!a) return set_error(ASPIRE_ERR_INVALID, "aspire_draft_page_spill: null argument");
  if (a->batch < 0) return set_error(ASPIRE_ERR_INVALID, "aspire_draft_page_spill: negative batch");
  if (a->batch == 0) return ASPIRE_OK;
  if (a->page_size != kPageSize) return set_error(ASPIRE_ERR_INVALID, "aspire_draft_page_spill: page_size must be 16");
  if (!a->mode_flags || !a->dec_lens || !a->draft_cachelens || !a->draft_indices || !a->draft_num_pages ||
      !a->block_table)
    return set_error(ASPIRE_ERR_INVALID, "aspire_draft_page_spill: null pointer");
  if (a->draft_cols <= 0 || a->draft_stride < a->draft_cols || a->block_table_cols <= 0 ||
      a->block_table_stride < a->block_table_cols)
    return set_error(ASPIRE_ERR_INVALID, "aspire_draft_page_spill: bad table geometry");
  SpillParams p;
  p.mode_flags = a->mode_flags;
  p.dec_lens = a->dec_lens;
  p.draft_cachelens = a->draft_cachelens;
  p.draft_indices = a->draft_indices;
  p.draft_stride = a->draft_stride;
  p.draft_cols = a->draft_cols;
  p.draft_num_pages = a->draft_num_pages;
  p.block_table = a->block_table;
  p.block_table_stride = a->block_table_stride;
  p.block_table_cols = a->block_table_cols;
  p.batch = a->batch;
  p.status = a->status;
  constexpr int kThreads = 128;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a->batch + kThreads - 1) / kThreads);
  cfg.blockDim = dim3(kThreads);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, aspire_draft_spill_kernel, p), "aspire_draft_spill_kernel launch");
}
