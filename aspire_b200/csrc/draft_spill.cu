// Draft-page spill insert: one thread per request row.
//
// A draft step appends its token through the row's sparse draft table, whose
// last listed page must therefore be the page that holds the token.  When the
// token is the first of a new page, that page is appended to the table
// (LMBackendBase.prepare_forward_inputs, aspire/backends/base.py:1222-1236,
// and _handle_draft_page_spill, :718-742).  The reference computes the mask
// with several torch operations and synchronises the host on need_spill.any()
// before the insert; here the check and the insert are one launch.
//
// The entry point of the cleared slots' dump-state reset (kernel in
// dump_state.cu) sits here too, with the other slot-bookkeeping launch.
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

extern "C" int aspire_clear_dump_slots(const AspireClearDumpArgs* a, void* stream) {
  clear_error();
  if (!a) return set_error(ASPIRE_ERR_INVALID, "aspire_clear_dump_slots: null argument");
  if (a->n_slots < 0) return set_error(ASPIRE_ERR_INVALID, "aspire_clear_dump_slots: negative n_slots");
  if (a->n_slots == 0) return ASPIRE_OK;
  if (!a->dump || !a->slot_ids) return set_error(ASPIRE_ERR_INVALID, "aspire_clear_dump_slots: null pointer");
  if (a->dump_dtype != ASPIRE_DUMP_F16 && a->dump_dtype != ASPIRE_DUMP_F32)
    return set_error(ASPIRE_ERR_INVALID, "aspire_clear_dump_slots: bad dump_dtype");
  if (a->num_heads <= 0 || (a->slots != 1 && a->slots != 2) || a->kv_stride <= 0 || a->dump_rows <= 0)
    return set_error(ASPIRE_ERR_INVALID, "aspire_clear_dump_slots: bad dump geometry");
  if (reinterpret_cast<uintptr_t>(a->dump) & (a->dump_dtype == ASPIRE_DUMP_F32 ? 3 : 1))
    return set_error(ASPIRE_ERR_INVALID, "aspire_clear_dump_slots: dump not aligned to its element type");
  if (a->lse && (!a->qo_indptr || a->lse_rows <= 0 || a->qo_len <= 0))
    return set_error(ASPIRE_ERR_INVALID, "aspire_clear_dump_slots: lse needs qo_indptr, lse_rows and qo_len");
  ClearDumpParams p;
  p.dump = a->dump;
  p.dump_f32 = a->dump_dtype == ASPIRE_DUMP_F32 ? 1 : 0;
  p.row_elems = int64_t(a->num_heads) * a->slots * a->kv_stride;
  p.dump_rows = a->dump_rows;
  p.slot_ids = a->slot_ids;
  p.lse = a->lse;
  p.lse_rows = a->lse_rows;
  p.num_heads = a->num_heads;
  p.qo_indptr = a->qo_indptr;
  p.qo_len = a->qo_len;
  p.mode_flags = a->mode_flags;
  p.mode_value = a->mode_value;
  p.status = a->status;
  const int64_t pieces = (p.row_elems + kClearPieceElems - 1) / kClearPieceElems;
  if (pieces > 65535) return set_error(ASPIRE_ERR_CAPACITY, "aspire_clear_dump_slots: dump rows too long");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a->n_slots), static_cast<unsigned>(pieces));
  cfg.blockDim = dim3(kClearThreads);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, aspire_clear_dump_kernel, p), "aspire_clear_dump_kernel launch");
}
