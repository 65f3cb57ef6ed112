// Slot-local dump state reset: the refilled slots' dump rows back to -inf,
// the LSE row of each slot's last query to 0 and its dump mode flag to a
// given value, in one launch.  Restates LMBackendBase._clear_variant_slot_state
// (aspire/backends/base.py:1404-1419), which the engine runs as three torch
// indexing ops whenever slots are cleared:
//   dump.view(B, H, slots, kv_stride)[slot_ids] = -inf
//   lse[(qo_indptr[slot_ids + 1] - 1).clamp(0, lse_rows - 1)] = 0
//   dump_mode_flags[slot_ids] = VERIFY_MODE
// The -inf fill matters for parity: a first/last dump row of a slot whose
// next verify has q_len == 1 keeps its slot 1 from the slot's previous
// request otherwise (the dump writes only the slots its queries reach).
//
// Grid (n_slots, row pieces): each CTA fills one piece of one slot's row with
// 16-byte stores when the row is 16-byte aligned; the first piece's CTA also
// clears the LSE row and sets the flag.  A slot id outside [0, dump_rows), or
// whose qo_indptr entry lies past qo_len, is skipped and reported as
// ASPIRE_STATUS_BAD_ROW.
#include "kernels.cuh"

namespace aspire {

__global__ void __launch_bounds__(kClearThreads) aspire_clear_dump_kernel(ClearDumpParams p) {
  pdl_begin();
  const int32_t s = p.slot_ids[blockIdx.x];
  if (s < 0 || int64_t(s) >= p.dump_rows) {
    if (blockIdx.y == 0 && threadIdx.x == 0) record_status(p.status, ASPIRE_STATUS_BAD_ROW);
    return;
  }
  // This CTA's piece of the row.
  const int64_t begin = int64_t(blockIdx.y) * kClearPieceElems;
  const int64_t end = begin + kClearPieceElems < p.row_elems ? begin + kClearPieceElems : p.row_elems;
  const int esize = p.dump_f32 ? 4 : 2;
  char* row = static_cast<char*>(p.dump) + int64_t(s) * p.row_elems * esize;
  const uint32_t word = p.dump_f32 ? 0xff800000u : 0xfc00fc00u;  // -inf as fp32, as two fp16
  const bool vec = ((reinterpret_cast<uintptr_t>(row) | uintptr_t(begin * esize) | uintptr_t(end * esize)) & 15) == 0;
  if (vec) {
    const uint4 v = make_uint4(word, word, word, word);
    uint4* dst = reinterpret_cast<uint4*>(row + begin * esize);
    const int64_t n = (end - begin) * esize / 16;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = v;
  } else if (p.dump_f32) {
    float* dst = reinterpret_cast<float*>(row);
    for (int64_t i = begin + threadIdx.x; i < end; i += blockDim.x) dst[i] = __uint_as_float(word);
  } else {
    __half* dst = reinterpret_cast<__half*>(row);
    const __half ninf = __ushort_as_half(static_cast<unsigned short>(word & 0xffffu));
    for (int64_t i = begin + threadIdx.x; i < end; i += blockDim.x) dst[i] = ninf;
  }
  if (blockIdx.y != 0) return;
  if (p.mode_flags && threadIdx.x == 0) p.mode_flags[s] = p.mode_value;
  if (p.lse) {
    if (int64_t(s) + 1 >= p.qo_len) {
      if (threadIdx.x == 0) record_status(p.status, ASPIRE_STATUS_BAD_ROW);
      return;
    }
    int64_t r = int64_t(p.qo_indptr[s + 1]) - 1;
    r = r < 0 ? 0 : (r > p.lse_rows - 1 ? p.lse_rows - 1 : r);
    for (int h = threadIdx.x; h < p.num_heads; h += blockDim.x) p.lse[r * p.num_heads + h] = 0.f;
  }
}

}  // namespace aspire
