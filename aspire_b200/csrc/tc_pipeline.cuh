// Pieces shared by the tcgen05 attention kernels (decode and prefill):
// bounded mbarrier waits, the run-time item sequence, the paged K/V TMA
// producers and the query-tile load.  A kernel's shared-memory struct
// provides the fields these templates name: abort_flag, the seq ring
// (seq, seq_full, seq_empty), q_full, the two 64-dim query halves q[0..1]
// and wait_ns (the bound of one pipeline wait, from the launch parameters).
#pragma once

#include <cuda.h>

#include "kernels.cuh"
#include "tc_ptx.cuh"

namespace aspire {
namespace pipe {

constexpr int kTile = 128;                          // KV tokens per tile
constexpr int kPagesPerTile = kTile / kPageSize;
constexpr uint32_t kHalfBytes = kTile * 128;        // 128 rows x 128 B (64 dims)
constexpr uint32_t kSlotBytes = 2 * kHalfBytes;     // one K or V tile: two 64-dim halves
constexpr uint64_t kDrainLimitNs = 1000000000ull;   // 1 s: bound of the waits of a stopping CTA
constexpr int kSeqDepth = 8;                        // item-sequence ring (claimed items in flight per CTA)

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

template <class Sh>
__device__ __forceinline__ bool aborted(Sh& sm) {
  return *reinterpret_cast<volatile int*>(&sm.abort_flag) != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and stops the CTA) when
// the phase does not complete within sm.wait_ns (the launch's wait limit: 1 s
// unless aspire_set_wait_limit_ns set another) or another role aborted.
template <class Sh>
__device__ __forceinline__ bool wait_bar(Sh& sm, uint64_t& bar, uint32_t parity, uint32_t* status) {
  const uint32_t a = ptx::smem_addr(&bar);
  if (ptx::mbar_try_wait(a, parity)) return true;
  // Each failed try_wait has already suspended the thread for a while, so the
  // clock is read after every poll (a check every few hundred polls would
  // only fire for waits far longer than any short bound).
  const uint64_t t0 = global_ns();
  for (;;) {
    if (ptx::mbar_try_wait(a, parity)) return true;
    if (*reinterpret_cast<volatile int*>(&sm.abort_flag)) return false;
    if (global_ns() - t0 > sm.wait_ns) break;
  }
  *reinterpret_cast<volatile int*>(&sm.abort_flag) = 1;
  if (status) atomicOr(status, ASPIRE_STATUS_TIMEOUT);
  return false;
}

// Wait used while draining after an abort: ignores the abort flag and keeps
// the fixed 1 s bound whatever the launch's wait limit, so that copies and
// MMAs already issued (which always complete) land before the CTA releases
// its shared memory and TMEM.
__device__ __forceinline__ void drain_bar(uint64_t& bar, uint32_t parity) {
  const uint32_t a = ptx::smem_addr(&bar);
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (ptx::mbar_try_wait(a, parity)) return;
    if ((i & 255) == 0 && global_ns() - t0 > kDrainLimitNs) return;
  }
}

__device__ __forceinline__ int n_tiles_of(const WorkItem& it) {
  return it.tok_end > it.tok_begin ? (it.tok_end - it.tok_begin + kTile - 1) / kTile : 0;
}

// Items every role skips identically (the planner never emits them).
__device__ __forceinline__ bool item_valid(const AttnParams& p, const WorkItem& it, int max_rows) {
  const int nrows = it.pq_end - it.pq_begin;
  return nrows > 0 && nrows <= max_rows && it.kv_head >= 0 && it.kv_head < p.num_kv_heads &&
         it.tok_begin >= 0 && it.tok_begin % kTile == 0 && it.tok_end <= it.kv_len;
}

// ------------------------------------------------------------------ item sequence
// The CTAs share one of the plan's item lists ([first, first + n)) and claim
// items from it at run time, longest first (a global counter in the plan
// header, word claim_word).  In each CTA the K producer claims an item when it
// is ready to load it and publishes the index (-1 once the list is exhausted)
// in a small ring; the other roles read the same sequence in order.  Every
// warp reads through its lane 0, which returns -2 when a wait times out.
template <class Sh>
__device__ __forceinline__ int seq_claim(const AttnParams& p, Sh& sm, uint32_t& k, int lane, int first, int n,
                                         int claim_word) {
  int item = -2;
  if (lane == 0) {
    const int s = int(k % kSeqDepth);
    if (wait_bar(sm, sm.seq_empty[s], ((k / kSeqDepth) & 1) ^ 1, p.status)) {
      const int c = atomicAdd(const_cast<int32_t*>(p.plan) + claim_word, 1);
      item = c < n ? first + c : -1;
      *reinterpret_cast<volatile int*>(&sm.seq[s]) = item;
      ptx::mbar_arrive(ptx::smem_addr(&sm.seq_full[s]));
    }
  }
  ++k;
  return __shfl_sync(0xffffffffu, item, 0);
}

template <class Sh>
__device__ __forceinline__ int seq_read(Sh& sm, uint32_t& k, int lane, uint32_t* status) {
  int item = -2;
  if (lane == 0) {
    const int s = int(k % kSeqDepth);
    if (wait_bar(sm, sm.seq_full[s], (k / kSeqDepth) & 1, status)) {
      item = *reinterpret_cast<volatile int*>(&sm.seq[s]);
      ptx::mbar_arrive(ptx::smem_addr(&sm.seq_empty[s]));
    }
  }
  ++k;
  return __shfl_sync(0xffffffffu, item, 0);
}

// Next item of the sequence that has KV tiles (the roles skip the same items);
// -1 at the end of the sequence, -2 on a timeout.
template <class Sh>
__device__ __forceinline__ int next_item_with_tiles(const AttnParams& p, Sh& sm, uint32_t& k, int lane,
                                                    int max_rows) {
  for (;;) {
    const int ii = seq_read(sm, k, lane, p.status);
    if (ii < 0) return ii;
    const WorkItem it = load_item(p.plan, ii);
    if (item_valid(p, it, max_rows) && n_tiles_of(it) > 0) return ii;
  }
}

// ------------------------------------------------------------------ fused append
// Writes the item's share of its row's new tokens (K for kv_sel 0, V for 1)
// into the cache before the item's tiles are requested: the positions
// kv_len - q_len + i (i < q_len) inside the item's key range, at the row's own
// pages, as aspire_append_kv places them.  The chunks of a decode group
// partition its key range, so every new token is written once, by the item
// that reads it; half a warp copies one 256-byte token row.  The writes are
// fenced into the async proxy before the warp's TMA loads.
__device__ __forceinline__ void append_new_tokens(const AttnParams& p, const WorkItem& it, int kv_sel, int lane) {
  const int64_t first_new = int64_t(it.kv_len) - it.q_len;
  int64_t lo = first_new > it.tok_begin ? first_new : int64_t(it.tok_begin);
  lo = lo > 0 ? lo : 0;
  const int64_t hi = it.tok_end;
  const __nv_bfloat16* src_base = kv_sel ? p.v_new : p.k_new;
  const int64_t sn = kv_sel ? p.v_new_stride_n : p.k_new_stride_n;
  const int64_t sh = kv_sel ? p.v_new_stride_h : p.k_new_stride_h;
  __nv_bfloat16* cache = const_cast<__nv_bfloat16*>(p.kv);
  const int col = (lane & 15) * 8;
  for (int64_t pos = lo + (lane >> 4); pos < hi; pos += 2) {
    const int64_t t = int64_t(it.q_start) + (pos - first_new);
    if (t >= p.q_rows) {
      record_status(p.status, ASPIRE_STATUS_BAD_ROW);
      continue;
    }
    const int32_t page = row_page(p.kv_indices, it.kv_page_base, p.mode_flags, p.draft_table, p.draft_stride,
                                  p.block_table, p.block_table_stride, it.row, int(pos / kPageSize));
    if (page < 0 || int64_t(page) >= p.num_pages_total) {
      record_status(p.status, ASPIRE_STATUS_BAD_PAGE);
      continue;
    }
    const __nv_bfloat16* src = src_base + t * sn + int64_t(it.kv_head) * sh + col;
    const int64_t dst = ((int64_t(page) * 2 + kv_sel) * kPageSize + pos % kPageSize) * int64_t(p.num_kv_heads) *
                            kHeadDim + int64_t(it.kv_head) * kHeadDim + col;
    *reinterpret_cast<uint4*>(cache + dst) = *reinterpret_cast<const uint4*>(src);
  }
  ptx::fence_proxy_async_global();
  __syncwarp();
}

// ------------------------------------------------------------------ producers
// Lane pg (< 8) owns page pg of every tile: it reads the page id one tile
// ahead (the read overlaps the wait for a free slot) and issues the page's two
// 64-dim boxes of K (kv_sel 0) or V (kv_sel 1) into the ring slot.  The leader
// (the K producer) claims the items; the other producer reads the sequence.
// `k` is the warp's position in the item sequence (carried across the
// kernel's phases, which share the sequence ring).  Returns false on a timeout.
template <int STAGES, class Sh>
__device__ bool run_producer(const AttnParams& p, const CUtensorMap* tmap, Sh& sm, uint8_t (*ring)[kSlotBytes],
                             uint64_t* full, uint64_t* empty, int kv_sel, bool leader, int first, int n,
                             int claim_word, int max_rows, int lane, uint32_t& k) {
  uint32_t g = 0;
  int64_t last_issue[STAGES];
#pragma unroll
  for (int s = 0; s < STAGES; ++s) last_issue[s] = -1;
  bool ok = true;
  while (ok) {
    const int ii = leader ? seq_claim(p, sm, k, lane, first, n, claim_word) : seq_read(sm, k, lane, p.status);
    if (ii == -2) ok = false;
    if (ii < 0) break;
    const WorkItem it = load_item(p.plan, ii);
    if (!item_valid(p, it, max_rows)) continue;
    // The new tokens sit in the item's last tile or two: they are written just
    // before the first tile that holds one is requested, while the earlier
    // tiles stream (the writes overlap the wait for a free ring slot).
    const int64_t first_new = (p.k_new != nullptr && it.kind == 1) ? int64_t(it.kv_len) - it.q_len : INT64_MAX;
    bool appended = first_new >= it.tok_end;
    const int nt = n_tiles_of(it);
    const int first_page = it.tok_begin / kPageSize;
    const int end_page = (it.tok_end + kPageSize - 1) / kPageSize;
    auto page_id = [&](int t) -> int32_t {
      const int lp = first_page + t * kPagesPerTile + lane;
      if (lane >= kPagesPerTile || lp >= end_page) return -1;
      return row_page(p.kv_indices, it.kv_page_base, p.mode_flags, p.draft_table, p.draft_stride, p.block_table,
                      p.block_table_stride, it.row, lp);
    };
    int32_t next_id = nt > 0 ? page_id(0) : -1;
    for (int t = 0; t < nt; ++t, ++g) {
      const int32_t id = next_id;
      if (t + 1 < nt) next_id = page_id(t + 1);
      const int s = g % STAGES;
      const uint32_t ph = (g / STAGES) & 1;
      if (!appended && int64_t(it.tok_begin) + int64_t(t + 1) * kTile > first_new) {
        append_new_tokens(p, it, kv_sel, lane);
        appended = true;
      }
      if (!wait_bar(sm, empty[s], ph ^ 1, p.status)) {
        ok = false;
        break;
      }
      const uint32_t fb = ptx::smem_addr(&full[s]);
      if (lane == 0) ptx::mbar_arrive_expect_tx(fb, kSlotBytes);
      __syncwarp();
      if (lane < kPagesPerTile) {
        int page = static_cast<int>(p.num_pages_total);  // out of range: TMA fills zeros
        const int lp = first_page + t * kPagesPerTile + lane;
        if (lp < end_page) {
          if (id < 0 || int64_t(id) >= p.num_pages_total)
            record_status(p.status, ASPIRE_STATUS_BAD_PAGE);
          else
            page = id;
        }
        const uint32_t base = ptx::smem_addr(ring[s]) + uint32_t(lane) * kPageSize * 128;
        ptx::tma_load_5d(base, tmap, fb, 0, it.kv_head, 0, kv_sel, page);
        ptx::tma_load_5d(base + kHalfBytes, tmap, fb, 64, it.kv_head, 0, kv_sel, page);
      }
      last_issue[s] = g;
      __syncwarp();
    }
  }
  if (!ok || aborted(sm)) {
    // Let this CTA's own copies land before the CTA releases its shared memory.
#pragma unroll
    for (int s = 0; s < STAGES; ++s)
      if (last_issue[s] >= 0) drain_bar(full[s], uint32_t(last_issue[s] / STAGES) & 1);
    return false;
  }
  return true;
}

// A tile's tokens past the item's last one ([valid, 128)) that share a page
// with its last token hold whatever the cache has there, possibly NaN; their
// P entries are zero, but 0 x NaN is NaN in the PV product.  The MMA warp
// clears those V rows after the tile has landed and before its PV.  Whole
// pages past the item arrive zero-filled (their page index is out of range).
__device__ __forceinline__ void clear_v_tail(uint8_t* slot, int valid, int lane) {
  if (valid >= kTile || (valid & (kPageSize - 1)) == 0) return;
  const int n = (kPageSize - (valid & (kPageSize - 1))) * 16;  // rows x (2 halves x 8 chunks of 16 B)
  for (int i = lane; i < n; i += 32) {
    const int row = valid + (i >> 4), c = i & 15;
    *reinterpret_cast<uint4*>(slot + (c >> 3) * kHalfBytes + row * 128 + (c & 7) * 16) = make_uint4(0, 0, 0, 0);
  }
  ptx::fence_proxy_async_smem();
}

// Requests item `idx`'s query tile: one box of (64 dims x group heads x
// box_tokens tokens) per 64-dim half, starting at the item's first query.
// Rows past the item's queries are other queries or zero fill; they only feed
// ignored rows / columns.
template <class Sh>
__device__ __forceinline__ void issue_q(const AttnParams& p, const CUtensorMap* qmap, Sh& sm, int idx,
                                        int box_tokens) {
  const WorkItem it = load_item(p.plan, idx);
  const int q_idx0 = it.pq_begin / p.group;
  const uint32_t bytes = 2u * 128u * uint32_t(p.group) * uint32_t(box_tokens);
  const uint32_t bar = ptx::smem_addr(&sm.q_full);
  ptx::mbar_arrive_expect_tx(bar, bytes);
  ptx::tma_load_3d(ptx::smem_addr(sm.q[0]), qmap, bar, 0, it.kv_head * p.group, it.q_start + q_idx0);
  ptx::tma_load_3d(ptx::smem_addr(sm.q[1]), qmap, bar, 64, it.kv_head * p.group, it.q_start + q_idx0);
}

}  // namespace pipe
}  // namespace aspire
