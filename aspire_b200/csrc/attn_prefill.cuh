// Prefill phase of the tcgen05 attention kernel: work items of long-query
// rows (prefill chunks), up to 256 packed (query, head-in-group) rows each.
//
// The contraction is the direct one: packed query rows are the MMA's M
// dimension, KV tokens its N (QK^T) or K (PV) dimension.  An item holds two
// halves of up to 128 packed rows (whole query positions each) that share
// every 128-token K/V tile.  Each tile is consumed as two 64-key sub-tiles,
// and each half h keeps two S buffers in TMEM, so the tensor core computes
// sub-tile j+1's scores while half h's softmax works on sub-tile j:
//
//   S_h[b][128 rows x 64 keys] = Q_h . K_j^T   (A: Q_h, B: K_j; K-major SW128, SMEM)
//   O_h[128 rows x 128 d]     += P_h[b] . V_j  (A: P_h[b] in TMEM, B: V_j MN-major SW128)
//
// P_h[b] is written as bf16 pairs into the first 32 columns of S_h[b]
// (TMEM), so sub-tile j+2's Q_h.K^T (same buffer) waits until the PV that
// reads P_h[b] has completed.  Each half has its own MMA-issuing warp, which
// issues PV_h(j) and then QK_h(j+2) per sub-tile: that completion wait
// stalls only its own half's stream, while its softmax works on the other
// buffer and the other half's products keep the tensor core busy.
//
// Softmax warpgroup h owns half h; thread r owns TMEM lane r, i.e. packed row
// r of the half, so every row statistic is thread-local.  The running row max
// is lazy: the reference max moves (and O_h's row is rescaled in TMEM, once
// the previous sub-tile's PV has landed) only when a sub-tile's max exceeds
// it by more than 2^8 in the exp2 domain, so P stays <= 256 and most
// sub-tiles need no rescale.  The epilogue reads O_h's row, divides by the
// row sum and stores the row (bf16 output + base-2 LSE, or an fp32 partial
// for split-KV items).
//
// TMEM (512 columns): S_0[0..1] [0, 128), S_1[0..1] [128, 256),
// O_0 [256, 384), O_1 [384, 512).  Shared memory overlays the decode phase's
// data buffers.
#pragma once

#include <cuda.h>

#include "tc_pipeline.cuh"

namespace aspire {
namespace pf {

using namespace pipe;

constexpr int kKStages = 2;
constexpr int kVStages = 2;
constexpr int kSub = 64;                          // keys per sub-tile
constexpr uint32_t kQHalfBytes = kPfQTile * 128;  // 128 rows x 64 dims
constexpr uint32_t kTmemCols = 512;
constexpr float kLazyLog2 = 8.0f;

__host__ __device__ constexpr uint32_t col_s(int h, int b) { return uint32_t(h) * 128u + uint32_t(b) * 64u; }
__host__ __device__ constexpr uint32_t col_o(int h) { return 256u + uint32_t(h) * 128u; }

struct Buffers {
  uint8_t q[2][2][kQHalfBytes];  // [item half][64-dim half]
  uint8_t k[kKStages][kSlotBytes];
  uint8_t v[kVStages][kSlotBytes];
};

// Per half h and S buffer b: s_full (scores ready), p_full (P written),
// pv_done (the PV reading P_h[b] has completed); each completes one phase
// per K/V tile of the half.  o_free[h]: the epilogue has read O_h.
// k_empty / v_empty / q_empty complete when both MMA warps have released the
// slot (a commit after their MMAs, or a plain arrival for a single-half item
// that the second warp does not compute).  v_ready[s]: the first MMA warp has
// cleared a V tile's tail rows (two-half items only).
struct Barriers {
  uint64_t k_full[kKStages], k_empty[kKStages];
  uint64_t v_full[kVStages], v_empty[kVStages], v_ready[kVStages];
  uint64_t s_full[2][2], p_full[2][2], pv_done[2][2], o_free[2], done[2];
  uint64_t q_full, q_empty;
};

// Run by one thread before the CTA's first barrier.
__device__ inline void init_barriers(Barriers& b) {
  for (int s = 0; s < kKStages; ++s) {
    ptx::mbar_init(ptx::smem_addr(&b.k_full[s]), 1);
    ptx::mbar_init(ptx::smem_addr(&b.k_empty[s]), 2);
  }
  for (int s = 0; s < kVStages; ++s) {
    ptx::mbar_init(ptx::smem_addr(&b.v_full[s]), 1);
    ptx::mbar_init(ptx::smem_addr(&b.v_empty[s]), 2);
    ptx::mbar_init(ptx::smem_addr(&b.v_ready[s]), 1);
  }
  for (int h = 0; h < 2; ++h) {
    for (int u = 0; u < 2; ++u) {
      ptx::mbar_init(ptx::smem_addr(&b.s_full[h][u]), 1);
      ptx::mbar_init(ptx::smem_addr(&b.p_full[h][u]), 128);
      ptx::mbar_init(ptx::smem_addr(&b.pv_done[h][u]), 1);
    }
    ptx::mbar_init(ptx::smem_addr(&b.o_free[h]), 128);
    ptx::mbar_init(ptx::smem_addr(&b.done[h]), 1);
  }
  ptx::mbar_init(ptx::smem_addr(&b.q_full), 1);
  ptx::mbar_init(ptx::smem_addr(&b.q_empty), 2);
}

__device__ __forceinline__ int halves_of(const AttnParams& p, const WorkItem& it) {
  return (it.pq_end - it.pq_begin) > pf_half_rows(p.group) ? 2 : 1;
}

// Requests item `idx`'s query rows: half h holds query positions
// [q0 + h T, q0 + (h + 1) T) x the group's heads (T = 128 / group), one
// (64 dims x group x box) TMA box per 64-dim half.  Rows past the item's
// queries are other queries or zero fill and only feed ignored rows.
__device__ __forceinline__ void issue_q(const AttnParams& p, const CUtensorMap* qmap, Buffers& buf,
                                        Barriers& b, int idx) {
  const WorkItem it = load_item(p.plan, idx);
  const int half_tokens = kPfQTile / p.group;
  const int q0 = it.q_start + it.pq_begin / p.group;
  const int halves = halves_of(p, it);
  const uint32_t bytes = uint32_t(halves) * 2u * 128u * uint32_t(p.group) * uint32_t(p.pf_box_tokens);
  const uint32_t bar = ptx::smem_addr(&b.q_full);
  ptx::mbar_arrive_expect_tx(bar, bytes);
  for (int h = 0; h < halves; ++h)
    for (int d = 0; d < 2; ++d)
      ptx::tma_load_3d(ptx::smem_addr(buf.q[h][d]), qmap, bar, 64 * d, it.kv_head * p.group, q0 + h * half_tokens);
}

// ------------------------------------------------------------------ MMA issuers
// The MMA warp of half h.  Both warps walk every item and tile in the same
// order (the K/V ring and the query buffer are shared); warp 0 also loads
// the query rows and clears the V tiles' tail rows.
template <class Sh>
__device__ void run_mma(const AttnParams& p, const CUtensorMap* qmap, Sh& sm, Buffers& buf, int h, int lane,
                        uint32_t& k) {
  Barriers& b = sm.pf;
  const uint32_t tmem = sm.tmem_base;
  constexpr uint32_t idesc_qk = ptx::idesc_bf16(128, kSub, false, false);
  constexpr uint32_t idesc_pv = ptx::idesc_bf16(128, 128, false, true);
  const uint32_t k0 = ptx::smem_addr(buf.k[0]);
  const uint32_t v0 = ptx::smem_addr(buf.v[0]);
  const uint64_t qdesc0 = ptx::smem_desc(ptx::smem_addr(buf.q[h][0]), 16, 1024, ptx::kLayoutSw128);
  const bool leader = h == 0;
  uint32_t g = 0, items_done = 0;
  uint32_t nth = 0;  // this half's K/V tiles before the current item (s_full / p_full / pv_done phases)
  uint32_t nit = 0;  // this half's items so far (o_free phases)
  uint32_t ntail0 = 0, ntail1 = 0;  // tail clears waited for, per V stage (warp 1)
  bool ok = true, q_pending = false;

  // QK_h of sub-tile j of the item (its K tile in stage ks).
  auto issue_qk = [&](int j, int ks) {
    if (lane == 0) {
      const uint64_t kdesc0 = ptx::smem_desc(k0 + uint32_t(ks) * kSlotBytes + uint32_t(j & 1) * (kSub * 128), 16,
                                             1024, ptx::kLayoutSw128);
#pragma unroll
      for (int kk = 0; kk < 128 / 16; ++kk) {
        const uint32_t koff = uint32_t(kk / 4) * kHalfBytes + uint32_t(kk % 4) * 32;
        const uint32_t qoff = uint32_t(kk / 4) * kQHalfBytes + uint32_t(kk % 4) * 32;
        ptx::mma_bf16(tmem + col_s(h, j & 1), qdesc0 + (qoff >> 4), kdesc0 + (koff >> 4), idesc_qk, kk > 0 ? 1u : 0u);
      }
      ptx::mma_commit(ptx::smem_addr(&b.s_full[h][j & 1]));
    }
    __syncwarp();
  };
  // This warp's release of K stage ks (and of the query rows after the item's
  // last tile): a commit after its MMAs, or a plain arrival.
  auto release_k = [&](int ks, bool last_tile, bool active) {
    if (lane == 0) {
      if (active) {
        ptx::mma_commit(ptx::smem_addr(&b.k_empty[ks]));
        if (last_tile) ptx::mma_commit(ptx::smem_addr(&b.q_empty));
      } else {
        ptx::mbar_arrive(ptx::smem_addr(&b.k_empty[ks]));
        if (last_tile) ptx::mbar_arrive(ptx::smem_addr(&b.q_empty));
      }
    }
    __syncwarp();
  };

  int ii = next_item_with_tiles(p, sm, k, lane, kPfMaxRows);
  if (ii == -2) ok = false;
  if (ii >= 0 && leader) {
    if (lane == 0) issue_q(p, qmap, buf, b, ii);
    q_pending = true;
    __syncwarp();
  }
  while (ii >= 0 && ok) {
    const WorkItem it = load_item(p.plan, ii);
    const int nt = n_tiles_of(it);
    const int nh = halves_of(p, it);
    const bool active = h < nh;
    // (The second warp waits too: it releases the query buffer only after
    // this item's rows have landed.)
    if (!wait_bar(sm, b.q_full, items_done & 1, p.status)) {
      ok = false;
      break;
    }
    q_pending = false;
    // Scores of the first tile's two sub-tiles, once each S buffer is free
    // (the previous item's last PV on it has completed).
    if (!wait_bar(sm, b.k_full[g % kKStages], (g / kKStages) & 1, p.status)) {
      ok = false;
      break;
    }
    if (active) {
      for (int j = 0; j < 2 && ok; ++j) {
        if (nth > 0 && !wait_bar(sm, b.pv_done[h][j], (nth - 1) & 1, p.status)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        issue_qk(j, g % kKStages);
      }
      if (!ok) break;
    }
    release_k(g % kKStages, nt == 1, active);

    for (int t = 0; t < nt && ok; ++t) {
      const uint32_t gt = g + uint32_t(t);
      const int vs = gt % kVStages;
      if (!wait_bar(sm, b.v_full[vs], (gt / kVStages) & 1, p.status)) {
        ok = false;
        break;
      }
      const int valid = it.tok_end - (it.tok_begin + t * kTile);
      const bool tail = valid < kTile && (valid & (kPageSize - 1)) != 0;
      if (leader) {
        clear_v_tail(buf.v[vs], valid, lane);
        __syncwarp();
        if (tail && nh > 1 && lane == 0) ptx::mbar_arrive(ptx::smem_addr(&b.v_ready[vs]));
      } else if (tail && active) {
        if (!wait_bar(sm, b.v_ready[vs], (vs ? ntail1 : ntail0) & 1, p.status)) {
          ok = false;
          break;
        }
        if (vs) ++ntail1; else ++ntail0;
      }
      if (active) {
        const uint32_t th = nth + uint32_t(t);  // this half's tile index
        for (int bj = 0; bj < 2 && ok; ++bj) {
          const int j = 2 * t + bj;
          // The item's first PV overwrites O_h: the previous item's epilogue has read it.
          if (j == 0 && nit > 0 && !wait_bar(sm, b.o_free[h], (nit - 1) & 1, p.status)) {
            ok = false;
            break;
          }
          if (!wait_bar(sm, b.p_full[h][bj], th & 1, p.status)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          if (lane == 0) {
            const uint64_t vdesc0 = ptx::smem_desc(v0 + uint32_t(vs) * kSlotBytes + uint32_t(bj) * (kSub / 16) * 2048,
                                                   kHalfBytes, 1024, ptx::kLayoutSw128);
#pragma unroll
            for (int kk = 0; kk < kSub / 16; ++kk)
              ptx::mma_bf16_ts(tmem + col_o(h), tmem + col_s(h, bj) + uint32_t(kk) * 8,
                               vdesc0 + uint64_t(kk * 2048 >> 4), idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
            ptx::mma_commit(ptx::smem_addr(&b.pv_done[h][bj]));
          }
          __syncwarp();
          if (t + 1 < nt) {
            // Sub-tile j + 2 (tile t + 1) reuses S buffer bj once PV(j) has read P from it.
            const uint32_t gt2 = gt + 1;
            if (bj == 0 && !wait_bar(sm, b.k_full[gt2 % kKStages], (gt2 / kKStages) & 1, p.status)) {
              ok = false;
              break;
            }
            if (!wait_bar(sm, b.pv_done[h][bj], th & 1, p.status)) {
              ok = false;
              break;
            }
            ptx::tc_fence_after();
            issue_qk(j + 2, gt2 % kKStages);
            if (bj == 1) release_k(gt2 % kKStages, t + 1 == nt - 1, true);
          }
        }
        if (!ok) break;
        if (lane == 0) ptx::mma_commit(ptx::smem_addr(&b.v_empty[vs]));
        __syncwarp();
      } else {
        // The second warp on a single-half item releases the slots unused.
        if (t + 1 < nt) {
          const uint32_t gt2 = gt + 1;
          if (!wait_bar(sm, b.k_full[gt2 % kKStages], (gt2 / kKStages) & 1, p.status)) {
            ok = false;
            break;
          }
          release_k(gt2 % kKStages, t + 1 == nt - 1, false);
        }
        if (lane == 0) ptx::mbar_arrive(ptx::smem_addr(&b.v_empty[vs]));
        __syncwarp();
      }
    }
    if (!ok) break;
    g += uint32_t(nt);
    if (active) {
      nth += uint32_t(nt);
      ++nit;
    }
    // The next item's query rows load while this item's last PVs and epilogue run.
    const int nxt = next_item_with_tiles(p, sm, k, lane, kPfMaxRows);
    if (nxt == -2) {
      ok = false;
      break;
    }
    if (nxt >= 0 && leader) {
      if (!wait_bar(sm, b.q_empty, items_done & 1, p.status)) {
        ok = false;
        break;
      }
      if (lane == 0) issue_q(p, qmap, buf, b, nxt);
      q_pending = true;
      __syncwarp();
    }
    ++items_done;
    ii = nxt;
  }
  // A query load still in flight lands before the CTA reuses its memory.
  if (q_pending) drain_bar(b.q_full, items_done & 1);
  // Every MMA this thread issued has completed once `done` fires.
  if (lane == 0) ptx::mma_commit(ptx::smem_addr(&b.done[h]));
  __syncwarp();
  drain_bar(b.done[h], 0);
}

// ------------------------------------------------------------------ softmax / epilogue
// Packed pairs of fp32 (Blackwell's paired FP32 instructions).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  return uint64_t(__float_as_uint(lo)) | (uint64_t(__float_as_uint(hi)) << 32);
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float(uint32_t(v)); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float(uint32_t(v >> 32)); }
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float max64(const float* s) {
  float m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = max3(s[i], s[8 + i], s[16 + i]);
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = max3(m[i], s[24 + i], s[32 + i]);
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = max3(m[i], s[40 + i], s[48 + i]);
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = fmaxf(m[i], s[56 + i]);
  return max3(max3(m[0], m[1], m[2]), max3(m[3], m[4], m[5]), fmaxf(m[6], m[7]));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// One item for softmax warpgroup h (thread = packed row r of half h).  `gt`
// counts the K/V tiles this warpgroup has consumed (its barrier phases).
template <class Sh>
__device__ bool consume_item(const AttnParams& p, Sh& sm, const WorkItem& it, bool causal, int h, int r,
                             uint32_t tmem_lane, uint32_t& gt) {
  Barriers& b = sm.pf;
  const int group = p.group;
  const int nrows = it.pq_end - it.pq_begin;
  const int nj = 2 * n_tiles_of(it);
  const int j_row = h * pf_half_rows(group) + r;  // row within the item
  const bool valid = r < pf_half_rows(group) && j_row < nrows;
  const int pq = it.pq_begin + j_row;
  const int q_idx = pq / group;
  const int head = it.kv_head * group + (pq - q_idx * group);
  // Keys [tok_begin, vis_end) of the item are visible to this row (bottom-right
  // causal mask); padding rows see none.
  int vis_end = it.tok_begin;
  if (valid) vis_end = causal ? min(it.tok_end, it.kv_len - it.q_len + q_idx + 1) : it.tok_end;
  // Logit dump (raw q.k before scale and mask, dump_index): query 0 to the
  // first slot, query q_len-1 to the last one, as the dump kind has them.
  int64_t dump_at = -1;
  if (valid && dump_row_on(p, it.row)) {
    const bool first = dump_has_first(p) && q_idx == 0;
    const bool last = !first && dump_has_last(p, it.q_len) && q_idx == it.q_len - 1;
    if (first || last) dump_at = dump_index(p, it.row, head, last);
  }
  const int dump_end = p.dump_kv_stride < it.tok_end ? int(p.dump_kv_stride) : it.tok_end;
  const bool warp_dumps = __any_sync(0xffffffffu, dump_at >= 0);
  const float scale = p.scale_log2;
  const uint64_t scale2 = f2_pack(scale, scale);
  const uint32_t o_addr = tmem_lane + col_o(h);
  float m_ref = -INFINITY;  // reference row max x scale (log2 domain)
  float l = 0.f;

  for (int j = 0; j < nj; ++j) {
    const int bj = j & 1;
    const uint32_t th = gt + uint32_t(j >> 1);
    if (!wait_bar(sm, b.s_full[h][bj], th & 1, p.status)) return false;
    ptx::tc_fence_after();
    const int sub0 = it.tok_begin + j * kSub;
    const uint32_t s_addr = tmem_lane + col_s(h, bj);
    float s[kSub];
    ptx::tmem_ld32(s_addr, s);
    ptx::tmem_ld32(s_addr + 32, s + 32);
    ptx::tmem_wait_ld();
    if (warp_dumps && dump_at >= 0) {
#pragma unroll
      for (int c = 0; c < kSub; ++c)
        if (sub0 + c < dump_end) dump_store(p, dump_at + sub0 + c, s[c]);
    }
    const int nvis = vis_end - sub0;
    if (nvis < kSub) {
#pragma unroll
      for (int c = 0; c < kSub; ++c)
        if (c >= nvis) s[c] = -INFINITY;
    }
    const float ms = max64(s) * scale;
    const bool need = ms > m_ref + kLazyLog2;
    float alpha = 1.f;
    if (need) {
      alpha = (m_ref == -INFINITY) ? 0.f : ex2(m_ref - ms);
      l *= alpha;
      m_ref = ms;
    }
    if (j > 0 && __any_sync(0xffffffffu, need)) {
      // Rescale this row of O_h once the previous sub-tile's PV has landed
      // (tcgen05.ld/st are warp-collective, hence the warp vote).
      const uint32_t tp = gt + uint32_t((j - 1) >> 1);
      if (!wait_bar(sm, b.pv_done[h][bj ^ 1], tp & 1, p.status)) return false;
      ptx::tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < kHeadDim; c += 16) {
        float o[16];
        ptx::tmem_ld16(o_addr + c, o);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] *= alpha;
        ptx::tmem_st16(o_addr + c, o);
      }
    }
    // P = exp2(s * scale - m_ref), as bf16 pairs into the first 32 columns of S_h[b].
    const float mb = (m_ref == -INFINITY) ? 0.f : m_ref;
    const uint64_t nmb2 = f2_pack(-mb, -mb);
    uint64_t acc2[2] = {0, 0};
    uint32_t pk[kSub / 2];
#pragma unroll
    for (int i = 0; i < kSub / 2; ++i) {
      const uint64_t x = f2_fma(f2_pack(s[2 * i], s[2 * i + 1]), scale2, nmb2);
      const float p0 = ex2(f2_lo(x)), p1 = ex2(f2_hi(x));
      acc2[i & 1] = f2_add(acc2[i & 1], f2_pack(p0, p1));
      pk[i] = pack_bf16x2(p0, p1);
    }
    ptx::tmem_st32(s_addr, pk);
    const uint64_t acc = f2_add(acc2[0], acc2[1]);
    l += f2_lo(acc) + f2_hi(acc);
    ptx::tmem_wait_st();
    ptx::tc_fence_before();
    ptx::mbar_arrive(ptx::smem_addr(&b.p_full[h][bj]));
  }
  gt += uint32_t(nj >> 1);

  // Final O_h row once the item's last PV (buffer 1 of its last tile, issued
  // after every other) has completed, 32 dims at a time; then O_h is free.
  if (!wait_bar(sm, b.pv_done[h][1], (gt - 1) & 1, p.status)) return false;
  ptx::tc_fence_after();
  const float inv = l > 0.f ? 1.f / l : 0.f;
  const float lse = l > 0.f ? m_ref + lg2(l) : -INFINITY;
  const int64_t tok = int64_t(it.q_start) + q_idx;
  const bool final_rows = it.n_chunks <= 1;
  const int64_t prow = int64_t(it.partial_base) + int64_t(it.chunk) * nrows + j_row;
  bool store = valid;
  if (store && final_rows && tok >= p.q_rows) {
    record_status(p.status, ASPIRE_STATUS_BAD_ROW);
    store = false;
  }
  uint4* dst_bf16 = reinterpret_cast<uint4*>(p.out + tok * p.o_stride_n + int64_t(head) * p.o_stride_h);
  float4* dst_f32 = reinterpret_cast<float4*>(p.partial_o + prow * kHeadDim);
#pragma unroll
  for (int c = 0; c < kHeadDim; c += 32) {
    float o[32];
    ptx::tmem_ld32(o_addr + c, o);
    ptx::tmem_wait_ld();
    if (store && final_rows) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        uint4 u;
        u.x = pack_bf16x2(o[8 * e + 0] * inv, o[8 * e + 1] * inv);
        u.y = pack_bf16x2(o[8 * e + 2] * inv, o[8 * e + 3] * inv);
        u.z = pack_bf16x2(o[8 * e + 4] * inv, o[8 * e + 5] * inv);
        u.w = pack_bf16x2(o[8 * e + 6] * inv, o[8 * e + 7] * inv);
        dst_bf16[c / 8 + e] = u;
      }
    } else if (store) {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        dst_f32[c / 4 + e] = make_float4(o[4 * e] * inv, o[4 * e + 1] * inv, o[4 * e + 2] * inv, o[4 * e + 3] * inv);
    }
  }
  ptx::tc_fence_before();
  ptx::mbar_arrive(ptx::smem_addr(&b.o_free[h]));
  if (store) {
    if (!final_rows)
      partial_lse_ptr(p)[prow] = lse;
    else if (p.lse)
      p.lse[tok * p.num_qo_heads + head] = lse;
  }
  return true;
}

// Softmax warpgroup h's share of the item sequence: both halves of two-half
// items, half 0 of the others.  `quarter` is the warp's TMEM lane quarter.
template <class Sh>
__device__ void consume_items(const AttnParams& p, Sh& sm, bool causal, int h, int quarter, int lane, uint32_t& k) {
  const int r = quarter * 32 + lane;
  const uint32_t tmem_lane = sm.tmem_base + (uint32_t(quarter * 32) << 16);
  uint32_t gt = 0;
  for (;;) {
    if (aborted(sm)) return;
    const int ii = seq_read(sm, k, lane, p.status);
    if (ii < 0) return;
    const WorkItem it = load_item(p.plan, ii);
    if (!item_valid(p, it, kPfMaxRows)) {
      if (h == 0 && r == 0) record_status(p.status, ASPIRE_STATUS_BAD_PLAN);
      continue;
    }
    const int nrows = it.pq_end - it.pq_begin;
    if (n_tiles_of(it) == 0) {
      // No keys: zero output, -inf LSE (chunked items always have keys).
      for (int jr = h; jr < nrows; jr += 2) store_final(p, it, it.pq_begin + jr, r, 0.f, -INFINITY);
      continue;
    }
    if (h >= halves_of(p, it)) continue;
    if (!consume_item(p, sm, it, causal, h, r, tmem_lane, gt)) return;
  }
}

}  // namespace pf
}  // namespace aspire
