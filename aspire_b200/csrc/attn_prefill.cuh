// Prefill phase of the tcgen05 attention kernel: work items of long-query
// rows (prefill chunks), up to 256 packed (query, head-in-group) rows each.
//
// The contraction is the direct one: packed query rows are the MMA's M
// dimension, KV tokens its N (QK^T) or K (PV) dimension.  An item holds two
// halves of up to 128 packed rows (whole query positions each) that share
// every K/V tile; each half has its own S and O accumulators in TMEM:
//
//   S_h[128 rows x 128 tok] = Q_h . K^T        (A: Q_h, B: K; both K-major SW128, SMEM)
//   O_h[128 rows x 128 d ] += P_h . V          (A: P_h in TMEM, B: V MN-major SW128)
//
// P_h is written as bf16 pairs into the first 64 columns of S_h (TMEM), so
// the next tile's Q_h.K^T waits until the PV that reads P_h has completed.
// The MMA warp issues QK_0, QK_1, PV_0, PV_1 per tile: while one softmax
// warpgroup works on its S the tensor core runs the other half's products.
//
// Softmax warpgroup h owns half h; thread r owns TMEM lane r, i.e. packed row
// r of the half, so every row statistic is thread-local.  The running row max
// is lazy: the reference max moves (and O_h's row is rescaled in TMEM) only
// when a tile's max exceeds it by more than 2^8 in the exp2 domain, so P
// stays <= 256 and most tiles need no rescale.  The epilogue reads O_h's row,
// divides by the row sum and stores the row (bf16 output + base-2 LSE, or an
// fp32 partial for split-KV items).
//
// TMEM (512 columns): S_0 [0, 128), S_1 [128, 256), O_0 [256, 384),
// O_1 [384, 512).  Shared memory overlays the decode phase's data buffers.
#pragma once

#include <cuda.h>

#include "tc_pipeline.cuh"

namespace aspire {
namespace pf {

using namespace pipe;

constexpr int kKStages = 2;
constexpr int kVStages = 2;
constexpr uint32_t kQHalfBytes = kPfQTile * 128;  // 128 rows x 64 dims
constexpr uint32_t kTmemCols = 512;
constexpr float kLazyLog2 = 8.0f;

__host__ __device__ constexpr uint32_t col_s(int h) { return uint32_t(h) * 128u; }
__host__ __device__ constexpr uint32_t col_o(int h) { return 256u + uint32_t(h) * 128u; }

struct Buffers {
  uint8_t q[2][2][kQHalfBytes];  // [item half][64-dim half]
  uint8_t k[kKStages][kSlotBytes];
  uint8_t v[kVStages][kSlotBytes];
};

struct Barriers {
  uint64_t k_full[kKStages], k_empty[kKStages];
  uint64_t v_full[kVStages], v_empty[kVStages];
  uint64_t s_full[2], p_full[2], pv_done[2], o_free[2];
  uint64_t q_full, q_empty, done;
};

// Run by one thread before the CTA's first barrier.
__device__ inline void init_barriers(Barriers& b) {
  for (int s = 0; s < kKStages; ++s) {
    ptx::mbar_init(ptx::smem_addr(&b.k_full[s]), 1);
    ptx::mbar_init(ptx::smem_addr(&b.k_empty[s]), 1);
  }
  for (int s = 0; s < kVStages; ++s) {
    ptx::mbar_init(ptx::smem_addr(&b.v_full[s]), 1);
    ptx::mbar_init(ptx::smem_addr(&b.v_empty[s]), 1);
  }
  for (int h = 0; h < 2; ++h) {
    ptx::mbar_init(ptx::smem_addr(&b.s_full[h]), 1);
    ptx::mbar_init(ptx::smem_addr(&b.p_full[h]), 128);
    ptx::mbar_init(ptx::smem_addr(&b.pv_done[h]), 1);
    ptx::mbar_init(ptx::smem_addr(&b.o_free[h]), 128);
  }
  ptx::mbar_init(ptx::smem_addr(&b.q_full), 1);
  ptx::mbar_init(ptx::smem_addr(&b.q_empty), 1);
  ptx::mbar_init(ptx::smem_addr(&b.done), 1);
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

// ------------------------------------------------------------------ MMA issuer
template <class Sh>
__device__ void run_mma(const AttnParams& p, const CUtensorMap* qmap, Sh& sm, Buffers& buf, int lane,
                        uint32_t& k) {
  Barriers& b = sm.pf;
  const uint32_t tmem = sm.tmem_base;
  constexpr uint32_t idesc_qk = ptx::idesc_bf16(128, 128, false, false);
  constexpr uint32_t idesc_pv = ptx::idesc_bf16(128, 128, false, true);
  const uint32_t k0 = ptx::smem_addr(buf.k[0]);
  const uint32_t v0 = ptx::smem_addr(buf.v[0]);
  const uint32_t q0 = ptx::smem_addr(buf.q[0][0]);
  uint32_t g = 0, items_done = 0;
  // PVs issued per half (= pv_done / p_full phases) and items finished per
  // half (= o_free phases); scalars, so that they stay in registers.
  uint32_t npv0 = 0, npv1 = 0, nit0 = 0, nit1 = 0;
  bool ok = true, q_pending = false;

  int ii = next_item_with_tiles(p, sm, k, lane, kPfMaxRows);
  if (ii == -2) ok = false;
  if (ii >= 0) {
    if (lane == 0) issue_q(p, qmap, buf, b, ii);
    q_pending = true;
    __syncwarp();
  }
  while (ii >= 0 && ok) {
    const WorkItem it = load_item(p.plan, ii);
    const int nt = n_tiles_of(it);
    const int nh = halves_of(p, it);
    if (!wait_bar(sm, b.q_full, items_done & 1, p.status)) {
      ok = false;
      break;
    }
    q_pending = false;
    for (int t = 0; t < nt && ok; ++t, ++g) {
      const int ks = g % kKStages;
      if (!wait_bar(sm, b.k_full[ks], (g / kKStages) & 1, p.status)) {
        ok = false;
        break;
      }
      for (int h = 0; h < nh && ok; ++h) {
        // S_h holds P_h of the previous tile until that PV has completed.
        const uint32_t npv = h ? npv1 : npv0;
        if (npv > 0 && !wait_bar(sm, b.pv_done[h], (npv - 1) & 1, p.status)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        if (lane == 0) {
          const uint32_t kbase = k0 + uint32_t(ks) * kSlotBytes;
          const uint32_t qbase = q0 + uint32_t(h) * 2u * kQHalfBytes;
#pragma unroll
          for (int kk = 0; kk < 128 / 16; ++kk) {
            const uint32_t koff = uint32_t(kk / 4) * kHalfBytes + uint32_t(kk % 4) * 32;
            const uint32_t qoff = uint32_t(kk / 4) * kQHalfBytes + uint32_t(kk % 4) * 32;
            const uint64_t a = ptx::smem_desc(qbase + qoff, 16, 1024, ptx::kLayoutSw128);
            const uint64_t bd = ptx::smem_desc(kbase + koff, 16, 1024, ptx::kLayoutSw128);
            ptx::mma_bf16(tmem + col_s(h), a, bd, idesc_qk, kk > 0 ? 1u : 0u);
          }
          ptx::mma_commit(ptx::smem_addr(&b.s_full[h]));
        }
        __syncwarp();
      }
      if (!ok) break;
      if (lane == 0) {
        ptx::mma_commit(ptx::smem_addr(&b.k_empty[ks]));
        if (t == nt - 1) ptx::mma_commit(ptx::smem_addr(&b.q_empty));
      }
      __syncwarp();
      const int vs = g % kVStages;
      if (!wait_bar(sm, b.v_full[vs], (g / kVStages) & 1, p.status)) {
        ok = false;
        break;
      }
      clear_v_tail(buf.v[vs], it.tok_end - (it.tok_begin + t * kTile), lane);
      __syncwarp();
      for (int h = 0; h < nh && ok; ++h) {
        // The first PV of an item overwrites O_h: the previous item's epilogue has read it.
        const uint32_t nit = h ? nit1 : nit0;
        if (t == 0 && nit > 0 && !wait_bar(sm, b.o_free[h], (nit - 1) & 1, p.status)) {
          ok = false;
          break;
        }
        if (!wait_bar(sm, b.p_full[h], (h ? npv1 : npv0) & 1, p.status)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        if (lane == 0) {
          const uint32_t vbase = v0 + uint32_t(vs) * kSlotBytes;
#pragma unroll
          for (int kk = 0; kk < kTile / 16; ++kk) {
            const uint64_t bd = ptx::smem_desc(vbase + kk * 2048, kHalfBytes, 1024, ptx::kLayoutSw128);
            ptx::mma_bf16_ts(tmem + col_o(h), tmem + col_s(h) + uint32_t(kk) * 8, bd, idesc_pv,
                             (t > 0 || kk > 0) ? 1u : 0u);
          }
          ptx::mma_commit(ptx::smem_addr(&b.pv_done[h]));
        }
        __syncwarp();
        if (h) ++npv1; else ++npv0;
      }
      if (!ok) break;
      if (lane == 0) ptx::mma_commit(ptx::smem_addr(&b.v_empty[vs]));
      __syncwarp();
    }
    if (!ok) break;
    ++nit0;
    if (nh > 1) ++nit1;
    // The next item's query rows load while this item's last PVs and epilogue run.
    const int nxt = next_item_with_tiles(p, sm, k, lane, kPfMaxRows);
    if (nxt == -2) {
      ok = false;
      break;
    }
    if (nxt >= 0) {
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
  if (lane == 0) ptx::mma_commit(ptx::smem_addr(&b.done));
  __syncwarp();
  drain_bar(b.done, 0);
}

// ------------------------------------------------------------------ softmax / epilogue
__device__ __forceinline__ float max128(const float* s) {
  float m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = s[i];
#pragma unroll
  for (int c = 8; c < kTile; c += 8) {
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = fmaxf(m[i], s[c + i]);
  }
  return fmaxf(fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3])), fmaxf(fmaxf(m[4], m[5]), fmaxf(m[6], m[7])));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// One item for softmax warpgroup h (thread = packed row r of half h).  `gw`
// counts the tiles this warpgroup has consumed (its S / P / PV phases).
template <class Sh>
__device__ bool consume_item(const AttnParams& p, Sh& sm, const WorkItem& it, bool causal, int h, int r,
                             uint32_t tmem_lane, uint32_t& gw) {
  Barriers& b = sm.pf;
  const int group = p.group;
  const int nrows = it.pq_end - it.pq_begin;
  const int nt = n_tiles_of(it);
  const int j = h * pf_half_rows(group) + r;  // row within the item
  const bool valid = r < pf_half_rows(group) && j < nrows;
  const int pq = it.pq_begin + j;
  const int q_idx = pq / group;
  const int head = it.kv_head * group + (pq - q_idx * group);
  // Keys [tok_begin, vis_end) of the item are visible to this row (bottom-right
  // causal mask); padding rows see none.
  int vis_end = it.tok_begin;
  if (valid) vis_end = causal ? min(it.tok_end, it.kv_len - it.q_len + q_idx + 1) : it.tok_end;
  // First/last-query logit dump (raw q.k before scale and mask, fp16): query 0
  // to slot 0, query q_len-1 (q_len > 1) to slot 1.
  __half* dump_row = nullptr;
  if (p.dump != nullptr && valid && (q_idx == 0 || q_idx == it.q_len - 1)) {
    dump_row = p.dump + (int64_t(it.row) * p.dump_num_heads + head) * 2 * p.dump_kv_stride;
    if (q_idx != 0) dump_row += p.dump_kv_stride;
  }
  const int dump_end = p.dump_kv_stride < it.tok_end ? int(p.dump_kv_stride) : it.tok_end;
  const bool warp_dumps = __any_sync(0xffffffffu, dump_row != nullptr);
  const float scale = p.scale_log2;
  const uint32_t s_addr = tmem_lane + col_s(h);
  const uint32_t o_addr = tmem_lane + col_o(h);
  float m_ref = -INFINITY;  // reference row max x scale (log2 domain)
  float l = 0.f;

  for (int t = 0; t < nt; ++t, ++gw) {
    if (!wait_bar(sm, b.s_full[h], gw & 1, p.status)) return false;
    ptx::tc_fence_after();
    const int tile0 = it.tok_begin + t * kTile;
    float s[kTile];
#pragma unroll
    for (int c = 0; c < kTile; c += 32) ptx::tmem_ld32(s_addr + c, s + c);
    ptx::tmem_wait_ld();
    if (warp_dumps && dump_row != nullptr) {
#pragma unroll
      for (int c = 0; c < kTile; ++c)
        if (tile0 + c < dump_end) dump_row[tile0 + c] = __float2half_rn(s[c]);
    }
    const int nvis = vis_end - tile0;
    if (nvis < kTile) {
#pragma unroll
      for (int c = 0; c < kTile; ++c)
        if (c >= nvis) s[c] = -INFINITY;
    }
    const float ms = max128(s) * scale;
    const bool need = ms > m_ref + kLazyLog2;
    float alpha = 1.f;
    if (need) {
      alpha = (m_ref == -INFINITY) ? 0.f : ex2(m_ref - ms);
      l *= alpha;
      m_ref = ms;
    }
    // The previous tile's PV completed before this tile's QK^T was issued, so
    // O_h is at rest: rescale this row in place (tcgen05.ld/st are
    // warp-collective, hence the warp vote).
    if (t > 0 && __any_sync(0xffffffffu, need)) {
      // (In 8-column pieces: S is live in registers meanwhile.)
#pragma unroll 1
      for (int c = 0; c < kHeadDim; c += 8) {
        float o[8];
        ptx::tmem_ld8(o_addr + c, o);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] *= alpha;
        ptx::tmem_st8(o_addr + c, o);
      }
    }
    const float mb = (m_ref == -INFINITY) ? 0.f : m_ref;
    float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float pk[16];  // 16 columns of bf16 pairs (32 keys), as raw bits
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float p0 = ex2(fmaf(s[32 * c + 2 * i], scale, -mb));
        const float p1 = ex2(fmaf(s[32 * c + 2 * i + 1], scale, -mb));
        part[i & 3] += p0 + p1;
        pk[i] = __uint_as_float(pack_bf16x2(p0, p1));
      }
      ptx::tmem_st16(s_addr + 16 * c, pk);
    }
    l += (part[0] + part[1]) + (part[2] + part[3]);
    ptx::tmem_wait_st();
    ptx::tc_fence_before();
    ptx::mbar_arrive(ptx::smem_addr(&b.p_full[h]));
  }

  // Final O_h row once the item's last PV has completed, 32 dims at a time;
  // then O_h is free for the next item.
  if (!wait_bar(sm, b.pv_done[h], (gw - 1) & 1, p.status)) return false;
  ptx::tc_fence_after();
  const float inv = l > 0.f ? 1.f / l : 0.f;
  const float lse = l > 0.f ? m_ref + lg2(l) : -INFINITY;
  int64_t tok = int64_t(it.q_start) + q_idx;
  const bool final_rows = it.n_chunks <= 1;
  const int64_t prow = int64_t(it.partial_base) + int64_t(it.chunk) * nrows + j;
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
  uint32_t gw = 0;
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
      for (int j = h; j < nrows; j += 2) store_final(p, it, it.pq_begin + j, r, 0.f, -INFINITY);
      continue;
    }
    if (h >= halves_of(p, it)) continue;
    if (!consume_item(p, sm, it, causal, h, r, tmem_lane, gw)) return;
  }
}

}  // namespace pf
}  // namespace aspire
