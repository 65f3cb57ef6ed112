// tcgen05 paged-attention kernel for wide packed-query tiles (verify rows,
// and any row whose q_len x group exceeds the gather kernel's 4-row tile).
//
// One persistent CTA per SM walks its list of work items (a KV chunk of one
// (row, KV head, packed-query tile)).  The contraction is laid out "swapped":
// the 128 KV tokens of a tile are the MMA's M dimension and the packed
// (query, head-in-group) rows are its N dimension (16, 32 or 48), so one
// 128-token K/V tile feeds the whole GQA group and N stays small:
//
//   S^T[128 tok x N]  = K[128 tok x 128 d]  . Q^T      (A: K, K-major SW128)
//   O^T[128 d   x N]  = V^T[128 d x 128 tok] . P^T     (A: V, MN-major SW128)
//
// Warp roles (192 threads):
//   warp 0     TMA producer: gathers the tile's 8 pages through the page table
//              as 2 KiB boxes (16 tokens x 64 dims, 128-byte swizzle) of a
//              5-D tensor map over the paged cache; two 64 KiB stages.
//   warp 1     MMA issuer (one thread) and TMEM owner (256 columns: two S and
//              two O buffers).
//   warps 2-5  softmax / epilogue: thread r owns TMEM lane r, i.e. token r of
//              the S tile and dim r of the O tile.  Column maxima are reduced
//              with warp shuffles and shared memory, P^T is written as bf16
//              in the no-swizzle MN-major layout, O is accumulated in
//              registers with the online-softmax rescale.
// Every mbarrier wait is bounded: on timeout the CTA records
// ASPIRE_STATUS_TIMEOUT, stops, drains its own TMA loads and MMAs, frees TMEM
// and returns.
//
// Semantics are those of the gather kernel (FlashInfer's persistent paged
// attention as ASPIRE drives it): bottom-right causal mask, base-2 LSE of the
// scaled logits, fp16 first/last logit dump of the raw q.k.
#include <cuda.h>

#include "kernels.cuh"
#include "tc_ptx.cuh"

namespace aspire {

namespace {

constexpr int kTcThreads = 192;
constexpr int kTile = 128;
constexpr int kPagesPerTile = kTile / kPageSize;
constexpr int kTcStages = 2;
constexpr int kNMax = kTcQTile;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kKvHalfBytes = kTile * 128;          // 128 rows x 128 B
constexpr uint32_t kStageBytes = 4 * kKvHalfBytes;      // K lo, K hi, V lo, V hi
constexpr uint32_t kQHalfBytes = kNMax * 128;
constexpr uint32_t kPBufBytes = (kNMax / 8) * kTile * 16;
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s: far above any legitimate wait

__host__ __device__ constexpr uint32_t col_s(int b) { return uint32_t(b) * 64u; }
__host__ __device__ constexpr uint32_t col_o(int b) { return 128u + uint32_t(b) * 64u; }

struct TcShared {
  uint8_t kv[kTcStages][kStageBytes];
  uint8_t q[2][kQHalfBytes];
  uint8_t p[2][kPBufBytes];
  float red[2][4][kNMax];
  float red_l[4][kNMax];
  float mrun[3][kNMax];
  uint64_t kv_full[kTcStages], kv_empty[kTcStages];
  uint64_t s_full[2], s_empty[2], p_full[2], p_empty[2], o_full[2], o_empty[2];
  uint64_t q_full, done, grp;
  uint32_t tmem_base;
  int abort_flag;
  int merge_flag;
};
static_assert(sizeof(TcShared) + 1024 <= 227 * 1024, "tcgen05 kernel shared memory too large");
static_assert(kNMax % 16 == 0 && kNMax <= 64, "N tile must be a multiple of 16 and fit a 64-column buffer");

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on an mbarrier phase.  Returns false (and stops the CTA) when
// the phase does not complete within kWaitLimitNs or another role aborted.
__device__ __forceinline__ bool wait_bar(TcShared& sm, uint64_t& bar, uint32_t parity, uint32_t* status) {
  const uint32_t a = ptx::smem_addr(&bar);
  if (ptx::mbar_try_wait(a, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (ptx::mbar_try_wait(a, parity)) return true;
    if (*reinterpret_cast<volatile int*>(&sm.abort_flag)) return false;
    if ((i & 255) == 0 && global_ns() - t0 > kWaitLimitNs) break;
  }
  *reinterpret_cast<volatile int*>(&sm.abort_flag) = 1;
  if (status) atomicOr(status, ASPIRE_STATUS_TIMEOUT);
  return false;
}

// Wait used while draining after an abort: ignores the abort flag, still bounded.
__device__ __forceinline__ void drain_bar(uint64_t& bar, uint32_t parity) {
  const uint32_t a = ptx::smem_addr(&bar);
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (ptx::mbar_try_wait(a, parity)) return;
    if ((i & 255) == 0 && global_ns() - t0 > kWaitLimitNs) return;
  }
}

// Barrier of the 128 softmax threads on an mbarrier (bounded, so that a thread
// that stopped on a timeout cannot leave the others blocked).
__device__ __forceinline__ bool group_sync(TcShared& sm, uint32_t& uses, uint32_t* status) {
  ptx::mbar_arrive(ptx::smem_addr(&sm.grp));
  const uint32_t parity = uses & 1;
  ++uses;
  return wait_bar(sm, sm.grp, parity, status);
}

__device__ __forceinline__ int n_tiles_of(const WorkItem& it) {
  return it.tok_end > it.tok_begin ? (it.tok_end - it.tok_begin + kTile - 1) / kTile : 0;
}

// Items every role skips identically (the planner never emits them).
__device__ __forceinline__ bool item_valid(const AttnParams& p, const WorkItem& it) {
  const int nrows = it.pq_end - it.pq_begin;
  return nrows > 0 && nrows <= kNMax && it.kv_head >= 0 && it.kv_head < p.num_kv_heads &&
         it.tok_begin >= 0 && it.tok_begin % kTile == 0 && it.tok_end <= it.kv_len;
}

__device__ __forceinline__ bool aborted(TcShared& sm) {
  return *reinterpret_cast<volatile int*>(&sm.abort_flag) != 0;
}

// ------------------------------------------------------------------ producer
__device__ void run_producer(const AttnParams& p, const CUtensorMap* tmap, TcShared& sm, int item_begin,
                             int item_end, int lane) {
  uint32_t g = 0;
  int64_t last_issue[kTcStages] = {-1, -1};
  bool ok = true;
  for (int ii = item_begin; ii < item_end && ok; ++ii) {
    const WorkItem it = load_item(p.plan, ii);
    if (!item_valid(p, it)) continue;
    const int nt = n_tiles_of(it);
    const int first_page = it.tok_begin / kPageSize;
    const int end_page = (it.tok_end + kPageSize - 1) / kPageSize;
    for (int t = 0; t < nt; ++t, ++g) {
      const int s = g % kTcStages;
      const uint32_t ph = (g / kTcStages) & 1;
      if (!wait_bar(sm, sm.kv_empty[s], ph ^ 1, p.status)) {
        ok = false;
        break;
      }
      if (lane == 0) {
        const uint32_t full = ptx::smem_addr(&sm.kv_full[s]);
        ptx::mbar_arrive_expect_tx(full, kStageBytes);
        const uint32_t base = ptx::smem_addr(sm.kv[s]);
        for (int pg = 0; pg < kPagesPerTile; ++pg) {
          const int lp = first_page + t * kPagesPerTile + pg;
          int page = static_cast<int>(p.num_pages_total);  // out of range: TMA fills zeros
          if (lp < end_page) {
            const int32_t id = p.kv_indices[it.kv_page_base + lp];
            if (id < 0 || int64_t(id) >= p.num_pages_total) {
              record_status(p.status, ASPIRE_STATUS_BAD_PAGE);
            } else {
              page = id;
            }
          }
          const uint32_t off = uint32_t(pg) * kPageSize * 128;
          ptx::tma_load_5d(base + 0 * kKvHalfBytes + off, tmap, full, 0, it.kv_head, 0, 0, page);
          ptx::tma_load_5d(base + 1 * kKvHalfBytes + off, tmap, full, 64, it.kv_head, 0, 0, page);
          ptx::tma_load_5d(base + 2 * kKvHalfBytes + off, tmap, full, 0, it.kv_head, 0, 1, page);
          ptx::tma_load_5d(base + 3 * kKvHalfBytes + off, tmap, full, 64, it.kv_head, 0, 1, page);
        }
      }
      last_issue[s] = g;
      __syncwarp();
    }
  }
  if (!ok || aborted(sm)) {
    // Let this CTA's own copies land before the CTA releases its shared memory.
    for (int s = 0; s < kTcStages; ++s)
      if (last_issue[s] >= 0) drain_bar(sm.kv_full[s], uint32_t(last_issue[s] / kTcStages) & 1);
  }
}

// ------------------------------------------------------------------ MMA issuer
__device__ void run_mma(const AttnParams& p, TcShared& sm, int item_begin, int item_end, int lane) {
  const uint32_t tmem = sm.tmem_base;
  uint32_t g = 0, items_done = 0;
  bool ok = true;
  const uint32_t kv0 = ptx::smem_addr(sm.kv[0]);
  const uint32_t q0 = ptx::smem_addr(sm.q[0]);
  const uint32_t p0 = ptx::smem_addr(sm.p[0]);

  auto issue_pv = [&](uint32_t u, uint32_t idesc_pv) -> bool {
    const int b = u % 2;
    const uint32_t ph = (u / 2) & 1;
    if (!wait_bar(sm, sm.p_full[b], ph, p.status)) return false;
    if (!wait_bar(sm, sm.o_empty[b], ph ^ 1, p.status)) return false;
    ptx::tc_fence_after();
    if (lane == 0) {
      const uint32_t vbase = kv0 + uint32_t(b) * kStageBytes + 2 * kKvHalfBytes;
      const uint32_t pbase = p0 + uint32_t(b) * kPBufBytes;
#pragma unroll
      for (int kk = 0; kk < kTile / 16; ++kk) {
        const uint64_t a = ptx::smem_desc(vbase + kk * 2048, kKvHalfBytes, 1024, ptx::kLayoutSw128);
        const uint64_t bd = ptx::smem_desc(pbase + kk * 256, 128, kTile * 16, ptx::kLayoutNone);
        ptx::mma_bf16(tmem + col_o(b), a, bd, idesc_pv, kk > 0 ? 1u : 0u);
      }
      ptx::mma_commit(ptx::smem_addr(&sm.o_full[b]));
      ptx::mma_commit(ptx::smem_addr(&sm.kv_empty[b]));
      ptx::mma_commit(ptx::smem_addr(&sm.p_empty[b]));
    }
    __syncwarp();
    return true;
  };

  for (int ii = item_begin; ii < item_end && ok; ++ii) {
    const WorkItem it = load_item(p.plan, ii);
    if (!item_valid(p, it)) continue;
    const int nt = n_tiles_of(it);
    if (nt == 0) continue;
    const int nrows = it.pq_end - it.pq_begin;
    const uint32_t N = uint32_t((nrows + 15) / 16 * 16);
    const uint32_t idesc_qk = ptx::idesc_bf16(128, N, false, false);
    const uint32_t idesc_pv = ptx::idesc_bf16(128, N, true, true);
    if (!wait_bar(sm, sm.q_full, items_done & 1, p.status)) {
      ok = false;
      break;
    }
    for (int t = 0; t < nt && ok; ++t, ++g) {
      const int b = g % 2;
      const uint32_t ph = (g / 2) & 1;
      if (!wait_bar(sm, sm.kv_full[b], ph, p.status) || !wait_bar(sm, sm.s_empty[b], ph ^ 1, p.status)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      if (lane == 0) {
        const uint32_t kbase = kv0 + uint32_t(b) * kStageBytes;
#pragma unroll
        for (int kk = 0; kk < 128 / 16; ++kk) {
          const uint32_t koff = uint32_t(kk / 4) * kKvHalfBytes + uint32_t(kk % 4) * 32;
          const uint32_t qoff = uint32_t(kk / 4) * kQHalfBytes + uint32_t(kk % 4) * 32;
          const uint64_t a = ptx::smem_desc(kbase + koff, 16, 1024, ptx::kLayoutSw128);
          const uint64_t bd = ptx::smem_desc(q0 + qoff, 16, 1024, ptx::kLayoutSw128);
          ptx::mma_bf16(tmem + col_s(b), a, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        ptx::mma_commit(ptx::smem_addr(&sm.s_full[b]));
      }
      __syncwarp();
      if (t > 0 && !issue_pv(g - 1, idesc_pv)) ok = false;
    }
    if (ok && !issue_pv(g - 1, idesc_pv)) ok = false;
    ++items_done;
  }
  // Every MMA this thread issued has completed once `done` fires.
  if (lane == 0) ptx::mma_commit(ptx::smem_addr(&sm.done));
  __syncwarp();
  drain_bar(sm.done, 0);
}

// ------------------------------------------------------------------ softmax / epilogue
template <int N>
__device__ bool consume_item(const AttnParams& p, TcShared& sm, const WorkItem& it, bool causal, int r,
                             int ctid, int wq, int lane, uint32_t& g, uint32_t& grp_uses) {
  const int nrows = it.pq_end - it.pq_begin;
  const int nt = n_tiles_of(it);
  const uint32_t tmem_lane = sm.tmem_base + (uint32_t(wq * 32) << 16);
  const float scale = p.scale_log2;
  const int group = p.group;

  // Stage Q (K-major, 128-byte swizzle; rows >= nrows are zero).
  for (int e = ctid; e < N * 16; e += 128) {
    const int j = e >> 4, c = e & 15;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (j < nrows) {
      int q_idx, head;
      packed_row(p, it, it.pq_begin + j, q_idx, head);
      v = *reinterpret_cast<const uint4*>(p.q + int64_t(it.q_start + q_idx) * p.q_stride_n +
                                          int64_t(head) * p.q_stride_h + c * 8);
    }
    uint8_t* dst = sm.q[c >> 3] + j * 128 + (((c & 7) ^ (j & 7)) << 4);
    *reinterpret_cast<uint4*>(dst) = v;
  }
  ptx::fence_proxy_async_smem();
  ptx::mbar_arrive(ptx::smem_addr(&sm.q_full));

  // Per-column facts: query index, causal limit, dump slot.
  const int q_idx0 = it.pq_begin / group;
  float o_acc[N], l[N];
#pragma unroll
  for (int j = 0; j < N; ++j) {
    o_acc[j] = 0.f;
    l[j] = 0.f;
  }
  bool ok = true;
  const uint32_t g0 = g;

  auto acc_o = [&](int u) -> bool {
    const uint32_t gu = g0 + u;
    const int b = gu % 2;
    const uint32_t ph = (gu / 2) & 1;
    if (!wait_bar(sm, sm.o_full[b], ph, p.status)) return false;
    ptx::tc_fence_after();
    float ov[N];
#pragma unroll
    for (int i = 0; i < N / 16; ++i) ptx::tmem_ld16(tmem_lane + col_o(b) + 16 * i, ov + 16 * i);
    ptx::tmem_wait_ld();
    ptx::tc_fence_before();
    ptx::mbar_arrive(ptx::smem_addr(&sm.o_empty[b]));
    const float* m_now = sm.mrun[u % 3];
    const float* m_prev = sm.mrun[(u + 2) % 3];
#pragma unroll
    for (int j = 0; j < N; ++j) {
      float alpha = 0.f;
      if (u > 0) {
        const float mp = m_prev[j], mn = m_now[j];
        alpha = (mp == -INFINITY) ? 0.f : (mp == mn ? 1.f : ex2((mp - mn) * scale));
      }
      o_acc[j] = fmaf(o_acc[j], alpha, ov[j]);
    }
    return true;
  };

  for (int t = 0; t < nt; ++t) {
    const uint32_t gt = g0 + t;
    const int b = gt % 2;
    const uint32_t ph = (gt / 2) & 1;
    if (!wait_bar(sm, sm.s_full[b], ph, p.status)) {
      ok = false;
      break;
    }
    ptx::tc_fence_after();
    float sv[N];
#pragma unroll
    for (int i = 0; i < N / 16; ++i) ptx::tmem_ld16(tmem_lane + col_s(b) + 16 * i, sv + 16 * i);
    ptx::tmem_wait_ld();
    ptx::tc_fence_before();
    ptx::mbar_arrive(ptx::smem_addr(&sm.s_empty[b]));

    const int tile0 = it.tok_begin + t * kTile;
    const int tok = tile0 + r;
    const bool in_chunk = tok < it.tok_end;
    if (p.dump != nullptr && in_chunk) {
#pragma unroll
      for (int j = 0; j < N; ++j) {
        if (j < nrows) {
          const int pq = it.pq_begin + j;
          const int q_idx = pq / group;
          const bool s0 = q_idx == 0, s1 = q_idx != 0 && q_idx + 1 == it.q_len;
          if (s0 || s1) {
            const int head = it.kv_head * group + (pq - q_idx * group);
            const int64_t idx = ((int64_t(it.row) * p.dump_num_heads + head) * 2 + (s0 ? 0 : 1)) * p.dump_kv_stride + tok;
            p.dump[idx] = __float2half_rn(sv[j]);
          }
        }
      }
    }
    const int limit_min = causal ? (it.kv_len - it.q_len + q_idx0 + 1) : it.kv_len;
    // Padded columns (j >= nrows) only feed ignored O columns: they need no mask.
    const bool full_tile = tile0 + kTile <= it.tok_end && tile0 + kTile <= limit_min;
    if (!full_tile) {
#pragma unroll
      for (int j = 0; j < N; ++j) {
        const int q_idx = (it.pq_begin + j) / group;
        const int lim = causal ? (it.kv_len - it.q_len + q_idx + 1) : it.kv_len;
        if (!(in_chunk && tok < lim)) sv[j] = -INFINITY;
      }
    }
    // Column maxima of the tile: butterfly within the warp, then across the 4 warps.
    float* red = sm.red[t & 1][wq];
#pragma unroll
    for (int j = 0; j < N; ++j) {
      float mx = sv[j];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      if (lane == (j & 31)) red[j] = mx;
    }
    if (!group_sync(sm, grp_uses, p.status)) {
      ok = false;
      break;
    }
    const float* r0 = sm.red[t & 1][0];
    const float* r1 = sm.red[t & 1][1];
    const float* r2 = sm.red[t & 1][2];
    const float* r3 = sm.red[t & 1][3];
    const float* m_prev = sm.mrun[(t + 2) % 3];
    float* m_cur = sm.mrun[t % 3];
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const float tmax = fmaxf(fmaxf(r0[j], r1[j]), fmaxf(r2[j], r3[j]));
      const float mp = t > 0 ? m_prev[j] : -INFINITY;
      const float mn = fmaxf(mp, tmax);
      if (ctid == j) m_cur[j] = mn;
      const float alpha = (mp == -INFINITY) ? 0.f : (mp == mn ? 1.f : ex2((mp - mn) * scale));
      const float pv = (mn == -INFINITY) ? 0.f : ex2(fmaf(sv[j], scale, -mn * scale));
      l[j] = fmaf(l[j], alpha, pv);
      sv[j] = pv;
    }
    // P^T as bf16, MN-major without swizzle: 8 queries x 16 B per token, token-major.
    if (!wait_bar(sm, sm.p_empty[b], ph ^ 1, p.status)) {
      ok = false;
      break;
    }
    uint8_t* pbuf = sm.p[b];
#pragma unroll
    for (int c = 0; c < N / 8; ++c) {
      uint4 v;
      __nv_bfloat162 h0 = __floats2bfloat162_rn(sv[8 * c + 0], sv[8 * c + 1]);
      __nv_bfloat162 h1 = __floats2bfloat162_rn(sv[8 * c + 2], sv[8 * c + 3]);
      __nv_bfloat162 h2 = __floats2bfloat162_rn(sv[8 * c + 4], sv[8 * c + 5]);
      __nv_bfloat162 h3 = __floats2bfloat162_rn(sv[8 * c + 6], sv[8 * c + 7]);
      v.x = *reinterpret_cast<uint32_t*>(&h0);
      v.y = *reinterpret_cast<uint32_t*>(&h1);
      v.z = *reinterpret_cast<uint32_t*>(&h2);
      v.w = *reinterpret_cast<uint32_t*>(&h3);
      *reinterpret_cast<uint4*>(pbuf + c * (kTile * 16) + r * 16) = v;
    }
    ptx::fence_proxy_async_smem();
    ptx::mbar_arrive(ptx::smem_addr(&sm.p_full[b]));
    if (t > 0 && !acc_o(t - 1)) {
      ok = false;
      break;
    }
  }
  if (ok && nt > 0 && !acc_o(nt - 1)) ok = false;
  g = g0 + nt;
  if (!ok) return false;

  // Column sums of l across the 128 threads.
#pragma unroll
  for (int j = 0; j < N; ++j) {
    float sum = l[j];
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if (lane == (j & 31)) sm.red_l[wq][j] = sum;
  }
  if (!group_sync(sm, grp_uses, p.status)) return false;
  const float* m_fin = sm.mrun[(nt + 2) % 3];  // m of the last tile
  float o_fin[N];
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const float L = sm.red_l[0][j] + sm.red_l[1][j] + sm.red_l[2][j] + sm.red_l[3][j];
    o_fin[j] = L > 0.f ? o_acc[j] / L : 0.f;
  }
  float my_lse = -INFINITY;  // LSE of column ctid
  if (ctid < nrows) {
    const float L = sm.red_l[0][ctid] + sm.red_l[1][ctid] + sm.red_l[2][ctid] + sm.red_l[3][ctid];
    my_lse = L > 0.f ? fmaf(m_fin[ctid], scale, lg2(L)) : -INFINITY;
  }
  const int d = r;  // this thread's output dim
  if (it.n_chunks <= 1) {
#pragma unroll
    for (int j = 0; j < N; ++j) {
      if (j < nrows) {
        int q_idx, head;
        packed_row(p, it, it.pq_begin + j, q_idx, head);
        const int64_t tokrow = int64_t(it.q_start) + q_idx;
        p.out[tokrow * p.o_stride_n + int64_t(head) * p.o_stride_h + d] = __float2bfloat16_rn(o_fin[j]);
      }
    }
    if (ctid < nrows && p.lse) {
      int q_idx, head;
      packed_row(p, it, it.pq_begin + ctid, q_idx, head);
      p.lse[(int64_t(it.q_start) + q_idx) * p.num_qo_heads + head] = my_lse;
    }
  } else {
    float* plse = partial_lse_ptr(p);
    const int64_t base = int64_t(it.partial_base) + int64_t(it.chunk) * nrows;
#pragma unroll
    for (int j = 0; j < N; ++j)
      if (j < nrows) p.partial_o[(base + j) * kHeadDim + d] = o_fin[j];
    if (ctid < nrows) plse[base + ctid] = my_lse;
    __threadfence();
    if (!group_sync(sm, grp_uses, p.status)) return false;
    int32_t* counters = const_cast<int32_t*>(p.plan) + p.plan[kHdrOffCounters];
    if (ctid == 0) {
      const int prev = atomicAdd(&counters[it.merge_id], 1);
      sm.merge_flag = (prev == it.n_chunks - 1);
    }
    if (!group_sync(sm, grp_uses, p.status)) return false;
    if (sm.merge_flag) {
      __threadfence();
      for (int j = 0; j < nrows; ++j) {
        float m = -INFINITY;
        for (int c = 0; c < it.n_chunks; ++c)
          m = fmaxf(m, __ldcg(plse + it.partial_base + int64_t(c) * nrows + j));
        float acc = 0.f, wsum = 0.f;
        if (m != -INFINITY) {
          for (int c = 0; c < it.n_chunks; ++c) {
            const int64_t prow = it.partial_base + int64_t(c) * nrows + j;
            const float w = ex2(__ldcg(plse + prow) - m);
            wsum += w;
            acc += w * __ldcg(p.partial_o + prow * kHeadDim + d);
          }
        }
        store_final(p, it, it.pq_begin + j, d, wsum > 0.f ? acc / wsum : 0.f,
                    wsum > 0.f ? m + lg2(wsum) : -INFINITY);
      }
      if (ctid == 0) counters[it.merge_id] = 0;
    }
  }
  // The ring buffers are reused by the next item.
  return group_sync(sm, grp_uses, p.status);
}

__device__ void run_consumer(const AttnParams& p, TcShared& sm, int item_begin, int item_end, bool causal,
                             int warp, int lane) {
  const int wq = warp & 3;
  const int r = wq * 32 + lane;          // TMEM lane = S-tile token = O-tile dim
  const int ctid = threadIdx.x - 64;     // 0..127
  uint32_t g = 0, grp_uses = 0;
  for (int ii = item_begin; ii < item_end; ++ii) {
    if (aborted(sm)) return;
    const WorkItem it = load_item(p.plan, ii);
    const int nrows = it.pq_end - it.pq_begin;
    if (!item_valid(p, it)) {
      if (ctid == 0) record_status(p.status, ASPIRE_STATUS_BAD_PLAN);
      continue;
    }
    if (n_tiles_of(it) == 0) {
      // No keys: zero output, -inf LSE (chunked items always have keys).
      for (int j = 0; j < nrows; ++j) store_final(p, it, it.pq_begin + j, r, 0.f, -INFINITY);
      continue;
    }
    const int N = (nrows + 15) / 16 * 16;
    bool ok;
    if (N == 16)
      ok = consume_item<16>(p, sm, it, causal, r, ctid, wq, lane, g, grp_uses);
    else if (N == 32)
      ok = consume_item<32>(p, sm, it, causal, r, ctid, wq, lane, g, grp_uses);
    else
      ok = consume_item<48>(p, sm, it, causal, r, ctid, wq, lane, g, grp_uses);
    if (!ok) return;
  }
}

}  // namespace

__global__ void __launch_bounds__(kTcThreads, 1)
    aspire_attn_tc_kernel(AttnParams p, const __grid_constant__ CUtensorMap tmap) {
  extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
  const uint32_t raw = ptx::smem_addr(tc_smem_raw);
  TcShared& sm = *reinterpret_cast<TcShared*>(tc_smem_raw + ((1024 - (raw & 1023)) & 1023));
  const int32_t* plan = p.plan;
  if (plan[kHdrMagic] != kPlanMagic) return;
  if (int(blockIdx.x) >= plan[kHdrNumTcCtas]) return;
  const int32_t* indptr = plan + plan[kHdrOffTcIndptr];
  const int item_begin = indptr[blockIdx.x], item_end = indptr[blockIdx.x + 1];
  if (item_begin >= item_end) return;
  const bool causal = plan[kHdrCausal] != 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      ptx::mbar_init(ptx::smem_addr(&sm.kv_full[s]), 1);
      ptx::mbar_init(ptx::smem_addr(&sm.kv_empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(ptx::smem_addr(&sm.s_full[b]), 1);
      ptx::mbar_init(ptx::smem_addr(&sm.s_empty[b]), 128);
      ptx::mbar_init(ptx::smem_addr(&sm.p_full[b]), 128);
      ptx::mbar_init(ptx::smem_addr(&sm.p_empty[b]), 1);
      ptx::mbar_init(ptx::smem_addr(&sm.o_full[b]), 1);
      ptx::mbar_init(ptx::smem_addr(&sm.o_empty[b]), 128);
    }
    ptx::mbar_init(ptx::smem_addr(&sm.q_full), 128);
    ptx::mbar_init(ptx::smem_addr(&sm.done), 1);
    ptx::mbar_init(ptx::smem_addr(&sm.grp), 128);
    sm.abort_flag = 0;
    sm.merge_flag = 0;
    ptx::mbar_fence_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_addr(&sm.tmem_base), kTmemCols);
    ptx::tmem_relinquish();
  }
  if (warp == 0 && lane == 0) ptx::prefetch_tmap(&tmap);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();

  if (warp == 0) {
    run_producer(p, &tmap, sm, item_begin, item_end, lane);
  } else if (warp == 1) {
    run_mma(p, sm, item_begin, item_end, lane);
  } else {
    run_consumer(p, sm, item_begin, item_end, causal, warp, lane);
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(sm.tmem_base, kTmemCols);
}

size_t tc_smem_bytes() { return sizeof(TcShared) + 1024; }

bool tc_kernel_available() { return true; }

}  // namespace aspire
