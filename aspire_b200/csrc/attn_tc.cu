// tcgen05 paged-attention kernel for wide packed-query tiles (verify rows,
// and any row whose q_len x group exceeds the gather kernel's 4-row tile).
//
// One persistent CTA per SM claims work items (a KV chunk of one (row, KV
// head, packed-query tile)) from the plan's shared list, longest first.  The contraction is laid out "swapped":
// the 128 KV tokens of a tile are the MMA's M dimension and the packed
// (query, head-in-group) rows are its N dimension (16, 32 or 48), so one
// 128-token K/V tile feeds the whole GQA group and N stays small:
//
//   S^T[128 tok x N]  = K[128 tok x 128 d]  . Q^T      (A: K, K-major SW128)
//   O^T[128 d   x N] += V^T[128 d x 128 tok] . P^T     (A: V, MN-major SW128)
//
// Warp roles (384 threads):
//   warp 0     K producer: TMA-gathers the tile's 8 pages (2 KiB boxes of 16
//              tokens x 64 dims, 128-byte swizzle, through a 5-D tensor map
//              over the paged cache) into a 2-stage K ring.
//   warp 10    V producer: the same into a 3-stage V ring.
//   warp 1     QK^T issuer (one thread) and TMEM owner (two S tiles and the
//              O accumulator).  A K stage is released as soon as its QK^T
//              completes.  It also TMA-loads each item's query tile while the
//              previous item finishes.
//   warp 11    P.V issuer: a V stage is released when its PV completes.
//              (In the prefill phase warps 1 and 11 issue the products of
//              the item's two halves.)
//   warps 2-9  softmax / epilogue in two warpgroups that split the item's N
//              columns in halves: thread r of a group owns TMEM lane r, i.e.
//              token r of the S tile and dim r of the O tile, for the group's
//              columns.  The running column max is kept lazily: a tile only
//              triggers the cross-thread max reduction (warp reduce-scatter +
//              shared memory) and the O/l rescale when one of its logits
//              exceeds the current max by more than 2^8 in the exp2 domain,
//              so P stays <= 256 and the common tile needs one warp vote and
//              one 128-thread barrier per group.  P^T is written as bf16
//              (no-swizzle MN-major), O accumulates in TMEM, finished rows
//              leave through shared memory by bulk stores.
// Every mbarrier wait is time-bounded (1 s unless aspire_set_wait_limit_ns
// sets another bound): on timeout the CTA records ASPIRE_STATUS_TIMEOUT,
// stops, drains its own TMA loads and MMAs (those waits keep a fixed 1 s
// bound), frees TMEM and returns.
//
// The same launch then serves the plan's prefill list (long-query rows; see
// attn_prefill.cuh): a CTA that finds the decode list exhausted waits for its
// own decode work to drain and switches roles in place (same warps, same
// item-sequence ring, prefill buffers over the decode buffers, 512 TMEM
// columns allocated once), so batches without prefill rows pay no extra
// launch and mixed batches need no second grid.
//
// Semantics are those of the gather kernel (FlashInfer's persistent paged
// attention as ASPIRE drives it): bottom-right causal mask, base-2 LSE of the
// scaled logits, logit dump of the raw q.k (first/last or last-token).
#include <cuda.h>

#include "attn_prefill.cuh"
#include "kernels.cuh"
#include "tc_pipeline.cuh"
#include "tc_ptx.cuh"

namespace aspire {

namespace {

using namespace pipe;

constexpr int kTcThreads = 384;
constexpr int kFirstSoftmaxWarp = 2;  // warps 2-5: softmax group 0, warps 6-9: group 1
constexpr int kVProducerWarp = 10;
constexpr int kPvWarp = 11;           // decode phase: the P.V issuer
constexpr int kSeqReaders = 11;       // V producer, the two MMA warps and the 8 softmax warps
constexpr int kKStages = 2;
constexpr int kVStages = 3;
constexpr int kNMax = kTcQTile;
constexpr uint32_t kTmemCols = pf::kTmemCols;  // the decode phase uses [0, 256)
constexpr uint32_t kQHalfBytes = kNMax * 128;
constexpr uint32_t kPBufBytes = (kNMax / 8) * kTile * 16;
constexpr float kLazyLog2 = 8.0f;                  // max growth tolerated before a rescale

__host__ __device__ constexpr uint32_t col_s(int b) { return uint32_t(b) * 64u; }
constexpr uint32_t kColO = 128;

struct TcShared {
  uint8_t k[kKStages][kSlotBytes];
  uint8_t v[kVStages][kSlotBytes];
  uint8_t q[2][kQHalfBytes];
  uint8_t p[2][kPBufBytes];
  uint8_t out_stage[kNMax * kHeadDim * 4];  // finished rows (fp32 partial or bf16) on their way out
  float red[2][4][kNMax];
  float red_l[4][kNMax];
  float alpha[2][kNMax];
  float inv_l[kNMax];     // 1 / column sum of the finished item
  float mref[2][kNMax];   // column reference max x scale (log2 domain), double buffered
  int flags[2][2][4];     // per softmax group: per-warp exceed votes, double buffered
  int grew[2][2];         // per softmax group: some column reference grew (exceed path)
  uint64_t k_full[kKStages], k_empty[kKStages];
  uint64_t v_full[kVStages], v_empty[kVStages];
  uint64_t s_full[2], s_empty[2], p_full[2], p_empty[2];
  uint64_t o_free, q_full, q_empty, done, done_pv, grp[2];
  pf::Barriers pf;  // prefill phase
  uint64_t seq_full[kSeqDepth], seq_empty[kSeqDepth];
  int seq[kSeqDepth];
  uint64_t wait_ns;  // bound of one pipeline wait (launch parameter)
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(TcShared) + 1024 <= 227 * 1024, "tcgen05 kernel shared memory too large");
// The prefill phase's buffers overlay the decode phase's data buffers only.
static_assert(sizeof(pf::Buffers) <= offsetof(TcShared, red), "prefill buffers overlap decode state");
static_assert(kNMax % 16 == 0 && kNMax <= 64, "N tile must be a multiple of 16 and fit a 64-column buffer");

// Columns N of an item's products: its packed rows rounded up to 16, or the
// wider width its plan gives it (WorkItem::cols: the planners give the long
// groups' items one width when there are few items per CTA, so that those
// CTAs stream at one rate).  Each width has its own softmax loop
// (consume_item<N / 2>).  A value that is not a multiple of 16 between the
// rows' own width and kNMax is ignored, so every role derives the same N.
// Launches with the dump keep the exact widths (their dump path is longer
// per column).
__device__ __forceinline__ int item_columns(const WorkItem& it, bool use_cols) {
  const int exact = (it.pq_end - it.pq_begin + 15) / 16 * 16;
  return use_cols && it.cols > exact && it.cols <= kNMax && it.cols % 16 == 0 ? it.cols : exact;
}

// Barrier of one softmax warpgroup's 128 threads on an mbarrier (bounded, so that a thread
// that stopped on a timeout cannot leave the others blocked).
__device__ __forceinline__ bool group_sync(TcShared& sm, uint64_t& grp, uint32_t& uses, uint32_t* status) {
  ptx::mbar_arrive(ptx::smem_addr(&grp));
  const uint32_t parity = uses & 1;
  ++uses;
  return wait_bar(sm, grp, parity, status);
}

// ------------------------------------------------------------------ MMA issuers
// A tcgen05.mma issue proceeds at about the rate the tensor core takes the
// instruction (~90 cycles for these small-N products), so one thread issuing
// both products of a tile (16 instructions) plus its barrier traffic would
// take about as long as the tile's 64 KiB take to arrive from HBM at a
// power-capped clock.  The two products share no data (S buffers vs the O
// accumulator), so each has its own issuing warp.
//
// Shared-memory descriptors of consecutive K steps differ only in their
// start-address field (address >> 4, 14 bits, no carry for addresses inside
// the CTA's shared memory), so each loop adds offsets to a base descriptor.

// QK^T of every tile, and the query-tile loads (warp 1).
__device__ void run_qk(const AttnParams& p, const CUtensorMap* qmap, TcShared& sm, int lane, uint32_t& k,
                       bool use_cols) {
  const uint32_t tmem = sm.tmem_base;
  uint32_t g = 0, items_done = 0;
  bool ok = true;
  const uint32_t k0 = ptx::smem_addr(sm.k[0]);
  const uint32_t q0 = ptx::smem_addr(sm.q[0]);
  const uint64_t qdesc0 = ptx::smem_desc(q0, 16, 1024, ptx::kLayoutSw128);
  bool q_pending = false;  // a query-tile load is in flight

  int ii = next_item_with_tiles(p, sm, k, lane, kNMax);
  if (ii == -2) ok = false;
  if (ii >= 0) {
    if (lane == 0) issue_q(p, qmap, sm, ii, p.q_box_tokens);
    q_pending = true;
  }
  while (ii >= 0 && ok) {
    const WorkItem it = load_item(p.plan, ii);
    const int nt = n_tiles_of(it);
    const uint32_t N = uint32_t(item_columns(it, use_cols));
    const uint32_t idesc_qk = ptx::idesc_bf16(128, N, false, false);
    if (!wait_bar(sm, sm.q_full, items_done & 1, p.status)) {
      ok = false;
      break;
    }
    q_pending = false;
    for (int t = 0; t < nt && ok; ++t, ++g) {
      const int ks = g % kKStages, sb = g % 2;
      if (!wait_bar(sm, sm.k_full[ks], (g / kKStages) & 1, p.status) ||
          !wait_bar(sm, sm.s_empty[sb], ((g / 2) & 1) ^ 1, p.status)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      if (lane == 0) {
        const uint64_t kdesc0 = ptx::smem_desc(k0 + uint32_t(ks) * kSlotBytes, 16, 1024, ptx::kLayoutSw128);
#pragma unroll
        for (int kk = 0; kk < 128 / 16; ++kk) {
          const uint32_t koff = uint32_t(kk / 4) * kHalfBytes + uint32_t(kk % 4) * 32;
          const uint32_t qoff = uint32_t(kk / 4) * kQHalfBytes + uint32_t(kk % 4) * 32;
          ptx::mma_bf16(tmem + col_s(sb), kdesc0 + (koff >> 4), qdesc0 + (qoff >> 4), idesc_qk, kk > 0 ? 1u : 0u);
        }
        ptx::mma_commit(ptx::smem_addr(&sm.s_full[sb]));
        ptx::mma_commit(ptx::smem_addr(&sm.k_empty[ks]));
        if (t == nt - 1) ptx::mma_commit(ptx::smem_addr(&sm.q_empty));
      }
      __syncwarp();
    }
    if (!ok) break;
    // The next item's query tile loads while this item's last PV and epilogue run.
    const int nxt = next_item_with_tiles(p, sm, k, lane, kNMax);
    if (nxt == -2) {
      ok = false;
      break;
    }
    if (nxt >= 0) {
      if (!wait_bar(sm, sm.q_empty, items_done & 1, p.status)) {
        ok = false;
        break;
      }
      if (lane == 0) issue_q(p, qmap, sm, nxt, p.q_box_tokens);
      q_pending = true;
      __syncwarp();
    }
    ++items_done;
    ii = nxt;
  }
  // A query load still in flight lands before the CTA releases its memory.
  if (q_pending) drain_bar(sm.q_full, items_done & 1);
  // Every MMA this thread issued has completed once `done` fires.
  if (lane == 0) ptx::mma_commit(ptx::smem_addr(&sm.done));
  __syncwarp();
  drain_bar(sm.done, 0);
}

// P.V of every tile into the O accumulator (warp 11).
__device__ void run_pv(const AttnParams& p, TcShared& sm, int lane, uint32_t& k, bool use_cols) {
  const uint32_t tmem = sm.tmem_base;
  uint32_t g = 0, items_done = 0;
  bool ok = true;
  const uint32_t v0 = ptx::smem_addr(sm.v[0]);
  const uint32_t p0 = ptx::smem_addr(sm.p[0]);
  int ii = next_item_with_tiles(p, sm, k, lane, kNMax);
  if (ii == -2) ok = false;
  while (ii >= 0 && ok) {
    const WorkItem it = load_item(p.plan, ii);
    const int nt = n_tiles_of(it);
    const uint32_t N = uint32_t(item_columns(it, use_cols));
    const uint32_t idesc_pv = ptx::idesc_bf16(128, N, true, true);
    for (int t = 0; t < nt && ok; ++t, ++g) {
      const uint32_t vs = g % kVStages, pb = g % 2;
      // The item's first PV overwrites O: the previous item's epilogue has read it.
      if ((t == 0 && !wait_bar(sm, sm.o_free, (items_done & 1) ^ 1, p.status)) ||
          !wait_bar(sm, sm.v_full[vs], (g / kVStages) & 1, p.status)) {
        ok = false;
        break;
      }
      clear_v_tail(sm.v[vs], it.tok_end - (it.tok_begin + t * kTile), lane);
      __syncwarp();
      if (!wait_bar(sm, sm.p_full[pb], (g / 2) & 1, p.status)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      if (lane == 0) {
        const uint64_t vdesc0 = ptx::smem_desc(v0 + vs * kSlotBytes, kHalfBytes, 1024, ptx::kLayoutSw128);
        const uint64_t pdesc0 = ptx::smem_desc(p0 + pb * kPBufBytes, 128, kTile * 16, ptx::kLayoutNone);
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          ptx::mma_bf16(tmem + kColO, vdesc0 + uint64_t(kk * 2048 >> 4), pdesc0 + uint64_t(kk * 256 >> 4), idesc_pv,
                        (t > 0 || kk > 0) ? 1u : 0u);
        ptx::mma_commit(ptx::smem_addr(&sm.v_empty[vs]));
        ptx::mma_commit(ptx::smem_addr(&sm.p_empty[pb]));
      }
      __syncwarp();
    }
    if (!ok) break;
    ++items_done;
    ii = next_item_with_tiles(p, sm, k, lane, kNMax);
    if (ii == -2) ok = false;
  }
  if (lane == 0) ptx::mma_commit(ptx::smem_addr(&sm.done_pv));
  __syncwarp();
  drain_bar(sm.done_pv, 0);
}

// ------------------------------------------------------------------ warp reductions
template <bool kMax>
__device__ __forceinline__ float combine(float a, float b) {
  return kMax ? fmaxf(a, b) : a + b;
}

// v[0..2W) -> v[0..W): keep the half selected by this lane's `off` bit, send
// the other half to the partner lane, combine.
template <int W, bool kMax>
__device__ __forceinline__ void scatter_step(float* v, int lane, int off) {
  const bool hi = (lane & off) != 0;
#pragma unroll
  for (int i = 0; i < W; ++i) {
    const float keep = hi ? v[W + i] : v[i];
    const float send = hi ? v[i] : v[W + i];
    v[i] = combine<kMax>(keep, __shfl_xor_sync(0xffffffffu, send, off));
  }
}

// Reduce-scatter over the 32 lanes, in place (v is destroyed): lane l returns
// the reduction of column l.
template <bool kMax>
__device__ __forceinline__ float reduce_scatter32(float* v, int lane) {
  scatter_step<16, kMax>(v, lane, 16);
  scatter_step<8, kMax>(v, lane, 8);
  scatter_step<4, kMax>(v, lane, 4);
  scatter_step<2, kMax>(v, lane, 2);
  scatter_step<1, kMax>(v, lane, 1);
  return v[0];
}

// 16 columns over 32 lanes, in place: lane l returns the reduction of column l & 15.
template <bool kMax>
__device__ __forceinline__ float reduce_scatter16(float* v, int lane) {
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = combine<kMax>(v[i], __shfl_xor_sync(0xffffffffu, v[i], 16));
  scatter_step<8, kMax>(v, lane, 8);
  scatter_step<4, kMax>(v, lane, 4);
  scatter_step<2, kMax>(v, lane, 2);
  scatter_step<1, kMax>(v, lane, 1);
  return v[0];
}

// 8 columns over 32 lanes, in place: lane l returns the reduction of column l & 7.
template <bool kMax>
__device__ __forceinline__ float reduce_scatter8(float* v, int lane) {
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = combine<kMax>(v[i], __shfl_xor_sync(0xffffffffu, v[i], 16));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = combine<kMax>(v[i], __shfl_xor_sync(0xffffffffu, v[i], 8));
  scatter_step<4, kMax>(v, lane, 4);
  scatter_step<2, kMax>(v, lane, 2);
  scatter_step<1, kMax>(v, lane, 1);
  return v[0];
}

// Per-warp reduction of NH (8, 16 or 24) columns over the 32 lanes, written to
// out[0..NH).  Destroys v.
template <int NH, bool kMax>
__device__ __forceinline__ void warp_columns(float* v, float* out, int lane) {
  if constexpr (NH == 8) {
    const float r8 = reduce_scatter8<kMax>(v, lane);
    if (lane < 8) out[lane] = r8;
  } else {
    const float r16 = reduce_scatter16<kMax>(v, lane);
    if (lane < 16) out[lane] = r16;
    if constexpr (NH == 24) {
      const float r8 = reduce_scatter8<kMax>(v + 16, lane);
      if (lane < 8) out[16 + lane] = r8;
    }
  }
}

// NH consecutive TMEM columns of this warp's lanes (NH = 8, 16 or 24).
template <int NH>
__device__ __forceinline__ void tmem_load_cols(uint32_t taddr, float* v) {
  if constexpr (NH >= 16) ptx::tmem_ld16(taddr, v);
  if constexpr (NH == 8) ptx::tmem_ld8(taddr, v);
  if constexpr (NH == 24) ptx::tmem_ld8(taddr + 16, v + 16);
}

// ------------------------------------------------------------------ softmax / epilogue
// Writes dump columns [lo, hi) of one token (raw logits, dump_store); column
// c goes to element base + (c - base_col) * col_stride + tok.  The first 8
// are in dv, further pieces are read from the S tile at s_addr.  Kept out of
// line: the three column-count instantiations of the consumer loop share it,
// which keeps their hot loops small.
__device__ __noinline__ void dump_columns(const AttnParams& p, int lo, int hi, int64_t base, int base_col,
                                          int64_t col_stride, int tok, bool store, uint32_t s_addr,
                                          const float* dv_in) {
  float dv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) dv[i] = dv_in[i];
  for (int c = lo; c < hi; c += 8) {
    if (c > lo) {
      ptx::tmem_ld8(s_addr + c, dv);
      ptx::tmem_wait_ld();
    }
    if (store) {
      const int64_t dst = base + int64_t(c - base_col) * col_stride + tok;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (c + i < hi) dump_store(p, dst + int64_t(i) * col_stride, dv[i]);
    }
  }
}

// The item's N packed columns are split between the two softmax warpgroups:
// warpgroup wg owns columns [c0, c0 + NH) with c0 = wg * NH, NH = N / 2.  A
// column's running statistics (reference max, sum, rescale factor) live with
// its owner, so the two groups never wait for each other; they meet only on
// the S / P / O barriers shared with the MMA warp.
template <int NH, bool kDump>
__device__ bool consume_item(const AttnParams& p, TcShared& sm, const WorkItem& it, bool causal, int r,
                             int ctid, int wg, int wq, int lane, uint32_t& g, uint32_t& grp_uses) {
  constexpr int N = 2 * NH;
  const int c0 = wg * NH;
  const int nrows = it.pq_end - it.pq_begin;
  const int nt = n_tiles_of(it);
  const uint32_t tmem_lane = sm.tmem_base + (uint32_t(wq * 32) << 16);
  const float scale = p.scale_log2;
  const int group = p.group;
  uint64_t& grp = sm.grp[wg];
  int(*flags)[4] = sm.flags[wg];
  int* grew = sm.grew[wg];

  const int q_idx0 = it.pq_begin / group;
  // Logit dump: the item's columns of query 0 (first slot) and of query
  // q_len-1 (last slot) are two runs of at most `group` consecutive S
  // columns; each tile reads this group's part of those runs.  Which runs
  // exist depends on the dump kind and the row's flag (dump_index).
  int d0_lo = 0, d0_hi = 0, d1_lo = 0, d1_hi = 0, dump_c1 = 0;
  int64_t dump_base0 = 0, dump_base1 = 0;
  const int64_t dump_col_stride = dump_head_stride(p);  // between heads
  if (kDump && dump_row_on(p, it.row)) {
    const int last_lo = (it.q_len - 1) * group;  // first packed row of the last query
    const int64_t head0 = int64_t(it.kv_head) * group;
    if (dump_has_first(p) && it.pq_begin < group) {
      const int n0 = min(group - it.pq_begin, nrows);
      d0_lo = c0;
      d0_hi = min(n0, c0 + NH);
      dump_base0 = dump_index(p, it.row, head0 + it.pq_begin, false);
    }
    if (dump_has_last(p, it.q_len) && last_lo < it.pq_end) {
      dump_c1 = max(last_lo - it.pq_begin, 0);
      d1_lo = max(dump_c1, c0);
      d1_hi = min(nrows, c0 + NH);
      dump_base1 = dump_index(p, it.row, head0 + it.pq_begin + dump_c1 - last_lo, true);
    }
  }
  const bool dumping = kDump && (d0_lo < d0_hi || d1_lo < d1_hi);
  // The column reference max (times scale) is uniform across the group's
  // threads and lives in shared memory (mref[cur]); the first tile of an item
  // always sets it.
  float l[NH];
#pragma unroll
  for (int j = 0; j < NH; ++j) l[j] = 0.f;
  int cur = 0;
  const uint32_t g0 = g;

  for (int t = 0; t < nt; ++t) {
    const uint32_t gt = g0 + t;
    const int b = gt % 2;
    const uint32_t ph = (gt / 2) & 1;
    if (!wait_bar(sm, sm.s_full[b], ph, p.status)) return false;
    ptx::tc_fence_after();
    const int tile0 = it.tok_begin + t * kTile;
    const int tok = tile0 + r;
    const bool in_chunk = tok < it.tok_end;
    const int limit_min = causal ? (it.kv_len - it.q_len + q_idx0 + 1) : it.kv_len;
    // Padded columns (j >= nrows) only feed ignored O columns: they need no mask.
    const bool full_tile = tile0 + kTile <= it.tok_end && tile0 + kTile <= limit_min;
    const uint32_t s_cols = tmem_lane + col_s(b) + c0;
    auto load_s = [&](float* sv) {
      tmem_load_cols<NH>(s_cols, sv);
      ptx::tmem_wait_ld();
    };
    // Token `tok` is visible to packed column j iff it lies in the chunk and,
    // under the bottom-right causal mask, q_idx(j) >= tok - (kv_len - q_len),
    // i.e. j >= jmin: one threshold per thread instead of a division per column.
    int jmin = 0;
    if (!full_tile) {
      if (!in_chunk || tok >= it.kv_len) {
        jmin = N;
      } else if (causal) {
        const int d0 = tok - (it.kv_len - it.q_len);
        jmin = d0 <= 0 ? 0 : min(d0 * group - it.pq_begin, N);
      }
    }
    auto mask_s = [&](float* sv) {
      if (!full_tile) {
#pragma unroll
        for (int j = 0; j < NH; ++j)
          if (c0 + j < jmin) sv[j] = -INFINITY;
      }
    };
    float sv[NH];
    if (dumping) {
      // Raw logits before scale and mask of the dump columns: each slot's
      // columns are a run [lo, hi) of this group's columns; the first 8 of
      // each run load with the tile (one wait), longer runs in more pieces.
      float dv0[8], dv1[8];
      tmem_load_cols<NH>(s_cols, sv);
      if (d0_lo < d0_hi) ptx::tmem_ld8(tmem_lane + col_s(b) + d0_lo, dv0);
      if (d1_lo < d1_hi) ptx::tmem_ld8(tmem_lane + col_s(b) + d1_lo, dv1);
      ptx::tmem_wait_ld();
      const bool store = in_chunk && tok < p.dump_kv_stride;
      if (d0_lo < d0_hi)
        dump_columns(p, d0_lo, d0_hi, dump_base0, 0, dump_col_stride, tok, store, tmem_lane + col_s(b), dv0);
      if (d1_lo < d1_hi)
        dump_columns(p, d1_lo, d1_hi, dump_base1, dump_c1, dump_col_stride, tok, store, tmem_lane + col_s(b), dv1);
    } else {
      load_s(sv);
    }
    mask_s(sv);

    // Lazy running max: does any logit of the tile exceed its column's reference by > 2^8?
    const float* mr = sm.mref[cur] + c0;
    bool exceed = (t == 0);
    if (t > 0) {
#pragma unroll
      for (int j = 0; j < NH; ++j) exceed |= fmaf(sv[j], scale, -mr[j]) > kLazyLog2;
    }
    const bool warp_exceed = __any_sync(0xffffffffu, exceed);
    if (lane == 0) flags[t & 1][wq] = warp_exceed ? 1 : 0;
    if (!group_sync(sm, grp, grp_uses, p.status)) return false;
    const bool any_exceed = (flags[t & 1][0] | flags[t & 1][1] | flags[t & 1][2] | flags[t & 1][3]) != 0;
    if (any_exceed) {
      // Exact column maxima of the tile (reduced in place; S is read again from
      // TMEM afterwards).  Thread j < NH then updates column c0 + j's reference
      // (mref[cur ^ 1]) and its rescale factor alpha; the per-column work is
      // spread over threads so that this once-per-item path stays short.
      warp_columns<NH, true>(sv, sm.red[t & 1][wq] + c0, lane);
      if (ctid == 0) grew[t & 1] = 0;
      if (!group_sync(sm, grp, grp_uses, p.status)) return false;
      if (ctid < NH) {
        const int c = c0 + ctid;
        const float mo = t > 0 ? sm.mref[cur][c] : -INFINITY;
        const float tmax = fmaxf(fmaxf(sm.red[t & 1][0][c], sm.red[t & 1][1][c]),
                                 fmaxf(sm.red[t & 1][2][c], sm.red[t & 1][3][c]));
        const float mn = fmaxf(mo, tmax * scale);
        sm.mref[cur ^ 1][c] = mn;
        sm.alpha[t & 1][c] = (mo == -INFINITY) ? 0.f : (mn == mo ? 1.f : ex2(mo - mn));
        if (mn != mo && mo != -INFINITY) grew[t & 1] = 1;
      }
      load_s(sv);
      mask_s(sv);
      ptx::tc_fence_before();
      ptx::mbar_arrive(ptx::smem_addr(&sm.s_empty[b]));
      // New references and alphas visible to every thread (uniform branch).
      if (!group_sync(sm, grp, grp_uses, p.status)) return false;
      cur ^= 1;
      if (t > 0 && grew[t & 1]) {
        const float* alpha_s = sm.alpha[t & 1] + c0;
#pragma unroll
        for (int j = 0; j < NH; ++j) l[j] *= alpha_s[j];
        // Rescale this group's O columns once the previous tile's PV has
        // landed.  PV completion is observed on its P buffer's empty barrier,
        // whose phases this thread waits on in order (so the parity test is
        // unambiguous).
        const uint32_t prev = gt - 1;
        if (!wait_bar(sm, sm.p_empty[prev % 2], (prev / 2) & 1, p.status)) return false;
        ptx::tc_fence_after();
        float ov[NH];
        tmem_load_cols<NH>(tmem_lane + kColO + c0, ov);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < NH; ++j) ov[j] *= alpha_s[j];
        if constexpr (NH >= 16) ptx::tmem_st16(tmem_lane + kColO + c0, ov);
        if constexpr (NH == 8) ptx::tmem_st8(tmem_lane + kColO + c0, ov);
        if constexpr (NH == 24) ptx::tmem_st8(tmem_lane + kColO + c0 + 16, ov + 16);
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
      }
    } else {
      ptx::tc_fence_before();
      ptx::mbar_arrive(ptx::smem_addr(&sm.s_empty[b]));
    }
    {
      const float* m = sm.mref[cur] + c0;
#pragma unroll
      for (int j = 0; j < NH; ++j) {
        const float pv = (m[j] == -INFINITY) ? 0.f : ex2(fmaf(sv[j], scale, -m[j]));
        l[j] += pv;
        sv[j] = pv;
      }
    }
    // P^T as bf16, MN-major without swizzle: 8 queries x 16 B per token, token-major.
    if (!wait_bar(sm, sm.p_empty[b], ph ^ 1, p.status)) return false;
    uint8_t* pbuf = sm.p[b] + (c0 / 8) * (kTile * 16);
#pragma unroll
    for (int c = 0; c < NH / 8; ++c) {
      uint4 val;
      __nv_bfloat162 h0 = __floats2bfloat162_rn(sv[8 * c + 0], sv[8 * c + 1]);
      __nv_bfloat162 h1 = __floats2bfloat162_rn(sv[8 * c + 2], sv[8 * c + 3]);
      __nv_bfloat162 h2 = __floats2bfloat162_rn(sv[8 * c + 4], sv[8 * c + 5]);
      __nv_bfloat162 h3 = __floats2bfloat162_rn(sv[8 * c + 6], sv[8 * c + 7]);
      val.x = *reinterpret_cast<uint32_t*>(&h0);
      val.y = *reinterpret_cast<uint32_t*>(&h1);
      val.z = *reinterpret_cast<uint32_t*>(&h2);
      val.w = *reinterpret_cast<uint32_t*>(&h3);
      *reinterpret_cast<uint4*>(pbuf + c * (kTile * 16) + r * 16) = val;
    }
    ptx::fence_proxy_async_smem();
    ptx::mbar_arrive(ptx::smem_addr(&sm.p_full[b]));
  }
  g = g0 + nt;

  // Final O: wait for the item's last PV (on its P buffer's empty barrier),
  // read this lane (dim r) of the group's columns, free the accumulator.
  if (!wait_bar(sm, sm.p_empty[(g - 1) % 2], ((g - 1) / 2) & 1, p.status)) return false;
  ptx::tc_fence_after();
  float o_fin[NH];
  tmem_load_cols<NH>(tmem_lane + kColO + c0, o_fin);
  ptx::tmem_wait_ld();
  ptx::tc_fence_before();
  ptx::mbar_arrive(ptx::smem_addr(&sm.o_free));

  // Column sums of l across the group's 128 threads; thread j < NH then turns
  // column c0 + j into its reciprocal and LSE once.
  warp_columns<NH, false>(l, sm.red_l[wq] + c0, lane);
  if (!group_sync(sm, grp, grp_uses, p.status)) return false;
  float my_lse = -INFINITY;  // LSE of column c0 + ctid
  if (ctid < NH) {
    const int c = c0 + ctid;
    const float L = sm.red_l[0][c] + sm.red_l[1][c] + sm.red_l[2][c] + sm.red_l[3][c];
    sm.inv_l[c] = L > 0.f ? 1.f / L : 0.f;
    my_lse = L > 0.f ? sm.mref[cur][c] + lg2(L) : -INFINITY;
  }
  // The previous item's bulk stores (issued by this group's thread 0) have
  // read the group's staging rows before anyone rewrites them.
  if (ctid == 0) ptx::bulk_wait_read();
  if (!group_sync(sm, grp, grp_uses, p.status)) return false;

  // Normalised rows are staged in shared memory and leave by bulk stores, so
  // the threads move on to the next item at once.
  const int d = r;  // this thread's output dim
  uint8_t* stage = sm.out_stage;
  const bool final_rows = it.n_chunks <= 1;
  const int row_end = min(c0 + NH, nrows);  // this group's rows are [c0, row_end)
  if (final_rows) {
    __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(stage);
#pragma unroll
    for (int j = 0; j < NH; ++j)
      if (c0 + j < nrows) st[(c0 + j) * kHeadDim + d] = __float2bfloat16_rn(o_fin[j] * sm.inv_l[c0 + j]);
    if (ctid < NH && c0 + ctid < nrows && p.lse) {
      int q_idx, head;
      packed_row(p, it, it.pq_begin + c0 + ctid, q_idx, head);
      if (int64_t(it.q_start) + q_idx < p.q_rows) p.lse[(int64_t(it.q_start) + q_idx) * p.num_qo_heads + head] = my_lse;
    }
  } else {
    float* st = reinterpret_cast<float*>(stage);
#pragma unroll
    for (int j = 0; j < NH; ++j)
      if (c0 + j < nrows) st[(c0 + j) * kHeadDim + d] = o_fin[j] * sm.inv_l[c0 + j];
    if (ctid < NH && c0 + ctid < nrows)
      partial_lse_ptr(p)[int64_t(it.partial_base) + int64_t(it.chunk) * nrows + c0 + ctid] = my_lse;
  }
  ptx::fence_proxy_async_smem();
  if (!group_sync(sm, grp, grp_uses, p.status)) return false;
  if (ctid == 0 && c0 < row_end) {
    if (final_rows) {
      const uint32_t src = ptx::smem_addr(stage);
      for (int j = c0; j < row_end; ++j) {
        int q_idx, head;
        packed_row(p, it, it.pq_begin + j, q_idx, head);
        if (int64_t(it.q_start) + q_idx >= p.q_rows) {
          record_status(p.status, ASPIRE_STATUS_BAD_ROW);
          continue;
        }
        __nv_bfloat16* dst = p.out + (int64_t(it.q_start) + q_idx) * p.o_stride_n + int64_t(head) * p.o_stride_h;
        ptx::bulk_store(dst, src + uint32_t(j) * kHeadDim * 2, kHeadDim * 2);
      }
    } else {
      const uint32_t src = ptx::smem_addr(stage) + uint32_t(c0) * kHeadDim * 4;
      const int64_t base = int64_t(it.partial_base) + int64_t(it.chunk) * nrows + c0;
      ptx::bulk_store(p.partial_o + base * kHeadDim, src, uint32_t(row_end - c0) * kHeadDim * 4);
    }
    ptx::bulk_commit();
  }
  return true;
}

__device__ void consume_items(const AttnParams& p, TcShared& sm, bool causal, int warp, int lane, uint32_t& k,
                              bool use_cols) {
  const int wq = warp & 3;
  const int wg = (warp - kFirstSoftmaxWarp) / 4;  // softmax warpgroup 0 or 1
  const int r = wq * 32 + lane;                    // TMEM lane = S-tile token = O-tile dim
  const int ctid = (warp - kFirstSoftmaxWarp - 4 * wg) * 32 + lane;  // 0..127 within the group
  uint32_t g = 0, grp_uses = 0;
  for (;;) {
    if (aborted(sm)) return;
    const int ii = seq_read(sm, k, lane, p.status);
    if (ii < 0) return;
    const WorkItem it = load_item(p.plan, ii);
    const int nrows = it.pq_end - it.pq_begin;
    if (!item_valid(p, it, kNMax)) {
      if (ctid == 0 && wg == 0) record_status(p.status, ASPIRE_STATUS_BAD_PLAN);
      continue;
    }
    if (n_tiles_of(it) == 0) {
      // No keys: zero output, -inf LSE (chunked items always have keys).
      for (int j = wg; j < nrows; j += 2) store_final(p, it, it.pq_begin + j, r, 0.f, -INFINITY);
      continue;
    }
    const int N = item_columns(it, use_cols);
    // Items whose columns include dumped rows (query 0 or the last query, as
    // the dump kind and the row's flag have it) take the instantiation that
    // carries the dump path.
    const bool dump_item = dump_row_on(p, it.row) &&
                           ((dump_has_first(p) && it.pq_begin < p.group) ||
                            (dump_has_last(p, it.q_len) && (it.q_len - 1) * p.group < it.pq_end));
    bool ok;
    if (dump_item) {
      if (N == 16)
        ok = consume_item<8, true>(p, sm, it, causal, r, ctid, wg, wq, lane, g, grp_uses);
      else if (N == 32)
        ok = consume_item<16, true>(p, sm, it, causal, r, ctid, wg, wq, lane, g, grp_uses);
      else
        ok = consume_item<24, true>(p, sm, it, causal, r, ctid, wg, wq, lane, g, grp_uses);
    } else {
      if (N == 16)
        ok = consume_item<8, false>(p, sm, it, causal, r, ctid, wg, wq, lane, g, grp_uses);
      else if (N == 32)
        ok = consume_item<16, false>(p, sm, it, causal, r, ctid, wg, wq, lane, g, grp_uses);
      else
        ok = consume_item<24, false>(p, sm, it, causal, r, ctid, wg, wq, lane, g, grp_uses);
    }
    if (!ok) return;
  }
}

__device__ void run_consumer(const AttnParams& p, TcShared& sm, bool causal, int warp, int lane, uint32_t& k,
                             bool use_cols) {
  consume_items(p, sm, causal, warp, lane, k, use_cols);
  // The bulk stores of each group's last item (issued by its thread 0) finish
  // before the CTA exits.
  if (lane == 0 && (warp - kFirstSoftmaxWarp) % 4 == 0) ptx::bulk_wait_all();
}

}  // namespace

__global__ void __launch_bounds__(kTcThreads, 1)
    aspire_attn_tc_kernel(AttnParams p, const __grid_constant__ CUtensorMap tmap,
                          const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap qmap_pf) {
  pdl_launch_dependents();
  extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
  const uint32_t raw = ptx::smem_addr(tc_smem_raw);
  TcShared& sm = *reinterpret_cast<TcShared*>(tc_smem_raw + ((1024 - (raw & 1023)) & 1023));
  pf::Buffers& pbuf = *reinterpret_cast<pf::Buffers*>(&sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Prologue: shared memory, TMEM and the tensor maps only (no global memory
  // written by earlier kernels), so it overlaps the preceding kernel's tail.

  if (threadIdx.x == 0) {
    for (int s = 0; s < kKStages; ++s) {
      ptx::mbar_init(ptx::smem_addr(&sm.k_full[s]), 1);
      ptx::mbar_init(ptx::smem_addr(&sm.k_empty[s]), 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      ptx::mbar_init(ptx::smem_addr(&sm.v_full[s]), 1);
      ptx::mbar_init(ptx::smem_addr(&sm.v_empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(ptx::smem_addr(&sm.s_full[b]), 1);
      ptx::mbar_init(ptx::smem_addr(&sm.s_empty[b]), 256);
      ptx::mbar_init(ptx::smem_addr(&sm.p_full[b]), 256);
      ptx::mbar_init(ptx::smem_addr(&sm.p_empty[b]), 1);
    }
    ptx::mbar_init(ptx::smem_addr(&sm.o_free), 256);
    ptx::mbar_init(ptx::smem_addr(&sm.q_full), 1);
    ptx::mbar_init(ptx::smem_addr(&sm.q_empty), 1);
    ptx::mbar_init(ptx::smem_addr(&sm.done), 1);
    ptx::mbar_init(ptx::smem_addr(&sm.done_pv), 1);
    ptx::mbar_init(ptx::smem_addr(&sm.grp[0]), 128);
    ptx::mbar_init(ptx::smem_addr(&sm.grp[1]), 128);
    pf::init_barriers(sm.pf);
    for (int s = 0; s < kSeqDepth; ++s) {
      ptx::mbar_init(ptx::smem_addr(&sm.seq_full[s]), 1);
      ptx::mbar_init(ptx::smem_addr(&sm.seq_empty[s]), kSeqReaders);
    }
    sm.abort_flag = 0;
    sm.wait_ns = p.wait_ns;
    ptx::mbar_fence_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_addr(&sm.tmem_base), kTmemCols);
    ptx::tmem_relinquish();
  }
  if (warp == 0 && lane == 0) ptx::prefetch_tmap(&tmap);
  if (warp == 1 && lane == 0) {
    ptx::prefetch_tmap(&qmap);
    ptx::prefetch_tmap(&qmap_pf);
  }
  // Query rows that no load writes (when kNMax is not a multiple of the group)
  // stay zero.
  for (int i = threadIdx.x; i < int(sizeof(sm.q) / 16); i += blockDim.x)
    reinterpret_cast<uint4*>(&sm.q[0][0])[i] = make_uint4(0, 0, 0, 0);
  ptx::fence_proxy_async_smem();
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();

  // The plan and every input are outputs of earlier kernels (or copies).
  pdl_wait();
  const int32_t* plan = p.plan;
  const bool live = plan[kHdrMagic] == kPlanMagic && int(blockIdx.x) < plan[kHdrNumTcCtas];
  const int tc_first = live ? plan[kHdrTcFirst] : 0;
  const int pf_first = live ? plan[kHdrPfFirst] : 0;
  const int n_tc = live ? pf_first - tc_first : 0;
  const int n_pf = live ? plan[kHdrNumItems] - pf_first : 0;
  const bool causal = live && plan[kHdrCausal] != 0;
  const bool use_cols = p.dump == nullptr;

  // Both phases read one item sequence (the ring of claimed item indices);
  // each warp keeps its position across the phase change.
  uint32_t k = 0;
  // Phase 1: the decode list.
  if (n_tc > 0) {
    if (warp == 0) {
      run_producer<kKStages>(p, &tmap, sm, sm.k, sm.k_full, sm.k_empty, 0, true, tc_first, n_tc, kHdrTcClaim, kNMax,
                             lane, k);
    } else if (warp == kVProducerWarp) {
      run_producer<kVStages>(p, &tmap, sm, sm.v, sm.v_full, sm.v_empty, 1, false, tc_first, n_tc, kHdrTcClaim,
                             kNMax, lane, k);
    } else if (warp == 1) {
      run_qk(p, &qmap, sm, lane, k, use_cols);
    } else if (warp == kPvWarp) {
      run_pv(p, sm, lane, k, use_cols);
    } else {
      run_consumer(p, sm, causal, warp, lane, k, use_cols);
    }
  }
  // Phase 2: the prefill list, in the same shared memory and TMEM.  Every
  // copy, MMA and bulk store of phase 1 has completed (each role drained its
  // own) before any role passes this barrier.
  if (n_pf > 0) {
    ptx::fence_proxy_async_smem();
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    if (!aborted(sm)) {
      if (warp == 0) {
        run_producer<pf::kKStages>(p, &tmap, sm, pbuf.k, sm.pf.k_full, sm.pf.k_empty, 0, true, pf_first, n_pf,
                                   kHdrPfClaim, kPfMaxRows, lane, k);
      } else if (warp == kVProducerWarp) {
        run_producer<pf::kVStages>(p, &tmap, sm, pbuf.v, sm.pf.v_full, sm.pf.v_empty, 1, false, pf_first, n_pf,
                                   kHdrPfClaim, kPfMaxRows, lane, k);
      } else if (warp == 1 || warp == kPvWarp) {
        // One MMA-issuing warp per item half.
        pf::run_mma(p, &qmap_pf, sm, pbuf, warp == 1 ? 0 : 1, lane, k);
      } else {
        pf::consume_items(p, sm, causal, (warp - kFirstSoftmaxWarp) / 4, warp & 3, lane, k);
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(sm.tmem_base, kTmemCols);
}

size_t tc_smem_bytes() { return sizeof(TcShared) + 1024; }

int tc_threads() { return kTcThreads; }

bool tc_kernel_available() { return true; }

}  // namespace aspire
