// CUDA-core paged-attention kernel for narrow packed-query tiles (draft /
// decode rows, <= 4 packed (query, head) rows per KV head).
//
// Treated as a memory-bound gather over the page table: each CTA streams the
// 16-token pages of one (row, KV head, chunk) through a cp.async ring of
// 8 KiB stages (K page + V page, 128-bit copies), and the GQA head group
// shares every staged K/V row.  Half-warps own tokens (16 lanes x 8 dims),
// reduce q.k with warp shuffles and keep an online softmax per half-warp;
// the eight half-warp states are merged through shared memory at the end of
// the chunk; split-KV chunks write partials combined by the merge kernel.
//
// Semantics follow FlashInfer's persistent paged attention as ASPIRE drives
// it (flashinfer include/flashinfer/attention/persistent.cuh:178-497,
// prefill.cuh logits_mask):  bottom-right causal mask (query i of a row of
// q_len sees KV positions < kv_len - q_len + i + 1), base-2 LSE of the
// scaled logits, GQA kv_head = q_head / group.  With a dump buffer the raw
// fp32 q.k (before scaling and masking) of the dumped queries is stored
// rounded to fp16 (dump_index / dump_store: first/last or last-token, as the
// reference's variants do, aspire/backends/jit_kernels.py:180-193).
#include "kernels.cuh"

namespace aspire {

namespace {

constexpr int kThreads = 128;
constexpr int kStages = 6;
constexpr int kQT = kGatherQTile;  // packed query rows per item

struct GatherSmem {
  union {
    __nv_bfloat16 ring[kStages][2][kPageSize][kHeadDim];   // 48 KiB
    struct {
      float m[8][kQT];
      float l[8][kQT];
      float o[8][kQT][kHeadDim];                            // 16 KiB
      float fo[kQT][kHeadDim];                              // merged rows
      float flse[kQT];
    } red;
  };
  int flag;
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

}  // namespace

__global__ void __launch_bounds__(kThreads, kGatherCtasPerSm) aspire_attn_gather_kernel(AttnParams p) {
  pdl_begin();
  extern __shared__ __align__(128) unsigned char smem_raw[];
  GatherSmem& sm = *reinterpret_cast<GatherSmem*>(smem_raw);
  const int32_t* plan = p.plan;
  if (plan[kHdrMagic] != kPlanMagic) return;
  if (int(blockIdx.x) >= plan[kHdrNumGatherCtas]) return;
  const int32_t* indptr = plan + plan[kHdrOffGatherIndptr];
  const int item_begin = indptr[blockIdx.x], item_end = indptr[blockIdx.x + 1];
  const bool causal = plan[kHdrCausal] != 0;

  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int l16 = lane & 15;
  const int grp = warp * 2 + (lane >> 4);  // half-warp id 0..7
  const int64_t tok_stride = int64_t(p.num_kv_heads) * kHeadDim;  // elements between tokens of a page
  const int64_t page_stride = 2 * kPageSize * tok_stride;

  for (int ii = item_begin; ii < item_end; ++ii) {
    const WorkItem it = load_item(plan, ii);
    const int nq = it.pq_end - it.pq_begin;
    if (nq <= 0 || nq > kQT || it.kv_head >= p.num_kv_heads) {
      if (tid == 0) record_status(p.status, ASPIRE_STATUS_BAD_PLAN);
      continue;
    }

    // Query rows of this item (raw bf16 -> fp32, 8 dims per lane).
    float qv[kQT][8];
    int lim[kQT];
    int64_t dump_at[kQT];  // dump element index of token 0 of row j, -1 when not dumped
    const bool row_dumps = dump_row_on(p, it.row);
#pragma unroll
    for (int j = 0; j < kQT; ++j) {
      int q_idx = 0, head = 0;
      if (j < nq) packed_row(p, it, it.pq_begin + j, q_idx, head);
      lim[j] = causal ? (it.kv_len - it.q_len + q_idx + 1) : it.kv_len;
      const bool first = (j < nq) && row_dumps && dump_has_first(p) && q_idx == 0;
      const bool last = (j < nq) && row_dumps && !first && dump_has_last(p, it.q_len) && q_idx + 1 == it.q_len;
      dump_at[j] = (first || last) ? dump_index(p, it.row, head, last) : -1;
      if (j < nq && int64_t(it.q_start) + q_idx < p.q_rows) {
        const uint4 u = *reinterpret_cast<const uint4*>(
            p.q + int64_t(it.q_start + q_idx) * p.q_stride_n + int64_t(head) * p.q_stride_h +
            l16 * 8);
        bf16x8_to_f32(u, qv[j]);
      } else {
#pragma unroll
        for (int d = 0; d < 8; ++d) qv[j][d] = 0.f;
      }
    }

    float m[kQT], l[kQT], o[kQT][8];
#pragma unroll
    for (int j = 0; j < kQT; ++j) {
      m[j] = -INFINITY;
      l[j] = 0.f;
#pragma unroll
      for (int d = 0; d < 8; ++d) o[j][d] = 0.f;
    }

    const int pg0 = it.tok_begin / kPageSize;
    const int npg = it.tok_end > it.tok_begin ? (it.tok_end + kPageSize - 1) / kPageSize - pg0 : 0;
    const __nv_bfloat16* kv_head_base = p.kv + int64_t(it.kv_head) * kHeadDim;

    // Page ids are read one issue ahead so their latency is off the copy path.
    auto page_of = [&](int pi) -> int32_t {
      return pi < npg ? row_page(p.kv_indices, it.kv_page_base, p.mode_flags, p.draft_table, p.draft_stride,
                                 p.block_table, p.block_table_stride, it.row, pg0 + pi)
                      : 0;
    };
    auto issue = [&](int pi, int32_t page) {
      const int stage = pi % kStages;
      int bytes = 16;
      if (page < 0 || int64_t(page) >= p.num_pages_total) {
        if (tid == 0) record_status(p.status, ASPIRE_STATUS_BAD_PAGE);
        page = 0;
        bytes = 0;  // zero-fill, read nothing
      }
      const __nv_bfloat16* kbase = kv_head_base + int64_t(page) * page_stride;
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2) {
        const int c = tid + c2 * kThreads;  // 0..255
        const int r = c >> 4, col = (c & 15) * 8;
        cp_async16(&sm.ring[stage][0][r][col], kbase + r * tok_stride + col, bytes);
        cp_async16(&sm.ring[stage][1][r][col], kbase + kPageSize * tok_stride + r * tok_stride + col,
                   bytes);
      }
    };

    int32_t ids[kStages - 1];
#pragma unroll
    for (int s = 0; s < kStages - 1; ++s) ids[s] = page_of(s);
#pragma unroll
    for (int s = 0; s < kStages - 1; ++s) {
      if (s < npg) issue(s, ids[s]);
      cp_async_commit();
    }
    int32_t next_id = page_of(kStages - 1);

    for (int pi = 0; pi < npg; ++pi) {
      cp_async_wait<kStages - 2>();
      __syncthreads();
      const int32_t id = next_id;
      next_id = page_of(pi + kStages);
      if (pi + kStages - 1 < npg) issue(pi + kStages - 1, id);
      cp_async_commit();

      const int stage = pi % kStages;
      const int tbase = (pg0 + pi) * kPageSize;
      float x[2][kQT];
      float vf[2][8];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int tl = grp + 8 * u;
        const int tok = tbase + tl;
        float kf[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(&sm.ring[stage][0][tl][l16 * 8]), kf);
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(&sm.ring[stage][1][tl][l16 * 8]), vf[u]);
        float s[kQT];
#pragma unroll
        for (int j = 0; j < kQT; ++j) {
          float acc = 0.f;
#pragma unroll
          for (int d = 0; d < 8; ++d) acc = fmaf(qv[j][d], kf[d], acc);
          s[j] = acc;
        }
#pragma unroll
        for (int off = 8; off >= 1; off >>= 1) {
#pragma unroll
          for (int j = 0; j < kQT; ++j) s[j] += __shfl_xor_sync(0xffffffffu, s[j], off);
        }
        const bool in_chunk = tok >= it.tok_begin && tok < it.tok_end;
        // A page's slots past the row's last token may hold anything (NaN
        // included); their weight is zero and so must be their values.
        if (!in_chunk) {
#pragma unroll
          for (int d = 0; d < 8; ++d) vf[u][d] = 0.f;
        }
        if (p.dump != nullptr && in_chunk && tok < p.dump_kv_stride) {
#pragma unroll
          for (int j = 0; j < kQT; ++j) {
            if (l16 == j && dump_at[j] >= 0) {
              dump_store(p, dump_at[j] + tok, s[j]);
            }
          }
        }
#pragma unroll
        for (int j = 0; j < kQT; ++j)
          x[u][j] = (in_chunk && tok < lim[j] && j < nq) ? s[j] * p.scale_log2 : -INFINITY;
      }
#pragma unroll
      for (int j = 0; j < kQT; ++j) {
        const float m_new = fmaxf(m[j], fmaxf(x[0][j], x[1][j]));
        if (m_new == -INFINITY) continue;
        const float alpha = ex2(m[j] - m_new);  // m[j] == -inf -> 0
        const float p0 = ex2(x[0][j] - m_new), p1 = ex2(x[1][j] - m_new);
        l[j] = fmaf(l[j], alpha, p0 + p1);
#pragma unroll
        for (int d = 0; d < 8; ++d) o[j][d] = fmaf(o[j][d], alpha, fmaf(p0, vf[0][d], p1 * vf[1][d]));
        m[j] = m_new;
      }
    }
    cp_async_wait<0>();
    __syncthreads();

    // Merge the eight half-warp states.
    if (l16 == 0) {
#pragma unroll
      for (int j = 0; j < kQT; ++j) {
        sm.red.m[grp][j] = m[j];
        sm.red.l[grp][j] = l[j];
      }
    }
#pragma unroll
    for (int j = 0; j < kQT; ++j) {
      float4* dst = reinterpret_cast<float4*>(&sm.red.o[grp][j][l16 * 8]);
      dst[0] = make_float4(o[j][0], o[j][1], o[j][2], o[j][3]);
      dst[1] = make_float4(o[j][4], o[j][5], o[j][6], o[j][7]);
    }
    __syncthreads();
    // Thread tid owns dim d = tid of every row.
    {
      const int d = tid;
#pragma unroll
      for (int j = 0; j < kQT; ++j) {
        if (j >= nq) break;
        float mm = -INFINITY;
#pragma unroll
        for (int g = 0; g < 8; ++g) mm = fmaxf(mm, sm.red.m[g][j]);
        float acc = 0.f, wl = 0.f;
        if (mm != -INFINITY) {
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            const float w = ex2(sm.red.m[g][j] - mm);
            wl = fmaf(w, sm.red.l[g][j], wl);
            acc = fmaf(w, sm.red.o[g][j][d], acc);
          }
        }
        sm.red.fo[j][d] = wl > 0.f ? acc / wl : 0.f;
        if (d == 0) sm.red.flse[j] = wl > 0.f ? mm + lg2(wl) : -INFINITY;
      }
    }
    __syncthreads();
    finish_item(
        p, it, tid, kThreads, [&](int r, int d) { return sm.red.fo[r][d]; },
        [&](int r) { return sm.red.flse[r]; });
    __syncthreads();
  }
}

size_t gather_smem_bytes() { return sizeof(GatherSmem); }

}  // namespace aspire
