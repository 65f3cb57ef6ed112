// Split-KV merge: combines the chunk partials of every split (row, KV head,
// packed-query tile) into the final output row and LSE.
//
// Each chunk wrote its normalised partial O row and its base-2 LSE; the merged
// row is  O = sum_c w_c O_c / sum_c w_c  with  w_c = exp2(lse_c - max_c lse_c),
// LSE = max + log2(sum_c w_c)  (the state merge of FlashInfer's
// BlockBatchReductionPersistent, flashinfer include/flashinfer/attention/
// persistent.cuh:526-637, which ASPIRE's persistent kernel ends with).
// One warp per (merge group, packed row): lanes split the chunks for the LSE
// reduction and the 128 dims (4 each, 16-byte loads) for the weighted sum;
// chunks are always combined in chunk order, so the result is deterministic.
// The pass waits on few memory round trips (the unit, its descriptor, then the
// LSEs and the first chunks' rows together), since a warp merges about one
// row and the kernel sits between two attention launches.
// The grid is fixed and the work list comes from the device plan, so a
// captured graph stays valid across re-plans.  It also rearms the tcgen05
// kernel's item counters.
#include "kernels.cuh"

namespace aspire {

__global__ void __launch_bounds__(kMergeThreads) aspire_attn_merge_kernel(AttnParams p) {
  pdl_begin();
  const int32_t* plan = p.plan;
  if (plan[kHdrMagic] != kPlanMagic) return;
  // The tcgen05 kernel of this call has finished: rearm its item counters for
  // the next launch of the same plan (graph replays upload no new plan).
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const_cast<int32_t*>(plan)[kHdrTcClaim] = 0;
    const_cast<int32_t*>(plan)[kHdrPfClaim] = 0;
  }
  const int num_units = plan[kHdrNumMergeUnits];
  if (num_units == 0) return;
  const MergeDesc* descs = reinterpret_cast<const MergeDesc*>(plan + plan[kHdrOffMerge]);
  const int32_t* units = plan + plan[kHdrOffMergeUnits];
  const float* plse = partial_lse_ptr(p);
  const int lane = threadIdx.x & 31;
  const int warps_per_block = blockDim.x >> 5;
  const int warp_global = blockIdx.x * warps_per_block + (threadIdx.x >> 5);
  const int total_warps = gridDim.x * warps_per_block;

  for (int u = warp_global; u < num_units; u += total_warps) {
    const int32_t code = units[u];
    const MergeDesc md = descs[code >> 8];
    const int j = code & 0xff;
    const int n = md.n_chunks;
    const int64_t row0 = int64_t(md.partial_base) + j;  // partial row of chunk c: row0 + c * nrows

    const float4* orow = reinterpret_cast<const float4*>(p.partial_o + row0 * kHeadDim) + lane;
    const int64_t ostep = int64_t(md.nrows) * (kHeadDim / 4);  // float4s between chunks of the row
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float wsum = 0.f;
    float m = -INFINITY;
    if (n <= 32) {
      // One memory round trip for the LSEs (one per lane) and the first eight
      // chunks' rows together, since the rows' loads do not need the weights.
      const float lse_lane = lane < n ? __ldcg(plse + row0 + int64_t(lane) * md.nrows) : -INFINITY;
      float4 ov[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) ov[i] = i < n ? __ldcg(orow + i * ostep) : make_float4(0.f, 0.f, 0.f, 0.f);
      m = lse_lane;
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      if (m != -INFINITY) {
        const float w_lane = lane < n ? ex2(lse_lane - m) : 0.f;
        for (int c0 = 0; c0 < n; c0 += 8) {
          if (c0 > 0) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              ov[i] = c0 + i < n ? __ldcg(orow + (c0 + i) * ostep) : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float w = __shfl_sync(0xffffffffu, w_lane, (c0 + i) & 31);
            if (c0 + i < n) {  // chunk order, as in the general path below
              wsum += w;
              acc.x = fmaf(w, ov[i].x, acc.x);
              acc.y = fmaf(w, ov[i].y, acc.y);
              acc.z = fmaf(w, ov[i].z, acc.z);
              acc.w = fmaf(w, ov[i].w, acc.w);
            }
          }
        }
      }
    } else {
      for (int c = lane; c < n; c += 32) m = fmaxf(m, __ldcg(plse + row0 + int64_t(c) * md.nrows));
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    }
    if (n > 32 && m != -INFINITY) {
      for (int c0 = 0; c0 < n; c0 += 32) {
        const int cl = c0 + lane;
        const float w_lane = cl < n ? ex2(__ldcg(plse + row0 + int64_t(cl) * md.nrows) - m) : 0.f;
        const int cn = min(32, n - c0);
#pragma unroll 4
        for (int i = 0; i < cn; ++i) {
          const float w = __shfl_sync(0xffffffffu, w_lane, i);
          const float4 o = __ldcg(reinterpret_cast<const float4*>(
                                      p.partial_o + (row0 + int64_t(c0 + i) * md.nrows) * kHeadDim) +
                                  lane);
          wsum += w;
          acc.x = fmaf(w, o.x, acc.x);
          acc.y = fmaf(w, o.y, acc.y);
          acc.z = fmaf(w, o.z, acc.z);
          acc.w = fmaf(w, o.w, acc.w);
        }
      }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    const int pq = md.pq_begin + j;
    const int q_idx = pq / p.group;
    const int head = md.kv_head * p.group + (pq - q_idx * p.group);
    const int64_t tok = int64_t(md.q_start) + q_idx;
    if (tok >= p.q_rows) {
      if (lane == 0) record_status(p.status, ASPIRE_STATUS_BAD_ROW);
      continue;
    }
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x * inv, acc.y * inv);
    __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z * inv, acc.w * inv);
    uint2 packed;
    packed.x = *reinterpret_cast<uint32_t*>(&lo);
    packed.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(p.out + tok * p.o_stride_n + int64_t(head) * p.o_stride_h + lane * 4) = packed;
    if (lane == 0 && p.lse) p.lse[tok * p.num_qo_heads + head] = wsum > 0.f ? m + lg2(wsum) : -INFINITY;
  }
}

}  // namespace aspire
