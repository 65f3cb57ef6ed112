// Parameter blocks and declarations of every kernel of libaspire_b200.
#pragma once

#include <cuda.h>

#include "attn_common.cuh"

namespace aspire {

// Programmatic dependent launch.  Every kernel of the library is launched
// with a programmatic dependency on the work before it in the stream and
// starts with both calls: the next kernel may then be scheduled while this
// one runs (its launch latency hides under this kernel's tail), and wait
// blocks until the preceding kernel has completed and its writes are visible.
// Without such a dependency both are no-ops.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// Waits until the preceding kernels of the stream have completed and their
// memory is visible; nothing that reads their outputs may run before it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_begin() {
  pdl_launch_dependents();
  pdl_wait();
}


struct AppendParams {
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t k_stride_n, k_stride_h, v_stride_n, v_stride_h;
  int64_t num_tokens;
  const int32_t* append_indptr;
  __nv_bfloat16* kv;
  int64_t num_pages_total;
  const int32_t* page_indices;  // flat page list, or NULL for the page tables below
  const int32_t* mode_flags;
  const int32_t* draft_table;
  int64_t draft_stride;
  const int32_t* block_table;
  int64_t block_table_stride;
  const int32_t* page_indptr;
  const int32_t* last_page_len;
  int32_t num_rows;
  int32_t num_kv_heads;
  uint32_t* status;
};

struct PrologueParams {
  AppendParams ap;              // k (before norm / rotation), v, rows, pages, cache
  const __nv_bfloat16* q;
  int64_t q_stride_n, q_stride_h;
  __nv_bfloat16* q_out;         // may alias q
  int64_t qo_stride_n, qo_stride_h;
  const __nv_bfloat16* q_norm_w;  // [128] bf16; NULL (with k_norm_w) = no norm / permutation
  const __nv_bfloat16* k_norm_w;
  float eps;
  const int32_t* rope_offsets;  // position of each row's first new token
  float rcp_theta, rcp_scale, smooth_a, smooth_b;
  int32_t num_qo_heads;
};
__global__ void aspire_qkv_prologue_kernel(PrologueParams p);

struct DevPlanParams {
  const int32_t* qo_indptr;     // device [batch + 1]
  const int32_t* kv_indptr;     // device [batch + 1] page offsets
  const int32_t* last_page_len; // device [batch]
  int32_t batch, group, num_kv_heads, causal, num_sms;
  int32_t* plan;                // int workspace + kStatusBytes
  int64_t plan_words;           // capacity of the plan area in int32 words
  int64_t float_ws_bytes;
  uint32_t* status;
};
constexpr int kDevPlanThreads = 1024;
__global__ void aspire_plan_device_kernel(DevPlanParams p);

struct SelectParams {
  const void* dump;  // fp16 or fp32 (dump_f32) [rows, num_heads, dump_slots, kv_stride]
  int32_t dump_slots;  // 2: first/last dump (first + last query), 1: last-token dump
  int32_t dump_f32;
  int64_t kv_stride, max_seq_len;
  const float* lse;
  int64_t lse_rows;
  const int32_t* qo_indptr;
  const int32_t* row_ids;
  const float* scores_in;
  const int32_t* num_pages;
  const int32_t* block_table;
  int64_t block_table_stride;
  int32_t block_table_cols;
  int32_t num_heads, pages_per_slot, L, subset_cache_size, min_draft_pages;
  float draft_percent;
  float scale_log2;
  int32_t* table_out;
  int64_t table_stride;
  int32_t table_width;
  int32_t* counts_out;
  float* scores_out;
  uint32_t* status;
  int32_t sort_cap;  // power of two >= pages_per_slot
  int32_t order_by_page;  // sort the selection by page index and write block ids in that order
};

struct IndicesParams {
  const int32_t* mode_flags;
  const int32_t* draft_indices;
  int64_t draft_stride;
  int32_t draft_cols;
  const int32_t* verify_indices;
  int64_t verify_stride;
  int32_t verify_cols;
  const int32_t* draft_num_pages;
  const int32_t* verify_num_pages;
  int32_t* indices_out;
  int32_t* indptr_out;
  uint32_t* status;
  int64_t indices_capacity;
};

struct SpillParams {
  const int32_t* mode_flags;
  const int32_t* dec_lens;
  const int32_t* draft_cachelens;
  int32_t* draft_indices;
  int64_t draft_stride;
  int32_t draft_cols;
  int32_t* draft_num_pages;
  const int32_t* block_table;
  int64_t block_table_stride;
  int32_t block_table_cols;
  int32_t batch;
  uint32_t* status;
};
__global__ void aspire_draft_spill_kernel(SpillParams p);

// Slot-local dump state reset (dump_state.cu).
struct ClearDumpParams {
  void* dump;                 // fp16 or fp32 (dump_f32) [dump_rows, row_elems]
  int32_t dump_f32;
  int64_t row_elems;          // heads x slots x kv_stride
  int64_t dump_rows;
  const int32_t* slot_ids;
  float* lse;                 // optional [lse_rows, num_heads]
  int64_t lse_rows;
  int32_t num_heads;
  const int32_t* qo_indptr;   // required with lse
  int64_t qo_len;
  int32_t* mode_flags;        // optional [dump_rows]
  int32_t mode_value;
  uint32_t* status;
};
constexpr int kClearThreads = 256;
constexpr int64_t kClearPieceElems = 32768;  // elements of a row one CTA fills
__global__ void aspire_clear_dump_kernel(ClearDumpParams p);

constexpr int kIndicesThreads = 128;
__global__ void aspire_build_indices_kernel(IndicesParams p);

constexpr int kSelThreads = 512;
constexpr int kScoreThreads = 128;
__global__ void aspire_page_scores_kernel(SelectParams p);
constexpr int kMaxSelHeads = 128;

__global__ void aspire_attn_gather_kernel(AttnParams p);
__global__ void aspire_attn_tc_kernel(AttnParams p, const __grid_constant__ CUtensorMap tmap,
                                      const __grid_constant__ CUtensorMap qmap,
                                      const __grid_constant__ CUtensorMap qmap_pf);
constexpr int kMergeThreads = 128;
constexpr int kMergeCtasPerSm = 4;
__global__ void aspire_attn_merge_kernel(AttnParams p);
__global__ void aspire_append_kv_kernel(AppendParams p);
__global__ void aspire_select_pages_kernel(SelectParams p);

size_t gather_smem_bytes();
size_t tc_smem_bytes();
int tc_threads();
bool tc_kernel_available();
size_t select_smem_bytes(int pages_per_slot, int sort_cap);

}  // namespace aspire
