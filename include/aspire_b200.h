/*
 * aspire_b200.h - C ABI of libaspire_b200.so, the sm_100a implementation of
 * ASPIRE's unified mixed forward hot path:
 *
 *   1. paged mixed draft/verify attention (draft rows attend a sparse page
 *      list with q_len 1, verify rows attend the full cache with a causal
 *      multi-token query), optionally dumping the first/last-query or the
 *      last-query logits at the refresh layer, and optionally appending the
 *      step's new tokens inside the same launch;
 *   2. refresh-layer page scoring + top-k page re-selection, written in place
 *      into the draft page table;
 *   3. the paged KV append of the step's new tokens, the mixed page-list
 *      build, the draft-page spill insert and the dump-state reset of cleared
 *      slots;
 *   4. planning: on the host, or on the device inside a CUDA graph.
 *
 * Every entry point takes plain pointers, sizes and a CUDA stream handle
 * (passed as void*); no framework types cross this boundary.  Every entry
 * point returns 0 on success or a negative ASPIRE_ERR_* code; the message of
 * the last failure on the calling thread is returned by aspire_last_error().
 *
 * Tensor layouts (all device pointers unless stated otherwise):
 *   q        bf16 [tokens, num_qo_heads, 128], head_dim contiguous, strides given
 *   kv_cache bf16 [num_pages_total, 2, 16, num_kv_heads, 128] contiguous
 *            (index 0 of dim 1 = K, 1 = V; "NHD" paged layout)
 *   out      bf16 [tokens, num_qo_heads, 128], strides given
 *   lse      fp32 [tokens, num_qo_heads], base-2 log-sum-exp of the scaled logits
 *   dump     raw q.k logits of chosen queries (fp16, or fp32 holding the
 *            fp16-rounded value): [batch, dump_num_heads, 2, dump_kv_stride]
 *            first/last (ASPIRE_DUMP_FIRST_LAST) or [batch, dump_num_heads,
 *            dump_kv_stride] last query only (ASPIRE_DUMP_LAST_TOKEN)
 *
 * Only page_size 16 and head_dim 128 are supported (every ASPIRE config).
 */
#ifndef ASPIRE_B200_H_
#define ASPIRE_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ASPIRE_API __attribute__((visibility("default")))
#else
#define ASPIRE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define ASPIRE_B200_ABI_VERSION 5

#define ASPIRE_OK 0
#define ASPIRE_ERR_INVALID (-1)  /* bad argument (shape, size, alignment)       */
#define ASPIRE_ERR_CUDA (-2)     /* a CUDA runtime call failed                   */
#define ASPIRE_ERR_CAPACITY (-3) /* a workspace or plan buffer is too small      */
#define ASPIRE_ERR_DEVICE (-4)   /* a kernel reported bad input via the status word */

/* Device status word bits (written by kernels instead of faulting). */
#define ASPIRE_STATUS_BAD_PAGE 1u  /* a page id >= num_pages_total was skipped */
#define ASPIRE_STATUS_BAD_PLAN 2u  /* a work item was inconsistent and skipped */
#define ASPIRE_STATUS_BAD_ROW 4u   /* attention row past q_rows, or selection
                                      row/argument out of range               */
#define ASPIRE_STATUS_TIMEOUT 8u   /* a bounded device wait expired; the CTA stopped */

/* Logit-dump variants (AspireAttnArgs.dump_kind, AspireSelectArgs.dump_kind),
 * the dump kinds of aspire/backends/jit_kernels.py:180-193: */
#define ASPIRE_DUMP_FIRST_LAST 0  /* "first_last_compact": query 0 -> slot 0, query
                                     q_len-1 (q_len > 1) -> slot 1 (ASPIRE backend) */
#define ASPIRE_DUMP_LAST_TOKEN 1  /* "last_token": query q_len-1 only, one slot
                                     (LMBackendBase, base.py:208-214)              */
#define ASPIRE_DUMP_F16 0         /* dump buffer element type: fp16                */
#define ASPIRE_DUMP_F32 1         /* fp32, holding the fp16-rounded logit          */

/* ------------------------------------------------------------------------ */
/* Plan (host).                                                             */
/* ------------------------------------------------------------------------ */

/*
 * Result of aspire_plan: where the work list lives inside the device int
 * workspace and how much of each workspace it needs.  Returned to the
 * caller, who passes it back unchanged to aspire_mixed_attention.  The
 * kernels read every plan-dependent quantity from the device int workspace,
 * so a CUDA graph captured around aspire_mixed_attention stays valid when a
 * later aspire_plan call rewrites the work list in place.
 */
typedef struct AspirePlanInfo {
  int32_t num_items;        /* work items over all kernel classes            */
  int32_t num_items_gather; /* items for the CUDA-core gather kernel         */
  int32_t num_items_tc;     /* decode items for the tcgen05 kernel           */
  int32_t num_ctas;         /* persistent grid of each kernel class          */
  int32_t num_merge;        /* (row, kv-head, q-tile) groups split over chunks */
  int32_t chunk_tokens;     /* KV tokens per split-KV chunk                   */
  int64_t partial_rows;     /* fp32 partial rows needed in the float workspace */
  int64_t int_bytes;        /* bytes of the int workspace used (and uploaded) */
  int64_t float_bytes;      /* bytes of the float workspace needed            */
  int32_t num_qo_heads;
  int32_t num_kv_heads;
  int32_t causal;
  int32_t batch_size;       /* rows planned (including padding rows)          */
  int32_t max_q_len;
  int32_t tc_enabled;       /* 1 when wide query tiles use the tcgen05 kernel */
  int32_t on_device;        /* 1 when aspire_plan_device rendered the plan: the
                               counts above are then upper bounds (int_bytes and
                               float_bytes the workspace capacities) or -1      */
  int32_t num_items_prefill;/* prefill items for the tcgen05 kernel (rows of
                               at least 128 packed query rows: prefill chunks,
                               up to 256 packed rows per item)                 */
} AspirePlanInfo;

/*
 * Builds the split-KV work list for one attention program and uploads it.
 * Replaces FlashInfer's TwoStageHolisticPlan as driven by
 * HolisticAttentionWrapper.plan / plan_host
 * (aspire/attention/holistic_wrapper.py:253-265, :323-335).
 *
 *   qo_indptr  host int32 [batch_size + 1]  query-row offsets per request
 *   kv_indptr  host int32 [batch_size + 1]  page-list offsets per request
 *   kv_len     host int32 [batch_size]      attended KV tokens per request
 *   host_buf   pinned host buffer the work list is rendered into
 *   dev_int_ws device int workspace (the work list is copied to its start)
 *
 * The copy host_buf -> dev_int_ws is enqueued on `stream` with
 * cudaMemcpyAsync; the caller must not reuse host_buf until that copy has
 * completed (the wrapper fences a small ring of pinned buffers with events).
 * num_ctas <= 0 selects one CTA per SM of the current device.
 */
ASPIRE_API int aspire_plan(const int32_t* qo_indptr, const int32_t* kv_indptr, const int32_t* kv_len,
                int32_t batch_size, int32_t num_qo_heads, int32_t num_kv_heads, int32_t head_dim,
                int32_t page_size, int32_t causal, int32_t num_ctas, void* host_buf,
                size_t host_buf_bytes, void* dev_int_ws, size_t dev_int_ws_bytes,
                size_t float_ws_bytes, void* stream, AspirePlanInfo* info);

/* Host-only variant of aspire_plan: renders the work list into host_buf
 * without touching the device (used by tests and by callers that upload the
 * list themselves).  num_ctas must be > 0. */
ASPIRE_API int aspire_plan_host_only(const int32_t* qo_indptr, const int32_t* kv_indptr,
                          const int32_t* kv_len, int32_t batch_size, int32_t num_qo_heads,
                          int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
                          int32_t causal, int32_t num_ctas, void* host_buf,
                          size_t host_buf_bytes, size_t float_ws_bytes, AspirePlanInfo* info);

/* ------------------------------------------------------------------------ */
/* Mixed paged attention (device).                                          */
/* ------------------------------------------------------------------------ */

typedef struct AspireAttnArgs {
  const void* q;            /* bf16 [tokens, num_qo_heads, 128]                   */
  int64_t q_stride_n;       /* elements between tokens                            */
  int64_t q_stride_h;       /* elements between heads                             */
  const void* kv_cache;     /* bf16 [num_pages_total, 2, 16, num_kv_heads, 128]   */
  int64_t num_pages_total;
  const int32_t* kv_indices; /* int32 page ids, indexed by the plan's kv_indptr    */
  void* out;                /* bf16 [tokens, num_qo_heads, 128]                   */
  int64_t o_stride_n;
  int64_t o_stride_h;
  float* lse;               /* optional fp32 [tokens, num_qo_heads] (NULL = skip) */
  void* dump;               /* optional logit dump (NULL = skip), see dump_kind   */
  int64_t dump_num_heads;   /* heads dimension of the dump buffer                 */
  int64_t dump_kv_stride;   /* last dimension of the dump buffer                  */
  float sm_scale;           /* <= 0 selects 1/sqrt(128)                           */
  int32_t num_qo_heads;
  int32_t num_kv_heads;
  int32_t head_dim;         /* must be 128                                        */
  int32_t page_size;        /* must be 16                                         */
  void* int_ws;             /* device int workspace holding the uploaded plan     */
  size_t int_ws_bytes;
  void* float_ws;           /* device float workspace for split-KV partials       */
  size_t float_ws_bytes;
  int64_t q_rows;           /* first dimension of q (rows the kernels may read)   */
  /* Page tables, read instead of kv_indices when kv_indices is NULL: logical
   * page lp of request row b is draft_table[b * draft_stride + lp] when
   * mode_flags[b] == 0 (draft row), else block_table[b * block_table_stride
   * + lp].  This absorbs build_unified_indices (aspire/models/
   * sparse_draft_runner.py:126-153) into the attention: the plan's kv_indptr
   * still gives each row's page count.  No counterpart in the reference's
   * attention interface. */
  const int32_t* mode_flags;
  const int32_t* draft_table;
  int64_t draft_stride;
  const int32_t* block_table;
  int64_t block_table_stride;
  /* Dump variant: ASPIRE_DUMP_FIRST_LAST or ASPIRE_DUMP_LAST_TOKEN, element
   * type ASPIRE_DUMP_F16 or ASPIRE_DUMP_F32, and optional per-row enable
   * flags (int32 [batch], NULL = every row): row b writes its dump only when
   * dump_flags[b] != 0, the dump_enabled guard of the use_mode_flags variant
   * (jit_kernels.py:196-203, :300-301).  A zero-initialised struct keeps the
   * fp16 first/last dump of every row. */
  int32_t dump_kind;
  int32_t dump_dtype;
  const int32_t* dump_flags;
  /* Optional fused KV append (NULL = none): bf16 [>= q_rows, num_kv_heads, 128]
   * rows of the step's new keys and values (the queries' own: new token i of
   * row b at row qo_indptr[b] + i), head_dim contiguous, strides multiples of
   * 8 elements.
   * Before reading a row's keys the attention writes its new tokens into the
   * cache at positions kv_len - q_len + i of the row's pages (the page list or
   * the page tables), exactly as aspire_append_kv with the same qo_indptr and
   * page source does, so the separate append launch before the attention
   * (mylib::update_kv_padded, aspire/attention/kv_ops.py:127-187) goes away.
   * Host plans whose rows all run as tcgen05 decode items only: a plan with
   * prefill or CUDA-core items, or a device-side plan, is rejected. */
  const void* k_new;
  const void* v_new;
  int64_t k_new_stride_n, k_new_stride_h;
  int64_t v_new_stride_n, v_new_stride_h;
} AspireAttnArgs;

/*
 * Runs the planned attention program on `stream`.  Replaces
 * HolisticAttentionWrapper.run (aspire/attention/holistic_wrapper.py:344-386)
 * and the persistent FlashInfer kernel with its split-KV merge; with `dump`
 * set it also replaces the logit-dump variants (first/last and last-token,
 * with or without mode flags, fp16 or fp32 buffer:
 * aspire/backends/jit_kernels.py:180-203, :240-256, :271-332;
 * aspire/attention/holistic_wrapper.py:401-434).
 * Capturable in a CUDA graph; allocates nothing.
 */
ASPIRE_API int aspire_mixed_attention(const AspireAttnArgs* args, const AspirePlanInfo* plan, void* stream);

/*
 * Sizes of the two device arrays that aspire_mixed_attention_noalloc uses
 * instead of caller-provided workspaces: the plan array (status word + work
 * list) and the split-KV partials array.  Every GPU that loads the library
 * holds both (8.5 MiB in total) until the process exits.
 */
#define ASPIRE_NOALLOC_INT_BYTES ((size_t)512 * 1024)
#define ASPIRE_NOALLOC_FLOAT_BYTES ((size_t)8 * 1024 * 1024)

/*
 * aspire_mixed_attention for callers that cannot allocate device memory --
 * a plug-in whose host application owns every byte of GPU memory, or a
 * serving loop whose device memory is fixed at start-up (cudaMalloc would
 * also synchronise the device mid-step).  This entry point has no
 * counterpart in the reference; it allocates nothing.
 *
 * The caller renders the plan on the host with aspire_plan_host_only (its
 * num_ctas = the device's SM count) into `host_plan` and passes the returned
 * info; the call uploads that plan into the library's built-in plan array on
 * `stream` (pinned host memory keeps the copy asynchronous: `host_plan` must
 * then stay unchanged until the stream has reached that copy) and runs the
 * attention with the built-in partials array.  The int_ws / float_ws fields
 * of `args` are ignored.  A plan rendered by aspire_plan_device (on_device
 * set) is rejected with ASPIRE_ERR_INVALID.  Plans larger than
 * ASPIRE_NOALLOC_INT_BYTES or needing more than ASPIRE_NOALLOC_FLOAT_BYTES of
 * partials are rejected with ASPIRE_ERR_CAPACITY.  Every argument is checked
 * before the built-in arrays are touched: a rejected call changes nothing on
 * the device.  The first call on a device looks up the arrays' device
 * addresses (make it before any stream capture).  All calls share the
 * arrays: calls that overlap on the GPU race and must be serialised.  The
 * kernels' status word (ASPIRE_STATUS_* bits) lives in the built-in plan
 * array; it is cleared by every call and read by aspire_noalloc_status.
 */
ASPIRE_API int aspire_mixed_attention_noalloc(const AspireAttnArgs* args, const AspirePlanInfo* plan,
                                              const void* host_plan, void* stream);

/*
 * Enqueues on `stream` a copy of the status word of the calls above (the
 * ASPIRE_STATUS_* bits their kernels set instead of faulting: a bad page id,
 * an inconsistent plan, a row past q_rows, a wait that timed out) into
 * *host_out, and with `clear` != 0 a reset of the word to zero after it.
 * *host_out holds the value once the stream has reached the copy
 * (synchronise the stream before reading it).  Allocates nothing.  Companion
 * of aspire_mixed_attention_noalloc; no counterpart in the reference.
 */
ASPIRE_API int aspire_noalloc_status(uint32_t* host_out, int32_t clear, void* stream);

/* ------------------------------------------------------------------------ */
/* Paged KV append (device).                                                */
/* ------------------------------------------------------------------------ */

typedef struct AspireAppendArgs {
  const void* k;            /* bf16 [num_tokens, num_kv_heads, 128]              */
  const void* v;
  int64_t k_stride_n, k_stride_h, v_stride_n, v_stride_h;
  int64_t num_tokens;       /* bucket tokens (rows past the last request skipped) */
  const int32_t* append_indptr; /* int32 [num_rows + 1] new-token offsets        */
  void* kv_cache;           /* bf16 [num_pages_total, 2, 16, num_kv_heads, 128]  */
  int64_t num_pages_total;
  const int32_t* page_indices;  /* int32 page ids                                */
  const int32_t* page_indptr;   /* int32 [num_rows + 1]                          */
  const int32_t* last_page_len; /* int32 [num_rows]                              */
  int32_t num_rows;
  int32_t num_kv_heads;
  int32_t head_dim;         /* must be 128 */
  int32_t page_size;        /* must be 16  */
  uint32_t* status;         /* optional device status word (NULL = none)         */
  /* Page tables, read instead of page_indices when page_indices is NULL (the
   * same rule as AspireAttnArgs). */
  const int32_t* mode_flags;
  const int32_t* draft_table;
  int64_t draft_stride;
  const int32_t* block_table;
  int64_t block_table_stride;
} AspireAppendArgs;

/*
 * Writes each new token's K and V row into its page.  Replaces
 * mylib::update_kv_padded (aspire/attention/kv_ops.py:63-187): a token whose
 * position is negative (bucket padding) or past its row's length is skipped.
 */
ASPIRE_API int aspire_append_kv(const AspireAppendArgs* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Page scoring + top-k re-selection (device).                              */
/* ------------------------------------------------------------------------ */

typedef struct AspireSelectArgs {
  const void* dump;         /* [dump_batch, num_heads, 2 or 1, kv_stride] (dump_kind,
                               dump_dtype); NULL when scores_in set                 */
  int64_t kv_stride;
  int64_t max_seq_len;      /* logits past this position are ignored              */
  const float* lse;         /* fp32 [lse_rows, num_heads]                         */
  int64_t lse_rows;
  const int32_t* qo_indptr; /* int32 [>= rows + 1] of the dump program            */
  const int32_t* row_ids;   /* optional int32 [batch]: dump / qo_indptr row of each
                               output row (NULL = identity), for select_subset      */
  const float* scores_in;   /* optional fp32 [batch, pages_per_slot] raw page scores:
                               when set, scoring is skipped and only the top-k runs */
  const int32_t* num_pages; /* int32 [batch] valid pages per request              */
  const int32_t* block_table; /* int32 [batch, block_table_stride]                */
  int64_t block_table_stride;
  int32_t block_table_cols; /* page indices are clamped to cols - 1 (as the reference's topk_idx) */
  int32_t batch;
  int32_t num_heads;
  int32_t page_size;        /* must be 16 */
  int32_t pages_per_slot;
  int32_t L;                /* trailing pages always kept                          */
  int32_t subset_cache_size;/* k of the top-k                                      */
  int32_t min_draft_pages;  /* < 0 means None                                      */
  float draft_percent;      /* < 0 means None                                      */
  float sm_scale;           /* <= 0 selects 1/sqrt(head_dim)                       */
  int32_t head_dim;
  int32_t* table_out;       /* int32 [batch, table_stride]: sorted ids, zero tail  */
  int64_t table_stride;
  int32_t table_width;      /* columns written per row                             */
  int32_t* counts_out;      /* int32 [batch] valid counts                          */
  float* scores_out;        /* optional fp32 [batch, pages_per_slot] final scores  */
  uint32_t* status;         /* optional device status word                         */
  float* scores_ws;         /* fp32 [batch, pages_per_slot] scratch for the page
                               scores; required when scores_in and scores_out are
                               both NULL                                           */
  int32_t order_by_page;    /* 1 (with scores_in): the last L pages are not forced
                               and a row lists its selected pages in page order;
                               with page-index scores this is the recent-page
                               seeding of LMBackendBase._build_recent_draft_rows
                               (aspire/backends/base.py:1522-1537).  0: ascending
                               block ids, as the replan path stores them          */
  int32_t dump_kind;        /* ASPIRE_DUMP_FIRST_LAST: PageSelectorFirstLastAvg's
                               score (page_selector.py:163-181); ASPIRE_DUMP_LAST_TOKEN:
                               PageSelector's (page_selector.py:110-130, 140-146)  */
  int32_t dump_dtype;       /* ASPIRE_DUMP_F16 or ASPIRE_DUMP_F32                  */
} AspireSelectArgs;

/*
 * Scores pages from the logit dump and the dump program's LSE, selects the
 * top pages (ties broken by the lower page index) and writes the ascending
 * page-id rows plus the valid counts in place.  Replaces
 * PageSelectorFirstLastAvg.select (aspire/backends/page_selector.py:206-214,
 * :163-181, :79-108), or with ASPIRE_DUMP_LAST_TOKEN PageSelector.select
 * (:140-146, :110-130), followed by LMBackendBase._store_draft_rows
 * (aspire/backends/base.py:1421-1471).
 */
ASPIRE_API int aspire_select_pages(const AspireSelectArgs* args, void* stream);

/*
 * Renders the same work list as aspire_plan on the device, from device
 * arrays, with no host round trip or synchronisation, so that planning can be
 * captured in a CUDA graph together with the step.  Replaces the per-step host
 * planning of HolisticAttentionWrapper.plan / plan_host
 * (aspire/attention/holistic_wrapper.py:200-342) and the HostPlanState upload
 * (aspire/backends/host_plan.py:154-306).  kv_len of row b is
 * max(pages_b - 1, 0) * 16 + last_page_len[b], as in plan().  Every row goes
 * to the tcgen05 kernel, as a decode item or, with 128 or more packed query
 * rows, a prefill item (the default routing; other routing thresholds are
 * rejected).  A malformed row or a plan beyond the workspaces is reported as
 * ASPIRE_STATUS_BAD_PLAN on the device (the kernels then skip the plan).
 * `info` receives the grid, the heads and the workspace capacities.
 */
ASPIRE_API int aspire_plan_device(const int32_t* qo_indptr, const int32_t* kv_indptr,
                                  const int32_t* last_page_len, int32_t batch_size, int32_t num_qo_heads,
                                  int32_t num_kv_heads, int32_t head_dim, int32_t page_size, int32_t causal,
                                  int32_t num_ctas, void* dev_int_ws, size_t dev_int_ws_bytes,
                                  size_t float_ws_bytes, void* stream, AspirePlanInfo* info);

/* ------------------------------------------------------------------------ */
/* Fused attention prologue: q/k norm + RoPE + paged append (device).       */
/* ------------------------------------------------------------------------ */

typedef struct AspirePrologueArgs {
  const void* q;            /* bf16 [num_tokens, num_qo_heads, 128] (wqkv output view) */
  int64_t q_stride_n, q_stride_h;
  const void* k;            /* bf16 [num_tokens, num_kv_heads, 128]               */
  int64_t k_stride_n, k_stride_h;
  const void* v;            /* bf16 [num_tokens, num_kv_heads, 128]               */
  int64_t v_stride_n, v_stride_h;
  void* q_out;              /* bf16 [num_tokens, num_qo_heads, 128]; may equal q  */
  int64_t qo_stride_n, qo_stride_h;
  int64_t num_tokens;
  int32_t num_qo_heads;
  int32_t num_kv_heads;
  int32_t head_dim;         /* must be 128 */
  const void* q_norm_weight;/* bf16 [128]; NULL together with k_norm_weight: no
                               qk-norm and no permutation (models without it)     */
  const void* k_norm_weight;
  float norm_eps;
  const int32_t* rope_offsets; /* int32 [num_rows]: position of each row's first new token */
  float rope_theta;
  float rope_scale;
  float low_freq_factor;    /* Llama-3.1 smoothing when > 0, else plain RoPE      */
  float high_freq_factor;
  float old_context_len;
  const int32_t* append_indptr; /* int32 [num_rows + 1]                           */
  int32_t num_rows;
  void* kv_cache;           /* bf16 [num_pages_total, 2, 16, num_kv_heads, 128]  */
  int64_t num_pages_total;
  int32_t page_size;        /* must be 16 */
  const int32_t* page_indices;  /* flat page list, or NULL for the page tables     */
  const int32_t* page_indptr;
  const int32_t* last_page_len;
  const int32_t* mode_flags;
  const int32_t* draft_table;
  int64_t draft_stride;
  const int32_t* block_table;
  int64_t block_table_stride;
  uint32_t* status;
} AspirePrologueArgs;

/*
 * One launch for the per-layer attention prologue: q_norm / k_norm with the
 * HF-to-interleaved permutation (aspire/models/sparse_draft_transformer.py:
 * 150-158, transformer.py:360-364, 505-515), the interleaved RoPE of q and k
 * (mylib::rope -> FlashInfer apply_rope_inplace / apply_llama31_rope_inplace,
 * aspire/models/mixed_transformer.py:159-197) and the paged append of the
 * rotated k and of v (mylib::update_kv_padded, aspire/attention/kv_ops.py:
 * 127-187).  Writes the rotated q to q_out.  No single counterpart in the
 * reference: it replaces three of its ops.
 */
ASPIRE_API int aspire_qkv_prologue(const AspirePrologueArgs* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Mixed page list (device).                                                */
/* ------------------------------------------------------------------------ */

typedef struct AspireIndicesArgs {
  const int32_t* mode_flags;      /* int32 [batch]: 0 = draft row, otherwise verify row   */
  const int32_t* draft_indices;   /* int32 [batch, draft_stride] draft page tables        */
  int64_t draft_stride;
  int32_t draft_cols;             /* usable columns of a draft table row                  */
  const int32_t* verify_indices;  /* int32 [batch, verify_stride] block tables            */
  int64_t verify_stride;
  int32_t verify_cols;
  const int32_t* draft_num_pages; /* int32 [batch]                                        */
  const int32_t* verify_num_pages;/* int32 [batch]                                        */
  int32_t batch;
  int32_t* indices_out;           /* int32 [sum of the rows' page counts]                 */
  int32_t* indptr_out;            /* int32 [batch + 1]: exclusive prefix sum              */
  uint32_t* status;               /* optional device status word                          */
  int64_t indices_capacity;       /* entries of indices_out: pages that would land past
                                     it are not written (ASPIRE_STATUS_BAD_ROW)          */
} AspireIndicesArgs;

/*
 * Builds the mixed page list of one step: row b's pages are its draft table
 * prefix (draft rows) or its block-table prefix (verify rows), concatenated
 * in row order, with indptr the prefix sum of the counts.  Replaces
 * build_unified_indices (aspire/models/sparse_draft_runner.py:126-153) and
 * its Triton _copy_indices_kernel (:93-123).  A count larger than its table's
 * width copies the width, a negative count counts as 0, and a page that
 * would land at or past indices_capacity is not written; each sets
 * ASPIRE_STATUS_BAD_ROW.  With batch 0 only indptr_out[0] = 0 is written, as
 * the reference does.
 */
ASPIRE_API int aspire_build_unified_indices(const AspireIndicesArgs* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Draft-page spill insert (device).                                        */
/* ------------------------------------------------------------------------ */

typedef struct AspireSpillArgs {
  const int32_t* mode_flags;      /* int32 [batch]: 0 = draft row                          */
  const int32_t* dec_lens;        /* int32 [batch]: the step's decode lengths (0 = finished) */
  const int32_t* draft_cachelens; /* int32 [batch]: draft cache lengths, this step's token
                                     counted                                                */
  int32_t* draft_indices;         /* int32 [batch, draft_stride] draft tables (in place)    */
  int64_t draft_stride;
  int32_t draft_cols;             /* usable columns of a draft table row                    */
  int32_t* draft_num_pages;       /* int32 [batch] draft page counts (in place)             */
  const int32_t* block_table;     /* int32 [batch, block_table_stride]                      */
  int64_t block_table_stride;
  int32_t block_table_cols;
  int32_t batch;
  int32_t page_size;              /* must be 16                                             */
  uint32_t* status;               /* optional device status word                            */
} AspireSpillArgs;

/*
 * Adds the page of a draft row's newest token to its draft table when that
 * token opened a new page: for a draft row with dec_len > 0 whose
 * (draft_cachelen - 1) is a multiple of the page size, the page
 * block_table[b, ceil(draft_cachelen / 16) - 1] is appended at column
 * draft_num_pages[b] (and the count incremented) unless the table's last
 * listed page already is that page or the row has no free column.  Replaces
 * the spill check and insert of LMBackendBase.prepare_forward_inputs
 * (aspire/backends/base.py:1222-1236) with _handle_draft_page_spill
 * (:718-742) and its host-identified variant _handle_draft_page_spill_ids
 * (:744-759): one launch, no host synchronisation, capturable.  A page index
 * past block_table_cols sets ASPIRE_STATUS_BAD_ROW and skips the row.
 */
ASPIRE_API int aspire_draft_page_spill(const AspireSpillArgs* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Dump-state reset of cleared slots (device).                              */
/* ------------------------------------------------------------------------ */

typedef struct AspireClearDumpArgs {
  void* dump;               /* [dump_rows, num_heads, slots, kv_stride], dump_dtype  */
  int32_t dump_dtype;       /* ASPIRE_DUMP_F16 or ASPIRE_DUMP_F32                    */
  int32_t num_heads;
  int32_t slots;            /* 2 (first/last dump) or 1 (last-token dump)            */
  int64_t kv_stride;
  int64_t dump_rows;        /* rows of the dump buffer (slot ids must be below it)   */
  const int32_t* slot_ids;  /* int32 [n_slots], device                               */
  int32_t n_slots;
  float* lse;               /* optional fp32 [lse_rows, num_heads] (NULL = skip)     */
  int64_t lse_rows;
  const int32_t* qo_indptr; /* int32 [qo_len] of the dump program; required with lse */
  int64_t qo_len;
  int32_t* mode_flags;      /* optional int32 [dump_rows] dump enable flags (NULL = skip) */
  int32_t mode_value;       /* value written to mode_flags[slot] (VERIFY_MODE = 1)   */
  uint32_t* status;         /* optional device status word                           */
} AspireClearDumpArgs;

/*
 * Resets the dump state of cleared slots in one launch: every element of the
 * slots' dump rows becomes -inf, the LSE row of each slot's last query
 * (qo_indptr[slot + 1] - 1, clamped to [0, lse_rows)) becomes 0 and
 * mode_flags[slot] becomes mode_value.  Replaces
 * LMBackendBase._clear_variant_slot_state (aspire/backends/base.py:1404-1419),
 * three torch indexing ops.  A slot id outside [0, dump_rows) or whose
 * qo_indptr entry is past qo_len is skipped and sets ASPIRE_STATUS_BAD_ROW.
 * Capturable; allocates nothing.
 */
ASPIRE_API int aspire_clear_dump_slots(const AspireClearDumpArgs* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Utilities.                                                               */
/* ------------------------------------------------------------------------ */

/* Message of the last failing call on this thread ("" when none). */
ASPIRE_API const char* aspire_last_error(void);

/* ABI version of the loaded library (ASPIRE_B200_ABI_VERSION). */
ASPIRE_API int aspire_abi_version(void);

/* Bytes of the int workspace reserved ahead of the plan for the status word;
 * the status word is the first uint32 of the int workspace. */
ASPIRE_API size_t aspire_status_offset(void);

/* Bound of one pipeline wait inside the tcgen05 attention kernel, in
 * nanoseconds, for launches made after the call (0 restores the default of
 * 1 s).  A wait that runs past it stops its CTA, which sets
 * ASPIRE_STATUS_TIMEOUT, waits (with a fixed 1 s bound) for its own copies and
 * MMAs in flight, frees its tensor memory and returns; the device stays
 * usable.  Process-wide.  No counterpart in the reference, whose waits are
 * unbounded. */
ASPIRE_API int aspire_set_wait_limit_ns(uint64_t ns);

/* Names of the kernels the library launches, one per line (diagnostics). */
ASPIRE_API const char* aspire_kernel_names(void);

#ifdef __cplusplus
}
#endif

#endif /* ASPIRE_B200_H_ */
