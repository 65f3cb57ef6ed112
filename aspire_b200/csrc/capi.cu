// extern "C" entry points of libaspire_b200.so (declared in
// include/aspire_b200.h): argument checking, launch configuration and
// error reporting.  No entry point allocates memory or synchronises.
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <algorithm>
#include <cstring>
#include <string>
#include <utility>

#include <cudaTypedefs.h>

#include "kernels.cuh"
#include "errors.h"

namespace aspire {

// ---- error state ----------------------------------------------------------
namespace {
thread_local std::string g_last_error;
}

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}
void clear_error() { g_last_error.clear(); }
const char* last_error() { return g_last_error.c_str(); }
int check_cuda(int st, const char* what) {
  if (st == cudaSuccess) return ASPIRE_OK;
  return set_error(ASPIRE_ERR_CUDA, std::string(what) + ": " +
                                        cudaGetErrorString(static_cast<cudaError_t>(st)));
}

// Launches `kernel` with a programmatic dependency on the preceding work in
// the stream (every kernel begins with griddepcontrol.launch_dependents +
// wait, so it is scheduled early but reads nothing before its predecessor
// has finished).
template <typename... KArgs, typename... Args>
int launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, const char* what,
           Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...), what);
}

int plan_impl(const int32_t* qo_indptr, const int32_t* kv_indptr, const int32_t* kv_len,
              int32_t batch_size, int32_t num_qo_heads, int32_t num_kv_heads, int32_t head_dim,
              int32_t page_size, int32_t causal, int32_t num_sms, bool tc_enabled, int32_t tc_min_rows,
              int32_t tc_min_kv, void* host_buf, size_t host_buf_bytes, size_t float_ws_bytes,
              AspirePlanInfo* info);

namespace {

int current_sm_count(int* out) {
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  return check_cuda(cudaDeviceGetAttribute(out, cudaDevAttrMultiProcessorCount, dev),
                    "cudaDeviceGetAttribute(SM count)");
}

// Dynamic shared memory a kernel has been opted in to, per device: the
// attribute set by cudaFuncSetAttribute applies to the current device only,
// so a host thread that drives several GPUs sets it once on each.
constexpr int kMaxDevices = 64;
struct SmemOptIn {
  std::atomic<int> bytes[kMaxDevices];
  SmemOptIn() {
    for (auto& b : bytes) b.store(48 * 1024);
  }
};

// Opt-in to large dynamic shared memory once per (kernel, device, size).
int ensure_smem(const void* func, size_t bytes, SmemOptIn& cache) {
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  const bool cached = dev >= 0 && dev < kMaxDevices;
  if (cached && int(bytes) <= cache.bytes[dev].load(std::memory_order_relaxed)) return ASPIRE_OK;
  rc = check_cuda(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)),
                  "cudaFuncSetAttribute(max dynamic smem)");
  if (rc == ASPIRE_OK && cached) {
    int cur = cache.bytes[dev].load(std::memory_order_relaxed);
    while (cur < int(bytes) && !cache.bytes[dev].compare_exchange_weak(cur, int(bytes))) {
    }
  }
  return rc;
}

SmemOptIn g_gather_smem, g_tc_smem, g_sel_smem;

// Bound of one pipeline wait of the tcgen05 kernel (aspire_set_wait_limit_ns);
// 0 selects the default.
constexpr uint64_t kDefaultWaitNs = 1000000000ull;
std::atomic<uint64_t> g_wait_limit_ns{0};

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}

// 5-D view of the paged cache [pages, 2, 16, Hkv, 128] (innermost first:
// dim, head, token, K/V, page) with a 64-dim x 16-token box, 128-byte swizzle.
// Query tile map over q [q_rows, num_qo_heads, 128]: boxes of 64 dims x
// `group` heads x `box_tokens` tokens, 128-byte swizzle (the K-major B operand
// of Q.K^T).
int encode_q_tensor_map(CUtensorMap* map, const void* q, int64_t q_rows, int num_qo_heads, int64_t stride_n,
                        int64_t stride_h, int group, int box_tokens) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return set_error(ASPIRE_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[3] = {cuuint64_t(kHeadDim), cuuint64_t(num_qo_heads), cuuint64_t(q_rows)};
  cuuint64_t strides[2] = {cuuint64_t(stride_h) * 2, cuuint64_t(stride_n) * 2};
  cuuint32_t box[3] = {64, cuuint32_t(group), cuuint32_t(box_tokens)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(ASPIRE_ERR_INVALID, "cuTensorMapEncodeTiled (q) failed with code " + std::to_string(int(r)));
  return ASPIRE_OK;
}

int encode_kv_tensor_map(CUtensorMap* map, const void* kv, int64_t num_pages, int num_kv_heads) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return set_error(ASPIRE_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const cuuint64_t row = kHeadDim * 2;  // bytes per (token, head)
  cuuint64_t dims[5] = {cuuint64_t(kHeadDim), cuuint64_t(num_kv_heads), cuuint64_t(kPageSize), 2,
                        cuuint64_t(num_pages)};
  cuuint64_t strides[4] = {row, row * num_kv_heads, row * num_kv_heads * kPageSize,
                           row * num_kv_heads * kPageSize * 2};
  cuuint32_t box[5] = {64, 1, cuuint32_t(kPageSize), 1, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(kv), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(ASPIRE_ERR_INVALID, "cuTensorMapEncodeTiled failed with code " + std::to_string(int(r)));
  return ASPIRE_OK;
}

// Routing thresholds of rows to the tcgen05 kernel (packed query rows, KV
// tokens); overridable for measurements through the environment.
int32_t env_int(const char* name, int32_t dflt) {
  const char* e = std::getenv(name);
  return (e && *e) ? static_cast<int32_t>(std::strtol(e, nullptr, 10)) : dflt;
}
int32_t tc_min_rows() {
  static const int32_t v = env_int("ASPIRE_B200_TC_MIN_ROWS", 1);
  return v;
}
int32_t tc_min_kv() {
  static const int32_t v = env_int("ASPIRE_B200_TC_MIN_KV", 4096);
  return v;
}

bool tc_env_enabled() {
  const char* e = std::getenv("ASPIRE_B200_DISABLE_TC");
  return !(e && e[0] == '1');
}

}  // namespace

int check_attention_args(const AspireAttnArgs* a, const AspirePlanInfo* plan, const char* who) {
  const std::string w(who);
  if (!a || !plan) return set_error(ASPIRE_ERR_INVALID, w + ": null argument");
  if (a->head_dim != kHeadDim) return set_error(ASPIRE_ERR_INVALID, w + ": head_dim must be 128");
  if (a->page_size != kPageSize) return set_error(ASPIRE_ERR_INVALID, w + ": page_size must be 16");
  if (a->num_kv_heads <= 0 || a->num_qo_heads % a->num_kv_heads != 0)
    return set_error(ASPIRE_ERR_INVALID, w + ": bad head counts");
  if (a->num_qo_heads != plan->num_qo_heads || a->num_kv_heads != plan->num_kv_heads)
    return set_error(ASPIRE_ERR_INVALID, w + ": head counts differ from the plan's");
  if (!a->q || !a->kv_cache || !a->out) return set_error(ASPIRE_ERR_INVALID, w + ": null tensor pointer");
  if (!a->kv_indices && (!a->mode_flags || !a->draft_table || !a->block_table))
    return set_error(ASPIRE_ERR_INVALID, w + ": kv_indices or the three page tables are required");
  if ((reinterpret_cast<uintptr_t>(a->q) | reinterpret_cast<uintptr_t>(a->kv_cache)) & 15)
    return set_error(ASPIRE_ERR_INVALID, w + ": q / kv_cache not 16-byte aligned");
  if ((a->q_stride_n | a->q_stride_h) & 7)
    return set_error(ASPIRE_ERR_INVALID, w + ": q strides must be multiples of 8 elements");
  if (a->dump && (a->dump_num_heads < a->num_qo_heads || a->dump_kv_stride <= 0))
    return set_error(ASPIRE_ERR_INVALID, w + ": bad dump geometry");
  if (a->dump_kind != ASPIRE_DUMP_FIRST_LAST && a->dump_kind != ASPIRE_DUMP_LAST_TOKEN)
    return set_error(ASPIRE_ERR_INVALID, w + ": dump_kind must be ASPIRE_DUMP_FIRST_LAST or ASPIRE_DUMP_LAST_TOKEN");
  if (a->dump_dtype != ASPIRE_DUMP_F16 && a->dump_dtype != ASPIRE_DUMP_F32)
    return set_error(ASPIRE_ERR_INVALID, w + ": dump_dtype must be ASPIRE_DUMP_F16 or ASPIRE_DUMP_F32");
  if (a->dump && (reinterpret_cast<uintptr_t>(a->dump) & (a->dump_dtype == ASPIRE_DUMP_F32 ? 3 : 1)))
    return set_error(ASPIRE_ERR_INVALID, w + ": dump buffer not aligned to its element type");
  if (a->q_rows <= 0 || a->q_rows > INT32_MAX)
    return set_error(ASPIRE_ERR_INVALID, w + ": q_rows (rows of q) must be set");
  if (a->k_new || a->v_new) {
    if (!a->k_new || !a->v_new) return set_error(ASPIRE_ERR_INVALID, w + ": fused append needs k_new and v_new");
    if (plan->on_device || plan->num_items_prefill > 0 || plan->num_items_gather > 0 || !plan->tc_enabled)
      return set_error(ASPIRE_ERR_INVALID,
                       w + ": fused append needs a host plan of tcgen05 decode items only (no prefill rows, "
                           "no CUDA-core rows); append with aspire_append_kv first otherwise");
    if ((reinterpret_cast<uintptr_t>(a->k_new) | reinterpret_cast<uintptr_t>(a->v_new)) & 15)
      return set_error(ASPIRE_ERR_INVALID, w + ": k_new / v_new not 16-byte aligned");
    if ((a->k_new_stride_n | a->k_new_stride_h | a->v_new_stride_n | a->v_new_stride_h) & 7)
      return set_error(ASPIRE_ERR_INVALID, w + ": k_new / v_new strides must be multiples of 8 elements");
  }
  const int group = a->num_qo_heads / a->num_kv_heads;
  const bool run_tc = plan->tc_enabled && group <= kTcQTile;
  if (run_tc && ((reinterpret_cast<uintptr_t>(a->out) & 15) || ((a->o_stride_n | a->o_stride_h) & 7)))
    return set_error(ASPIRE_ERR_INVALID, w + ": out must be 16-byte aligned with strides in multiples of 8");
  if (run_tc && (a->num_pages_total <= 0 || a->num_pages_total > INT32_MAX))
    return set_error(ASPIRE_ERR_INVALID, w + ": num_pages_total out of range");
  return ASPIRE_OK;
}

}  // namespace aspire

using namespace aspire;

extern "C" {

int aspire_abi_version(void) { return ASPIRE_B200_ABI_VERSION; }

const char* aspire_last_error(void) { return aspire::last_error(); }

size_t aspire_status_offset(void) { return kStatusBytes; }

int aspire_set_wait_limit_ns(uint64_t ns) {
  clear_error();
  g_wait_limit_ns.store(ns, std::memory_order_relaxed);
  return ASPIRE_OK;
}

const char* aspire_kernel_names(void) {
  return "aspire_attn_gather_kernel\naspire_attn_tc_kernel\naspire_attn_merge_kernel\naspire_append_kv_kernel\n"
         "aspire_select_pages_kernel\naspire_page_scores_kernel\naspire_build_indices_kernel\naspire_qkv_prologue_kernel\naspire_plan_device_kernel\n"
         "aspire_draft_spill_kernel\naspire_clear_dump_kernel\n";
}

int aspire_plan_host_only(const int32_t* qo_indptr, const int32_t* kv_indptr,
                          const int32_t* kv_len, int32_t batch_size, int32_t num_qo_heads,
                          int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
                          int32_t causal, int32_t num_ctas, void* host_buf,
                          size_t host_buf_bytes, size_t float_ws_bytes, AspirePlanInfo* info) {
  clear_error();
  return plan_impl(qo_indptr, kv_indptr, kv_len, batch_size, num_qo_heads, num_kv_heads, head_dim,
                   page_size, causal, num_ctas, tc_kernel_available() && tc_env_enabled(), tc_min_rows(),
                   tc_min_kv(), host_buf, host_buf_bytes, float_ws_bytes, info);
}

int aspire_plan_device(const int32_t* qo_indptr, const int32_t* kv_indptr, const int32_t* last_page_len,
                       int32_t batch_size, int32_t num_qo_heads, int32_t num_kv_heads, int32_t head_dim,
                       int32_t page_size, int32_t causal, int32_t num_ctas, void* dev_int_ws,
                       size_t dev_int_ws_bytes, size_t float_ws_bytes, void* stream, AspirePlanInfo* info) {
  clear_error();
  if (!qo_indptr || !kv_indptr || !last_page_len || !dev_int_ws || !info)
    return set_error(ASPIRE_ERR_INVALID, "aspire_plan_device: null pointer argument");
  if (batch_size < 0) return set_error(ASPIRE_ERR_INVALID, "aspire_plan_device: batch_size < 0");
  if (head_dim != kHeadDim || page_size != kPageSize)
    return set_error(ASPIRE_ERR_INVALID, "aspire_plan_device: head_dim must be 128 and page_size 16");
  if (num_kv_heads <= 0 || num_qo_heads <= 0 || num_qo_heads % num_kv_heads != 0)
    return set_error(ASPIRE_ERR_INVALID,
                     "aspire_plan_device: num_qo_heads must be a positive multiple of num_kv_heads");
  const int group = num_qo_heads / num_kv_heads;
  if (group > kTcQTile || !(tc_kernel_available() && tc_env_enabled()) || tc_min_rows() > 1)
    return set_error(ASPIRE_ERR_INVALID,
                     "aspire_plan_device: device planning routes every row to the tcgen05 kernel "
                     "(group <= 48, default routing)");
  if (dev_int_ws_bytes <= kStatusBytes + kHdrWords * 4)
    return set_error(ASPIRE_ERR_CAPACITY, "aspire_plan_device: int workspace too small");
  if (num_ctas <= 0) {
    int rc = current_sm_count(&num_ctas);
    if (rc) return rc;
  }
  DevPlanParams p;
  p.qo_indptr = qo_indptr;
  p.kv_indptr = kv_indptr;
  p.last_page_len = last_page_len;
  p.batch = batch_size;
  p.group = group;
  p.num_kv_heads = num_kv_heads;
  p.causal = causal;
  p.num_sms = num_ctas;
  p.plan = reinterpret_cast<int32_t*>(static_cast<char*>(dev_int_ws) + kStatusBytes);
  p.plan_words = int64_t((dev_int_ws_bytes - kStatusBytes) / 4);
  p.float_ws_bytes = int64_t(float_ws_bytes);
  p.status = static_cast<uint32_t*>(dev_int_ws);
  int rc = launch(aspire_plan_device_kernel, dim3(1), dim3(kDevPlanThreads), 0, static_cast<cudaStream_t>(stream),
                  "aspire_plan_device_kernel launch", p);
  if (rc) return rc;
  std::memset(info, 0, sizeof(*info));
  info->num_items = -1;
  info->num_items_gather = 0;
  info->num_items_tc = -1;
  info->num_ctas = num_ctas;
  info->num_merge = 1;  // may split: the float workspace is required
  info->chunk_tokens = -1;
  info->partial_rows = -1;
  info->int_bytes = int64_t(dev_int_ws_bytes) - kStatusBytes;
  info->float_bytes = int64_t(float_ws_bytes);
  info->num_qo_heads = num_qo_heads;
  info->num_kv_heads = num_kv_heads;
  info->causal = causal ? 1 : 0;
  info->batch_size = batch_size;
  info->max_q_len = -1;
  info->tc_enabled = 1;
  info->on_device = 1;
  info->num_items_prefill = -1;
  return ASPIRE_OK;
}

int aspire_plan(const int32_t* qo_indptr, const int32_t* kv_indptr, const int32_t* kv_len,
                int32_t batch_size, int32_t num_qo_heads, int32_t num_kv_heads, int32_t head_dim,
                int32_t page_size, int32_t causal, int32_t num_ctas, void* host_buf,
                size_t host_buf_bytes, void* dev_int_ws, size_t dev_int_ws_bytes,
                size_t float_ws_bytes, void* stream, AspirePlanInfo* info) {
  clear_error();
  if (!dev_int_ws) return set_error(ASPIRE_ERR_INVALID, "aspire_plan: null device workspace");
  if (num_ctas <= 0) {
    int rc = current_sm_count(&num_ctas);
    if (rc) return rc;
  }
  int rc = plan_impl(qo_indptr, kv_indptr, kv_len, batch_size, num_qo_heads, num_kv_heads, head_dim,
                     page_size, causal, num_ctas, tc_kernel_available() && tc_env_enabled(), tc_min_rows(),
                     tc_min_kv(), host_buf, host_buf_bytes, float_ws_bytes, info);
  if (rc) return rc;
  if (size_t(info->int_bytes) + kStatusBytes > dev_int_ws_bytes)
    return set_error(ASPIRE_ERR_CAPACITY, "aspire_plan: plan needs " +
                                              std::to_string(info->int_bytes + kStatusBytes) +
                                              " bytes of device int workspace, have " +
                                              std::to_string(dev_int_ws_bytes));
  return check_cuda(cudaMemcpyAsync(static_cast<char*>(dev_int_ws) + kStatusBytes, host_buf,
                                    size_t(info->int_bytes), cudaMemcpyHostToDevice,
                                    static_cast<cudaStream_t>(stream)),
                    "aspire_plan: cudaMemcpyAsync(plan upload)");
}

int aspire_mixed_attention(const AspireAttnArgs* a, const AspirePlanInfo* plan, void* stream) {
  clear_error();
  int rc = check_attention_args(a, plan, "aspire_mixed_attention");
  if (rc) return rc;
  if (!a->int_ws) return set_error(ASPIRE_ERR_INVALID, "aspire_mixed_attention: null int workspace");
  if (size_t(plan->int_bytes) + kStatusBytes > a->int_ws_bytes)
    return set_error(ASPIRE_ERR_CAPACITY, "aspire_mixed_attention: int workspace smaller than plan");
  if (size_t(plan->float_bytes) > a->float_ws_bytes)
    return set_error(ASPIRE_ERR_CAPACITY, "aspire_mixed_attention: float workspace smaller than plan");
  if (plan->num_merge > 0 && !a->float_ws)
    return set_error(ASPIRE_ERR_INVALID, "aspire_mixed_attention: split-KV needs a float workspace");
  const int group = a->num_qo_heads / a->num_kv_heads;
  // The tcgen05 kernel takes rows only when a whole query position fits its tile.
  const bool run_tc = plan->tc_enabled && group <= kTcQTile;

  AttnParams p;
  p.q = static_cast<const __nv_bfloat16*>(a->q);
  p.q_stride_n = a->q_stride_n;
  p.q_stride_h = a->q_stride_h;
  p.kv = static_cast<const __nv_bfloat16*>(a->kv_cache);
  p.num_pages_total = a->num_pages_total;
  p.kv_indices = a->kv_indices;
  p.mode_flags = a->mode_flags;
  p.draft_table = a->draft_table;
  p.draft_stride = a->draft_stride;
  p.block_table = a->block_table;
  p.block_table_stride = a->block_table_stride;
  p.out = static_cast<__nv_bfloat16*>(a->out);
  p.o_stride_n = a->o_stride_n;
  p.o_stride_h = a->o_stride_h;
  p.lse = a->lse;
  p.dump = a->dump;
  p.dump_num_heads = a->dump_num_heads;
  p.dump_kv_stride = a->dump_kv_stride;
  p.dump_kind = a->dump_kind;
  p.dump_f32 = a->dump_dtype == ASPIRE_DUMP_F32 ? 1 : 0;
  p.dump_flags = a->dump_flags;
  p.k_new = static_cast<const __nv_bfloat16*>(a->k_new);
  p.v_new = static_cast<const __nv_bfloat16*>(a->v_new);
  p.k_new_stride_n = a->k_new_stride_n;
  p.k_new_stride_h = a->k_new_stride_h;
  p.v_new_stride_n = a->v_new_stride_n;
  p.v_new_stride_h = a->v_new_stride_h;
  const float sm_scale = a->sm_scale > 0.f ? a->sm_scale : 1.0f / std::sqrt(float(kHeadDim));
  p.scale_log2 = sm_scale * 1.44269504088896340736f;
  p.num_qo_heads = a->num_qo_heads;
  p.num_kv_heads = a->num_kv_heads;
  p.group = group;
  p.q_box_tokens = static_cast<int32_t>(std::min<int64_t>(kTcQTile / group, a->q_rows));
  p.pf_box_tokens = static_cast<int32_t>(std::min<int64_t>(kPfQTile / group, a->q_rows));
  p.q_rows = a->q_rows;
  p.plan = reinterpret_cast<const int32_t*>(static_cast<const char*>(a->int_ws) + kStatusBytes);
  p.status = static_cast<uint32_t*>(a->int_ws);
  p.partial_o = static_cast<float*>(a->float_ws);
  const uint64_t wait_ns = g_wait_limit_ns.load(std::memory_order_relaxed);
  p.wait_ns = wait_ns ? wait_ns : kDefaultWaitNs;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Kernels are launched with plan-independent grids: items live in device
  // memory, so a captured graph stays valid across re-plans.  The CUDA-core
  // kernel is left out only when the routing thresholds send every row to
  // the tcgen05 kernel (no plan can then hold a CUDA-core item); the
  // thresholds are read from the environment once per process.
  static const bool all_rows_tc = tc_min_rows() <= 1;
  if (!(run_tc && all_rows_tc)) {
    const size_t smem = gather_smem_bytes();
    rc = ensure_smem(reinterpret_cast<const void*>(&aspire_attn_gather_kernel), smem, g_gather_smem);
    if (rc) return rc;
    rc = launch(aspire_attn_gather_kernel, dim3(plan->num_ctas * kGatherCtasPerSm), dim3(128), smem, st,
                "aspire_attn_gather_kernel launch", p);
    if (rc) return rc;
  }
  if (run_tc) {
    const size_t smem = tc_smem_bytes();
    rc = ensure_smem(reinterpret_cast<const void*>(&aspire_attn_tc_kernel), smem, g_tc_smem);
    if (rc) return rc;
    alignas(64) CUtensorMap tmap;
    rc = encode_kv_tensor_map(&tmap, a->kv_cache, a->num_pages_total, a->num_kv_heads);
    if (rc) return rc;
    alignas(64) CUtensorMap qmap;
    rc = encode_q_tensor_map(&qmap, a->q, a->q_rows, a->num_qo_heads, a->q_stride_n, a->q_stride_h, group,
                             p.q_box_tokens);
    if (rc) return rc;
    alignas(64) CUtensorMap qmap_pf;
    rc = encode_q_tensor_map(&qmap_pf, a->q, a->q_rows, a->num_qo_heads, a->q_stride_n, a->q_stride_h, group,
                             p.pf_box_tokens);
    if (rc) return rc;
    rc = launch(aspire_attn_tc_kernel, dim3(plan->num_ctas * kTcCtasPerSm), dim3(tc_threads()), smem, st,
                "aspire_attn_tc_kernel launch", p, tmap, qmap, qmap_pf);
    if (rc) return rc;
  }
  // Split-KV merge (exits at once when the current plan split nothing).
  return launch(aspire_attn_merge_kernel, dim3(plan->num_ctas * kMergeCtasPerSm), dim3(kMergeThreads), 0, st,
                "aspire_attn_merge_kernel launch", p);
}

int aspire_append_kv(const AspireAppendArgs* a, void* stream) {
  clear_error();
  if (!a) return set_error(ASPIRE_ERR_INVALID, "aspire_append_kv: null argument");
  if (a->head_dim != kHeadDim || a->page_size != kPageSize)
    return set_error(ASPIRE_ERR_INVALID, "aspire_append_kv: head_dim must be 128 and page_size 16");
  if (a->num_tokens <= 0 || a->num_rows <= 0) return ASPIRE_OK;
  if (!a->page_indices && (!a->mode_flags || !a->draft_table || !a->block_table))
    return set_error(ASPIRE_ERR_INVALID, "aspire_append_kv: page_indices or the three page tables are required");
  if (!a->k || !a->v || !a->kv_cache || !a->append_indptr || !a->page_indptr ||
      !a->last_page_len)
    return set_error(ASPIRE_ERR_INVALID, "aspire_append_kv: null pointer");
  if (((a->k_stride_n | a->k_stride_h | a->v_stride_n | a->v_stride_h) & 7) ||
      ((reinterpret_cast<uintptr_t>(a->k) | reinterpret_cast<uintptr_t>(a->v) |
        reinterpret_cast<uintptr_t>(a->kv_cache)) &
       15))
    return set_error(ASPIRE_ERR_INVALID,
                     "aspire_append_kv: k/v/kv_cache must be 16-byte aligned with 8-element strides");
  AppendParams p;
  p.k = static_cast<const __nv_bfloat16*>(a->k);
  p.v = static_cast<const __nv_bfloat16*>(a->v);
  p.k_stride_n = a->k_stride_n;
  p.k_stride_h = a->k_stride_h;
  p.v_stride_n = a->v_stride_n;
  p.v_stride_h = a->v_stride_h;
  p.num_tokens = a->num_tokens;
  p.append_indptr = a->append_indptr;
  p.kv = static_cast<__nv_bfloat16*>(a->kv_cache);
  p.num_pages_total = a->num_pages_total;
  p.page_indices = a->page_indices;
  p.mode_flags = a->mode_flags;
  p.draft_table = a->draft_table;
  p.draft_stride = a->draft_stride;
  p.block_table = a->block_table;
  p.block_table_stride = a->block_table_stride;
  p.page_indptr = a->page_indptr;
  p.last_page_len = a->last_page_len;
  p.num_rows = a->num_rows;
  p.num_kv_heads = a->num_kv_heads;
  p.status = a->status;
  // One CTA column per row; enough CTAs per row that each warp moves a few
  // (token, head) pairs when the rows hold a long append (prefill chunks).
  const int64_t pairs_per_row = (a->num_tokens * a->num_kv_heads + a->num_rows - 1) / a->num_rows;
  const unsigned ny = static_cast<unsigned>(std::min<int64_t>(std::max<int64_t>((pairs_per_row + 31) / 32, 1), 64));
  return launch(aspire_append_kv_kernel, dim3(static_cast<unsigned>(a->num_rows), ny), dim3(256), 0,
                static_cast<cudaStream_t>(stream), "aspire_append_kv_kernel launch", p);
}

int aspire_qkv_prologue(const AspirePrologueArgs* a, void* stream) {
  clear_error();
  if (!a) return set_error(ASPIRE_ERR_INVALID, "aspire_qkv_prologue: null argument");
  if (a->head_dim != kHeadDim || a->page_size != kPageSize)
    return set_error(ASPIRE_ERR_INVALID, "aspire_qkv_prologue: head_dim must be 128 and page_size 16");
  if (a->num_tokens <= 0 || a->num_rows < 0) return ASPIRE_OK;
  if (!a->q || !a->k || !a->v || !a->q_out || !a->kv_cache || !a->append_indptr || !a->page_indptr ||
      !a->last_page_len || (a->num_rows > 0 && !a->rope_offsets))
    return set_error(ASPIRE_ERR_INVALID, "aspire_qkv_prologue: null pointer");
  if (!a->page_indices && (!a->mode_flags || !a->draft_table || !a->block_table))
    return set_error(ASPIRE_ERR_INVALID, "aspire_qkv_prologue: page_indices or the three page tables are required");
  if ((a->q_norm_weight == nullptr) != (a->k_norm_weight == nullptr))
    return set_error(ASPIRE_ERR_INVALID, "aspire_qkv_prologue: give both norm weights or neither");
  if (a->num_qo_heads <= 0 || a->num_kv_heads <= 0)
    return set_error(ASPIRE_ERR_INVALID, "aspire_qkv_prologue: bad head counts");
  if (!(a->rope_theta > 0.f) || !(a->rope_scale > 0.f))
    return set_error(ASPIRE_ERR_INVALID, "aspire_qkv_prologue: rope_theta and rope_scale must be > 0");
  const uintptr_t ptrs = reinterpret_cast<uintptr_t>(a->q) | reinterpret_cast<uintptr_t>(a->k) |
                         reinterpret_cast<uintptr_t>(a->v) | reinterpret_cast<uintptr_t>(a->q_out) |
                         reinterpret_cast<uintptr_t>(a->kv_cache);
  const int64_t strides = a->q_stride_n | a->q_stride_h | a->k_stride_n | a->k_stride_h | a->v_stride_n |
                          a->v_stride_h | a->qo_stride_n | a->qo_stride_h;
  if ((ptrs & 15) || (strides & 7))
    return set_error(ASPIRE_ERR_INVALID,
                     "aspire_qkv_prologue: tensors must be 16-byte aligned with strides in multiples of 8");
  PrologueParams p;
  AppendParams& ap = p.ap;
  ap.k = static_cast<const __nv_bfloat16*>(a->k);
  ap.v = static_cast<const __nv_bfloat16*>(a->v);
  ap.k_stride_n = a->k_stride_n;
  ap.k_stride_h = a->k_stride_h;
  ap.v_stride_n = a->v_stride_n;
  ap.v_stride_h = a->v_stride_h;
  ap.num_tokens = a->num_tokens;
  ap.append_indptr = a->append_indptr;
  ap.kv = static_cast<__nv_bfloat16*>(a->kv_cache);
  ap.num_pages_total = a->num_pages_total;
  ap.page_indices = a->page_indices;
  ap.mode_flags = a->mode_flags;
  ap.draft_table = a->draft_table;
  ap.draft_stride = a->draft_stride;
  ap.block_table = a->block_table;
  ap.block_table_stride = a->block_table_stride;
  ap.page_indptr = a->page_indptr;
  ap.last_page_len = a->last_page_len;
  ap.num_rows = a->num_rows;
  ap.num_kv_heads = a->num_kv_heads;
  ap.status = a->status;
  p.q = static_cast<const __nv_bfloat16*>(a->q);
  p.q_stride_n = a->q_stride_n;
  p.q_stride_h = a->q_stride_h;
  p.q_out = static_cast<__nv_bfloat16*>(a->q_out);
  p.qo_stride_n = a->qo_stride_n;
  p.qo_stride_h = a->qo_stride_h;
  p.q_norm_w = static_cast<const __nv_bfloat16*>(a->q_norm_weight);
  p.k_norm_w = static_cast<const __nv_bfloat16*>(a->k_norm_weight);
  p.eps = a->norm_eps;
  p.rope_offsets = a->rope_offsets;
  // The constants FlashInfer derives on the host: reciprocals in fp32, the
  // Llama-3.1 smoothing line from double-precision pi.
  p.rcp_theta = 1.0f / a->rope_theta;
  p.rcp_scale = 1.0f / a->rope_scale;
  p.smooth_a = 0.f;
  p.smooth_b = 0.f;
  if (a->low_freq_factor > 0.f && a->high_freq_factor > a->low_freq_factor) {
    const double pi = 3.14159265358979323846;
    p.smooth_a = static_cast<float>(a->old_context_len /
                                    (2 * pi * a->high_freq_factor - 2 * pi * a->low_freq_factor));
    p.smooth_b = -1.0f / (a->high_freq_factor / a->low_freq_factor - 1.0f);
  }
  p.num_qo_heads = a->num_qo_heads;
  const int64_t units_per_row = (a->num_tokens * (a->num_qo_heads + 2 * a->num_kv_heads) + a->num_rows) /
                                std::max<int64_t>(a->num_rows, 1);
  const unsigned ny = static_cast<unsigned>(std::min<int64_t>(std::max<int64_t>((units_per_row + 31) / 32, 1), 64));
  return launch(aspire_qkv_prologue_kernel, dim3(static_cast<unsigned>(a->num_rows + 1), ny), dim3(256), 0,
                static_cast<cudaStream_t>(stream), "aspire_qkv_prologue_kernel launch", p);
}

int aspire_build_unified_indices(const AspireIndicesArgs* a, void* stream) {
  clear_error();
  if (!a) return set_error(ASPIRE_ERR_INVALID, "aspire_build_unified_indices: null argument");
  if (a->batch < 0) return set_error(ASPIRE_ERR_INVALID, "aspire_build_unified_indices: negative batch");
  if (a->batch == 0) {  // the reference still writes indptr[0] = 0
    if (!a->indptr_out) return set_error(ASPIRE_ERR_INVALID, "aspire_build_unified_indices: null indptr");
    return check_cuda(cudaMemsetAsync(a->indptr_out, 0, sizeof(int32_t), static_cast<cudaStream_t>(stream)),
                      "aspire_build_unified_indices memset");
  }
  if (!a->mode_flags || !a->draft_indices || !a->verify_indices || !a->draft_num_pages ||
      !a->verify_num_pages || !a->indices_out || !a->indptr_out)
    return set_error(ASPIRE_ERR_INVALID, "aspire_build_unified_indices: null pointer");
  if (a->draft_cols < 0 || a->verify_cols < 0 || a->draft_stride < a->draft_cols ||
      a->verify_stride < a->verify_cols)
    return set_error(ASPIRE_ERR_INVALID, "aspire_build_unified_indices: bad table geometry");
  if (a->indices_capacity < 0)
    return set_error(ASPIRE_ERR_INVALID, "aspire_build_unified_indices: negative indices_capacity");
  IndicesParams p;
  p.mode_flags = a->mode_flags;
  p.draft_indices = a->draft_indices;
  p.draft_stride = a->draft_stride;
  p.draft_cols = a->draft_cols;
  p.verify_indices = a->verify_indices;
  p.verify_stride = a->verify_stride;
  p.verify_cols = a->verify_cols;
  p.draft_num_pages = a->draft_num_pages;
  p.verify_num_pages = a->verify_num_pages;
  p.indices_out = a->indices_out;
  p.indptr_out = a->indptr_out;
  p.status = a->status;
  p.indices_capacity = a->indices_capacity;
  return launch(aspire_build_indices_kernel, dim3(a->batch), dim3(kIndicesThreads), 0,
                static_cast<cudaStream_t>(stream), "aspire_build_indices_kernel launch", p);
}

int aspire_select_pages(const AspireSelectArgs* a, void* stream) {
  clear_error();
  if (!a) return set_error(ASPIRE_ERR_INVALID, "aspire_select_pages: null argument");
  if (a->batch <= 0) return ASPIRE_OK;
  if (a->page_size != kPageSize)
    return set_error(ASPIRE_ERR_INVALID, "aspire_select_pages: page_size must be 16");
  if (!a->num_pages || !a->block_table || !a->table_out || !a->counts_out)
    return set_error(ASPIRE_ERR_INVALID, "aspire_select_pages: null pointer");
  if (!a->scores_in && (!a->dump || !a->lse || !a->qo_indptr))
    return set_error(ASPIRE_ERR_INVALID,
                     "aspire_select_pages: dump, lse and qo_indptr are required without scores_in");
  if (a->block_table_cols <= 0 || a->block_table_stride < a->block_table_cols)
    return set_error(ASPIRE_ERR_INVALID, "aspire_select_pages: bad block_table geometry");
  if (a->num_heads <= 0 || a->num_heads > kMaxSelHeads)
    return set_error(ASPIRE_ERR_INVALID, "aspire_select_pages: num_heads must be in [1, 128]");
  if (a->pages_per_slot <= 0 || a->subset_cache_size <= 0 || a->L < 0)
    return set_error(ASPIRE_ERR_INVALID, "aspire_select_pages: bad pages_per_slot / k / L");
  if (a->subset_cache_size > a->pages_per_slot)
    return set_error(ASPIRE_ERR_INVALID,
                     "aspire_select_pages: subset_cache_size exceeds pages_per_slot (topk would fail)");
  if (!a->scores_in && a->max_seq_len > a->kv_stride)
    return set_error(ASPIRE_ERR_INVALID, "aspire_select_pages: max_seq_len exceeds kv_stride");
  if (!a->scores_in && int64_t(a->pages_per_slot) * kPageSize < a->max_seq_len)
    return set_error(ASPIRE_ERR_INVALID, "aspire_select_pages: pages_per_slot*16 < max_seq_len");
  if (a->dump_kind != ASPIRE_DUMP_FIRST_LAST && a->dump_kind != ASPIRE_DUMP_LAST_TOKEN)
    return set_error(ASPIRE_ERR_INVALID, "aspire_select_pages: bad dump_kind");
  if (a->dump_dtype != ASPIRE_DUMP_F16 && a->dump_dtype != ASPIRE_DUMP_F32)
    return set_error(ASPIRE_ERR_INVALID, "aspire_select_pages: bad dump_dtype");
  if (a->dump && (reinterpret_cast<uintptr_t>(a->dump) & (a->dump_dtype == ASPIRE_DUMP_F32 ? 3 : 1)))
    return set_error(ASPIRE_ERR_INVALID, "aspire_select_pages: dump buffer not aligned to its element type");
  SelectParams p;
  p.dump = a->dump;
  p.dump_slots = a->dump_kind == ASPIRE_DUMP_LAST_TOKEN ? 1 : 2;
  p.dump_f32 = a->dump_dtype == ASPIRE_DUMP_F32 ? 1 : 0;
  p.kv_stride = a->kv_stride;
  p.max_seq_len = a->max_seq_len;
  p.lse = a->lse;
  p.lse_rows = a->lse_rows;
  p.qo_indptr = a->qo_indptr;
  p.row_ids = a->row_ids;
  p.scores_in = a->scores_in;
  p.num_pages = a->num_pages;
  p.block_table = a->block_table;
  p.block_table_stride = a->block_table_stride;
  p.block_table_cols = a->block_table_cols;
  p.num_heads = a->num_heads;
  p.pages_per_slot = a->pages_per_slot;
  p.L = a->L;
  p.subset_cache_size = a->subset_cache_size;
  p.min_draft_pages = a->min_draft_pages;
  p.draft_percent = a->draft_percent;
  const int hd = a->head_dim > 0 ? a->head_dim : kHeadDim;
  const double sm = a->sm_scale > 0.f ? double(a->sm_scale) : 1.0 / std::sqrt(double(hd));
  // PageSelector keeps sm_scale * log2(e) as a Python float (double); the
  // fp16 tensor multiply then uses it as an fp32 scalar.
  p.scale_log2 = static_cast<float>(sm * 1.4426950408889634);
  p.table_out = a->table_out;
  p.table_stride = a->table_stride;
  p.table_width = a->table_width;
  p.counts_out = a->counts_out;
  p.scores_out = a->scores_out;
  p.status = a->status;
  p.order_by_page = a->order_by_page ? 1 : 0;
  if (p.order_by_page && !a->scores_in)
    return set_error(ASPIRE_ERR_INVALID, "aspire_select_pages: order_by_page needs scores_in");
  int cap = 1;
  while (cap < std::min(a->pages_per_slot, a->subset_cache_size)) cap <<= 1;
  p.sort_cap = cap;
  const size_t smem = select_smem_bytes(a->pages_per_slot, cap);
  if (smem > 200 * 1024)
    return set_error(ASPIRE_ERR_CAPACITY, "aspire_select_pages: pages_per_slot too large");
  int rc = ensure_smem(reinterpret_cast<const void*>(&aspire_select_pages_kernel), smem, g_sel_smem);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!a->scores_in) {
    // Scoring on its own wide grid into scores_out (or the scratch), then the
    // per-row selection reads it back.
    float* ws = a->scores_out ? a->scores_out : a->scores_ws;
    if (!ws)
      return set_error(ASPIRE_ERR_INVALID, "aspire_select_pages: scores_ws is required without scores_out");
    p.scores_out = ws;
    const unsigned splits = static_cast<unsigned>((a->pages_per_slot + kScoreThreads - 1) / kScoreThreads);
    rc = launch(aspire_page_scores_kernel, dim3(static_cast<unsigned>(a->batch), splits), dim3(kScoreThreads), 0, st,
                "aspire_page_scores_kernel launch", p);
    if (rc) return rc;
    p.scores_in = ws;
    p.scores_out = nullptr;
  }
  return launch(aspire_select_pages_kernel, dim3(a->batch), dim3(kSelThreads), smem, st,
                "aspire_select_pages_kernel launch", p);
}

}  // extern "C"
