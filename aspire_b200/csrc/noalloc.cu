// Mixed attention without any device allocation by the caller or the library.
//
// Some callers of this library cannot obtain device memory for the
// attention's workspaces: a plug-in loaded into a host application that owns
// all GPU memory (and forbids cudaMalloc after start-up), or a serving loop
// whose memory budget is fixed when it starts and where a cudaMalloc would
// also synchronise the device in the middle of a step.  For them this file
// keeps the two workspaces in file-scope device arrays: the plan / status
// array (kNoAllocIntBytes) and the split-KV partials array
// (kNoAllocFloatBytes).  Every GPU that loads the library holds both arrays
// until the process exits.
//
// Host code may not pass the arrays' names to a kernel (in host code they are
// host-side stand-ins, not device addresses): the first call on each device
// looks up their device addresses with cudaGetSymbolAddress, with that device
// current, and caches them.  Make that first call before any stream capture.
//
// All calls share the arrays and the arrays keep the last call's contents.
// The status word is cleared on every call (aspire_noalloc_status reads it
// back); the plan and the partials are always written before they are read.  Calls that overlap on the GPU (two
// streams, two host threads) race on the arrays: serialise them.
#include <cstring>
#include <mutex>
#include <string>

#include "kernels.cuh"
#include "errors.h"

namespace aspire {
namespace {

constexpr size_t kNoAllocIntBytes = ASPIRE_NOALLOC_INT_BYTES;
constexpr size_t kNoAllocFloatBytes = ASPIRE_NOALLOC_FLOAT_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_int[kNoAllocIntBytes];
static __device__ __align__(256) unsigned char g_noalloc_float[kNoAllocFloatBytes];

struct DeviceScratch {
  void* int_ws = nullptr;
  void* float_ws = nullptr;
};
DeviceScratch g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

// Device addresses of the two arrays on the current device (looked up once).
int scratch_for_current_device(DeviceScratch* out) {
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "aspire_mixed_attention_noalloc: cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(ASPIRE_ERR_INVALID, "aspire_mixed_attention_noalloc: device index out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  DeviceScratch& s = g_scratch[dev];
  if (s.int_ws == nullptr || s.float_ws == nullptr) {
    void* ip = nullptr;
    void* fp = nullptr;
    rc = check_cuda(cudaGetSymbolAddress(&ip, g_noalloc_int),
                    "aspire_mixed_attention_noalloc: cudaGetSymbolAddress(plan scratch)");
    if (rc) return rc;
    rc = check_cuda(cudaGetSymbolAddress(&fp, g_noalloc_float),
                    "aspire_mixed_attention_noalloc: cudaGetSymbolAddress(partials scratch)");
    if (rc) return rc;
    s.int_ws = ip;
    s.float_ws = fp;
  }
  *out = s;
  return ASPIRE_OK;
}

}  // namespace
}  // namespace aspire

using namespace aspire;

extern "C" int aspire_mixed_attention_noalloc(const AspireAttnArgs* args, const AspirePlanInfo* plan,
                                              const void* host_plan, void* stream) {
  clear_error();
  if (!args || !plan || !host_plan)
    return set_error(ASPIRE_ERR_INVALID, "aspire_mixed_attention_noalloc: null argument");
  if (plan->on_device)
    return set_error(ASPIRE_ERR_INVALID,
                     "aspire_mixed_attention_noalloc: the plan must be rendered on the host with "
                     "aspire_plan_host_only (an aspire_plan_device plan has no host copy to upload)");
  // Every argument is checked before the shared arrays are touched, so a
  // rejected call leaves the previous call's plan and status in place.
  int rc = check_attention_args(args, plan, "aspire_mixed_attention_noalloc");
  if (rc) return rc;
  if (plan->int_bytes <= 0 || size_t(plan->int_bytes) + kStatusBytes > kNoAllocIntBytes)
    return set_error(ASPIRE_ERR_CAPACITY,
                     "aspire_mixed_attention_noalloc: the plan needs " +
                         std::to_string(plan->int_bytes + kStatusBytes) +
                         " bytes, the built-in plan scratch holds " + std::to_string(kNoAllocIntBytes));
  if (plan->float_bytes < 0 || size_t(plan->float_bytes) > kNoAllocFloatBytes)
    return set_error(ASPIRE_ERR_CAPACITY,
                     "aspire_mixed_attention_noalloc: split-KV partials need " +
                         std::to_string(plan->float_bytes) + " bytes, the built-in scratch holds " +
                         std::to_string(kNoAllocFloatBytes) + " (fewer, longer chunks: a smaller batch)");
  DeviceScratch s;
  rc = scratch_for_current_device(&s);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The status word must start at zero; the plan follows the control block.
  rc = check_cuda(cudaMemsetAsync(s.int_ws, 0, kStatusBytes, st),
                  "aspire_mixed_attention_noalloc: clearing the status word");
  if (rc) return rc;
  rc = check_cuda(cudaMemcpyAsync(static_cast<char*>(s.int_ws) + kStatusBytes, host_plan,
                                  size_t(plan->int_bytes), cudaMemcpyHostToDevice, st),
                  "aspire_mixed_attention_noalloc: plan upload");
  if (rc) return rc;
  AspireAttnArgs a = *args;
  a.int_ws = s.int_ws;
  a.int_ws_bytes = kNoAllocIntBytes;
  a.float_ws = s.float_ws;
  a.float_ws_bytes = kNoAllocFloatBytes;
  return aspire_mixed_attention(&a, plan, stream);
}

extern "C" int aspire_noalloc_status(uint32_t* host_out, int32_t clear, void* stream) {
  clear_error();
  if (!host_out) return set_error(ASPIRE_ERR_INVALID, "aspire_noalloc_status: null host_out");
  DeviceScratch s;
  int rc = scratch_for_current_device(&s);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = check_cuda(cudaMemcpyAsync(host_out, s.int_ws, sizeof(uint32_t), cudaMemcpyDeviceToHost, st),
                  "aspire_noalloc_status: status copy");
  if (rc || !clear) return rc;
  return check_cuda(cudaMemsetAsync(s.int_ws, 0, sizeof(uint32_t), st), "aspire_noalloc_status: clearing");
}
