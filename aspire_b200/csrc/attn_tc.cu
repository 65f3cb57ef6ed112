// tcgen05 paged-attention kernel for wide packed-query tiles (verify rows).
#include "kernels.cuh"

namespace aspire {

__global__ void aspire_attn_tc_kernel(AttnParams p) { (void)p; }

size_t tc_smem_bytes() { return 0; }

bool tc_kernel_available() { return false; }

}  // namespace aspire
