// Thread-local error reporting of the C ABI.
#pragma once

#include <string>

#include "aspire_b200.h"

namespace aspire {

// Records `msg` as the calling thread's last error and returns `code`.
int set_error(int code, const std::string& msg);

// Clears the calling thread's last error.
void clear_error();

const char* last_error();

// Returns ASPIRE_OK, or records the CUDA error of `what` and returns
// ASPIRE_ERR_CUDA.
int check_cuda(int cuda_status, const char* what);

// Argument checks of aspire_mixed_attention that do not involve the
// workspaces (shapes, alignment, pointers, dump geometry, q_rows).  `who`
// names the entry point in the message.  Returns ASPIRE_OK or an error code
// (with the message recorded).
int check_attention_args(const AspireAttnArgs* a, const AspirePlanInfo* plan, const char* who);

}  // namespace aspire
