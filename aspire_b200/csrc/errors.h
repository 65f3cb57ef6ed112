// Thread-local error reporting of the C ABI.
#pragma once

#include <string>

namespace aspire {

// Records `msg` as the calling thread's last error and returns `code`.
int set_error(int code, const std::string& msg);

// Clears the calling thread's last error.
void clear_error();

const char* last_error();

// Returns ASPIRE_OK, or records the CUDA error of `what` and returns
// ASPIRE_ERR_CUDA.
int check_cuda(int cuda_status, const char* what);

}  // namespace aspire
