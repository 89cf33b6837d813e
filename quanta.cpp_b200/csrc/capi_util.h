// Error reporting shared by the C ABI translation units (the message qnt_last_error returns, per thread).
#pragma once

#include <cuda_runtime.h>

#include <string>

namespace qnt_capi {

extern thread_local std::string g_err;
int set_err(int code, const std::string& message);                // stores the message, returns code
int cuda_err(cudaError_t e, const char* what);                     // QNT_ERR_CUDA with the runtime's message

}  // namespace qnt_capi
