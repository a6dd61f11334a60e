// Internal helpers shared by the C ABI translation units (q3s_capi.cpp owns
// the context and the per-thread error text).  Not installed.
#pragma once

#include <cstddef>
#include <string>

#include <cuda_runtime.h>

#include "../../include/q3s_sampler.h"

namespace q3s {

struct ContextInfo {
  int device;
  int sm_count;
  size_t smem_optin;
};

ContextInfo context_info(const q3s_context* ctx);

// Records `msg` as the calling thread's q3s_last_error() and returns `code`.
int record_error(int code, const std::string& msg);

// Records a CUDA failure of `what` and returns Q3S_E_CUDA (Q3S_E_OUT_OF_MEMORY
// for an allocation failure).
int record_cuda_error(cudaError_t e, const char* what);

}  // namespace q3s
