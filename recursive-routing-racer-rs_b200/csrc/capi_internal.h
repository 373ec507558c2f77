// capi_internal.h — the context object and error helpers shared by the C-ABI sources.
#pragma once
#include <cuda_runtime.h>

#include <string>

#include "../../include/rrr_cuda.h"
#include "internal.h"

struct rrr_ctx {
  int device = 0;
  int sm_count = 0;
  int* d_err = nullptr;  // device error flag written by kernels whose bounded waits give up
  bool pdl = true;       // launch kernels with programmatic dependent launch
  std::string last_error;
};

namespace rrr {
// Records a message for rrr_last_error and returns `code`.
int set_error(rrr_ctx* ctx, int code, const char* fmt, ...);
int cuda_error(rrr_ctx* ctx, cudaError_t e, const char* what);
int bind_device(rrr_ctx* ctx);
LaunchEnv make_env(rrr_ctx* ctx, void* stream);
}  // namespace rrr
