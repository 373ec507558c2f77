// gemm_kq_tc.cu — kernel (2): batched-token K-quant GEMM on the tcgen05 tensor cores.
#include "internal.h"

namespace rrr {

cudaError_t launch_gemm_kq_tc(const LaunchEnv&, int, const void*, const uint16_t*, float*, int,
                              int, int) {
  return cudaErrorNotSupported;
}

}  // namespace rrr
