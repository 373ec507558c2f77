// tp_exchange.cu — data movement of the tensor-parallel decode step that is not a
// collective between processes: the exchanges of the one-GPU emulation of a G-rank split
// (all ranks' buffers on this GPU, summed in rank order like the peer-memory all-reduce,
// so the emulated step has the bits of the peer-memory one) and the reorder after an NCCL
// all-gather of row-split logits; and the end of a step's fused exchanges (the last
// site's sum, the epoch advance). Plain grid-stride kernels; the sizes are small (3072
// floats per all-reduce, one row of logits per token).
#include <cuda_runtime.h>

#include <algorithm>

#include "internal.h"
#include "rrr_common.cuh"

namespace rrr {
namespace {

struct Ptrs {
  float* p[kMaxTpRanks];
};
struct CPtrs {
  const float* p[kMaxTpRanks];
};

__global__ void local_allreduce_kernel(Ptrs bufs, int G, int64_t n) {
  pdl_launch_dependents();
  pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float acc = bufs.p[0][i];
    for (int r = 1; r < G; ++r) acc += bufs.p[r][i];
    for (int r = 0; r < G; ++r) bufs.p[r][i] = acc;
  }
}

__global__ void local_allgather_rows_kernel(CPtrs parts, Ptrs outs, int G, int rows, int64_t npr) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t n = (int64_t)rows * G * npr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / (G * npr), rem = i % (G * npr);
    const int src = (int)(rem / npr);
    const float v = parts.p[src][row * npr + rem % npr];
    for (int r = 0; r < G; ++r) outs.p[r][i] = v;
  }
}

__global__ void rows_from_ranks_kernel(const float* tmp, float* out, int G, int rows, int64_t npr) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t n = (int64_t)rows * G * npr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / (G * npr), rem = i % (G * npr);
    const int64_t g = rem / npr;
    out[i] = tmp[(g * rows + row) * npr + rem % npr];
  }
}

// out[i] = sum over ranks in rank order of the tagged words slots[r*n + i] of epoch
// *epoch + 1 (the order and the bits of the exchange kernel's all-reduce).
__global__ void fused_sum_kernel(const unsigned long long* slots, float* out, int n, int G,
                                 const unsigned* epoch, int* err) {
  pdl_launch_dependents();
  pdl_wait();
  const unsigned e = *epoch + 1u;
  bool ok = true;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const unsigned long long* p = slots + i;
    float acc = __uint_as_float((unsigned)wait_tagged(p, ld_relaxed_sys_u64(p), e, ok, err));
    for (int r = 1; r < G; ++r) {
      p += n;
      acc += __uint_as_float((unsigned)wait_tagged(p, ld_relaxed_sys_u64(p), e, ok, err));
    }
    out[i] = acc;
  }
}

__global__ void epoch_advance_kernel(unsigned* epoch) {
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x == 0) *epoch += 1u;
}

int grid_for(int64_t n, int sms) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)sms * 8));
}

}  // namespace

cudaError_t launch_local_allreduce(const LaunchEnv& env, float* const* bufs, int G, int64_t n) {
  if (G < 1 || G > kMaxTpRanks || n < 1) return cudaErrorInvalidValue;
  Ptrs b{};
  for (int r = 0; r < G; ++r) b.p[r] = bufs[r];
  return rrr_launch_pdl(local_allreduce_kernel, dim3(grid_for(n, env.sm_count)), dim3(256), 0,
                        env.stream, env.pdl, b, G, n);
}

cudaError_t launch_local_allgather_rows(const LaunchEnv& env, const float* const* parts,
                                        float* const* outs, int G, int rows, int64_t npr) {
  if (G < 1 || G > kMaxTpRanks || rows < 1 || npr < 1) return cudaErrorInvalidValue;
  CPtrs a{};
  Ptrs b{};
  for (int r = 0; r < G; ++r) {
    a.p[r] = parts[r];
    b.p[r] = outs[r];
  }
  return rrr_launch_pdl(local_allgather_rows_kernel,
                        dim3(grid_for((int64_t)rows * G * npr, env.sm_count)), dim3(256), 0,
                        env.stream, env.pdl, a, b, G, rows, npr);
}

cudaError_t launch_fused_sum(const LaunchEnv& env, const unsigned long long* slots, float* out,
                             int n, int G, const unsigned* epoch) {
  if (G < 1 || G > kMaxTpRanks || n < 1) return cudaErrorInvalidValue;
  return rrr_launch_pdl(fused_sum_kernel, dim3((n + 255) / 256), dim3(256), 0, env.stream, env.pdl,
                        slots, out, n, G, epoch, env.d_err);
}

cudaError_t launch_epoch_advance(const LaunchEnv& env, unsigned* epoch) {
  return rrr_launch_pdl(epoch_advance_kernel, dim3(1), dim3(32), 0, env.stream, env.pdl, epoch);
}

cudaError_t launch_rows_from_ranks(const LaunchEnv& env, const float* tmp, float* out, int G,
                                   int rows, int64_t npr) {
  if (G < 1 || rows < 1 || npr < 1) return cudaErrorInvalidValue;
  return rrr_launch_pdl(rows_from_ranks_kernel, dim3(grid_for((int64_t)rows * G * npr, env.sm_count)),
                        dim3(256), 0, env.stream, env.pdl, tmp, out, G, rows, npr);
}

}  // namespace rrr
