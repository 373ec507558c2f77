// tp_exchange.cu — data movement of the tensor-parallel decode step that is not a
// collective between processes: the exchanges of the one-GPU emulation of a G-rank split
// (all ranks' buffers on this GPU, summed in rank order like the peer-memory all-reduce,
// so the emulated step has the bits of the peer-memory one) and the reorder after an NCCL
// all-gather of row-split logits. Plain grid-stride kernels; the sizes are small (3072
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

cudaError_t launch_rows_from_ranks(const LaunchEnv& env, const float* tmp, float* out, int G,
                                   int rows, int64_t npr) {
  if (G < 1 || rows < 1 || npr < 1) return cudaErrorInvalidValue;
  return rrr_launch_pdl(rows_from_ranks_kernel, dim3(grid_for((int64_t)rows * G * npr, env.sm_count)),
                        dim3(256), 0, env.stream, env.pdl, tmp, out, G, rows, npr);
}

}  // namespace rrr
