// argmax_noalloc.cu — greedy argmax over f32 logits for callers that cannot allocate
// device memory.
//
// rrr_argmax_f32 needs a context, and creating a context allocates (rrr_init reserves the
// context's error flag and the argmax's key/counter with cudaMalloc). Some callers cannot
// do that: a host whose device memory is entirely reserved by its own caching allocator
// (cudaMalloc fails or steals memory it accounts for), code that runs while someone else's
// stream capture is open (cudaMalloc is not allowed there), and latency-critical paths
// where the implicit device synchronisation of cudaMalloc / cudaFree is not acceptable.
// rrr_argmax_f32_noalloc takes no context and allocates nothing: its scratch (one 64-bit
// key per CTA plus a finish counter) lives in a file-scope __device__ array of fixed size,
// present on every GPU that loads this library until the process exits.
//
// Result semantics are those of rrr_argmax_f32 (the reference's CPU scan,
// src/model/phi4.rs:1172-1183): the first maximum wins, NaN is never selected, and the
// index is 0 when no element compares greater than -inf.
#include <cuda_runtime.h>

#include <mutex>

#include "capi_internal.h"
#include "rrr_common.cuh"

namespace {

// Elements per CTA (4 per thread of a 1024-thread CTA) and the scratch size: one 64-bit
// key per CTA, so n may be at most kMaxBlocks * kPerBlock = 8,388,608 elements (the
// 200,064-entry vocabulary needs 49 CTAs). The last slot is the finish counter.
constexpr int kPerBlock = 4096;
constexpr int kMaxBlocks = 2048;

static __device__ __align__(256) unsigned long long g_argmax_noalloc_scratch[kMaxBlocks + 1];

__device__ __forceinline__ unsigned long long noalloc_key(float v, int idx) {
  if (v == 0.f) v = 0.f;  // -0 and +0 compare equal in the reference's scan
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (uint32_t)(~(uint32_t)idx);
}

// CTA b reduces x[b*kPerBlock, (b+1)*kPerBlock) to one key in partials[b]; the last CTA
// to finish (counter) reduces the keys in index order, writes the index and sets the
// counter back to zero.
__global__ void __launch_bounds__(1024) argmax_noalloc_kernel(const float* __restrict__ x, int n,
                                                              int* __restrict__ out,
                                                              unsigned long long* partials) {
  __shared__ unsigned long long sh[32];
  __shared__ bool last;
  unsigned int* counter = reinterpret_cast<unsigned int*>(partials + kMaxBlocks);
  unsigned long long best = 0ull;
  const int base = blockIdx.x * kPerBlock;
#pragma unroll
  for (int i = 0; i < kPerBlock / 1024; ++i) {
    const int e = base + i * 1024 + threadIdx.x;
    if (e < n) {
      const float v = x[e];
      if (v == v && v > -INFINITY) {
        const unsigned long long k = noalloc_key(v, e);
        best = k > best ? k : best;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
    best = t > best ? t : best;
  }
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x < 32) {
    best = sh[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
      best = t > best ? t : best;
    }
    if (threadIdx.x == 0) {
      partials[blockIdx.x] = best;
      __threadfence();
      last = atomicAdd(counter, 1u) == gridDim.x - 1;
    }
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  best = 0ull;
  for (int i = threadIdx.x; i < (int)gridDim.x; i += 1024) {
    const unsigned long long k = *reinterpret_cast<volatile unsigned long long*>(partials + i);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
    best = t > best ? t : best;
  }
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    best = 0ull;
    for (int w = 0; w < 32; ++w) best = sh[w] > best ? sh[w] : best;
    *out = best ? (int)(~(uint32_t)(best & 0xFFFFFFFFull)) : 0;
    *counter = 0u;
  }
}

// Device address of the scratch array, looked up once per device (the name of a
// __device__ variable is not a device address in host code).
std::mutex g_setup_mutex;
unsigned long long* g_scratch_addr[64] = {};

}  // namespace

extern "C" int rrr_argmax_f32_noalloc(const float* x, int n, int* out_index, void* stream) {
  using rrr::set_error;
  if (!x || !out_index)
    return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_argmax_f32_noalloc: null pointer");
  if (n < 1 || n > kMaxBlocks * kPerBlock)
    return set_error(nullptr, RRR_ERR_BAD_SHAPE,
                     "rrr_argmax_f32_noalloc: n = %d outside [1, %d] (the fixed scratch holds "
                     "%d per-CTA keys of %d elements)",
                     n, kMaxBlocks * kPerBlock, kMaxBlocks, kPerBlock);
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64)
    return set_error(nullptr, RRR_ERR_CUDA, "rrr_argmax_f32_noalloc: cudaGetDevice: %s",
                     cudaGetErrorString(e));
  unsigned long long* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_addr[dev]) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_argmax_noalloc_scratch);
      if (e != cudaSuccess || !p)
        return set_error(nullptr, RRR_ERR_CUDA,
                         "rrr_argmax_f32_noalloc: cudaGetSymbolAddress: %s",
                         cudaGetErrorString(e));
      g_scratch_addr[dev] = static_cast<unsigned long long*>(p);
    }
    scratch = g_scratch_addr[dev];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the finish counter must start at zero (a call cut short would leave it set)
  e = cudaMemsetAsync(scratch + kMaxBlocks, 0, sizeof(unsigned int), s);
  if (e != cudaSuccess)
    return set_error(nullptr, RRR_ERR_CUDA, "rrr_argmax_f32_noalloc: clear counter: %s",
                     cudaGetErrorString(e));
  const int grid = (n + kPerBlock - 1) / kPerBlock;
  argmax_noalloc_kernel<<<grid, 1024, 0, s>>>(x, n, out_index, scratch);
  e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(nullptr, RRR_ERR_CUDA, "rrr_argmax_f32_noalloc launch: %s",
                     cudaGetErrorString(e));
  return RRR_OK;
}
