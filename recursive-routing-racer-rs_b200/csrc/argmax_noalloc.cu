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
#include <cuda.h>
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

// Device address of the scratch array (the name of a __device__ variable is not a device
// address in host code), looked up once per CUDA context and cached with that context's
// unique id. A context that is destroyed and created again (cudaDeviceReset, a host that
// swaps contexts) gets a new id, so a stale address from a previous module load is never
// used. The two driver queries come from cudaGetDriverEntryPoint, so the library does not
// link libcuda.
std::mutex g_setup_mutex;
struct ScratchSlot {
  unsigned long long ctx_id;
  unsigned long long* addr;
};
ScratchSlot g_slots[64] = {};
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;

// Id of the calling thread's current context (the runtime makes the device's primary
// context current first if none is). Returns false if the driver entry points are missing.
bool current_context_id(unsigned long long* id) {
  if (!g_ctx_get_current || !g_ctx_get_id) {
    void* f1 = nullptr;
    void* f2 = nullptr;
    cudaDriverEntryPointQueryResult q1 = cudaDriverEntryPointSymbolNotFound, q2 = q1;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f1, cudaEnableDefault, &q1) != cudaSuccess ||
        cudaGetDriverEntryPoint("cuCtxGetId", &f2, cudaEnableDefault, &q2) != cudaSuccess ||
        q1 != cudaDriverEntryPointSuccess || q2 != cudaDriverEntryPointSuccess || !f1 || !f2)
      return false;
    g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(f1);
    g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(f2);
  }
  CUcontext c = nullptr;
  if (g_ctx_get_current(&c) != CUDA_SUCCESS || !c) return false;
  return g_ctx_get_id(c, id) == CUDA_SUCCESS;
}

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
    // cudaGetDevice above made the device's primary context current if none was
    unsigned long long id = 0;
    if (!current_context_id(&id))
      return set_error(nullptr, RRR_ERR_CUDA, "rrr_argmax_f32_noalloc: no current CUDA context");
    ScratchSlot& slot = g_slots[dev];
    if (!slot.addr || slot.ctx_id != id) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_argmax_noalloc_scratch);
      if (e != cudaSuccess || !p)
        return set_error(nullptr, RRR_ERR_CUDA,
                         "rrr_argmax_f32_noalloc: cudaGetSymbolAddress: %s",
                         cudaGetErrorString(e));
      slot.addr = static_cast<unsigned long long*>(p);
      slot.ctx_id = id;
    }
    scratch = slot.addr;
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
