// comm_p2p.cu — all-reduce and all-gather of f32 vectors between the GPUs of one box over
// NVLink peer memory, for the tensor-parallel decode step (one process per GPU).
//
// Every rank owns an exchange buffer, mapped into the other ranks' processes through CUDA
// IPC handles: data[2][world][max_elems] f32 and flags[2][world][kMaxCtas] u32. A call
// of `n` elements runs C CTAs; CTA c owns elements [c*chunk, (c+1)*chunk). It
//   1. writes its chunk of this rank's input into slot `rank` of every rank's buffer
//      (peer stores over NVLink; the local one is an ordinary store),
//   2. makes the stores visible system-wide and sets flags[set][rank][c] = epoch on every
//      rank (epoch = this CTA's call counter + 1, set = epoch & 1),
//   3. waits until flags[set][r][c] == epoch for every r in its own buffer (bounded: it
//      gives up after about a second, records an error in the context's device flag and
//      returns), then
//   4. sums the slots in rank order (all-reduce: every rank gets identical bits) or copies
//      them in rank order (all-gather).
// The two buffer sets alternate between calls: a rank can be one call ahead of another
// but not two (it needs every rank's data of the previous call first), so a set is never
// rewritten while a slower rank still reads it. The epoch counters live in this rank's
// device memory, so a CUDA graph replays the calls correctly. All ranks must issue the
// same sequence of calls with the same sizes.
#include <cuda_runtime.h>

#include <string.h>

#include <algorithm>
#include <vector>

#include "capi_internal.h"
#include "rrr_common.cuh"

namespace rrr {
namespace {

constexpr int kMaxCtas = 64;
constexpr int kMaxWorld = 8;
constexpr int kThreadsX = 512;
constexpr int kDevErrCommTimeout = 5;

struct Peers {
  float* data[kMaxWorld];       // each rank's data region (this rank's own at index rank)
  unsigned* flags[kMaxWorld];   // each rank's flag region
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// mode 0: x[i] = sum over ranks (in place, `out` == `in`); mode 1: out[r*n + i] = rank r's in[i]
__global__ void __launch_bounds__(kThreadsX) exchange_kernel(Peers peers, const float* in, float* out,
                                                              int64_t n, int64_t chunk, int rank,
                                                              int world, int64_t max_elems,
                                                              unsigned* counters, int mode, int* err) {
  const int c = blockIdx.x;
  const int64_t i0 = (int64_t)c * chunk, i1 = min(n, i0 + chunk);
  __shared__ unsigned s_epoch;
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    s_epoch = counters[c] + 1;
    s_ok = 1;
  }
  __syncthreads();
  const unsigned e = s_epoch;
  const int set = e & 1;
  // 1. this rank's chunk into slot `rank` of every buffer
  for (int r = 0; r < world; ++r) {
    float* dst = peers.data[r] + ((int64_t)set * world + rank) * max_elems;
    for (int64_t i = i0 + threadIdx.x; i < i1; i += kThreadsX) dst[i] = in[i];
  }
  // 2. stores visible to the other GPUs, then the flags
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < world) {
    unsigned* f = peers.flags[threadIdx.x] + ((int64_t)set * world + rank) * kMaxCtas + c;
    st_release_sys(f, e);
  }
  // 3. every rank's chunk has arrived in this buffer
  if (threadIdx.x < world) {
    const unsigned* f = peers.flags[rank] + ((int64_t)set * world + threadIdx.x) * kMaxCtas + c;
    if (ld_acquire_sys(f) != e) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_sys(f) != e) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          atomicCAS(err, 0, kDevErrCommTimeout);
          s_ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  // 4. combine in rank order (the slots were written by other GPUs: read around L1)
  const float* base = peers.data[rank] + (int64_t)set * world * max_elems;
  if (s_ok) {
    if (mode == 0) {
      for (int64_t i = i0 + threadIdx.x; i < i1; i += kThreadsX) {
        float acc = __ldcg(base + i);
        for (int r = 1; r < world; ++r) acc += __ldcg(base + (int64_t)r * max_elems + i);
        out[i] = acc;
      }
    } else {
      for (int r = 0; r < world; ++r)
        for (int64_t i = i0 + threadIdx.x; i < i1; i += kThreadsX)
          out[(int64_t)r * n + i] = __ldcg(base + (int64_t)r * max_elems + i);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) counters[c] = e;
}

}  // namespace
}  // namespace rrr

struct rrr_comm {
  rrr_ctx* ctx = nullptr;
  int rank = 0, world = 0;
  int64_t max_elems = 0;
  char* local = nullptr;  // this rank's exchange buffer
  size_t bytes = 0;
  unsigned* counters = nullptr;
  std::vector<char*> mapped;  // peers' buffers (nullptr at this rank's index)
  rrr::Peers peers{};
  bool connected = false;
};

using namespace rrr;

static size_t data_bytes(int world, int64_t max_elems) {
  return (size_t)2 * world * max_elems * sizeof(float);
}

extern "C" {

int rrr_comm_create(rrr_ctx* ctx, int rank, int world, int64_t max_elems, rrr_comm** out,
                    void* handle_out) {
  if (!ctx) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context");
  if (!out || !handle_out) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_comm_create: null argument");
  *out = nullptr;
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || max_elems < 1)
    return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_comm_create: need 1 <= world <= %d, 0 <= rank < world, max_elems >= 1",
                     kMaxWorld);
  int rc = bind_device(ctx);
  if (rc) return rc;
  rrr_comm* c = new rrr_comm();
  c->ctx = ctx;
  c->rank = rank;
  c->world = world;
  c->max_elems = (max_elems + 3) / 4 * 4;
  c->bytes = data_bytes(world, c->max_elems) + (size_t)2 * world * kMaxCtas * sizeof(unsigned);
  cudaError_t e = cudaMalloc(&c->local, c->bytes);
  if (e == cudaSuccess) e = cudaMemset(c->local, 0, c->bytes);
  if (e == cudaSuccess) e = cudaMalloc(&c->counters, kMaxCtas * sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemset(c->counters, 0, kMaxCtas * sizeof(unsigned));
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->local);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (c->local) cudaFree(c->local);
    if (c->counters) cudaFree(c->counters);
    delete c;
    return cuda_error(ctx, e, "rrr_comm_create");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  memcpy(handle_out, &h, 64);
  c->mapped.assign(world, nullptr);
  *out = c;
  return RRR_OK;
}

int rrr_comm_connect(rrr_comm* c, const void* handles) {
  if (!c) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null communicator");
  if (!handles) return set_error(c->ctx, RRR_ERR_INVALID_ARG, "rrr_comm_connect: null handles");
  if (c->connected) return set_error(c->ctx, RRR_ERR_INVALID_ARG, "rrr_comm_connect: already connected");
  int rc = bind_device(c->ctx);
  if (rc) return rc;
  const char* hs = static_cast<const char*>(handles);
  for (int r = 0; r < c->world; ++r) {
    char* base = c->local;
    if (r != c->rank) {
      cudaIpcMemHandle_t h;
      memcpy(&h, hs + 64 * r, 64);
      void* p = nullptr;
      cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) {
        for (int q = 0; q < r; ++q)
          if (c->mapped[q]) cudaIpcCloseMemHandle(c->mapped[q]);
        c->mapped.assign(c->world, nullptr);
        return cuda_error(c->ctx, e, "rrr_comm_connect: cudaIpcOpenMemHandle");
      }
      c->mapped[r] = static_cast<char*>(p);
      base = c->mapped[r];
    }
    c->peers.data[r] = reinterpret_cast<float*>(base);
    c->peers.flags[r] = reinterpret_cast<unsigned*>(base + data_bytes(c->world, c->max_elems));
  }
  c->connected = true;
  return RRR_OK;
}

static int comm_launch(rrr_comm* c, const float* in, float* out, int64_t n, int mode, void* stream,
                       const char* what) {
  if (!c) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null communicator");
  if (!c->connected) return set_error(c->ctx, RRR_ERR_INVALID_ARG, "%s: not connected", what);
  if (!in || !out) return set_error(c->ctx, RRR_ERR_INVALID_ARG, "%s: null pointer", what);
  if (n < 1 || n > c->max_elems)
    return set_error(c->ctx, RRR_ERR_BAD_SHAPE, "%s: n = %lld outside [1, %lld]", what,
                     (long long)n, (long long)c->max_elems);
  int rc = bind_device(c->ctx);
  if (rc) return rc;
  // about 4 KB per CTA and rank, at most kMaxCtas CTAs
  int64_t chunk = std::max<int64_t>(1024, (n + kMaxCtas - 1) / kMaxCtas);
  chunk = (chunk + 3) / 4 * 4;
  const int ctas = (int)((n + chunk - 1) / chunk);
  const LaunchEnv env = make_env(c->ctx, stream);
  exchange_kernel<<<ctas, kThreadsX, 0, env.stream>>>(c->peers, in, out, n, chunk, c->rank, c->world,
                                                      c->max_elems, c->counters, mode, env.d_err);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(c->ctx, e, what);
  return RRR_OK;
}

int rrr_comm_allreduce_f32(rrr_comm* c, float* x, int64_t n, void* stream) {
  return comm_launch(c, x, x, n, 0, stream, "rrr_comm_allreduce_f32");
}

int rrr_comm_allgather_f32(rrr_comm* c, float* out, const float* part, int64_t n_per_rank,
                           void* stream) {
  // `part` may be this rank's own slot of `out` (in-place gather), else disjoint from out
  if (c && out && part && part != out + (int64_t)c->rank * n_per_rank &&
      !((const char*)out + (size_t)c->world * n_per_rank * 4 <= (const char*)part ||
        (const char*)part + (size_t)n_per_rank * 4 <= (const char*)out))
    return set_error(c->ctx, RRR_ERR_INVALID_ARG, "rrr_comm_allgather_f32: out overlaps part");
  return comm_launch(c, part, out, n_per_rank, 1, stream, "rrr_comm_allgather_f32");
}

int rrr_comm_disconnect(rrr_comm* c) {
  if (!c) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null communicator");
  int rc = bind_device(c->ctx);
  if (rc) return rc;
  cudaDeviceSynchronize();
  for (char*& p : c->mapped)
    if (p) {
      cudaIpcCloseMemHandle(p);
      p = nullptr;
    }
  c->connected = false;
  return RRR_OK;
}

int rrr_comm_destroy(rrr_comm* c) {
  if (!c) return RRR_OK;
  rrr_comm_disconnect(c);
  if (c->local) cudaFree(c->local);
  if (c->counters) cudaFree(c->counters);
  delete c;
  return RRR_OK;
}

}  // extern "C"
