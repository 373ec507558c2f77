// comm_p2p.cu — all-reduce and all-gather of f32 vectors between the GPUs of one box over
// NVLink peer memory, for the tensor-parallel decode step (one process per GPU).
//
// Every rank owns an exchange buffer, mapped into the other ranks' processes through CUDA
// IPC handles: slots[2][world][max_elems] of 8-byte words. Each word carries one value
// and the epoch of the call that wrote it (value bits low, epoch high), stored and loaded
// as one naturally aligned 64-bit access (single-copy atomic), so the receiver waits on
// the data itself: no fences and no separate flags, one NVLink trip per exchange. A call
// of `n` elements runs C CTAs; CTA c owns elements [c*chunk, (c+1)*chunk). It
//   1. stores its elements of this rank's input, tagged with the epoch, into slot `rank`
//      of every rank's buffer (peer stores over NVLink; the local one is an ordinary store;
//      epoch = this CTA's call counter + 1, set = epoch & 1),
//   2. waits, element by element, until every rank's slot carries the epoch (bounded: it
//      gives up after about a second, records an error in the context's device flag and
//      stops waiting), and
//   3. sums the slots in rank order (all-reduce: every rank gets identical bits) or copies
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
constexpr int kThreadsX = 256;  // few registers: co-resident with a finishing GEMV
constexpr int kDevErrCommTimeout = 5;

struct Peers {
  unsigned long long* slots[kMaxWorld];  // each rank's buffer (this rank's own at index rank)
};

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// The value of word p once its epoch is e; gives up (ok = false) after the context's wait
// limit (wait_limit_ns).
__device__ __forceinline__ float wait_word(const unsigned long long* p, unsigned e, bool& ok,
                                           int* err) {
  unsigned long long w = ld_relaxed_sys_u64(p);
  if ((unsigned)(w >> 32) != e && ok) {
    const uint64_t t0 = globaltimer_ns();
    const uint64_t limit = wait_limit_ns(err);
    for (int i = 0;; ++i) {
      w = ld_relaxed_sys_u64(p);
      if ((unsigned)(w >> 32) == e) break;
      if ((i & 63) == 63 && globaltimer_ns() - t0 > limit) {
        atomicCAS(err, 0, kDevErrCommTimeout);
        ok = false;
        break;
      }
    }
  }
  return __uint_as_float((unsigned)w);
}

// mode 0: x[i] = sum over ranks (in place allowed); mode 1: all-gather, element i of rank
// r's input to out[(i / npr) * world * npr + r * npr + i % npr] (npr = n: concatenation;
// npr < n: rows of npr elements interleaved by rank, the layout of row-split logits)
__global__ void __launch_bounds__(kThreadsX) exchange_kernel(Peers peers, const float* in, float* out,
                                                              int64_t n, int64_t chunk, int rank,
                                                              int world, int64_t max_elems,
                                                              unsigned* counters, int mode,
                                                              int64_t npr, int* err) {
  // launched with programmatic dependent launch: let the next kernel (a GEMV streaming its
  // weights) start now, and wait for the kernel that produced `in`
  pdl_launch_dependents();
  pdl_wait();
  const int c = blockIdx.x;
  const int64_t i0 = (int64_t)c * chunk, i1 = min(n, i0 + chunk);
  __shared__ unsigned s_epoch;
  if (threadIdx.x == 0) s_epoch = counters[c] + 1;
  __syncthreads();
  const unsigned e = s_epoch;
  const int set = e & 1;
  const unsigned long long tag = (unsigned long long)e << 32;
  // 1. this rank's elements, tagged, into slot `rank` of every buffer
  for (int r = 0; r < world; ++r) {
    unsigned long long* dst = peers.slots[r] + ((int64_t)set * world + rank) * max_elems;
    for (int64_t i = i0 + threadIdx.x; i < i1; i += kThreadsX)
      st_relaxed_sys_u64(dst + i, tag | __float_as_uint(in[i]));
  }
  // 2.-3. every rank's element, in rank order
  const unsigned long long* base = peers.slots[rank] + (int64_t)set * world * max_elems;
  bool ok = true;
  for (int64_t i = i0 + threadIdx.x; i < i1; i += kThreadsX) {
    if (mode == 0) {
      float acc = wait_word(base + i, e, ok, err);
      for (int r = 1; r < world; ++r) acc += wait_word(base + (int64_t)r * max_elems + i, e, ok, err);
      out[i] = acc;
    } else {
      float* o = out + (i / npr) * world * npr + i % npr;
      for (int r = 0; r < world; ++r)
        o[(int64_t)r * npr] = wait_word(base + (int64_t)r * max_elems + i, e, ok, err);
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
  return (size_t)2 * world * max_elems * sizeof(unsigned long long);
}

namespace rrr {
void comm_info(const rrr_comm* c, rrr_ctx** ctx, int* rank, int* world, int64_t* max_elems) {
  *ctx = c->ctx;
  *rank = c->rank;
  *world = c->world;
  *max_elems = c->max_elems;
}
}  // namespace rrr

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
  c->bytes = data_bytes(world, c->max_elems);
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
    c->peers.slots[r] = reinterpret_cast<unsigned long long*>(base);
  }
  c->connected = true;
  return RRR_OK;
}

static int comm_launch(rrr_comm* c, const float* in, float* out, int64_t n, int mode, int64_t npr,
                       void* stream, const char* what) {
  if (!c) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null communicator");
  if (!c->connected) return set_error(c->ctx, RRR_ERR_INVALID_ARG, "%s: not connected", what);
  if (!in || !out) return set_error(c->ctx, RRR_ERR_INVALID_ARG, "%s: null pointer", what);
  if (n < 1 || n > c->max_elems)
    return set_error(c->ctx, RRR_ERR_BAD_SHAPE, "%s: n = %lld outside [1, %lld]", what,
                     (long long)n, (long long)c->max_elems);
  int rc = bind_device(c->ctx);
  if (rc) return rc;
  // about 2 KB of values per CTA and rank, at most kMaxCtas CTAs
  int64_t chunk = std::max<int64_t>(512, (n + kMaxCtas - 1) / kMaxCtas);
  chunk = (chunk + 3) / 4 * 4;
  const int ctas = (int)((n + chunk - 1) / chunk);
  const LaunchEnv env = make_env(c->ctx, stream);
  cudaError_t e = rrr_launch_pdl(exchange_kernel, dim3(ctas), dim3(kThreadsX), 0, env.stream, env.pdl,
                                 c->peers, in, out, n, chunk, c->rank, c->world, c->max_elems,
                                 c->counters, mode, npr, env.d_err);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(c->ctx, e, what);
  return RRR_OK;
}

int rrr_comm_allreduce_f32(rrr_comm* c, float* x, int64_t n, void* stream) {
  return comm_launch(c, x, x, n, 0, n, stream, "rrr_comm_allreduce_f32");
}

int rrr_comm_allgather_f32(rrr_comm* c, float* out, const float* part, int64_t n_per_rank,
                           void* stream) {
  // `part` may be this rank's own slot of `out` (in-place gather), else disjoint from out
  if (c && out && part && part != out + (int64_t)c->rank * n_per_rank &&
      !((const char*)out + (size_t)c->world * n_per_rank * 4 <= (const char*)part ||
        (const char*)part + (size_t)n_per_rank * 4 <= (const char*)out))
    return set_error(c->ctx, RRR_ERR_INVALID_ARG, "rrr_comm_allgather_f32: out overlaps part");
  return comm_launch(c, part, out, n_per_rank, 1, n_per_rank, stream, "rrr_comm_allgather_f32");
}

int rrr_comm_allgather_rows_f32(rrr_comm* c, float* out, const float* part, int rows,
                                int64_t n_per_row, void* stream) {
  if (c && (rows < 1 || n_per_row < 1))
    return set_error(c->ctx, RRR_ERR_BAD_SHAPE, "rrr_comm_allgather_rows_f32: rows, n_per_row >= 1");
  if (c && out && part && !((const char*)out + (size_t)c->world * rows * n_per_row * 4 <= (const char*)part ||
                            (const char*)part + (size_t)rows * n_per_row * 4 <= (const char*)out))
    return set_error(c->ctx, RRR_ERR_INVALID_ARG, "rrr_comm_allgather_rows_f32: out overlaps part");
  return comm_launch(c, part, out, (int64_t)rows * n_per_row, 1, n_per_row, stream,
                     "rrr_comm_allgather_rows_f32");
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
