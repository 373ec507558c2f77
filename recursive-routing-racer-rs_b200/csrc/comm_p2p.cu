// comm_p2p.cu — all-reduce and all-gather of f32 vectors between the GPUs of one box over
// NVLink peer memory, for the tensor-parallel decode step (one process per GPU).
//
// Every rank owns an exchange buffer, mapped into the other ranks' processes through CUDA
// IPC handles: a 256-byte header (the owner's GPU UUID and region sizes, read by the peers
// when they connect), then slots[2][world][max_elems] of 8-byte words, then the optional
// fused-exchange region of the decode step's GEMVs. Each word carries one value
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
#include <cstdlib>
#include <vector>

#include "capi_internal.h"
#include "rrr_common.cuh"

namespace rrr {
namespace {

constexpr int kMaxCtas = 64;
constexpr int kMaxWorld = 8;
constexpr int kThreadsX = 256;  // few registers: co-resident with a finishing GEMV

constexpr size_t kHeaderBytes = 256;

// What a rank's buffer says about its owner (at offset 0; the peers read it at connect).
struct BufHeader {
  unsigned char uuid[16];  // the owner's GPU
  int64_t max_elems, fused_words;
  int32_t world, rank;
};

struct Peers {
  unsigned long long* slots[kMaxWorld];  // each rank's buffer (this rank's own at index rank)
};

// mode 0: x[i] = sum over ranks (in place allowed); mode 1: all-gather, element i of rank
// r's input to out[(i / npr) * world * npr + r * npr + i % npr] (npr = n: concatenation;
// npr < n: rows of npr elements interleaved by rank, the layout of row-split logits);
// mode 2: the mode-0 sum in two trips (reduce-scatter, then all-gather of the sums): rank
// s owns the slice [s*npr, (s+1)*npr) (npr = ceil(n / world)); every rank sends slice s
// only to its owner, the owner sums it in rank order (the bits of mode 0) and sends the
// sums to every rank. In rank r's buffer the owner's sums of slice s land in the slots of
// source s outside slice r, which the first trip leaves unused. A CTA covers slice
// positions [c*chunk, (c+1)*chunk) of every slice.
// Every call runs all kMaxCtas CTAs (those past the data only advance their epoch), so
// the epochs of all CTAs advance together and consecutive calls always use different slot
// sets, however differently two calls map elements to CTAs.
// The words p(u, r) = q[u] + r * rstride (u < B, r < W) once they carry epoch e, for the
// (u, r) where valid(u, r) holds: every load first, then a bounded wait on each word that
// had not arrived yet. B elements of a thread are collected together (4 to 8 words in
// flight) so that its waits cost one round trip per batch instead of one per word.
template <int W, int B, typename Valid>
__device__ __forceinline__ void collect(const unsigned long long* const (&q)[B], int64_t rstride,
                                        Valid valid, unsigned e, bool& ok, int* err,
                                        float (&v)[B][W]) {
  unsigned long long w[B][W];
#pragma unroll
  for (int u = 0; u < B; ++u)
#pragma unroll
    for (int r = 0; r < W; ++r)
      if (valid(u, r)) w[u][r] = ld_relaxed_sys_u64(q[u] + r * rstride);
#pragma unroll
  for (int u = 0; u < B; ++u)
#pragma unroll
    for (int r = 0; r < W; ++r)
      if (valid(u, r))
        v[u][r] = __uint_as_float((unsigned)wait_tagged(q[u] + r * rstride, w[u][r], e, ok, err));
}

// W = world (1..kMaxWorld ranks), B = elements collected together.
template <int W>
__global__ void __launch_bounds__(kThreadsX, 6) exchange_kernel(Peers peers, const float* in, float* out,
                                                                 int64_t n, int64_t chunk, int rank,
                                                                 int64_t max_elems, unsigned* counters,
                                                                 int mode, int64_t npr, int* err) {
  constexpr int world = W;
  constexpr int kBatch = W >= 4 ? 1 : 4 / W;
  // launched with programmatic dependent launch: let the next kernel (a GEMV streaming its
  // weights) start now, and wait for the kernel that produced `in`
  pdl_launch_dependents();
  pdl_wait();
  const int c = blockIdx.x;
  const int64_t i0 = (int64_t)c * chunk, i1 = min(mode == 2 ? npr : n, i0 + chunk);
  __shared__ unsigned s_epoch;
  if (threadIdx.x == 0) s_epoch = counters[c] + 1;
  __syncthreads();
  const unsigned e = s_epoch;
  const int set = e & 1;
  const unsigned long long tag = (unsigned long long)e << 32;
  const unsigned long long* base = peers.slots[rank] + (int64_t)set * world * max_elems;
  bool ok = true;
  float v[kBatch][W];
  if (mode == 2) {
    // 1. slice s of this rank's input, tagged, into slot `rank` of its owner's buffer
    for (int s = 0; s < world; ++s) {
      unsigned long long* dst = peers.slots[s] + ((int64_t)set * world + rank) * max_elems;
      for (int64_t j = i0 + threadIdx.x; j < i1; j += kThreadsX) {
        const int64_t i = (int64_t)s * npr + j;
        if (i < n) st_relaxed_sys_u64(dst + i, tag | __float_as_uint(in[i]));
      }
    }
    // 2. this rank's slice: every rank's element in rank order, the sum to every rank
    const int64_t own = (int64_t)rank * npr;
    for (int64_t jb = i0 + threadIdx.x; jb < i1; jb += kBatch * kThreadsX) {
      const unsigned long long* q[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) q[u] = base + own + jb + u * kThreadsX;
      auto valid = [&](int u, int) {
        const int64_t j = jb + u * kThreadsX;
        return j < i1 && own + j < n;
      };
      collect<W, kBatch>(q, max_elems, valid, e, ok, err, v);
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        if (!valid(u, 0)) continue;
        const int64_t i = own + jb + u * kThreadsX;
        float acc = v[u][0];
#pragma unroll
        for (int r = 1; r < W; ++r) acc += v[u][r];
        out[i] = acc;
        for (int r = 0; r < world; ++r)
          if (r != rank)
            st_relaxed_sys_u64(peers.slots[r] + ((int64_t)set * world + rank) * max_elems + i,
                               tag | __float_as_uint(acc));
      }
    }
    // 3. the other slices' sums from their owners: word (s, s*npr + j) of this buffer (for
    // s = rank that is this rank's own first-trip word, already there and not used)
    for (int64_t jb = i0 + threadIdx.x; jb < i1; jb += kBatch * kThreadsX) {
      const unsigned long long* q[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) q[u] = base + jb + u * kThreadsX;
      auto valid = [&](int u, int s) {
        const int64_t j = jb + u * kThreadsX;
        return j < i1 && (int64_t)s * npr + j < n;
      };
      collect<W, kBatch>(q, max_elems + npr, valid, e, ok, err, v);
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
#pragma unroll
        for (int s2 = 0; s2 < W; ++s2)
          if (s2 != rank && valid(u, s2))
            out[(int64_t)s2 * npr + jb + u * kThreadsX] = v[u][s2];
    }
    __syncthreads();
    if (threadIdx.x == 0) counters[c] = e;
    return;
  }
  // 1. this rank's elements, tagged, into slot `rank` of every buffer
  for (int r = 0; r < world; ++r) {
    unsigned long long* dst = peers.slots[r] + ((int64_t)set * world + rank) * max_elems;
    for (int64_t i = i0 + threadIdx.x; i < i1; i += kThreadsX)
      st_relaxed_sys_u64(dst + i, tag | __float_as_uint(in[i]));
  }
  // 2.-3. every rank's element: their sum in rank order (mode 0) or each in place (mode 1)
  for (int64_t ib = i0 + threadIdx.x; ib < i1; ib += kBatch * kThreadsX) {
    const unsigned long long* q[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) q[u] = base + ib + u * kThreadsX;
    auto valid = [&](int u, int) { return ib + u * kThreadsX < i1; };
    collect<W, kBatch>(q, max_elems, valid, e, ok, err, v);
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      if (!valid(u, 0)) continue;
      const int64_t i = ib + u * kThreadsX;
      if (mode == 0) {
        float acc = v[u][0];
#pragma unroll
        for (int r = 1; r < W; ++r) acc += v[u][r];
        out[i] = acc;
      } else {
        float* o = out + (i / npr) * world * npr + i % npr;
#pragma unroll
        for (int r = 0; r < W; ++r) o[(int64_t)r * npr] = v[u][r];
      }
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
  int64_t fused_words = 0;  // words of the fused-exchange region after the slots
  char* local = nullptr;  // this rank's exchange buffer
  size_t bytes = 0;       // slots + fused region
  size_t slot_bytes = 0;  // the exchange kernels' slots (the fused region starts here)
  unsigned* counters = nullptr;
  std::vector<char*> mapped;  // peers' buffers (nullptr at this rank's index)
  rrr::Peers peers{};
  bool connected = false;
  bool distinct_devices = false;  // every peer's buffer lives on another GPU
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

int64_t comm_fused(const rrr_comm* c, unsigned long long** bases, unsigned** epoch) {
  if (!c->connected || c->fused_words == 0 || !c->distinct_devices) return 0;
  *epoch = c->counters + kMaxCtas;
  for (int r = 0; r < c->world; ++r)
    bases[r] = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(c->peers.slots[r]) +
                                                     c->slot_bytes);
  return c->fused_words;
}
}  // namespace rrr

extern "C" {

int rrr_comm_create(rrr_ctx* ctx, int rank, int world, int64_t max_elems, rrr_comm** out,
                    void* handle_out) {
  return rrr_comm_create_ex(ctx, rank, world, max_elems, 0, out, handle_out);
}

int rrr_comm_create_ex(rrr_ctx* ctx, int rank, int world, int64_t max_elems, int64_t fused_words,
                       rrr_comm** out, void* handle_out) {
  if (!ctx) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context");
  if (fused_words < 0) return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_comm_create_ex: fused_words >= 0");
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
  c->slot_bytes = data_bytes(world, c->max_elems);
  c->fused_words = (fused_words + 31) / 32 * 32;
  c->bytes = kHeaderBytes + c->slot_bytes + (size_t)c->fused_words * sizeof(unsigned long long);
  BufHeader hdr{};
  cudaDeviceProp prop{};
  cudaError_t e = cudaGetDeviceProperties(&prop, ctx->device);
  memcpy(hdr.uuid, &prop.uuid, 16);
  hdr.max_elems = c->max_elems;
  hdr.fused_words = c->fused_words;
  hdr.world = world;
  hdr.rank = rank;
  if (e == cudaSuccess) e = cudaMalloc(&c->local, c->bytes);
  if (e == cudaSuccess) e = cudaMemset(c->local, 0, c->bytes);
  if (e == cudaSuccess) e = cudaMemcpy(c->local, &hdr, sizeof hdr, cudaMemcpyHostToDevice);
  // the exchange CTAs' call counters, then the fused exchanges' step epoch
  if (e == cudaSuccess) e = cudaMalloc(&c->counters, (kMaxCtas + 1) * sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemset(c->counters, 0, (kMaxCtas + 1) * sizeof(unsigned));
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
    c->peers.slots[r] = reinterpret_cast<unsigned long long*>(base + kHeaderBytes);
  }
  // The peers' headers: the same layout everywhere, and whose GPU each buffer is on. Kernels
  // that wait on one another's stores may only run on different GPUs: the fused exchanges
  // are enabled only then (the exchange kernels' waits stay bounded either way).
  BufHeader mine{};
  cudaError_t e = cudaMemcpy(&mine, c->local, sizeof mine, cudaMemcpyDeviceToHost);
  c->distinct_devices = true;
  for (int r = 0; r < c->world && e == cudaSuccess; ++r) {
    if (r == c->rank) continue;
    BufHeader h{};
    e = cudaMemcpy(&h, c->mapped[r], sizeof h, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) break;
    if (h.world != c->world || h.rank != r || h.max_elems != c->max_elems ||
        h.fused_words != c->fused_words) {
      for (char*& p : c->mapped)
        if (p) {
          cudaIpcCloseMemHandle(p);
          p = nullptr;
        }
      return set_error(c->ctx, RRR_ERR_INVALID_ARG,
                       "rrr_comm_connect: handle %d is rank %d of %d with %lld elements and %lld "
                       "fused words; this rank expects rank %d of %d with %lld and %lld",
                       r, (int)h.rank, (int)h.world, (long long)h.max_elems,
                       (long long)h.fused_words, r, c->world, (long long)c->max_elems,
                       (long long)c->fused_words);
    }
    if (memcmp(h.uuid, mine.uuid, 16) == 0) c->distinct_devices = false;
  }
  if (e != cudaSuccess) {
    for (char*& p : c->mapped)
      if (p) {
        cudaIpcCloseMemHandle(p);
        p = nullptr;
      }
    return cuda_error(c->ctx, e, "rrr_comm_connect: reading the peers' headers");
  }
  c->connected = true;
  return RRR_OK;
}

// RRR_COMM_TWO_TRIP: 1 = every all-reduce of two or more ranks takes two trips, 0 = none
// does; unset = large ones from 4 ranks (comm_launch). Read once per process (tests run the
// two-trip form on two GPUs with it).
static int two_trip_setting() {
  static const int v = [] {
    const char* s = std::getenv("RRR_COMM_TWO_TRIP");
    return s ? std::atoi(s) : -1;
  }();
  return v;
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
  // Large all-reduces from 4 ranks up take two trips (mode 2): each rank then writes about
  // 2n tagged words instead of world * n, which pays once the saved bytes outweigh the
  // second NVLink trip (n * (world - 2) * 8 bytes >= 2 MB, e.g. 64 tokens x 3072 at 8 ranks)
  const int forced = two_trip_setting();
  if (mode == 0 && c->world >= 2 &&
      (forced == 1 || (forced != 0 && c->world >= 4 && n * (c->world - 2) * 8 >= (int64_t)(2 << 20)))) {
    mode = 2;
    npr = (n + c->world - 1) / c->world;
  }
  // about 2 KB of values per CTA and rank (of each slice in mode 2), at most kMaxCtas CTAs
  // with data; all kMaxCtas CTAs run (see exchange_kernel)
  const int64_t span = mode == 2 ? npr : n;
  int64_t chunk = std::max<int64_t>(512, (span + kMaxCtas - 1) / kMaxCtas);
  chunk = (chunk + 3) / 4 * 4;
  const int ctas = kMaxCtas;
  const LaunchEnv env = make_env(c->ctx, stream);
  cudaError_t e;
  switch (c->world) {
#define RRR_EXCHANGE(W)                                                                          \
  case W:                                                                                        \
    e = rrr_launch_pdl(exchange_kernel<W>, dim3(ctas), dim3(kThreadsX), 0, env.stream, env.pdl,  \
                       c->peers, in, out, n, chunk, c->rank, c->max_elems, c->counters, mode, npr, \
                       env.d_err);                                                               \
    break;
    RRR_EXCHANGE(1) RRR_EXCHANGE(2) RRR_EXCHANGE(3) RRR_EXCHANGE(4)
    RRR_EXCHANGE(5) RRR_EXCHANGE(6) RRR_EXCHANGE(7) RRR_EXCHANGE(8)
#undef RRR_EXCHANGE
    default: e = cudaErrorInvalidValue;
  }
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
