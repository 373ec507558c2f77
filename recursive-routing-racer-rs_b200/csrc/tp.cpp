// tp.cpp — tensor parallelism of the decode step behind the C ABI (
// the reference has no multi-GPU code): the shard plan, the exchange channel of a rank
// (NCCL loaded at run time, or the peer-memory rrr_comm), and the host watchdog.
//
// The plan follows the split of the per-layer weight GEMVs that keeps every non-GEMV op
// local: QKV by KV-head group, the O-projection by head columns (super-block window), gate /
// up rows with the matching down columns, the logits by vocabulary rows.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <time.h>

#include <cstring>
#include <mutex>

#include "capi_internal.h"
#include "internal.h"
#include "tp_watchdog.h"

using namespace rrr;

namespace {

// The NCCL entry points this file uses, from the libnccl.so.2 already loaded in the
// process (for example by torch) or else loaded here; no link-time dependency.
struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t);
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*CommAbort)(ncclComm_t);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  const char* (*GetErrorString)(ncclResult_t);
  bool ok = false;
};

const NcclApi* nccl_api() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    auto sym = [&](const char* n) { return dlsym(h, n); };
    api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(sym("ncclGetUniqueId"));
    api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(sym("ncclCommInitRank"));
    api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(sym("ncclAllReduce"));
    api.AllGather = reinterpret_cast<decltype(api.AllGather)>(sym("ncclAllGather"));
    api.CommGetAsyncError =
        reinterpret_cast<decltype(api.CommGetAsyncError)>(sym("ncclCommGetAsyncError"));
    api.CommAbort = reinterpret_cast<decltype(api.CommAbort)>(sym("ncclCommAbort"));
    api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(sym("ncclCommDestroy"));
    api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(sym("ncclGetErrorString"));
    api.ok = api.GetUniqueId && api.CommInitRank && api.AllReduce && api.AllGather &&
             api.CommGetAsyncError && api.CommAbort && api.CommDestroy && api.GetErrorString;
  });
  return api.ok ? &api : nullptr;
}

int nccl_error(rrr_ctx* ctx, const NcclApi* api, ncclResult_t r, const char* what) {
  return set_error(ctx, RRR_ERR_NCCL, "%s: %s", what, api ? api->GetErrorString(r) : "NCCL unavailable");
}

}  // namespace

struct rrr_tp_comm {
  rrr_ctx* ctx = nullptr;
  int rank = 0, world = 1;
  rrr_comm* p2p = nullptr;      // peer-memory channel (not owned), or
  ncclComm_t nccl = nullptr;    // an NCCL communicator (owned)
  bool aborted = false;
  float* gather_tmp = nullptr;  // NCCL row all-gather staging [world][rows][n_per_row]
  size_t gather_cap = 0;        // floats
};

namespace rrr {

int tp_comm_world(const rrr_tp_comm* c) { return c ? c->world : 1; }
int tp_comm_rank(const rrr_tp_comm* c) { return c ? c->rank : 0; }
bool tp_comm_is_p2p(const rrr_tp_comm* c) { return c && c->p2p; }
rrr_comm* tp_comm_p2p_of(rrr_tp_comm* c) { return c ? c->p2p : nullptr; }

int tp_allreduce(rrr_tp_comm* c, float* x, int64_t n, void* stream) {
  if (c->p2p) return rrr_comm_allreduce_f32(c->p2p, x, n, stream);
  if (c->aborted) return set_error(c->ctx, RRR_ERR_NCCL, "tp all-reduce: communicator aborted");
  const NcclApi* api = nccl_api();
  const ncclResult_t r = api->AllReduce(x, x, (size_t)n, ncclFloat32, ncclSum, c->nccl,
                                        static_cast<cudaStream_t>(stream));
  return r == ncclSuccess ? RRR_OK : nccl_error(c->ctx, api, r, "tp all-reduce");
}

int tp_allgather_rows(rrr_tp_comm* c, float* out, const float* part, int rows, int64_t npr,
                      void* stream) {
  if (c->p2p) {
    if (rows == 1) return rrr_comm_allgather_f32(c->p2p, out, part, npr, stream);
    return rrr_comm_allgather_rows_f32(c->p2p, out, part, rows, npr, stream);
  }
  if (c->aborted) return set_error(c->ctx, RRR_ERR_NCCL, "tp all-gather: communicator aborted");
  const NcclApi* api = nccl_api();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 1) {
    const ncclResult_t r = api->AllGather(part, out, (size_t)npr, ncclFloat32, c->nccl, s);
    return r == ncclSuccess ? RRR_OK : nccl_error(c->ctx, api, r, "tp all-gather");
  }
  // [world][rows][npr] from NCCL, then rows of [world][npr]
  const size_t need = (size_t)c->world * rows * npr;
  if (need > c->gather_cap) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(s, &cs);
    if (cs != cudaStreamCaptureStatusNone)
      return set_error(c->ctx, RRR_ERR_INVALID_ARG,
                       "tp all-gather: staging must be sized by an eager call before capture");
    cudaError_t e = cudaStreamSynchronize(s);
    if (e == cudaSuccess && c->gather_tmp) e = cudaFree(c->gather_tmp);
    c->gather_tmp = nullptr;
    c->gather_cap = 0;
    if (e == cudaSuccess) e = cudaMalloc(&c->gather_tmp, need * sizeof(float));
    if (e != cudaSuccess) return cuda_error(c->ctx, e, "tp all-gather: staging");
    c->gather_cap = need;
  }
  const ncclResult_t r =
      api->AllGather(part, c->gather_tmp, (size_t)rows * npr, ncclFloat32, c->nccl, s);
  if (r != ncclSuccess) return nccl_error(c->ctx, api, r, "tp all-gather");
  const cudaError_t e = launch_rows_from_ranks(make_env(c->ctx, stream), c->gather_tmp, out,
                                               c->world, rows, npr);
  return e == cudaSuccess ? RRR_OK : cuda_error(c->ctx, e, "tp all-gather: reorder");
}

}  // namespace rrr

extern "C" {

int rrr_tp_plan(int d, int nq, int nkv, int hd, int F, int V, int G, int g, rrr_tp_shard* out) {
  if (!out) return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_tp_plan: null output");
  if (d <= 0 || nq <= 0 || nkv <= 0 || hd <= 0 || F <= 0 || V <= 0 || nq * hd != d)
    return set_error(nullptr, RRR_ERR_BAD_SHAPE, "rrr_tp_plan: bad model dimensions");
  if (G < 1 || g < 0 || g >= G)
    return set_error(nullptr, RRR_ERR_BAD_SHAPE, "rrr_tp_plan: bad rank %d of %d", g, G);
  if (nq % G || nkv % G || nq % nkv)
    return set_error(nullptr, RRR_ERR_BAD_SHAPE,
                     "rrr_tp_plan: %d query / %d KV heads do not split over %d GPUs", nq, nkv, G);
  if (F % (256 * G))
    return set_error(nullptr, RRR_ERR_BAD_SHAPE, "rrr_tp_plan: ffn_dim %d is not a multiple of 256*%d", F, G);
  if (V % G) return set_error(nullptr, RRR_ERR_BAD_SHAPE, "rrr_tp_plan: vocab %d is not a multiple of %d", V, G);
  rrr_tp_shard s{};
  s.G = G;
  s.g = g;
  s.q_head0 = nq * g / G;
  s.q_head1 = nq * (g + 1) / G;
  s.kv_head0 = nkv * g / G;
  s.kv_head1 = nkv * (g + 1) / G;
  s.qkv_rows[0][0] = s.q_head0 * hd;
  s.qkv_rows[0][1] = s.q_head1 * hd;
  s.qkv_rows[1][0] = nq * hd + s.kv_head0 * hd;
  s.qkv_rows[1][1] = nq * hd + s.kv_head1 * hd;
  s.qkv_rows[2][0] = (nq + nkv) * hd + s.kv_head0 * hd;
  s.qkv_rows[2][1] = (nq + nkv) * hd + s.kv_head1 * hd;
  s.qkv_dim = (s.q_head1 - s.q_head0) * hd + 2 * (s.kv_head1 - s.kv_head0) * hd;
  const int c0 = s.q_head0 * hd, c1 = s.q_head1 * hd;
  s.o_block0 = c0 / 256;
  s.o_block1 = (c1 + 255) / 256;
  s.o_k = 256 * (s.o_block1 - s.o_block0);
  s.o_k_offset = c0 - 256 * s.o_block0;
  s.ffn0 = F * g / G;
  s.ffn1 = F * (g + 1) / G;
  s.vocab0 = V * g / G;
  s.vocab1 = V * (g + 1) / G;
  *out = s;
  return RRR_OK;
}

int rrr_tp_nccl_unique_id(void* id_out) {
  if (!id_out) return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_tp_nccl_unique_id: null output");
  const NcclApi* api = nccl_api();
  if (!api) return set_error(nullptr, RRR_ERR_NCCL, "rrr_tp_nccl_unique_id: libnccl.so.2 not loadable");
  ncclUniqueId id;
  const ncclResult_t r = api->GetUniqueId(&id);
  if (r != ncclSuccess) return nccl_error(nullptr, api, r, "ncclGetUniqueId");
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
  memcpy(id_out, &id, sizeof id);
  return RRR_OK;
}

int rrr_tp_comm_nccl(rrr_ctx* ctx, const void* unique_id, int rank, int world, rrr_tp_comm** out) {
  if (!ctx) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context");
  if (!unique_id || !out) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_tp_comm_nccl: null argument");
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world)
    return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_tp_comm_nccl: bad rank %d of %d", rank, world);
  const NcclApi* api = nccl_api();
  if (!api) return set_error(ctx, RRR_ERR_NCCL, "rrr_tp_comm_nccl: libnccl.so.2 not loadable");
  int rc = bind_device(ctx);
  if (rc) return rc;
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof id);
  ncclComm_t comm = nullptr;
  const ncclResult_t r = api->CommInitRank(&comm, world, id, rank);
  if (r != ncclSuccess) return nccl_error(ctx, api, r, "ncclCommInitRank");
  rrr_tp_comm* c = new rrr_tp_comm();
  c->ctx = ctx;
  c->rank = rank;
  c->world = world;
  c->nccl = comm;
  *out = c;
  return RRR_OK;
}

int rrr_tp_comm_p2p(rrr_comm* comm, rrr_tp_comm** out) {
  if (!comm || !out) return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_tp_comm_p2p: null argument");
  rrr_tp_comm* c = new rrr_tp_comm();
  int64_t max_elems = 0;
  comm_info(comm, &c->ctx, &c->rank, &c->world, &max_elems);
  c->p2p = comm;
  *out = c;
  return RRR_OK;
}

int rrr_tp_wait(rrr_tp_comm* c, void* stream, int timeout_ms) {
  if (!c) return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_tp_wait: null communicator");
  if (timeout_ms < 0) return set_error(c->ctx, RRR_ERR_INVALID_ARG, "rrr_tp_wait: negative timeout");
  int rc = bind_device(c->ctx);
  if (rc) return rc;
  struct State {
    rrr_tp_comm* c;
    cudaStream_t s;
    cudaError_t err;
  } st{c, static_cast<cudaStream_t>(stream), cudaSuccess};
  WatchOps ops{};
  ops.user = &st;
  ops.stream_state = [](void* u) {
    State* p = static_cast<State*>(u);
    const cudaError_t e = cudaStreamQuery(p->s);
    if (e == cudaSuccess) return 1;
    if (e == cudaErrorNotReady) return 0;
    p->err = e;
    return -1;
  };
  ops.comm_failed = [](void* u) {
    State* p = static_cast<State*>(u);
    if (!p->c->nccl) return 0;
    ncclResult_t r = ncclSuccess;
    if (nccl_api()->CommGetAsyncError(p->c->nccl, &r) != ncclSuccess) return 1;
    return (r != ncclSuccess && r != ncclInProgress) ? 1 : 0;
  };
  ops.abort_comm = [](void* u) {
    State* p = static_cast<State*>(u);
    if (p->c->nccl && !p->c->aborted) {
      nccl_api()->CommAbort(p->c->nccl);
      p->c->aborted = true;
      p->c->nccl = nullptr;
    }
  };
  ops.now_ms = [](void*) {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e3 + ts.tv_nsec * 1e-6;
  };
  ops.pause = [](void*) {
    timespec ts{0, 50000};
    nanosleep(&ts, nullptr);
  };
  switch (tp_watch(ops, (double)timeout_ms)) {
    case kWatchDone: {
      int code = 0;
      return rrr_check_device_error(c->ctx, &code);
    }
    case kWatchStreamError:
      return cuda_error(c->ctx, st.err, "rrr_tp_wait: the step failed");
    case kWatchCommError:
      return set_error(c->ctx, RRR_ERR_NCCL,
                       "rrr_tp_wait: the communicator reported an error; it was aborted");
    default:
      return set_error(c->ctx, RRR_ERR_TIMEOUT,
                       "rrr_tp_wait: the step did not complete within %d ms; the communicator was "
                       "aborted", timeout_ms);
  }
}

int rrr_tp_comm_destroy(rrr_tp_comm* c) {
  if (!c) return RRR_OK;
  if (c->ctx) bind_device(c->ctx);
  if (c->nccl && !c->aborted) nccl_api()->CommDestroy(c->nccl);
  if (c->gather_tmp) cudaFree(c->gather_tmp);
  delete c;
  return RRR_OK;
}

}  // extern "C"
