// dispatch.cpp — named dispatch and prebuilt dispatch tables.
//
// rrr_dispatch_by_name mirrors ComputeEngine::dispatch_by_name (src/gpu/engine.rs:476-554):
// a kernel is identified by the reference's shader name, its bindings are a list of
// buffers with byte sizes, its arguments raw push-constant bytes. Unlike the reference
// (which trusts the sizes and panics on misuse) every binding size and push layout is
// validated and reported as a status code.
//
// rrr_batch mirrors the prebuilt table of pre_allocate_desc_set +
// dispatch_batch_persistent_v2 (engine.rs:244-268, 317-370; built at phi4.rs:969-1064):
// the recorded dispatches are captured once into a CUDA graph and replayed with one
// launch. Stream order replaces the reference's explicit pipeline barriers. A single-token
// GEMV dispatch whose input no earlier dispatch of the table writes prepares that input
// before its grid dependency wait (the kernel writes its rows only after it), so the
// preparation overlaps the tail of the dispatch before it.
#include <cuda_runtime.h>

#include <cstring>
#include <string>
#include <vector>

#include "capi_internal.h"
#include "internal.h"

using namespace rrr;

namespace {

struct Op {
  std::string name;
  std::vector<void*> bufs;
  std::vector<uint64_t> sizes;
  std::vector<uint8_t> push;
};

uint32_t push_u32(const void* push, int i) {
  uint32_t v;
  std::memcpy(&v, static_cast<const uint8_t*>(push) + 4 * i, 4);
  return v;
}

int kq_from_name(const std::string& n, bool* batch) {
  *batch = false;
  std::string base = n;
  const std::string suf = "_batch";
  if (base.size() > suf.size() && base.compare(base.size() - suf.size(), suf.size(), suf) == 0) {
    base = base.substr(0, base.size() - suf.size());
    *batch = true;
  }
  if (base == "matmul_q4k") return RRR_Q4_K;
  if (base == "matmul_q5k") return RRR_Q5_K;
  if (base == "matmul_q6k") return RRR_Q6_K;
  return 0;
}

// Validates one dispatch; when `run` is set, launches it on `stream`.
int run_named(rrr_ctx* ctx, const char* cname, void* const* b, const uint64_t* sz, int nb,
              const void* push, int push_bytes, void* stream, bool run) {
  if (!cname) return set_error(ctx, RRR_ERR_INVALID_ARG, "dispatch: null name");
  const std::string name(cname);
  auto need = [&](int nbuf, int npush) -> int {
    if (nb != nbuf || !b || !sz)
      return set_error(ctx, RRR_ERR_INVALID_ARG, "%s: expects %d buffers, got %d", cname, nbuf, nb);
    for (int i = 0; i < nbuf; ++i)
      if (!b[i]) return set_error(ctx, RRR_ERR_INVALID_ARG, "%s: binding %d is null", cname, i);
    if (push_bytes != 4 * npush || (npush && !push))
      return set_error(ctx, RRR_ERR_INVALID_ARG, "%s: expects %d push bytes, got %d", cname,
                       4 * npush, push_bytes);
    return RRR_OK;
  };
  auto small = [&](int i, uint64_t want) -> bool { return sz[i] < want; };
  int rc;
  bool batch = false;
  const int qt = kq_from_name(name, &batch);
  if (qt) {
    if (!batch) {
      if ((rc = need(3, 2))) return rc;
      const uint32_t K = push_u32(push, 0), N = push_u32(push, 1);
      const uint64_t wb = (uint64_t)N * (K / 256) * (qt == RRR_Q4_K ? 144 : qt == RRR_Q5_K ? 176 : 210);
      if (small(0, 4ull * K) || small(1, wb) || small(2, 4ull * N))
        return set_error(ctx, RRR_ERR_BUFFER_TOO_SMALL, "%s: binding smaller than [K, N] = [%u, %u] needs",
                         cname, K, N);
      if (!run) return RRR_OK;
      return rrr_gemv_kq(ctx, qt, b[1], static_cast<const float*>(b[0]), static_cast<float*>(b[2]),
                         (int)K, (int)N, nullptr, stream);
    }
    if ((rc = need(3, 3))) return rc;
    const uint32_t K = push_u32(push, 0), N = push_u32(push, 1), M = push_u32(push, 2);
    const uint64_t wb = (uint64_t)N * (K / 256) * (qt == RRR_Q4_K ? 144 : qt == RRR_Q5_K ? 176 : 210);
    if (small(0, 2ull * M * K) || small(1, wb) || small(2, 4ull * M * N))
      return set_error(ctx, RRR_ERR_BUFFER_TOO_SMALL, "%s: binding smaller than [K, N, M] needs", cname);
    if (!run) return RRR_OK;
    return rrr_gemm_kq_batched(ctx, qt, b[1], static_cast<const uint16_t*>(b[0]),
                               static_cast<float*>(b[2]), (int)M, (int)K, (int)N, stream);
  }
  if (name == "rmsnorm") {
    if ((rc = need(3, 2))) return rc;
    const uint32_t rows = push_u32(push, 0), d = push_u32(push, 1);
    if (small(0, 4ull * rows * d) || small(1, 4ull * d) || small(2, 4ull * rows * d))
      return set_error(ctx, RRR_ERR_BUFFER_TOO_SMALL, "rmsnorm: binding smaller than [rows, d] needs");
    if (!run) return RRR_OK;
    return rrr_rmsnorm(ctx, static_cast<const float*>(b[0]), static_cast<const float*>(b[1]),
                       static_cast<float*>(b[2]), (int)rows, (int)d, 1e-5f, stream);
  }
  if (name == "matmul_tiled" || name == "matmul_reg_tiled") {
    if ((rc = need(3, 3))) return rc;
    const uint32_t M = push_u32(push, 0), K = push_u32(push, 1), N = push_u32(push, 2);
    if (small(0, 4ull * M * K) || small(1, 4ull * K * N) || small(2, 4ull * M * N))
      return set_error(ctx, RRR_ERR_BUFFER_TOO_SMALL, "%s: binding smaller than [M, K, N] needs", cname);
    if (!run) return RRR_OK;
    return rrr_matmul_f32(ctx, static_cast<const float*>(b[0]), static_cast<const float*>(b[1]),
                          static_cast<float*>(b[2]), (int)M, (int)K, (int)N, stream);
  }
  if (name == "silu_gate") {
    if ((rc = need(2, 1))) return rc;
    const uint32_t F = push_u32(push, 0);
    if (small(0, 8ull * F) || small(1, 4ull * F))
      return set_error(ctx, RRR_ERR_BUFFER_TOO_SMALL, "silu_gate: binding smaller than [F] needs");
    if (!run) return RRR_OK;
    return rrr_silu_gate(ctx, static_cast<const float*>(b[0]), static_cast<float*>(b[1]), (int)F, stream);
  }
  if (name == "residual_add") {
    if ((rc = need(3, 1))) return rc;
    const uint32_t n = push_u32(push, 0);
    if (small(0, 4ull * n) || small(1, 4ull * n) || small(2, 4ull * n))
      return set_error(ctx, RRR_ERR_BUFFER_TOO_SMALL, "residual_add: binding smaller than [n] needs");
    if (!run) return RRR_OK;
    return rrr_residual_add(ctx, static_cast<const float*>(b[0]), static_cast<const float*>(b[1]),
                            static_cast<float*>(b[2]), (int)n, stream);
  }
  if (name.rfind("matmul_gpuq", 0) == 0 || name.rfind("fused_norm_matmul", 0) == 0)
    return set_error(ctx, RRR_ERR_UNSUPPORTED,
                     "%s: repacked / fused-norm shader layouts are not provided; upload raw GGUF "
                     "blocks and use matmul_q{4,5,6}k (or rrr_gemv_kq_ex with RRR_X_RMSNORM)", cname);
  if (name == "rope_kv_store") {
    // push [pos, n_heads, n_kv_heads, head_dim, rope_dim, q_dim, kv_stride], bindings
    // [qkv, rope_factors, kbuf, vbuf] (phi4.rs:1115-1117, 1016-1017). The push carries no
    // theta / attention factor: the reference's constants ROPE_THETA and ROPE_ATTN_FACTOR
    // (phi4.rs:115-116) apply, and the factor table is the whole rope_factors binding.
    if ((rc = need(4, 7))) return rc;
    rrr_attn_desc a{};
    const uint32_t pos = push_u32(push, 0);
    a.n_heads = (int)push_u32(push, 1);
    a.n_kv_heads = (int)push_u32(push, 2);
    a.head_dim = (int)push_u32(push, 3);
    a.rope_dim = (int)push_u32(push, 4);
    const uint32_t q_dim = push_u32(push, 5), kv_stride = push_u32(push, 6);
    if (q_dim != (uint32_t)(a.n_heads * a.head_dim) || kv_stride != (uint32_t)(a.n_kv_heads * a.head_dim) ||
        kv_stride == 0)
      return set_error(ctx, RRR_ERR_BAD_SHAPE, "rope_kv_store: q_dim / kv_stride disagree with the heads");
    a.rope_theta = 10000.0f;
    a.rope_attn_factor = 1.190238f;
    a.rope_factors = static_cast<const float*>(b[1]);
    a.n_rope_factors = (int)(sz[1] / 4);
    a.max_seq = (int)(sz[2] / (2ull * kv_stride));
    if (small(0, 4ull * (q_dim + 2ull * kv_stride)) || sz[3] < sz[2] || pos >= (uint32_t)a.max_seq)
      return set_error(ctx, RRR_ERR_BUFFER_TOO_SMALL, "rope_kv_store: binding smaller than the push needs");
    if (!run) return RRR_OK;
    return rrr_rope_kv_store(ctx, &a, static_cast<float*>(b[0]), q_dim + 2ll * kv_stride, 1, (int)pos,
                             nullptr, static_cast<uint16_t*>(b[2]), static_cast<uint16_t*>(b[3]), stream);
  }
  if (name == "kv_store") {
    // push [pos, q_dim, kv_stride], bindings [qkv, kbuf, vbuf] (phi4.rs:1663-1677): K and
    // V of the QKV row (after RoPE) rounded to f16 into cache row pos
    if ((rc = need(3, 3))) return rc;
    const uint32_t pos = push_u32(push, 0), q_dim = push_u32(push, 1), kv_stride = push_u32(push, 2);
    if (kv_stride == 0 || kv_stride % 2)
      return set_error(ctx, RRR_ERR_BAD_SHAPE, "kv_store: kv_stride must be even and > 0");
    if (small(0, 4ull * (q_dim + 2ull * kv_stride)) || small(1, 2ull * (pos + 1) * kv_stride) ||
        small(2, 2ull * (pos + 1) * kv_stride))
      return set_error(ctx, RRR_ERR_BUFFER_TOO_SMALL, "kv_store: binding smaller than the push needs");
    if ((reinterpret_cast<uintptr_t>(b[1]) | reinterpret_cast<uintptr_t>(b[2])) & 3)
      return set_error(ctx, RRR_ERR_MISALIGNED, "kv_store: caches must be 4-byte aligned");
    if (!run) return RRR_OK;
    if ((rc = bind_device(ctx))) return rc;
    // one "head" of kv_stride values, no rotation
    cudaError_t e = launch_rope_kv_store(make_env(ctx, stream), static_cast<float*>(b[0]) + q_dim,
                                         q_dim + 2ll * kv_stride, 1, (int)pos, nullptr, 0, 1,
                                         (int)kv_stride, 0, 1.f, 1.f, nullptr, 0,
                                         static_cast<uint16_t*>(b[1]), static_cast<uint16_t*>(b[2]),
                                         (int)pos + 1);
    return e == cudaSuccess ? RRR_OK : cuda_error(ctx, e, "kv_store launch");
  }
  if (name == "attention") {
    // push [seq_len, n_kv_heads, heads_per_kv, head_dim], bindings [q, kbuf, vbuf, out],
    // one query row (phi4.rs:1118-1121, 1680-1688)
    if ((rc = need(4, 4))) return rc;
    rrr_attn_desc a{};
    const uint32_t seq = push_u32(push, 0);
    a.n_kv_heads = (int)push_u32(push, 1);
    a.n_heads = (int)(push_u32(push, 1) * push_u32(push, 2));
    a.head_dim = (int)push_u32(push, 3);
    a.max_seq = (int)seq;
    const uint64_t qn = (uint64_t)a.n_heads * a.head_dim, kvn = (uint64_t)seq * a.n_kv_heads * a.head_dim;
    if (seq == 0 || small(0, 4 * qn) || small(1, 2 * kvn) || small(2, 2 * kvn) || small(3, 4 * qn))
      return set_error(ctx, RRR_ERR_BUFFER_TOO_SMALL, "attention: binding smaller than the push needs");
    if (!run) return RRR_OK;
    return rrr_attention_f16kv(ctx, &a, static_cast<const float*>(b[0]), (int64_t)qn, 1, (int)seq - 1,
                               nullptr, static_cast<const uint16_t*>(b[1]),
                               static_cast<const uint16_t*>(b[2]), static_cast<float*>(b[3]), stream);
  }
  if (name == "rope" || name == "layer_norm" || name == "gelu" || name == "add")
    return set_error(ctx, RRR_ERR_UNSUPPORTED, "%s: outside the weight path; not provided", cname);
  return set_error(ctx, RRR_ERR_INVALID_ARG, "unknown dispatch name '%s'", cname);
}

}  // namespace

struct rrr_batch {
  rrr_ctx* ctx = nullptr;
  std::vector<Op> ops;
  cudaGraphExec_t exec = nullptr;
  cudaGraph_t graph = nullptr;
  cudaStream_t capture_stream = nullptr;
};

extern "C" {

int rrr_dispatch_by_name(rrr_ctx* ctx, const char* name, void* const* buffers,
                         const uint64_t* sizes, int n_buffers, const void* push, int push_bytes,
                         void* stream) {
  if (!ctx) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context");
  return run_named(ctx, name, buffers, sizes, n_buffers, push, push_bytes, stream, true);
}

int rrr_batch_create(rrr_ctx* ctx, rrr_batch** out) {
  if (!ctx) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context");
  if (!out) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_batch_create: null output");
  *out = new rrr_batch();
  (*out)->ctx = ctx;
  return RRR_OK;
}

int rrr_batch_add(rrr_batch* bt, const char* name, void* const* buffers, const uint64_t* sizes,
                  int n_buffers, const void* push, int push_bytes) {
  if (!bt) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null batch");
  int rc = run_named(bt->ctx, name, buffers, sizes, n_buffers, push, push_bytes, nullptr, false);
  if (rc) return rc;
  Op op;
  op.name = name;
  op.bufs.assign(buffers, buffers + n_buffers);
  op.sizes.assign(sizes, sizes + n_buffers);
  if (push_bytes > 0)
    op.push.assign(static_cast<const uint8_t*>(push), static_cast<const uint8_t*>(push) + push_bytes);
  bt->ops.push_back(std::move(op));
  if (bt->exec) {  // the table changed: capture again on the next launch
    cudaGraphExecDestroy(bt->exec);
    cudaGraphDestroy(bt->graph);
    bt->exec = nullptr;
    bt->graph = nullptr;
  }
  return RRR_OK;
}

int rrr_batch_launch(rrr_batch* bt, void* stream) {
  if (!bt) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null batch");
  rrr_ctx* ctx = bt->ctx;
  int rc = bind_device(ctx);
  if (rc) return rc;
  if (!bt->exec) {
    if (!bt->capture_stream) {
      cudaError_t e = cudaStreamCreateWithFlags(&bt->capture_stream, cudaStreamNonBlocking);
      if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_batch_launch: stream");
    }
    cudaError_t e = cudaStreamBeginCapture(bt->capture_stream, cudaStreamCaptureModeRelaxed);
    if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_batch_launch: begin capture");
    int first_rc = RRR_OK;
    // byte ranges written by the dispatches so far (a single-token GEMV writes its output
    // binding; every binding of any other dispatch counts as written)
    std::vector<std::pair<const char*, const char*>> written;
    auto overlaps = [&](const void* p, uint64_t n) {
      const char* a = static_cast<const char*>(p);
      for (const auto& w : written)
        if (a < w.second && w.first < a + n) return true;
      return false;
    };
    for (const Op& op : bt->ops) {
      bool batch = false;
      const int qt = kq_from_name(op.name, &batch);
      const uint32_t K = qt && !batch ? push_u32(op.push.data(), 0) : 0;
      const uint32_t N = qt && !batch ? push_u32(op.push.data(), 1) : 0;
      if (qt && !batch &&
          check_gemv(ctx, qt, op.bufs[1], static_cast<const float*>(op.bufs[0]),
                     static_cast<float*>(op.bufs[2]), (int)K, (int)N, nullptr, nullptr, false) == RRR_OK) {
        const bool early = !overlaps(op.bufs[0], 4ull * K);
        cudaError_t e2 = launch_gemv_kq(make_env(ctx, bt->capture_stream), qt, op.bufs[1],
                                        static_cast<const float*>(op.bufs[0]),
                                        static_cast<float*>(op.bufs[2]), (int)K, (int)N, nullptr,
                                        nullptr, nullptr, early);
        if (e2 == cudaSuccess) e2 = cudaGetLastError();
        if (e2 != cudaSuccess && !first_rc) first_rc = cuda_error(ctx, e2, "rrr_batch_launch: GEMV");
        const char* y = static_cast<const char*>(op.bufs[2]);
        written.emplace_back(y, y + 4ull * N);
        continue;
      }
      rc = run_named(ctx, op.name.c_str(), op.bufs.data(), op.sizes.data(), (int)op.bufs.size(),
                     op.push.empty() ? nullptr : op.push.data(), (int)op.push.size(),
                     bt->capture_stream, true);
      if (rc && !first_rc) first_rc = rc;
      for (size_t i = 0; i < op.bufs.size(); ++i) {
        const char* b = static_cast<const char*>(op.bufs[i]);
        written.emplace_back(b, b + op.sizes[i]);
      }
    }
    cudaGraph_t g = nullptr;
    e = cudaStreamEndCapture(bt->capture_stream, &g);
    if (first_rc) {
      if (g) cudaGraphDestroy(g);
      return first_rc;
    }
    if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_batch_launch: end capture");
    e = cudaGraphInstantiate(&bt->exec, g, 0);
    if (e != cudaSuccess) {
      cudaGraphDestroy(g);
      return cuda_error(ctx, e, "rrr_batch_launch: instantiate");
    }
    bt->graph = g;
  }
  cudaError_t e = cudaGraphLaunch(bt->exec, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_batch_launch: graph launch");
  return RRR_OK;
}

int rrr_batch_size(rrr_batch* bt, int* n) {
  if (!bt || !n) return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_batch_size: null argument");
  *n = (int)bt->ops.size();
  return RRR_OK;
}

int rrr_batch_destroy(rrr_batch* bt) {
  if (!bt) return RRR_OK;
  bind_device(bt->ctx);
  if (bt->exec) cudaGraphExecDestroy(bt->exec);
  if (bt->graph) cudaGraphDestroy(bt->graph);
  if (bt->capture_stream) cudaStreamDestroy(bt->capture_stream);
  delete bt;
  return RRR_OK;
}

}  // extern "C"
