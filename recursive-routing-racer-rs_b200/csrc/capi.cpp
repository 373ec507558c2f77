// capi.cpp — the C ABI (include/rrr_cuda.h): context, memory, validation and the
// entry points that replace RRR's Vulkan ComputeEngine dispatch API
// (src/gpu/engine.rs:15-29, 200-229, 476-554; src/model/phi4.rs:616-697).
// Nothing here throws or aborts across the ABI: every failure is a negative status with
// a message retrievable through rrr_last_error.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "capi_internal.h"
#include "internal.h"

using namespace rrr;

static thread_local std::string g_noctx_error;

int rrr::set_error(rrr_ctx* ctx, int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (ctx)
    ctx->last_error = buf;
  else
    g_noctx_error = buf;
  return code;
}

int rrr::cuda_error(rrr_ctx* ctx, cudaError_t e, const char* what) {
  if (e == cudaErrorMemoryAllocation)
    return set_error(ctx, RRR_ERR_OOM, "%s: %s", what, cudaGetErrorString(e));
  return set_error(ctx, RRR_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int rrr::bind_device(rrr_ctx* ctx) {
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != ctx->device) {
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return cuda_error(ctx, e, "cudaSetDevice");
  }
  return RRR_OK;
}

LaunchEnv rrr::make_env(rrr_ctx* ctx, void* stream) {
  LaunchEnv env;
  env.stream = static_cast<cudaStream_t>(stream);
  env.sm_count = ctx->sm_count;
  env.d_err = ctx->d_err;
  env.pdl = ctx->pdl;
  if (ctx->trace) {
    env.trace = ctx->trace;
    env.trace_cap = ctx->trace_cap;
    env.trace_next = &ctx->trace_next;
    env.trace_seq = &ctx->trace_seq;
  }
  return env;
}

static inline bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

static inline bool overlap(const void* a, size_t an, const void* b, size_t bn) {
  const char* pa = static_cast<const char*>(a);
  const char* pb = static_cast<const char*>(b);
  return pa < pb + bn && pb < pa + an;
}

#define RRR_CHECK_CTX(ctx)                                                   \
  do {                                                                       \
    if (!(ctx)) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context"); \
  } while (0)

#define RRR_BIND(ctx)                 \
  do {                                \
    int _rc = bind_device(ctx);       \
    if (_rc != RRR_OK) return _rc;    \
  } while (0)

#define RRR_LAUNCH_CHECK(ctx, expr, what)            \
  do {                                               \
    cudaError_t _e = (expr);                         \
    if (_e != cudaSuccess) return cuda_error(ctx, _e, what); \
  } while (0)

namespace rrr {

static int check_qtype(rrr_ctx* ctx, int qtype, const char* fn) {
  if (qtype != RRR_Q4_K && qtype != RRR_Q5_K && qtype != RRR_Q6_K)
    return set_error(ctx, RRR_ERR_BAD_QTYPE,
                     "%s: qtype %d is not a supported K-quant (12=Q4_K, 13=Q5_K, 14=Q6_K)", fn,
                     qtype);
  return RRR_OK;
}

// Bytes of the GEMV input that a prologue mode reads.
static size_t gemv_x_bytes(int K, const rrr_gemv_prologue* pro) {
  const int mode = pro ? pro->mode : RRR_X_PLAIN;
  if (mode == RRR_X_SILU_GATE) return 8 * (size_t)K;
  if (mode == RRR_X_GQA_V)
    return 4 * (size_t)(pro->n_q_heads + 2 * pro->n_kv_heads) * pro->head_dim;
  return 4 * (size_t)K;
}

int check_gemv(rrr_ctx* ctx, int qtype, const void* w, const float* x, float* y, int K, int N,
               const float* residual, const rrr_gemv_prologue* pro, bool swiglu) {
  const char* fn = swiglu ? "rrr_gemv_kq_swiglu" : "rrr_gemv_kq";
  int rc = check_qtype(ctx, qtype, fn);
  if (rc) return rc;
  if (!w || !x || !y) return set_error(ctx, RRR_ERR_INVALID_ARG, "%s: null pointer", fn);
  if (K < 256 || K % 256 != 0 || K > kGemvMaxK || N < 1)
    return set_error(ctx, RRR_ERR_BAD_SHAPE,
                     "%s: need K %% 256 == 0, 256 <= K <= %d, %s >= 1 (K=%d %s=%d)", fn,
                     kGemvMaxK, swiglu ? "F" : "N", K, swiglu ? "F" : "N", N);
  const int mode = pro ? pro->mode : RRR_X_PLAIN;
  if (swiglu && (mode != RRR_X_PLAIN && mode != RRR_X_RMSNORM))
    return set_error(ctx, RRR_ERR_INVALID_ARG, "%s: prologue must be PLAIN or RMSNORM", fn);
  if (swiglu && residual)
    return set_error(ctx, RRR_ERR_INVALID_ARG, "%s: no residual with the SwiGLU epilogue", fn);
  if (!aligned(w, 16) || !aligned(x, 16) || !aligned(y, 4) || (residual && !aligned(residual, 4)))
    return set_error(ctx, RRR_ERR_MISALIGNED,
                     "%s: W and x must be 16-byte aligned, y/residual 4-byte aligned", fn);
  if (mode == RRR_X_RMSNORM) {
    if (!pro->gamma)
      return set_error(ctx, swiglu ? RRR_ERR_MISALIGNED : RRR_ERR_INVALID_ARG,
                       "%s: RMSNORM needs gamma", fn);
    if (!aligned(pro->gamma, 16))
      return set_error(ctx, RRR_ERR_MISALIGNED, "%s: gamma must be 16-byte aligned", fn);
  } else if (mode == RRR_X_GQA_V) {
    const int nq = pro->n_q_heads, nkv = pro->n_kv_heads, hd = pro->head_dim;
    const int ko = pro->k_offset;
    if (nq <= 0 || nkv <= 0 || hd <= 0 || nq % nkv != 0 || hd % 8 != 0 || ko < 0 || ko % 8 != 0 ||
        ko + nq * hd > K)
      return set_error(ctx, RRR_ERR_BAD_SHAPE,
                       "%s: GQA_V needs n_q %% n_kv == 0, head_dim %% 8 == 0, "
                       "k_offset %% 8 == 0 and k_offset + n_q*head_dim <= K "
                       "(n_q=%d n_kv=%d hd=%d k_offset=%d K=%d)", fn, nq, nkv, hd, ko, K);
  } else if (mode != RRR_X_PLAIN && mode != RRR_X_SILU_GATE) {
    return set_error(ctx, RRR_ERR_INVALID_ARG, "%s: unknown prologue mode %d", fn, mode);
  }
  if (overlap(y, (size_t)N * 4, x, gemv_x_bytes(K, pro)))
    return set_error(ctx, RRR_ERR_INVALID_ARG, "%s: y must not overlap the input", fn);
  if (residual && residual != y && overlap(y, (size_t)N * 4, residual, (size_t)N * 4))
    return set_error(ctx, RRR_ERR_INVALID_ARG, "%s: residual must equal y or not overlap it", fn);
  return RRR_OK;
}

}  // namespace rrr

extern "C" {

int rrr_abi_version(void) { return RRR_ABI_VERSION; }

const char* rrr_status_string(int s) {
  switch (s) {
    case RRR_OK: return "RRR_OK";
    case RRR_ERR_INVALID_ARG: return "RRR_ERR_INVALID_ARG";
    case RRR_ERR_BAD_QTYPE: return "RRR_ERR_BAD_QTYPE";
    case RRR_ERR_BAD_SHAPE: return "RRR_ERR_BAD_SHAPE";
    case RRR_ERR_MISALIGNED: return "RRR_ERR_MISALIGNED";
    case RRR_ERR_CUDA: return "RRR_ERR_CUDA";
    case RRR_ERR_NCCL: return "RRR_ERR_NCCL";
    case RRR_ERR_TIMEOUT: return "RRR_ERR_TIMEOUT";
    case RRR_ERR_OOM: return "RRR_ERR_OOM";
    case RRR_ERR_UNSUPPORTED: return "RRR_ERR_UNSUPPORTED";
    case RRR_ERR_IO: return "RRR_ERR_IO";
    case RRR_ERR_BUFFER_TOO_SMALL: return "RRR_ERR_BUFFER_TOO_SMALL";
    default: return "RRR_ERR_UNKNOWN";
  }
}

const char* rrr_last_error(rrr_ctx* ctx) {
  return ctx ? ctx->last_error.c_str() : g_noctx_error.c_str();
}

int rrr_init(int device, rrr_ctx** out) {
  if (!out) return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_init: null output pointer");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0)
    return set_error(nullptr, RRR_ERR_CUDA, "rrr_init: no CUDA device (%s)",
                     e != cudaSuccess ? cudaGetErrorString(e) : "count is 0");
  if (device < 0 || device >= n)
    return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_init: device %d out of range [0,%d)",
                     device, n);
  e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_error(nullptr, e, "rrr_init: cudaSetDevice");
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return cuda_error(nullptr, e, "rrr_init: cudaGetDeviceProperties");
  if (prop.major != 10)
    return set_error(nullptr, RRR_ERR_UNSUPPORTED,
                     "rrr_init: device %d is sm_%d%d; this library is built for sm_100a only",
                     device, prop.major, prop.minor);
  rrr_ctx* c = new rrr_ctx();
  c->device = device;
  c->sm_count = prop.multiProcessorCount;
  c->pdl = true;
  e = cudaMalloc(&c->d_err, 256);
  if (e != cudaSuccess) {
    delete c;
    return cuda_error(nullptr, e, "rrr_init: cudaMalloc(error flag)");
  }
  cudaMemset(c->d_err, 0, 256);
  e = cudaMalloc(&c->xdig, rrr::i8_scratch_bytes(rrr::kGemvMaxK));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(c->d_err);
    if (c->xdig) cudaFree(c->xdig);
    delete c;
    return cuda_error(nullptr, e, "rrr_init: synchronize");
  }
  *out = c;
  return RRR_OK;
}

int rrr_destroy(rrr_ctx* ctx) {
  RRR_CHECK_CTX(ctx);
  bind_device(ctx);
  cudaDeviceSynchronize();
  if (ctx->d_err) cudaFree(ctx->d_err);
  if (ctx->xdig) cudaFree(ctx->xdig);
  delete ctx;
  return RRR_OK;
}

int rrr_alloc(rrr_ctx* ctx, size_t bytes, void** dptr) {
  RRR_CHECK_CTX(ctx);
  if (!dptr) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_alloc: null output pointer");
  *dptr = nullptr;
  RRR_BIND(ctx);
  cudaError_t e = cudaMalloc(dptr, bytes ? bytes : 1);
  if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_alloc");
  return RRR_OK;
}

int rrr_free(rrr_ctx* ctx, void* dptr) {
  RRR_CHECK_CTX(ctx);
  RRR_BIND(ctx);
  if (!dptr) return RRR_OK;
  RRR_LAUNCH_CHECK(ctx, cudaFree(dptr), "rrr_free");
  return RRR_OK;
}

int rrr_alloc_host(rrr_ctx* ctx, size_t bytes, void** hptr) {
  RRR_CHECK_CTX(ctx);
  if (!hptr) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_alloc_host: null output pointer");
  *hptr = nullptr;
  RRR_BIND(ctx);
  cudaError_t e = cudaMallocHost(hptr, bytes ? bytes : 1);
  if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_alloc_host");
  return RRR_OK;
}

int rrr_free_host(rrr_ctx* ctx, void* hptr) {
  RRR_CHECK_CTX(ctx);
  if (!hptr) return RRR_OK;
  RRR_LAUNCH_CHECK(ctx, cudaFreeHost(hptr), "rrr_free_host");
  return RRR_OK;
}

static int copy(rrr_ctx* ctx, void* dst, const void* src, size_t bytes, cudaMemcpyKind kind,
                void* stream, const char* what) {
  RRR_CHECK_CTX(ctx);
  if (bytes == 0) return RRR_OK;
  if (!dst || !src) return set_error(ctx, RRR_ERR_INVALID_ARG, "%s: null pointer", what);
  RRR_BIND(ctx);
  RRR_LAUNCH_CHECK(ctx, cudaMemcpyAsync(dst, src, bytes, kind, static_cast<cudaStream_t>(stream)),
                   what);
  return RRR_OK;
}

int rrr_h2d(rrr_ctx* ctx, void* dst, const void* src, size_t bytes, void* stream) {
  return copy(ctx, dst, src, bytes, cudaMemcpyHostToDevice, stream, "rrr_h2d");
}
int rrr_d2h(rrr_ctx* ctx, void* dst, const void* src, size_t bytes, void* stream) {
  return copy(ctx, dst, src, bytes, cudaMemcpyDeviceToHost, stream, "rrr_d2h");
}
int rrr_d2d(rrr_ctx* ctx, void* dst, const void* src, size_t bytes, void* stream) {
  return copy(ctx, dst, src, bytes, cudaMemcpyDeviceToDevice, stream, "rrr_d2d");
}

int rrr_memset(rrr_ctx* ctx, void* dst, int value, size_t bytes, void* stream) {
  RRR_CHECK_CTX(ctx);
  if (bytes == 0) return RRR_OK;
  if (!dst) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_memset: null pointer");
  RRR_BIND(ctx);
  RRR_LAUNCH_CHECK(ctx, cudaMemsetAsync(dst, value, bytes, static_cast<cudaStream_t>(stream)),
                   "rrr_memset");
  return RRR_OK;
}

int rrr_sync(rrr_ctx* ctx, void* stream) {
  RRR_CHECK_CTX(ctx);
  RRR_BIND(ctx);
  RRR_LAUNCH_CHECK(ctx, cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "rrr_sync");
  return RRR_OK;
}

int rrr_set_wait_limit(rrr_ctx* ctx, uint64_t ns) {
  RRR_CHECK_CTX(ctx);
  if (ns != 0 && (ns < 100000ull || ns > 60000000000ull))
    return set_error(ctx, RRR_ERR_INVALID_ARG,
                     "rrr_set_wait_limit: %llu ns outside [1e5, 6e10] (0 = the 1 s default)",
                     (unsigned long long)ns);
  RRR_BIND(ctx);
  const unsigned long long v = ns;
  RRR_LAUNCH_CHECK(ctx, cudaMemcpy(ctx->d_err + rrr::kWaitLimitSlot, &v, sizeof v, cudaMemcpyHostToDevice),
                   "rrr_set_wait_limit: write");
  return RRR_OK;
}

int rrr_set_trace(rrr_ctx* ctx, void* buffer, int64_t bytes) {
  RRR_CHECK_CTX(ctx);
  if (buffer && (bytes < 64 || (reinterpret_cast<uintptr_t>(buffer) & 7)))
    return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_set_trace: need an 8-byte aligned buffer of >= 64 bytes");
  ctx->trace = static_cast<unsigned long long*>(buffer);
  ctx->trace_cap = buffer ? bytes / 64 : 0;
  ctx->trace_next = 0;
  ctx->trace_seq = 0;
  return RRR_OK;
}

int rrr_trace_position(rrr_ctx* ctx, int64_t* next_record, int64_t* launches) {
  RRR_CHECK_CTX(ctx);
  if (!next_record || !launches) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_trace_position: null argument");
  *next_record = ctx->trace_next;
  *launches = ctx->trace_seq;
  return RRR_OK;
}

int rrr_check_device_error(rrr_ctx* ctx, int* code) {
  RRR_CHECK_CTX(ctx);
  if (!code) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_check_device_error: null code");
  RRR_BIND(ctx);
  RRR_LAUNCH_CHECK(ctx, cudaDeviceSynchronize(), "rrr_check_device_error: synchronize");
  int v = 0;
  RRR_LAUNCH_CHECK(ctx, cudaMemcpy(&v, ctx->d_err, sizeof v, cudaMemcpyDeviceToHost),
                   "rrr_check_device_error: read");
  RRR_LAUNCH_CHECK(ctx, cudaMemset(ctx->d_err, 0, sizeof v), "rrr_check_device_error: clear");
  *code = v;
  if (v == 6)
    return set_error(ctx, RRR_ERR_BAD_SHAPE,
                     "a kernel met a position outside the KV cache or a token id outside the "
                     "embedding table (device code 6)");
  if (v != 0)
    return set_error(ctx, RRR_ERR_TIMEOUT, "a kernel gave up a bounded wait (device code %d)", v);
  return RRR_OK;
}

int rrr_set_pdl(rrr_ctx* ctx, int enable) {
  RRR_CHECK_CTX(ctx);
  ctx->pdl = enable != 0;
  return RRR_OK;
}

int rrr_device_sm_count(rrr_ctx* ctx, int* sms) {
  RRR_CHECK_CTX(ctx);
  if (!sms) return set_error(ctx, RRR_ERR_INVALID_ARG, "null output");
  *sms = ctx->sm_count;
  return RRR_OK;
}

// ------------------------------------------------------------------ GEMV
int rrr_gemv_kq_ex(rrr_ctx* ctx, int qtype, const void* w, const float* x, float* y, int K,
                   int N, const float* residual, const rrr_gemv_prologue* pro, void* stream) {
  RRR_CHECK_CTX(ctx);
  int rc = check_gemv(ctx, qtype, w, x, y, K, N, residual, pro, false);
  if (rc) return rc;
  RRR_BIND(ctx);
  RRR_LAUNCH_CHECK(ctx, launch_gemv_kq(make_env(ctx, stream), qtype, w, x, y, K, N, residual, pro),
                   "rrr_gemv_kq launch");
  return RRR_OK;
}

int rrr_gemv_kq(rrr_ctx* ctx, int qtype, const void* w, const float* x, float* y, int K, int N,
                const float* residual, void* stream) {
  return rrr_gemv_kq_ex(ctx, qtype, w, x, y, K, N, residual, nullptr, stream);
}

int rrr_gemv_kq_swiglu(rrr_ctx* ctx, int qtype, const void* w, const float* x, float* y, int K,
                       int F, const rrr_gemv_prologue* pro, void* stream) {
  RRR_CHECK_CTX(ctx);
  int rc = check_gemv(ctx, qtype, w, x, y, K, F, nullptr, pro, true);
  if (rc) return rc;
  RRR_BIND(ctx);
  RRR_LAUNCH_CHECK(ctx, launch_gemv_kq_swiglu(make_env(ctx, stream), qtype, w, x, y, K, F, pro),
                   "rrr_gemv_kq_swiglu launch");
  return RRR_OK;
}

int rrr_dequant_kq(rrr_ctx* ctx, int qtype, const void* w, float* out, int64_t n_blocks,
                   void* stream) {
  RRR_CHECK_CTX(ctx);
  int rc = check_qtype(ctx, qtype, "rrr_dequant_kq");
  if (rc) return rc;
  if (n_blocks < 0) return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_dequant_kq: n_blocks < 0");
  if (n_blocks == 0) return RRR_OK;
  if (!w || !out) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_dequant_kq: null pointer");
  if (!aligned(w, 2) || !aligned(out, 4))
    return set_error(ctx, RRR_ERR_MISALIGNED, "rrr_dequant_kq: W 2-byte, out 4-byte aligned");
  RRR_BIND(ctx);
  RRR_LAUNCH_CHECK(ctx, launch_dequant_kq(make_env(ctx, stream), qtype, w, out, n_blocks),
                   "rrr_dequant_kq launch");
  return RRR_OK;
}

int rrr_gemm_kq_batched_ex(rrr_ctx* ctx, int qtype, const void* w, const uint16_t* x, float* y,
                           int M, int K, int N, const float* residual, void* stream) {
  return rrr_gemm_kq_batched_path(ctx, qtype, w, x, y, M, K, N, residual, RRR_GEMM_AUTO, stream);
}

int rrr_gemm_kq_batched_path(rrr_ctx* ctx, int qtype, const void* w, const uint16_t* x, float* y,
                             int M, int K, int N, const float* residual, int path, void* stream) {
  RRR_CHECK_CTX(ctx);
  if (path < RRR_GEMM_AUTO || path > RRR_GEMM_MMA_I8)
    return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_gemm_kq_batched_path: unknown path %d", path);
  int rc = check_qtype(ctx, qtype, "rrr_gemm_kq_batched");
  if (rc) return rc;
  if (!w || !x || !y) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_gemm_kq_batched: null pointer");
  if (M < 1 || N < 1 || K < 256 || K % 256 != 0 || K > kGemvMaxK)
    return set_error(ctx, RRR_ERR_BAD_SHAPE,
                     "rrr_gemm_kq_batched: need M, N >= 1, K %% 256 == 0, 256 <= K <= %d", kGemvMaxK);
  if (!aligned(w, 16) || !aligned(x, 16) || !aligned(y, 16) || (residual && !aligned(residual, 16)))
    return set_error(ctx, RRR_ERR_MISALIGNED, "rrr_gemm_kq_batched: W, X, Y, residual must be 16-byte aligned");
  if (overlap(y, (size_t)M * N * 4, x, (size_t)M * K * 2))
    return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_gemm_kq_batched: Y must not overlap X");
  if (residual && residual != y && overlap(y, (size_t)M * N * 4, residual, (size_t)M * N * 4))
    return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_gemm_kq_batched: residual must equal Y or not overlap it");
  RRR_BIND(ctx);
  const LaunchEnv env = make_env(ctx, stream);
  I8Plan iplan;
  // Automatic choice for short rows (K <= 1024, e.g. the O-projection shard of a 4- or
  // 8-way tensor-parallel split): the integer kernel's 16-token tiles give its grid
  // enough CTAs where the bf16 kernel cannot split K further (measured 7.2 vs 11.8 us at
  // 64 tokens, K = 768).
  const bool auto_i8 = path == RRR_GEMM_AUTO && M >= kMmaMinTokens && K <= 1024;
  if (path == RRR_GEMM_MMA_I8 || (auto_i8 && plan_gemm_kq_i8(qtype, M, K, N, ctx->sm_count, &iplan))) {
    if (!plan_gemm_kq_i8(qtype, M, K, N, ctx->sm_count, &iplan))
      return set_error(ctx, RRR_ERR_BAD_SHAPE,
                       "rrr_gemm_kq_batched_path: the integer mma.sync kernel takes 1 <= M <= 64 "
                       "and rows of a multiple of 16 bytes");
    RRR_LAUNCH_CHECK(ctx, launch_gemm_kq_i8(env, qtype, w, x, y, M, K, N, iplan, residual, ctx->xdig),
                     "rrr_gemm_kq_batched (integer mma.sync) launch");
    return RRR_OK;
  }
  MmaPlan mplan;
  // Automatic choice: the mma.sync kernel from 3 tokens (a 16-token tile with the rows past
  // M zero-filled by the X copy reads each weight once, where one GEMV per token reads the
  // weights M times), the tcgen05 kernel above 64 tokens.
  if ((path == RRR_GEMM_MMA || (path == RRR_GEMM_AUTO && M >= kMmaMinTokens)) &&
      plan_gemm_kq_mma(qtype, M, K, N, ctx->sm_count, &mplan)) {
    RRR_LAUNCH_CHECK(ctx, launch_gemm_kq_mma(env, qtype, w, x, y, M, K, N, mplan, residual),
                     "rrr_gemm_kq_batched (mma.sync) launch");
    return RRR_OK;
  }
  if (path == RRR_GEMM_MMA)
    return set_error(ctx, RRR_ERR_BAD_SHAPE,
                     "rrr_gemm_kq_batched_path: the mma.sync kernel takes 1 <= M <= 64 and rows "
                     "of a multiple of 16 bytes");
  TcPlan plan;
  if ((path == RRR_GEMM_AUTO || path == RRR_GEMM_TCGEN05) && M >= 16 &&
      plan_gemm_kq_tc(qtype, M, K, N, ctx->sm_count, &plan)) {
    RRR_LAUNCH_CHECK(ctx, launch_gemm_kq_tc(env, qtype, w, x, y, M, K, N, plan, residual),
                     "rrr_gemm_kq_batched (tensor cores) launch");
    return RRR_OK;
  }
  if (path == RRR_GEMM_TCGEN05)
    return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_gemm_kq_batched_path: the tcgen05 kernel takes M >= 16");
  for (int m = 0; m < M; ++m)
    RRR_LAUNCH_CHECK(ctx, launch_gemv_kq_bf16(env, qtype, w, x + (size_t)m * K, y + (size_t)m * N, K, N,
                                              residual ? residual + (size_t)m * N : nullptr),
                     "rrr_gemm_kq_batched (per-token) launch");
  return RRR_OK;
}

int rrr_gemm_kq_batched(rrr_ctx* ctx, int qtype, const void* w, const uint16_t* x, float* y,
                        int M, int K, int N, void* stream) {
  return rrr_gemm_kq_batched_ex(ctx, qtype, w, x, y, M, K, N, nullptr, stream);
}

int rrr_rmsnorm(rrr_ctx* ctx, const float* x, const float* gamma, float* y, int rows, int d,
                float eps, void* stream) {
  RRR_CHECK_CTX(ctx);
  if (!x || !gamma || !y) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_rmsnorm: null pointer");
  if (rows < 0 || d < 1) return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_rmsnorm: rows >= 0, d >= 1");
  if (!aligned(x, 4) || !aligned(gamma, 4) || !aligned(y, 4))
    return set_error(ctx, RRR_ERR_MISALIGNED, "rrr_rmsnorm: pointers must be 4-byte aligned");
  if (x != y && overlap(x, (size_t)rows * d * 4, y, (size_t)rows * d * 4))
    return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_rmsnorm: y must equal x or not overlap it");
  RRR_BIND(ctx);
  RRR_LAUNCH_CHECK(ctx, launch_rmsnorm(make_env(ctx, stream), x, gamma, y, rows, d, eps),
                   "rrr_rmsnorm launch");
  return RRR_OK;
}

int rrr_logits_f32(rrr_ctx* ctx, const float* W, const float* x, float* y, int V, int K,
                   int chunk_rows, const float* gamma, float eps, void* stream) {
  RRR_CHECK_CTX(ctx);
  if (!W || !x || !y) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_logits_f32: null pointer");
  if (V < 1 || K < 4 || K % 4 != 0 || K > 16384 || chunk_rows < 0)
    return set_error(ctx, RRR_ERR_BAD_SHAPE,
                     "rrr_logits_f32: need V >= 1, K %% 4 == 0, 4 <= K <= 16384, chunk_rows >= 0");
  if (!aligned(W, 16) || !aligned(x, 4) || !aligned(y, 4) || (gamma && !aligned(gamma, 4)))
    return set_error(ctx, RRR_ERR_MISALIGNED, "rrr_logits_f32: W 16-byte, x/y/gamma 4-byte aligned");
  if (overlap(y, (size_t)V * 4, x, (size_t)K * 4))
    return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_logits_f32: y must not overlap x");
  RRR_BIND(ctx);
  const LaunchEnv env = make_env(ctx, stream);
  const int chunk = chunk_rows > 0 ? chunk_rows : V;
  for (int v0 = 0; v0 < V; v0 += chunk) {
    const int n = chunk < V - v0 ? chunk : V - v0;
    RRR_LAUNCH_CHECK(ctx, launch_logits_f32(env, W + (size_t)v0 * K, x, y + v0, n, K, gamma, eps),
                     "rrr_logits_f32 launch");
  }
  return RRR_OK;
}

int rrr_silu_gate(rrr_ctx* ctx, const float* gu, float* out, int F, void* stream) {
  RRR_CHECK_CTX(ctx);
  if (!gu || !out) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_silu_gate: null pointer");
  if (F < 0) return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_silu_gate: F < 0");
  if (overlap(out, (size_t)F * 4, gu, (size_t)2 * F * 4) && out != gu)
    return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_silu_gate: out overlaps gate_up");
  RRR_BIND(ctx);
  RRR_LAUNCH_CHECK(ctx, launch_silu_gate(make_env(ctx, stream), gu, out, F), "rrr_silu_gate launch");
  return RRR_OK;
}

int rrr_residual_add(rrr_ctx* ctx, const float* a, const float* b, float* out, int n,
                     void* stream) {
  RRR_CHECK_CTX(ctx);
  if (!a || !b || !out) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_residual_add: null pointer");
  if (n < 0) return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_residual_add: n < 0");
  RRR_BIND(ctx);
  RRR_LAUNCH_CHECK(ctx, launch_residual_add(make_env(ctx, stream), a, b, out, n),
                   "rrr_residual_add launch");
  return RRR_OK;
}

int rrr_argmax_f32(rrr_ctx* ctx, const float* x, int n, int* out_index, void* stream) {
  RRR_CHECK_CTX(ctx);
  if (!x || !out_index) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_argmax_f32: null pointer");
  if (n < 1) return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_argmax_f32: n < 1");
  RRR_BIND(ctx);
  RRR_LAUNCH_CHECK(ctx, launch_argmax(make_env(ctx, stream), x, n, out_index, ctx->argmax_scratch()),
                   "rrr_argmax_f32 launch");
  return RRR_OK;
}

int rrr_matmul_f32(rrr_ctx* ctx, const float* A, const float* B, float* C, int M, int K, int N,
                   void* stream) {
  RRR_CHECK_CTX(ctx);
  if (!A || !B || !C) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_matmul_f32: null pointer");
  if (M < 0 || K < 0 || N < 0 || M > 65535)
    return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_matmul_f32: bad shape (M <= 65535)");
  RRR_BIND(ctx);
  RRR_LAUNCH_CHECK(ctx, launch_matmul_f32(make_env(ctx, stream), A, B, C, M, K, N),
                   "rrr_matmul_f32 launch");
  return RRR_OK;
}

int rrr_fill_kquant_random(rrr_ctx* ctx, int qtype, void* dst, int64_t n_blocks, uint64_t seed,
                           void* stream) {
  RRR_CHECK_CTX(ctx);
  int rc = check_qtype(ctx, qtype, "rrr_fill_kquant_random");
  if (rc) return rc;
  if (!dst || n_blocks < 0) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_fill_kquant_random: bad args");
  RRR_BIND(ctx);
  RRR_LAUNCH_CHECK(ctx, launch_fill_kquant(make_env(ctx, stream), qtype, dst, 1, n_blocks,
                                           n_blocks, 0, seed),
                   "rrr_fill_kquant_random launch");
  return RRR_OK;
}

int rrr_fill_kquant_random_2d(rrr_ctx* ctx, int qtype, void* dst, int64_t rows,
                              int64_t blocks_per_row, int64_t src_row_blocks, int64_t block0,
                              uint64_t seed, void* stream) {
  RRR_CHECK_CTX(ctx);
  int rc = check_qtype(ctx, qtype, "rrr_fill_kquant_random_2d");
  if (rc) return rc;
  if (!dst || rows < 0 || blocks_per_row < 0 || src_row_blocks < blocks_per_row || block0 < 0)
    return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_fill_kquant_random_2d: bad args");
  RRR_BIND(ctx);
  if (blocks_per_row == 0) return RRR_OK;
  RRR_LAUNCH_CHECK(ctx, launch_fill_kquant(make_env(ctx, stream), qtype, dst, rows,
                                           blocks_per_row, src_row_blocks, block0, seed),
                   "rrr_fill_kquant_random_2d launch");
  return RRR_OK;
}

int rrr_fill_f32_range(rrr_ctx* ctx, float* dst, int64_t n, int64_t offset, int normal, float a,
                       float b, uint64_t seed, void* stream) {
  RRR_CHECK_CTX(ctx);
  if (!dst || n < 0 || offset < 0)
    return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_fill_f32_range: bad args");
  RRR_BIND(ctx);
  RRR_LAUNCH_CHECK(ctx, launch_fill_f32(make_env(ctx, stream), dst, n, offset, normal ? 1 : 0, a, b, seed),
                   "rrr_fill_f32_range launch");
  return RRR_OK;
}

int rrr_fill_f32_normal(rrr_ctx* ctx, float* dst, int64_t n, float mean, float std, uint64_t seed,
                        void* stream) {
  RRR_CHECK_CTX(ctx);
  if (!dst || n < 0) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_fill_f32_normal: bad args");
  RRR_BIND(ctx);
  RRR_LAUNCH_CHECK(ctx, launch_fill_f32(make_env(ctx, stream), dst, n, 0, 1, mean, std, seed),
                   "rrr_fill_f32_normal launch");
  return RRR_OK;
}

int rrr_fill_f32_uniform(rrr_ctx* ctx, float* dst, int64_t n, float lo, float hi, uint64_t seed,
                         void* stream) {
  RRR_CHECK_CTX(ctx);
  if (!dst || n < 0) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_fill_f32_uniform: bad args");
  RRR_BIND(ctx);
  RRR_LAUNCH_CHECK(ctx, launch_fill_f32(make_env(ctx, stream), dst, n, 0, 0, lo, hi, seed),
                   "rrr_fill_f32_uniform launch");
  return RRR_OK;
}

int rrr_selftest_mma(rrr_ctx* ctx, int* ok) {
  RRR_CHECK_CTX(ctx);
  if (!ok) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_selftest_mma: null output");
  RRR_BIND(ctx);
  int* d = nullptr;
  RRR_LAUNCH_CHECK(ctx, cudaMalloc(&d, sizeof(int)), "rrr_selftest_mma: alloc");
  cudaMemset(d, 0, sizeof(int));
  cudaError_t e = launch_mma_selftest(make_env(ctx, nullptr), d);
  if (e == cudaSuccess) e = cudaMemcpy(ok, d, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(d);
  if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_selftest_mma");
  return RRR_OK;
}

}  // extern "C"
