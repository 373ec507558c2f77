// batch_kernels.cu — glue of the batched-token decode step (M tokens at position 0, the
// batched-prefill call sites of the reference, src/model/phi4.rs:1198-1445): the producers
// of the bf16 inputs of rrr_gemm_kq_batched and the batched logits.
//
//   rmsnorm_bf16   y[m] = bf16((gamma * x[m]) * inv_rms(x[m]))        (phi4.rs:593-599)
//   gqa_v_bf16     y[m][k] = bf16(V of head (k - k_offset)/hd's KV group) in the head
//                  window, 0 elsewhere (position-0 attention output, phi4.rs:1120)
//   silu_gate_bf16 y[m][i] = bf16(silu(gate[m][i]) * up[m][i])      (phi4.rs:1359-1378)
//   window_bf16    y[m][k] = bf16(x[m][k - k_offset]) inside the window, 0 outside (the
//                  attention output of a tensor-parallel rank's heads placed in its
//                  O-projection column window)
//   logits         rows normalised in f32, then one GEMM (cuBLAS SGEMM, a plain library
//                  GEMM: W row-major [V, K] times the normalised rows), on the TF32 tensor
//                  cores for 16+ rows (f32 storage and accumulation)
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "capi_internal.h"
#include "rrr_common.cuh"

namespace rrr {
namespace {

__device__ __forceinline__ float block_sum(float v, float* sh) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) sh[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += sh[i];
  __syncthreads();
  return t;
}

__global__ void __launch_bounds__(256) rmsnorm_bf16_kernel(const float* __restrict__ x,
                                                           const float* __restrict__ gamma,
                                                           __nv_bfloat16* __restrict__ y, int d,
                                                           float eps) {
  __shared__ float sh[8];
  pdl_launch_dependents();
  pdl_wait();
  const float* xr = x + (int64_t)blockIdx.x * d;
  __nv_bfloat16* yr = y + (int64_t)blockIdx.x * d;
  float ss = 0.f;
  for (int i = threadIdx.x; i < d; i += 256) ss += xr[i] * xr[i];
  const float tot = block_sum(ss, sh);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)d), eps)));
  for (int i = threadIdx.x; i < d; i += 256)
    yr[i] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(gamma[i], xr[i]), inv));
}

// Vector forms (rows of a multiple of 4 values, 16-byte aligned inputs, 8-byte aligned
// outputs): float4 loads, four bf16 per 8-byte store; the RMSNorm keeps its row slice in
// registers between the sum of squares and the scaling (one pass over global memory).
constexpr int kVecMax = 4;  // float4 per thread of a 256-thread RMSNorm row: d <= 4096

__device__ __forceinline__ uint2 pack_bf16x4(float a, float b, float c, float d) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
  return make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}

__global__ void __launch_bounds__(256) rmsnorm_bf16_vec_kernel(const float* __restrict__ x,
                                                               const float* __restrict__ gamma,
                                                               __nv_bfloat16* __restrict__ y,
                                                               int d, float eps) {
  __shared__ float sh[8];
  pdl_launch_dependents();
  pdl_wait();
  const float4* xr = reinterpret_cast<const float4*>(x + (int64_t)blockIdx.x * d);
  uint2* yr = reinterpret_cast<uint2*>(y + (int64_t)blockIdx.x * d);
  const int n4 = d >> 2;
  float4 v[kVecMax];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kVecMax; ++j) {
    const int i = threadIdx.x + 256 * j;
    v[j] = i < n4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
  }
  const float tot = block_sum(ss, sh);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)d), eps)));
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
#pragma unroll
  for (int j = 0; j < kVecMax; ++j) {
    const int i = threadIdx.x + 256 * j;
    if (i < n4) {
      const float4 g = g4[i];
      yr[i] = pack_bf16x4(__fmul_rn(__fmul_rn(g.x, v[j].x), inv), __fmul_rn(__fmul_rn(g.y, v[j].y), inv),
                          __fmul_rn(__fmul_rn(g.z, v[j].z), inv), __fmul_rn(__fmul_rn(g.w, v[j].w), inv));
    }
  }
}

__device__ __forceinline__ float silu_mul(float a, float u) {
  return __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, expf(-a))), u);
}

__global__ void silu_gate_bf16_vec_kernel(const float* __restrict__ gu,
                                          __nv_bfloat16* __restrict__ y, int F) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.y;
  const float4* g = reinterpret_cast<const float4*>(gu + (int64_t)m * 2 * F);
  const float4* u = reinterpret_cast<const float4*>(gu + (int64_t)m * 2 * F + F);
  uint2* yr = reinterpret_cast<uint2*>(y + (int64_t)m * F);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < (F >> 2); i += gridDim.x * blockDim.x) {
    const float4 a = g[i], b = u[i];
    yr[i] = pack_bf16x4(silu_mul(a.x, b.x), silu_mul(a.y, b.y), silu_mul(a.z, b.z), silu_mul(a.w, b.w));
  }
}

__global__ void gqa_v_bf16_kernel(const float* __restrict__ qkv, __nv_bfloat16* __restrict__ y,
                                  int nq, int nkv, int hd, int kwin, int koff) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.y;
  const int qkv_dim = (nq + 2 * nkv) * hd;
  const float* v = qkv + (int64_t)m * qkv_dim + (nq + nkv) * hd;
  __nv_bfloat16* yr = y + (int64_t)m * kwin;
  const int hpk = nq / nkv;
  for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < kwin; k += gridDim.x * blockDim.x) {
    const int kh = k - koff;
    float val = 0.f;
    if (kh >= 0 && kh < nq * hd) val = v[(kh / hd / hpk) * hd + kh % hd];
    yr[k] = __float2bfloat16_rn(val);
  }
}

__global__ void silu_gate_bf16_kernel(const float* __restrict__ gu, __nv_bfloat16* __restrict__ y,
                                      int F) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.y;
  const float* g = gu + (int64_t)m * 2 * F;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < F; i += gridDim.x * blockDim.x) {
    const float a = g[i];
    const float s = __fdiv_rn(a, __fadd_rn(1.0f, expf(-a)));
    y[(int64_t)m * F + i] = __float2bfloat16_rn(__fmul_rn(s, g[F + i]));
  }
}

__global__ void window_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, int n,
                                   int kwin, int koff) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.y;
  for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < kwin; k += gridDim.x * blockDim.x) {
    const int i = k - koff;
    y[(int64_t)m * kwin + k] = __float2bfloat16_rn(i >= 0 && i < n ? x[(int64_t)m * n + i] : 0.f);
  }
}

}  // namespace


}  // namespace rrr

using namespace rrr;

static int grid_x(int n) { return n < 256 ? 1 : (n + 255) / 256 > 64 ? 64 : (n + 255) / 256; }
static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

extern "C" {

int rrr_rmsnorm_bf16(rrr_ctx* ctx, const float* x, const float* gamma, uint16_t* y, int rows,
                     int d, float eps, void* stream) {
  if (!ctx) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context");
  if (!x || !gamma || !y) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_rmsnorm_bf16: null pointer");
  if (rows < 0 || d < 1) return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_rmsnorm_bf16: rows >= 0, d >= 1");
  int rc = bind_device(ctx);
  if (rc) return rc;
  if (rows == 0) return RRR_OK;
  const LaunchEnv env = make_env(ctx, stream);
  const bool vec = d % 4 == 0 && d <= 1024 * kVecMax && aligned16(x) && aligned16(gamma) &&
                   (reinterpret_cast<uintptr_t>(y) & 7) == 0;
  cudaError_t e = vec ? rrr_launch_pdl(rmsnorm_bf16_vec_kernel, dim3(rows), dim3(256), 0, env.stream,
                                       env.pdl, x, gamma, reinterpret_cast<__nv_bfloat16*>(y), d, eps)
                      : rrr_launch_pdl(rmsnorm_bf16_kernel, dim3(rows), dim3(256), 0, env.stream,
                                       env.pdl, x, gamma, reinterpret_cast<__nv_bfloat16*>(y), d, eps);
  return e == cudaSuccess ? RRR_OK : cuda_error(ctx, e, "rrr_rmsnorm_bf16 launch");
}

int rrr_gqa_v_bf16(rrr_ctx* ctx, const float* qkv, uint16_t* y, int rows, int n_q, int n_kv,
                   int head_dim, int k_window, int k_offset, void* stream) {
  if (!ctx) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context");
  if (!qkv || !y) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_gqa_v_bf16: null pointer");
  if (rows < 0 || n_q < 1 || n_kv < 1 || n_q % n_kv || head_dim < 1 || k_offset < 0 ||
      k_offset + n_q * head_dim > k_window)
    return set_error(ctx, RRR_ERR_BAD_SHAPE,
                     "rrr_gqa_v_bf16: need n_q %% n_kv == 0 and k_offset + n_q*head_dim <= k_window");
  int rc = bind_device(ctx);
  if (rc) return rc;
  if (rows == 0) return RRR_OK;
  const LaunchEnv env = make_env(ctx, stream);
  cudaError_t e = rrr_launch_pdl(gqa_v_bf16_kernel, dim3(grid_x(k_window), rows), dim3(256), 0,
                                 env.stream, env.pdl, qkv, reinterpret_cast<__nv_bfloat16*>(y), n_q,
                                 n_kv, head_dim, k_window, k_offset);
  return e == cudaSuccess ? RRR_OK : cuda_error(ctx, e, "rrr_gqa_v_bf16 launch");
}

int rrr_silu_gate_bf16(rrr_ctx* ctx, const float* gu, uint16_t* y, int rows, int F, void* stream) {
  if (!ctx) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context");
  if (!gu || !y) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_silu_gate_bf16: null pointer");
  if (rows < 0 || F < 1) return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_silu_gate_bf16: rows >= 0, F >= 1");
  int rc = bind_device(ctx);
  if (rc) return rc;
  if (rows == 0) return RRR_OK;
  const LaunchEnv env = make_env(ctx, stream);
  const bool vec = F % 4 == 0 && aligned16(gu) && (reinterpret_cast<uintptr_t>(y) & 7) == 0;
  cudaError_t e = vec ? rrr_launch_pdl(silu_gate_bf16_vec_kernel, dim3(grid_x(F / 4), rows), dim3(256), 0,
                                       env.stream, env.pdl, gu, reinterpret_cast<__nv_bfloat16*>(y), F)
                      : rrr_launch_pdl(silu_gate_bf16_kernel, dim3(grid_x(F), rows), dim3(256), 0,
                                       env.stream, env.pdl, gu, reinterpret_cast<__nv_bfloat16*>(y), F);
  return e == cudaSuccess ? RRR_OK : cuda_error(ctx, e, "rrr_silu_gate_bf16 launch");
}

int rrr_window_bf16(rrr_ctx* ctx, const float* x, uint16_t* y, int rows, int n, int k_window,
                    int k_offset, void* stream) {
  if (!ctx) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context");
  if (!x || !y) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_window_bf16: null pointer");
  if (rows < 0 || n < 1 || k_offset < 0 || k_offset + n > k_window)
    return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_window_bf16: need k_offset + n <= k_window");
  int rc = bind_device(ctx);
  if (rc) return rc;
  if (rows == 0) return RRR_OK;
  const LaunchEnv env = make_env(ctx, stream);
  cudaError_t e = rrr_launch_pdl(window_bf16_kernel, dim3(grid_x(k_window), rows), dim3(256), 0,
                                 env.stream, env.pdl, x, reinterpret_cast<__nv_bfloat16*>(y), n,
                                 k_window, k_offset);
  return e == cudaSuccess ? RRR_OK : cuda_error(ctx, e, "rrr_window_bf16 launch");
}

int rrr_logits_f32_batched(rrr_ctx* ctx, const float* W, const float* x, float* x_norm, float* y,
                           int M, int V, int K, const float* gamma, float eps, void* stream) {
  if (!ctx) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context");
  if (!W || !x || !y || !x_norm)
    return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_logits_f32_batched: null pointer");
  if (M < 1 || V < 1 || K < 1) return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_logits_f32_batched: M, V, K >= 1");
  int rc = bind_device(ctx);
  if (rc) return rc;
  const float* xin = gamma ? x_norm : x;
  if (K % 4 || (reinterpret_cast<uintptr_t>(W) & 15) || (reinterpret_cast<uintptr_t>(xin) & 15))
    return set_error(ctx, RRR_ERR_MISALIGNED,
                     "rrr_logits_f32_batched: K %% 4 == 0 and 16-byte aligned W and GEMM input "
                     "(x_norm with gamma, else x) are required");
  if (gamma) {
    rc = rrr_rmsnorm(ctx, x, gamma, x_norm, M, K, eps, stream);
    if (rc) return rc;
  }
  // 3xTF32 tensor-core kernel (logits_tc.cu): f32-level products, W streamed once per
  // 128-token tile
  const cudaError_t e = launch_logits_tc(make_env(ctx, stream), W, xin, y, M, V, K);
  if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_logits_f32_batched launch");
  return RRR_OK;
}

}  // extern "C"
