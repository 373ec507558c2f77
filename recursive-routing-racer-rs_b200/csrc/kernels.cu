// kernels.cu — the non-GEMV kernels of the weight path:
//   * bit-exact K-quant dequantisation (reference dequant_q{4,5,6}_k, phi4.rs:444-542);
//   * kernel (3) RMSNorm, one 256-thread CTA per row (reference `rmsnorm` shader,
//     README "256-thread parallel reduction", CPU form phi4.rs:593-599);
//   * kernel (4) F32 logits GEMV over a row-major [V, K] matrix with the output RMSNorm
//     fused into its prologue (reference logits chunks, phi4.rs:866-893, 1049-1064);
//   * decode glue: silu_gate, residual_add (phi4.rs:601-610), greedy argmax
//     (phi4.rs:1172-1183), the f32 matmul_tiled GEMM (ops.rs:65-84);
//   * seeded synthetic data generators (splitmix64; identical bytes to the oracle's).
#include <algorithm>

#include "internal.h"
#include "kquant.cuh"

namespace rrr {
namespace {

// ------------------------------------------------------------------ dequant
template <int QT>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ w,
                                                      float* __restrict__ out, int64_t n_blocks) {
  for (int64_t b = blockIdx.x; b < n_blocks; b += gridDim.x) {
    const uint8_t* blk = w + b * KQ<QT>::kBlockBytes;
    out[b * 256 + threadIdx.x] = kq_dequant_elem<QT>(blk, threadIdx.x);
  }
}

// ------------------------------------------------------------------ rmsnorm
__device__ __forceinline__ float block_sum_256(float v, float* sh) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sh[w] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) t += sh[i];
  return t;
}

__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* __restrict__ x,
                                                      const float* __restrict__ gamma,
                                                      float* __restrict__ y, int d, float eps) {
  __shared__ float sh[8];
  pdl_launch_dependents();
  pdl_wait();
  const float* xr = x + (int64_t)blockIdx.x * d;
  float* yr = y + (int64_t)blockIdx.x * d;
  float ss = 0.f;
  for (int i = threadIdx.x; i < d; i += 256) ss += xr[i] * xr[i];
  const float tot = block_sum_256(ss, sh);
  // inv_rms = 1 / sqrt(sum_sq / n + eps); out = (w * x) * inv_rms (phi4.rs:596-598)
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)d), eps)));
  for (int i = threadIdx.x; i < d; i += 256) yr[i] = __fmul_rn(__fmul_rn(gamma[i], xr[i]), inv);
}

// ------------------------------------------------------------------ logits (f32 GEMV)
// Persistent CTAs of 8 warps; each warp owns 4 rows at a time and streams them with
// 16-B vector loads (evict-first); the normalised x lives in shared memory.
constexpr int kLogitRowsPerWarp = 4;

__global__ void __launch_bounds__(256) logits_f32_kernel(const float* __restrict__ W,
                                                         const float* __restrict__ x,
                                                         float* __restrict__ y, int V, int K,
                                                         const float* __restrict__ gamma,
                                                         float eps) {
  extern __shared__ __align__(16) float xs[];
  __shared__ float sh[8];
  pdl_launch_dependents();
  pdl_wait();
  float inv = 1.f;
  if (gamma) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < K; i += 256) ss += x[i] * x[i];
    const float tot = block_sum_256(ss, sh);
    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), eps)));
  }
  for (int i = threadIdx.x; i < K; i += 256)
    xs[i] = gamma ? __fmul_rn(__fmul_rn(gamma[i], x[i]), inv) : x[i];
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K4 = K >> 2;
  const float4* xs4 = reinterpret_cast<const float4*>(xs);
  const int groups = (V + kLogitRowsPerWarp - 1) / kLogitRowsPerWarp;
  for (int grp = blockIdx.x * 8 + warp; grp < groups; grp += gridDim.x * 8) {
    const int r0 = grp * kLogitRowsPerWarp;
    const float4* wr[kLogitRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kLogitRowsPerWarp; ++r)
      wr[r] = reinterpret_cast<const float4*>(W + (int64_t)min(r0 + r, V - 1) * K);
    float acc[kLogitRowsPerWarp] = {0.f, 0.f, 0.f, 0.f};
    int i = lane;
    for (; i + 96 < K4; i += 128) {
      float4 wv[4][kLogitRowsPerWarp];
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int r = 0; r < kLogitRowsPerWarp; ++r) wv[u][r] = __ldcs(wr[r] + i + 32 * u);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4 xv = xs4[i + 32 * u];
#pragma unroll
        for (int r = 0; r < kLogitRowsPerWarp; ++r)
          acc[r] += wv[u][r].x * xv.x + wv[u][r].y * xv.y + wv[u][r].z * xv.z + wv[u][r].w * xv.w;
      }
    }
    for (; i < K4; i += 32) {
      const float4 xv = xs4[i];
#pragma unroll
      for (int r = 0; r < kLogitRowsPerWarp; ++r) {
        const float4 wv = __ldcs(wr[r] + i);
        acc[r] += wv.x * xv.x + wv.y * xv.y + wv.z * xv.z + wv.w * xv.w;
      }
    }
#pragma unroll
    for (int r = 0; r < kLogitRowsPerWarp; ++r) {
      const float v = warp_sum(acc[r]);
      if (lane == 0 && r0 + r < V) y[r0 + r] = v;
    }
  }
}

// ------------------------------------------------------------------ glue
__global__ void silu_gate_kernel(const float* __restrict__ gu, float* __restrict__ out, int F) {
  pdl_launch_dependents();
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < F; i += gridDim.x * blockDim.x) {
    const float g = gu[i];
    const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
    out[i] = __fmul_rn(s, gu[F + i]);
  }
}

__global__ void residual_add_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                    float* out, int n) {
  pdl_launch_dependents();
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[i] = __fadd_rn(a[i], b[i]);
}

// Order-preserving key of a float for an unsigned max (NaN handled by the caller); ties
// resolve to the smallest index through the complemented index in the low half.
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  if (v == 0.f) v = 0.f;  // -0 and +0 compare equal in the reference's scan
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (uint32_t)(~(uint32_t)idx);
}

// Greedy argmax: first maximum wins, NaN is skipped (reference scan
// `if src[j] > best_val`, phi4.rs:1172-1183); index 0 when nothing compares greater than
// -inf. Each CTA reduces its range to one order-preserving key and folds it into `key`
// with an atomic max (order-independent, so the result is deterministic); the last CTA to
// finish (counter) converts the key to the index and resets key and counter to zero for
// the next call.
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ x, int n,
                                                      int* __restrict__ out,
                                                      unsigned long long* key,
                                                      unsigned int* counter) {
  __shared__ unsigned long long sh[32];
  __shared__ bool last;
  pdl_launch_dependents();
  pdl_wait();
  unsigned long long best = 0ull;
  for (int i = blockIdx.x * 1024 + threadIdx.x; i < n; i += gridDim.x * 1024) {
    const float v = x[i];
    if (v == v && v > -INFINITY) {
      const unsigned long long k = argmax_key(v, i);
      best = k > best ? k : best;
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
      if (best) atomicMax(key, best);
      __threadfence();
      last = atomicAdd(counter, 1u) == gridDim.x - 1;
    }
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    const unsigned long long k = atomicExch(key, 0ull);
    *out = k ? (int)(~(uint32_t)(k & 0xFFFFFFFFull)) : 0;
    atomicExch(counter, 0u);
  }
}

// Greedy argmax of each of `rows` rows (row r at x + r * ld, n values), one CTA per row:
// the same order-preserving keys as argmax_kernel (first maximum wins, NaN skipped, index
// 0 when nothing compares greater than -inf), reduced in the CTA without atomics.
__global__ void __launch_bounds__(1024) argmax_rows_kernel(const float* __restrict__ x, int n,
                                                           long long ld, int* __restrict__ out) {
  __shared__ unsigned long long sh[32];
  pdl_launch_dependents();
  pdl_wait();
  const float* row = x + (long long)blockIdx.x * ld;
  unsigned long long best = 0ull;
  for (int i = threadIdx.x; i < n; i += 1024) {
    const float v = row[i];
    if (v == v && v > -INFINITY) {
      const unsigned long long k = argmax_key(v, i);
      best = k > best ? k : best;
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
    if (threadIdx.x == 0) out[blockIdx.x] = best ? (int)(~(uint32_t)(best & 0xFFFFFFFFull)) : 0;
  }
}

// C[M,N] = A[M,K] B[K,N], B row-major [K, N] (the reference's transposed chunk layout).
__global__ void matmul_f32_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                  float* __restrict__ C, int M, int K, int N) {
  pdl_launch_dependents();
  pdl_wait();
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = blockIdx.y;
  if (n >= N || m >= M) return;
  const float* a = A + (int64_t)m * K;
  float acc = 0.f;
  for (int k = 0; k < K; ++k) acc += a[k] * B[(int64_t)k * N + n];
  C[(int64_t)m * N + n] = acc;
}

// ------------------------------------------------------------------ generators
__device__ __forceinline__ uint64_t splitmix64(uint64_t& s) {
  uint64_t z = (s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ uint32_t f32_to_f16_rne(float f) {
  const uint32_t x = __float_as_uint(f);
  const uint32_t sign = (x >> 16) & 0x8000u, exp = (x >> 23) & 0xFFu, man = x & 0x7FFFFFu;
  if (exp == 0xFF) return sign | 0x7C00u | (man ? (0x200u | (man >> 13)) : 0u);
  const int e = (int)exp - 127 + 15;
  if (e >= 31) return sign | 0x7C00u;
  if (e <= 0) {
    if (e < -10) return sign;
    const uint32_t mm = man | 0x800000u;
    const int shift = 14 - e;
    uint32_t m = mm >> shift;
    const uint32_t rem = mm & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (m & 1u))) m++;
    return sign | m;
  }
  uint32_t h = sign | ((uint32_t)e << 10) | (man >> 13);
  const uint32_t rem = man & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return h;
}

// f16 of a value uniform in [1e-4, 1e-2]: lo + u*step with u a 24-bit integer (the same
// binary32 operations as the oracle's generator; no contraction).
__device__ __forceinline__ uint32_t gen_scale_f16(uint64_t r) {
  const float lo = 0x1.a36e2ep-14f, step = 0x1.446738p-31f;
  const float u = (float)(uint32_t)(r >> 40);
  return f32_to_f16_rne(__fadd_rn(lo, __fmul_rn(u, step)));
}

// dst block i = (r, c) of a rows x bpr block grid is generator block
// block0 + r * src_row + c (a row range, or a column window of every row)
template <int QT>
__global__ void fill_kquant_kernel(uint8_t* __restrict__ dst, int64_t n_blocks, int64_t bpr,
                                   int64_t src_row, int64_t block0, uint64_t seed) {
  constexpr int BB = KQ<QT>::kBlockBytes;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_blocks;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t gi = block0 + (i / bpr) * src_row + i % bpr;
    uint64_t s = seed ^ ((uint64_t)gi * 0xD1B54A32D192ED03ull);
    uint8_t buf[BB + 8];
    for (int o = 0; o < BB; o += 8) {
      const uint64_t r = splitmix64(s);
#pragma unroll
      for (int k = 0; k < 8; ++k) buf[o + k] = (uint8_t)(r >> (8 * k));
    }
    if (QT == RRR_Q6_K) {
#pragma unroll
      for (int k = 0; k < 16; ++k) buf[192 + k] = (uint8_t)(int8_t)((int)(buf[192 + k] & 63) - 32);
      const uint32_t d = gen_scale_f16(splitmix64(s));
      buf[208] = (uint8_t)d;
      buf[209] = (uint8_t)(d >> 8);
    } else {
      const uint32_t d = gen_scale_f16(splitmix64(s));
      const uint32_t dm = gen_scale_f16(splitmix64(s));
      buf[0] = (uint8_t)d; buf[1] = (uint8_t)(d >> 8);
      buf[2] = (uint8_t)dm; buf[3] = (uint8_t)(dm >> 8);
    }
    uint8_t* o = dst + i * BB;
    for (int k = 0; k < BB; ++k) o[k] = buf[k];
  }
}

__global__ void fill_f32_kernel(float* __restrict__ dst, int64_t n, int64_t offset, int normal,
                                float a, float b, uint64_t seed) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    uint64_t s = seed ^ ((uint64_t)(offset + i) * 0xD1B54A32D192ED03ull);
    const uint64_t r = splitmix64(s);
    const float u1 = ((float)(uint32_t)(r >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = (float)(uint32_t)(r & 0xFFFFFFu) * (1.0f / 16777216.0f);
    if (normal) {
      const float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
      dst[i] = a + b * z;
    } else {
      dst[i] = a + (b - a) * u2;
    }
  }
}

}  // namespace

// ------------------------------------------------------------------ launchers
cudaError_t launch_dequant_kq(const LaunchEnv& env, int qtype, const void* w, float* out,
                              int64_t n_blocks) {
  if (n_blocks <= 0) return cudaSuccess;
  const int grid = (int)std::min<int64_t>(n_blocks, (int64_t)env.sm_count * 16);
  const uint8_t* src = static_cast<const uint8_t*>(w);
  switch (qtype) {
    case RRR_Q4_K: dequant_kernel<RRR_Q4_K><<<grid, 256, 0, env.stream>>>(src, out, n_blocks); break;
    case RRR_Q5_K: dequant_kernel<RRR_Q5_K><<<grid, 256, 0, env.stream>>>(src, out, n_blocks); break;
    case RRR_Q6_K: dequant_kernel<RRR_Q6_K><<<grid, 256, 0, env.stream>>>(src, out, n_blocks); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm(const LaunchEnv& env, const float* x, const float* gamma, float* y,
                           int rows, int d, float eps) {
  if (rows <= 0) return cudaSuccess;
  return rrr_launch_pdl(rmsnorm_kernel, dim3(rows), dim3(256), 0, env.stream, env.pdl, x, gamma,
                        y, d, eps);
}

cudaError_t launch_logits_f32(const LaunchEnv& env, const float* W, const float* x, float* y,
                              int V, int K, const float* gamma, float eps) {
  if (V <= 0) return cudaSuccess;
  const size_t smem = (size_t)K * sizeof(float);
  static unsigned long long configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured & (1ull << (dev & 63)))) {
    cudaError_t e = cudaFuncSetAttribute(logits_f32_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
    if (e != cudaSuccess) return e;
    configured |= 1ull << (dev & 63);
  }
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, logits_f32_kernel, 256,
                                                                smem);
  if (e != cudaSuccess) return e;
  const int groups = (V + kLogitRowsPerWarp - 1) / kLogitRowsPerWarp;
  const int grid = std::max(1, std::min((groups + 7) / 8, std::max(per_sm, 1) * env.sm_count));
  return rrr_launch_pdl(logits_f32_kernel, dim3(grid), dim3(256), smem, env.stream, env.pdl, W,
                        x, y, V, K, gamma, eps);
}

cudaError_t launch_silu_gate(const LaunchEnv& env, const float* gu, float* out, int F) {
  if (F <= 0) return cudaSuccess;
  const int grid = std::min((F + 255) / 256, env.sm_count * 8);
  return rrr_launch_pdl(silu_gate_kernel, dim3(grid), dim3(256), 0, env.stream, env.pdl, gu, out,
                        F);
}

cudaError_t launch_residual_add(const LaunchEnv& env, const float* a, const float* b,
                                float* out, int n) {
  if (n <= 0) return cudaSuccess;
  const int grid = std::min((n + 255) / 256, env.sm_count * 8);
  return rrr_launch_pdl(residual_add_kernel, dim3(grid), dim3(256), 0, env.stream, env.pdl, a, b,
                        out, n);
}

cudaError_t launch_argmax(const LaunchEnv& env, const float* x, int n, int* out_index,
                          void* scratch) {
  unsigned long long* key = static_cast<unsigned long long*>(scratch);
  unsigned int* counter = reinterpret_cast<unsigned int*>(key + 1);
  const int grid = std::max(1, std::min((n + 4095) / 4096, env.sm_count));
  return rrr_launch_pdl(argmax_kernel, dim3(grid), dim3(1024), 0, env.stream, env.pdl, x, n,
                        out_index, key, counter);
}

cudaError_t launch_argmax_rows(const LaunchEnv& env, const float* x, int n, long long ld,
                               int* out_index, int rows) {
  if (rows <= 0) return cudaSuccess;
  return rrr_launch_pdl(argmax_rows_kernel, dim3(rows), dim3(1024), 0, env.stream, env.pdl, x, n,
                        ld, out_index);
}

cudaError_t launch_matmul_f32(const LaunchEnv& env, const float* A, const float* B, float* C,
                              int M, int K, int N) {
  if (M <= 0 || N <= 0) return cudaSuccess;
  return rrr_launch_pdl(matmul_f32_kernel, dim3((N + 255) / 256, M), dim3(256), 0, env.stream,
                        env.pdl, A, B, C, M, K, N);
}

// An empty kernel launched without programmatic stream serialisation: it starts only once
// every earlier kernel of the stream has completed and its writes are visible. Kernels
// that read weights before their griddepcontrol.wait (the GEMV producers stream weight
// blocks ahead of the dependency wait) may then overlap with this one safely, which they
// could not with a fill kernel that has just written those weights.
__global__ void full_dependency_marker_kernel() {}

cudaError_t end_with_full_dependency(const LaunchEnv& env) {
  full_dependency_marker_kernel<<<1, 32, 0, env.stream>>>();
  return cudaGetLastError();
}

cudaError_t launch_fill_kquant(const LaunchEnv& env, int qtype, void* dst, int64_t rows,
                               int64_t bpr, int64_t src_row, int64_t block0, uint64_t seed) {
  const int64_t n_blocks = rows * bpr;
  if (n_blocks <= 0) return cudaSuccess;
  const int grid = (int)std::min<int64_t>((n_blocks + 127) / 128, (int64_t)env.sm_count * 32);
  uint8_t* d = static_cast<uint8_t*>(dst);
  switch (qtype) {
    case RRR_Q4_K:
      fill_kquant_kernel<RRR_Q4_K><<<grid, 128, 0, env.stream>>>(d, n_blocks, bpr, src_row, block0, seed);
      break;
    case RRR_Q5_K:
      fill_kquant_kernel<RRR_Q5_K><<<grid, 128, 0, env.stream>>>(d, n_blocks, bpr, src_row, block0, seed);
      break;
    case RRR_Q6_K:
      fill_kquant_kernel<RRR_Q6_K><<<grid, 128, 0, env.stream>>>(d, n_blocks, bpr, src_row, block0, seed);
      break;
    default: return cudaErrorInvalidValue;
  }
  const cudaError_t e = cudaGetLastError();
  return e != cudaSuccess ? e : end_with_full_dependency(env);
}

cudaError_t launch_fill_f32(const LaunchEnv& env, float* dst, int64_t n, int64_t offset,
                            int normal, float a, float b, uint64_t seed) {
  if (n <= 0) return cudaSuccess;
  const int grid = (int)std::min<int64_t>((n + 255) / 256, (int64_t)env.sm_count * 32);
  fill_f32_kernel<<<grid, 256, 0, env.stream>>>(dst, n, offset, normal, a, b, seed);
  const cudaError_t e = cudaGetLastError();
  return e != cudaSuccess ? e : end_with_full_dependency(env);
}

}  // namespace rrr
