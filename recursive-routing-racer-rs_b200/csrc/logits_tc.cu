// logits_tc.cu — kernel (4), batched form: F32 logits of M tokens on the tcgen05 tensor
// cores, Y[M, V] = X[M, K] · W[V, K]^T with W the f32 output matrix (row-major [V, K],
// 2.46 GB for Phi-4-mini's 200,064 x 3072). Replaces the logits `matmul_tiled` chunks of
// the batched prefill (src/model/phi4.rs:1408-1434) and of the decode step
// (phi4.rs:1049-1064) when several tokens share one pass over W.
//
// Accuracy: f32 products from three tf32 tensor-core products (3xTF32). Every element of
// W and X is split into big = the element with its 13 low mantissa bits cleared (an
// exact tf32 value) and small = element - big (exact in f32, itself truncated to tf32 by
// the MMA, a relative error of 2^-21 of the element). The tf32 MMA reads an f32 operand
// as exactly that truncation (the low 13 bits are ignored; the parity tests at the f32
// bar pin it), so the staged raw values serve as the big parts and only the remainders
// are written. Y = Wb·Xb + Wb·Xs + Ws·Xb; the
// dropped Ws·Xs term is 2^-22 of the product. The two products that share Wb run as one
// MMA with the B operand [Xb; Xs] stacked along N (N = 2·TN): its first TN columns hold
// Wb·Xb and its last TN columns Wb·Xs; a second MMA (N = TN) computes Ws·Xb into its own
// TN columns. So each 8-deep K step is two MMAs, not three. Consecutive MMAs into one
// accumulator wait for each other, and at these small N that latency, not the tensor
// throughput, would set the pace; so the K steps rotate over `nslot` independent
// accumulator slots of 3·TN columns, and the epilogue adds the 3·nslot partial columns of
// each output in a fixed order (deterministic).
//
// One CTA (persistent, one per SM) takes 128-row tiles of W x TN-token tiles of X in turn,
// through a ring of stages [W | X | Xs] in shared memory plus a 32-column Ws stage in
// tensor memory, one 32-wide K chunk each:
//   warp 0     TMA producer: per chunk one box of W (128 rows x 128 bytes) and one of X
//              (TN rows x 128 bytes), both with the 128-byte swizzle;
//   warps 2-5  split each chunk: Xs next to X, elementwise on the swizzled bytes (so it
//              keeps the layout the MMA reads), and Ws into tensor memory: warp w reads the
//              32 elements of each row of TMEM lane quarter w % 4 from the stage and stores
//              their remainders with one tcgen05.st (Ws never passes through shared memory,
//              which the copies, the split and the MMA operand reads otherwise saturate);
//   warp 1     allocates TMEM (nbuf x nslot accumulator slots of 3·TN f32 columns, then
//              the Ws stages); one thread issues the MMAs (kind::tf32, M = 128, K = 8;
//              Ws·Xb with A from tensor memory) and tcgen05.commit's the three slots of a
//              chunk back and each finished tile to the epilogue;
//   warps 6-9  epilogue: tcgen05.ld of the partial columns, their sum, coalesced stores of
//              Y (32 consecutive vocabulary rows per warp and token); with two accumulator
//              sets (nbuf = 2) the MMAs of the next tile run meanwhile.
// W and X tiles past V / M / K are zero-filled by the TMA unit; their rows are not stored.
// All waits are bounded; a wait that gives up records an error in the context's device
// flag, the CTA stops issuing work, waits for its copies and MMAs in flight, frees its TMEM
// and returns.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <string.h>

#include <algorithm>

#include "internal.h"
#include "rrr_common.cuh"
#include "tile_common.cuh"

namespace rrr {
namespace {

constexpr int kRows = 128;                // W rows per tile = MMA M = TMEM lanes
constexpr int kBK = 32;                   // K per stage: one 128-byte swizzle row of f32
constexpr int kThreads = 320;             // 10 warps
constexpr int kABytes = kRows * kBK * 4;  // 16 KB: one W chunk
constexpr int kMaxStages = 8;
constexpr int kSmemBudget = 232448;       // 227 KB opt-in maximum on sm_100

struct LgParams {
  float* y;
  int M, V, K;
  int tn;                 // tokens per tile (multiple of 16, <= kMaxTokTile)
  int v_tiles, m_tiles, n_k;
  int stages;
  uint32_t stage_bytes;   // [W 16 KB | X tn*128 | Xs tn*128]
  uint32_t off_bar;
  uint32_t idesc_2n, idesc_n;
  uint32_t tmem_cols;
  int nbuf, nslot;        // accumulator sets (1 or 2) x K-step slots per set
  uint32_t a_col0;        // TMEM column of the first Ws stage (32 columns per stage)
  int* err;
};

// small = x - big with big = x with its low 13 mantissa bits cleared (the tf32 value the
// MMA reads for x); the difference is exact.
__device__ __forceinline__ void split4(const float4* x, float4* small) {
  const float4 w = *x;
  float4 h, l;
  h.x = __uint_as_float(__float_as_uint(w.x) & 0xFFFFE000u);
  h.y = __uint_as_float(__float_as_uint(w.y) & 0xFFFFE000u);
  h.z = __uint_as_float(__float_as_uint(w.z) & 0xFFFFE000u);
  h.w = __uint_as_float(__float_as_uint(w.w) & 0xFFFFE000u);
  l.x = __fsub_rn(w.x, h.x);
  l.y = __fsub_rn(w.y, h.y);
  l.z = __fsub_rn(w.z, h.z);
  l.w = __fsub_rn(w.w, h.w);
  *small = l;
}

__global__ void __launch_bounds__(kThreads, 1)
    logits_tc_kernel(const __grid_constant__ CUtensorMap wmap,
                     const __grid_constant__ CUtensorMap xmap, const LgParams p) {
  extern __shared__ uint8_t smem_dyn[];
  // 1024-byte-aligned base (the swizzle pattern is a function of the address bits)
  uint8_t* smem = smem_dyn + ((1024u - (smem_addr(smem_dyn) & 1023u)) & 1023u);
  const int S = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_bar);  // TMA bytes landed
  uint64_t* ready = full + S;                                      // chunk split (4 warps)
  uint64_t* empty = ready + S;                                     // MMAs done with the stage
  uint64_t* acc_full = empty + S;                                  // [nbuf] tile accumulated
  uint64_t* acc_empty = acc_full + 2;                              // [nbuf] tile stored (4 warps)
  uint64_t* fin = acc_empty + 2;                                   // every MMA completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fin + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = p.v_tiles * p.m_tiles;
  const int my_tiles =
      (int)blockIdx.x < n_tiles ? (n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int total = my_tiles * p.n_k;  // K chunks this CTA streams
  const uint32_t b_bytes = (uint32_t)p.tn * 128u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(fin, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Programmatic dependent launch: the next grid may be scheduled now; X (written by the
  // preceding RMSNorm) and Y are touched only after the preceding grid has completed.
  pdl_launch_dependents();
  pdl_wait();

  if (warp == 0) {
    // ---------------- TMA producer
    int issued = 0;
    for (int it = 0; it < total; ++it) {
      if (warp_aborted(abort_flag)) break;
      const int s = it % S;
      if (it >= S && !warp_wait(&empty[s], (uint32_t)((it / S) - 1) & 1u, p.err)) {
        *abort_flag = 1;
        break;
      }
      const int t = (int)blockIdx.x + (it / p.n_k) * (int)gridDim.x;
      const int vt = t % p.v_tiles, mt = t / p.v_tiles;
      const int k = (it % p.n_k) * kBK;
      uint8_t* st = smem + (size_t)s * p.stage_bytes;
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[s], (uint32_t)kABytes + b_bytes);
        tma_load_2d(st, &wmap, k, vt * kRows, &full[s]);
        tma_load_2d(st + kABytes, &xmap, k, mt * p.tn, &full[s]);
      }
      __syncwarp();
      ++issued;
    }
    // copies in flight (only after an abort) must land before the CTA exits
    for (int s = 0; s < S; ++s) {
      const int cnt = issued > s ? (issued - s + S - 1) / S : 0;
      if (cnt) warp_wait(&full[s], (uint32_t)(cnt - 1) & 1u, p.err);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      const uint32_t slot_cols = 3u * (uint32_t)p.tn;
      for (int tl = 0; tl < my_tiles && ok; ++tl) {
        const int b = tl % p.nbuf;
        if (tl >= p.nbuf && !mbar_wait_bounded(&acc_empty[b], (uint32_t)((tl / p.nbuf) - 1) & 1u,
                                               p.err, kDevErrTileWait)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t dset = tmem + (uint32_t)(b * p.nslot) * slot_cols;
        int step = 0;  // K step of the tile
        for (int kc = 0; kc < p.n_k; ++kc, ++it) {
          const int s = it % S;
          if (*abort_flag ||
              !mbar_wait_bounded(&ready[s], (uint32_t)(it / S) & 1u, p.err, kDevErrTileWait)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_addr(smem + (size_t)s * p.stage_bytes);
          const uint32_t bx = a + (uint32_t)kABytes;
          const uint32_t ta = tmem + p.a_col0 + 32u * (uint32_t)s;  // Ws of the stage
#pragma unroll
          for (int kk = 0; kk < kBK / 8; ++kk, ++step) {
            // slot j: [Wb·Xb | Wb·Xs] into its columns [0, 2tn), Ws·Xb into [2tn, 3tn)
            const int j = step % p.nslot;
            const uint32_t d = dset + (uint32_t)j * slot_cols;
            const uint32_t acc = step >= p.nslot ? 1u : 0u;
            umma_tf32(d, sw128_desc(a + 32u * kk), sw128_desc(bx + 32u * kk), p.idesc_2n, acc);
            umma_tf32_ta(d + 2u * (uint32_t)p.tn, ta + 8u * (uint32_t)kk, sw128_desc(bx + 32u * kk),
                         p.idesc_n, acc);
          }
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[b]);
      }
      umma_commit(fin);  // arrives once every MMA issued above has completed
    }
    __syncwarp();
  } else if (warp < 6) {
    // ---------------- remainders (warps 2-5, 128 threads)
    const int t = (int)threadIdx.x - 64;
    for (int it = 0; it < total; ++it) {
      if (warp_aborted(abort_flag)) break;
      const int s = it % S;
      if (!warp_wait(&full[s], (uint32_t)(it / S) & 1u, p.err)) {
        *abort_flag = 1;
        break;
      }
      uint8_t* st = smem + (size_t)s * p.stage_bytes;
      // Ws: row r = 32*(warp % 4) + lane of the swizzled W box (16-byte chunk c at c ^ (r % 8))
      {
        const int r = 32 * (warp & 3) + lane;
        uint32_t u[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 w = *reinterpret_cast<const float4*>(st + r * 128 + ((c ^ (r & 7)) << 4));
          const float wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int i = 0; i < 4; ++i)
            u[4 * c + i] = __float_as_uint(
                __fsub_rn(wv[i], __uint_as_float(__float_as_uint(wv[i]) & 0xFFFFE000u)));
        }
        tmem_st32(tmem + ((uint32_t)(32 * (warp & 3)) << 16) + p.a_col0 + 32u * (uint32_t)s, u);
      }
      const float4* B = reinterpret_cast<const float4*>(st + kABytes);
      float4* Bs = reinterpret_cast<float4*>(st + kABytes + b_bytes);
      for (int i = t; i < (int)(b_bytes / 16); i += 128) split4(B + i, Bs + i);
      tmem_wait_st();
      fence_proxy_async_smem();  // generic-proxy stores -> the tensor core's async proxy
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ready[s]);
    }
  } else {
    // ---------------- epilogue (warps 6-9: TMEM lane quarter warp % 4)
    const int q = warp & 3;
    const uint32_t slot_cols = 3u * (uint32_t)p.tn;
    for (int tl = 0; tl < my_tiles; ++tl) {
      const int b = tl % p.nbuf;
      if (!warp_wait(&acc_full[b], (uint32_t)(tl / p.nbuf) & 1u, p.err)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int t = (int)blockIdx.x + tl * (int)gridDim.x;
      const int vt = t % p.v_tiles, mt = t / p.v_tiles;
      const int v = vt * kRows + q * 32 + lane;
      const uint32_t base =
          tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * p.nslot) * slot_cols;
      for (int c = 0; c < p.tn; c += 8) {
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.f;
        for (int j = 0; j < p.nslot; ++j) {
#pragma unroll
          for (int part = 0; part < 3; ++part) {
            uint32_t u[8];
            tmem_ld8(base + (uint32_t)j * slot_cols + (uint32_t)(part * p.tn + c), u);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], __uint_as_float(u[i]));
          }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int m = mt * p.tn + c + i;
          if (m < p.M && v < p.V) p.y[(size_t)m * p.V + v] = acc[i];
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    // no MMA may still be running when its TMEM is freed
    warp_wait(fin, 0u, p.err);
    tc_fence_after();
    tmem_dealloc(tmem, p.tmem_cols);
  }
}

uint32_t tf32_idesc(int n) {
  // f32 accumulator (bits 4-5 = 1), A and B tf32 (bits 7-9 and 10-12 = 2), both K-major
  // (bits 15, 16 = 0), N >> 3 (bits 17-22), M >> 4 (bits 24-28)
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(kRows >> 4) << 24);
}

}  // namespace

cudaError_t launch_logits_tc(const LaunchEnv& env, const float* W, const float* x, float* y,
                             int M, int V, int K) {
  if (M < 1 || V < 1 || K < 1 || K % 4) return cudaErrorInvalidValue;
  LgParams p{};
  p.y = y;
  p.M = M;
  p.V = V;
  p.K = K;
  p.m_tiles = (M + kMaxTokTile - 1) / kMaxTokTile;
  p.tn = ((M + p.m_tiles - 1) / p.m_tiles + 15) / 16 * 16;
  p.v_tiles = (V + kRows - 1) / kRows;
  p.n_k = (K + kBK - 1) / kBK;
  p.stage_bytes = (uint32_t)kABytes + 2u * (uint32_t)p.tn * 128u;
  const int bar_bytes = 256;
  const int smem_stages = std::min(kMaxStages, (kSmemBudget - 1024 - bar_bytes) / (int)p.stage_bytes);
  // TMEM (512 columns): nbuf sets of nslot slots of 3·tn accumulator columns, then one
  // 32-column Ws stage per ring stage. Two sets (the epilogue of a tile overlaps the next
  // tile's MMAs) when four stages still fit beside them, else one set and more stages.
  // (At 64 tokens, one set of two slots instead of two sets of one measured 835 against
  // 815 µs for the step's logits.)
  const int slot = 3 * p.tn;
  p.nbuf = (512 - 2 * slot) / 32 >= 4 ? 2 : 1;
  p.stages = std::min(smem_stages, (512 - p.nbuf * slot) / 32);
  if (p.stages < 2) return cudaErrorInvalidValue;
  p.nslot = std::max(1, std::min(4, (512 - 32 * p.stages) / (p.nbuf * slot)));
  if (p.nbuf * p.nslot * slot + 32 * p.stages > 512) return cudaErrorInvalidValue;
  p.a_col0 = (uint32_t)(p.nbuf * p.nslot * slot);
  p.tmem_cols = 512;
  p.off_bar = (uint32_t)p.stages * p.stage_bytes;
  const int smem = (int)p.off_bar + bar_bytes + 1024;
  p.idesc_2n = tf32_idesc(2 * p.tn);
  p.idesc_n = tf32_idesc(p.tn);
  p.err = env.d_err;

  CUtensorMap wmap, xmap;
  if (!encode_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, W, (uint64_t)K, (uint64_t)V,
                 (uint64_t)K * 4, (uint32_t)kBK, (uint32_t)kRows, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, x, (uint64_t)K, (uint64_t)M,
                 (uint64_t)K * 4, (uint32_t)kBK, (uint32_t)p.tn, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;

  auto kern = logits_tc_kernel;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  const int grid = std::max(1, std::min(p.v_tiles * p.m_tiles, env.sm_count));
  return rrr_launch_pdl(kern, dim3(grid), dim3(kThreads), (size_t)smem, env.stream, env.pdl,
                        wmap, xmap, p);
}

}  // namespace rrr
