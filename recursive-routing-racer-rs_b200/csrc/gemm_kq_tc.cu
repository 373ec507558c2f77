// gemm_kq_tc.cu — kernel (2): batched-token K-quant GEMM on the tcgen05 tensor cores,
// Y[M,N] = X[M,K] · W[N,K]^T with W in raw GGUF Q4_K / Q5_K / Q6_K super-blocks and X bf16.
// Replaces the `matmul_gpuq{4,5,6}_batch` dispatches of the reference's batched prefill
// (push [K, N, M], one workgroup per (row, token): src/model/phi4.rs:1257-1268,
// 1346-1357, 1380-1391).
//
// One CTA computes a 128-row x TN-token tile of Y^T (TN <= 256 tokens, a multiple of 16)
// over a contiguous range of K super-blocks (split-K when the tile grid is smaller than
// the GPU):
//   warp 0     raw producer: per super-block, one 1-D bulk copy (cp.async.bulk, no
//              multicast) of each weight row's raw block into a two-stage raw ring.
//   warp 1     allocates the TMEM accumulator (128 lanes x TN f32 columns); one thread
//              issues 4 tcgen05.mma.kind::f16 (bf16 x bf16 -> f32, K = 16 each) per chunk
//              and tcgen05.commit's each ring slot back to its producers.
//   warp 2     X producer: per 64-wide K chunk, one TMA tile load of X[m0:m0+TN, k:k+64]
//              (bf16, 128-byte swizzle) into the B ring.
//   warps 3-10 dequantise each 64-wide chunk of the raw blocks to bf16 directly into the
//              A ring in the K-major 128-byte-swizzled layout the MMA reads (the same layout
//              the TMA writes for X), then run the epilogue: tcgen05.ld of the accumulator
//              and coalesced f32 stores. With split-K the CTAs of one tile form a
//              thread-block cluster and sum their partial tiles over distributed shared
//              memory in split order (deterministic, no workspace).
// All mbarrier waits are bounded (about one second); a wait that gives up records an error
// in the context's device flag and the CTA stops issuing work, waits for its copies in
// flight, frees its TMEM and returns.
//
// Dequantised weights are rounded once to bf16 (the MMA operand type) from an f32 value
// q*(d*scale) - dmin*min; the result is within the tensor-core tolerance (1e-2 relative L2),
// not bit-exact (the exact dequant lives in kquant.cuh and rrr_dequant_kq).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <string.h>

#include <mutex>

#include "internal.h"
#include "kquant.cuh"
#include "rrr_common.cuh"
#include "tile_common.cuh"

namespace rrr {
namespace {

constexpr int kBM = 128;              // weight rows per tile = MMA M = TMEM lanes
constexpr int kBK = 64;               // K per ring slot: one 128-byte swizzle row of bf16
constexpr int kThreads = 352;         // 11 warps
constexpr int kDqThreads = 256;       // warps 3..10
constexpr int kMaxRawStages = 4;
constexpr int kABytes = kBM * kBK * 2;  // 16 KB per A slot
constexpr int kMaxSplits = 8;         // portable cluster size
constexpr int kMaxKbs = 4;            // super-blocks per raw stage
constexpr int kSmemBudget = 232448;   // 227 KB opt-in maximum on sm_100

constexpr int kDevErrTcWait = kDevErrTileWait;

struct TcParams {
  const uint8_t* w;
  const uint8_t* w_end;
  float* y;
  const float* residual;  // optional [M, N] f32 added in the epilogue (may equal y)
  long long row_bytes;
  int M, K, N, nb, bb;  // nb super-blocks per row, bb bytes per super-block
  int tn, splits, stages, slot, tmem_cols, n_tiles;
  int raw_stages;       // depth of the raw-block ring (2..4)
  int kbs;              // super-blocks per raw stage (per row); `slot` = its row pitch
  int raw_tma;          // 1: one 2-D TMA box per raw stage (rows 16-byte aligned)
  uint32_t off_b, off_raw, off_bar;  // byte offsets from the 1024-aligned smem base
  uint32_t idesc;
  int* err;
};

// ---- tcgen05 primitives: tile_common.cuh -------------------------------------------

// ---- dequantisation of one 64-wide K chunk: 32 values per thread ---------------------
// Thread half h handles l in [16h, 16h+16) of the two 32-element runs of the chunk and
// writes the bf16 words of K positions [16h, 16h+16) to out[0..7] and
// [32+16h, 32+16h+16) to out[8..15].

// ---- dequantisation: half a super-block (chunks 2u, 2u+1) per call -------------------
// Thread H (0/1) of a weight row produces K positions [32H, 32H+32) of each 64-wide
// chunk: out[16*jj + 0..15] for chunk 2u+jj (16-byte chunks 4H..4H+3 of the row).

template <int QT> struct TcDq;

// Q4_K: chunk j = qs bytes [32j, 32j+32); nibble H is sub-block 2j+H; value
// q*(d*sc) - dmin*m (phi4.rs:481-510).
template <> struct TcDq<RRR_Q4_K> {
  template <int H>
  static __device__ __forceinline__ void half(const uint8_t* blk, int u, uint32_t* out) {
    const uint4 hd = *reinterpret_cast<const uint4*>(blk);
    const float d = f16_bits_to_f32(hd.x & 0xFFFFu), dmin = f16_bits_to_f32(hd.x >> 16);
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int j = 2 * u + jj;
      float sv, mv;
      scale_min_w(hd.y, hd.z, hd.w, 2 * j + H, sv, mv);
      const RunScale sc = run_scale(d * sv, dmin * mv);
      const uint4 q0 = *reinterpret_cast<const uint4*>(blk + 16 + 32 * j);
      const uint4 q1 = *reinterpret_cast<const uint4*>(blk + 16 + 32 * j + 16);
      const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
        emit4((qw[i] >> (4 * H)) & 0x0F0F0F0Fu, sc, out + 16 * jj + 2 * i);
    }
  }
};

// Q5_K: as Q4_K plus the fifth bit, bit s of qh[l] for sub-block s (phi4.rs:512-542).
template <> struct TcDq<RRR_Q5_K> {
  template <int H>
  static __device__ __forceinline__ void half(const uint8_t* blk, int u, uint32_t* out) {
    const uint4 hd = *reinterpret_cast<const uint4*>(blk);
    const float d = f16_bits_to_f32(hd.x & 0xFFFFu), dmin = f16_bits_to_f32(hd.x >> 16);
    const uint4 h0 = *reinterpret_cast<const uint4*>(blk + 16);
    const uint4 h1 = *reinterpret_cast<const uint4*>(blk + 32);
    const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int j = 2 * u + jj, sb = 2 * j + H;
      float sv, mv;
      scale_min_w(hd.y, hd.z, hd.w, sb, sv, mv);
      const RunScale sc = run_scale(d * sv, dmin * mv);
      const uint4 q0 = *reinterpret_cast<const uint4*>(blk + 48 + 32 * j);
      const uint4 q1 = *reinterpret_cast<const uint4*>(blk + 48 + 32 * j + 16);
      const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t v = ((qw[i] >> (4 * H)) & 0x0F0F0F0Fu) | (((hw[i] >> sb) & 0x01010101u) << 4);
        emit4(v, sc, out + 16 * jj + 2 * i);
      }
    }
  }
};

// Q6_K: chunks 2u, 2u+1 are half g = u of the block; chunk 2u+jj holds runs k = 2jj
// (K positions 0-31) and 2jj+1 (32-63), so thread H takes run k = 2jj+H: nibble jj of
// ql[64g + 32H + l], bits 2k of qh[32g + l], scale index e/16 = 8g + 2k + l/16; value
// (d*scale) * (q - 32) (phi4.rs:444-479). `blk` is only 2-byte aligned.
template <> struct TcDq<RRR_Q6_K> {
  template <int H>
  static __device__ __forceinline__ void half(const uint8_t* blk, int u, uint32_t* out) {
    uint32_t ql[8], qh[8];
    ld16_a2(blk + 64 * u + 32 * H, ql);
    ld16_a2(blk + 64 * u + 32 * H + 16, ql + 4);
    ld16_a2(blk + 128 + 32 * u, qh);
    ld16_a2(blk + 128 + 32 * u + 16, qh + 4);
    const float d = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(blk + 208));
    const int8_t* scp = reinterpret_cast<const int8_t*>(blk + 192 + 8 * u);
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int k = 2 * jj + H;
      const float a0 = d * (float)scp[2 * k], a1 = d * (float)scp[2 * k + 1];
      const RunScale sc0 = run_scale(a0, 32.f * a0), sc1 = run_scale(a1, 32.f * a1);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t v = ((ql[i] >> (4 * jj)) & 0x0F0F0F0Fu) | (((qh[i] >> (2 * k)) & 0x03030303u) << 4);
        emit4(v, i < 4 ? sc0 : sc1, out + 16 * jj + 2 * i);
      }
    }
  }
};

// The dequantisation warps' loop: thread (row r, half H) over the CTA's super-blocks.
template <int QT, int H>
__device__ __forceinline__ void dequant_rows(const TcParams& p, int r, int n0, int kb0, int n_blk,
                                             uint8_t* sA, const uint8_t* sRaw,
                                             uint32_t raw_stage_bytes, uint64_t* full,
                                             uint64_t* empty, uint64_t* raw_full,
                                             uint64_t* raw_empty, volatile int* abort_flag) {
  const int lane = threadIdx.x & 31;
  const int S = p.stages, R = p.raw_stages;
  const bool row_ok = n0 + r < p.N;
  uint32_t soff[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) soff[c] = sw128_off(r, 4 * H + c);
  const int n_st = (n_blk + p.kbs - 1) / p.kbs;
  for (int st = 0; st < n_st; ++st) {
    if (warp_aborted(abort_flag)) return;
    const int rs = st % R;
    if (!warp_wait(&raw_full[rs], (st / R) & 1, p.err)) {
      *abort_flag = 1;
      return;
    }
    const uint8_t* row = sRaw + rs * raw_stage_bytes + r * p.slot;
    const long long off = (long long)(n0 + r) * p.row_bytes + (long long)(kb0 + st * p.kbs) * p.bb;
    const uint8_t* row0 = row + (reinterpret_cast<uintptr_t>(p.w + off) & 15);
    const int nk = min(p.kbs, n_blk - st * p.kbs);
    for (int kk = 0; kk < nk; ++kk) {
    const int blk = st * p.kbs + kk;
    const uint8_t* bp = row0 + kk * p.bb;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      uint32_t out[32];
      if (row_ok) {
        TcDq<QT>::template half<H>(bp, u, out);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) out[i] = 0u;
      }
      const int it = 4 * blk + 2 * u;
      const int s0 = it % S, s1 = (it + 1) % S;
      if ((it >= S && !warp_wait(&empty[s0], ((it / S) - 1) & 1, p.err)) ||
          (it + 1 >= S && !warp_wait(&empty[s1], (((it + 1) / S) - 1) & 1, p.err))) {
        *abort_flag = 1;
        return;
      }
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        uint8_t* a = sA + (jj ? s1 : s0) * kABytes;
        const uint32_t* o = out + 16 * jj;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          *reinterpret_cast<uint4*>(a + soff[c]) = make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&full[s0]);
        mbar_arrive(&full[s1]);
        if (u == 1 && kk == nk - 1) mbar_arrive(&raw_empty[rs]);
      }
    }
    }
  }
}

// ---- the kernel ---------------------------------------------------------------------

template <int QT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kq_tc_kernel(const __grid_constant__ CUtensorMap xmap,
                      const __grid_constant__ CUtensorMap wmap, const TcParams p) {
  extern __shared__ uint8_t smem_dyn[];
  // 1024-byte-aligned base (the swizzle pattern is a function of the address bits);
  // derived from smem_dyn by pointer arithmetic so that accesses stay shared-space
  uint8_t* smem = smem_dyn + ((1024u - (smem_addr(smem_dyn) & 1023u)) & 1023u);
  const int S = p.stages;
  uint8_t* sA = smem;
  uint8_t* sB = smem + p.off_b;
  uint8_t* sRaw = smem + p.off_raw;
  // ring slot s = A tile (dequantised weights) + B tile (X); full[s] completes with the
  // 8 dequantisation warps' arrivals and the X tile's TMA bytes, empty[s] with the MMAs'
  // commit
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  uint64_t* empty = full + S;
  uint64_t* raw_full = empty + S;
  const int R = p.raw_stages;
  uint64_t* raw_empty = raw_full + R;
  uint64_t* acc_full = raw_empty + R;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBM, m0 = blockIdx.y * p.tn, z = blockIdx.z;
  const int kb0 = (int)((long long)z * p.nb / p.splits);
  const int kb1 = (int)((long long)(z + 1) * p.nb / p.splits);
  const int n_chunks = 4 * (kb1 - kb0);
  const uint32_t b_bytes = (uint32_t)p.tn * 128u;
  const uint32_t raw_stage_bytes = (uint32_t)kBM * (uint32_t)p.slot;  // slot = row pitch

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], kDqThreads / 32 + 1);
      mbar_init(&empty[s], 1);
    }
    for (int r = 0; r < R; ++r) {
      mbar_init(&raw_full[r], 1);
      mbar_init(&raw_empty[r], kDqThreads / 32);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, (uint32_t)p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Programmatic dependent launch: the next grid may be scheduled now; every global
  // access of this one comes after the previous grid's results are visible.
  pdl_launch_dependents();
  pdl_wait();

  if (warp == 0) {
    // ---------------- raw-block producer: runs up to R super-blocks ahead
    const int n_blk = kb1 - kb0;
    int n_raw = 0;
    const int n_st = (n_blk + p.kbs - 1) / p.kbs;
    for (int st = 0; st < n_st; ++st) {
      if (warp_aborted(abort_flag)) break;
      const int r = st % R;
      if (st >= R && !warp_wait(&raw_empty[r], ((st / R) - 1) & 1, p.err)) {
        *abort_flag = 1;
        break;
      }
      uint8_t* dst_stage = sRaw + r * raw_stage_bytes;
      const long long kb = kb0 + st * p.kbs;
      const int nk = min(p.kbs, n_blk - st * p.kbs);
      if (p.raw_tma) {
        // one box of 128 rows x `slot` bytes from the 16-byte-aligned envelope of blocks
        // kb.. (rows past N and bytes past the row end are zero-filled by the TMA unit;
        // bytes past the stage's blocks are not used)
        if (lane == 0) {
          mbar_arrive_expect_tx(&raw_full[r], raw_stage_bytes);
          tma_load_2d(dst_stage, &wmap, (int)(((kb * p.bb) & ~15ll) >> 3), n0, &raw_full[r]);
        }
        __syncwarp();
        ++n_raw;
        continue;
      }
      // rows not 16-byte aligned: one 1-D bulk copy per row
      const uint8_t* srcs[4];
      uint32_t lens[4];
      uint32_t tot = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = lane + 32 * i, n = n0 + row;
        lens[i] = 0;
        srcs[i] = nullptr;
        if (n < p.N) {
          const uint8_t* src = p.w + (long long)n * p.row_bytes + kb * p.bb;
          const uint8_t* a0 = reinterpret_cast<const uint8_t*>(
              reinterpret_cast<uintptr_t>(src) & ~(uintptr_t)15);
          const uint8_t* end = src + (long long)nk * p.bb;
          uint32_t len = (uint32_t)((end - a0 + 15) & ~15);
          if (a0 + len > p.w_end) {
            // the 16-byte envelope would read past the weights: copy the aligned part
            // and the few tail bytes with plain loads
            len = (uint32_t)((p.w_end - a0) & ~15);
            for (const uint8_t* t = a0 + len; t < end; ++t)
              dst_stage[row * p.slot + (t - a0)] = *t;
          }
          srcs[i] = a0;
          lens[i] = len;
          tot += len;
        }
      }
      tot = __reduce_add_sync(0xffffffffu, tot);
      __syncwarp();
      if (lane == 0) mbar_arrive_expect_tx(&raw_full[r], tot);
      __syncwarp();
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (lens[i]) bulk_g2s(dst_stage + (lane + 32 * i) * p.slot, srcs[i], lens[i], &raw_full[r]);
      ++n_raw;
    }
    // copies still in flight (only after an abort) must land before the CTA exits
    for (int r = 0; r < R; ++r) {
      const int cnt = n_raw > r ? (n_raw - r + R - 1) / R : 0;
      if (cnt) warp_wait(&raw_full[r], (cnt - 1) & 1, p.err);
    }
  } else if (warp == 2) {
    // ---------------- X-tile producer (TMA)
    int n_b = 0;
    for (int it = 0; it < n_chunks; ++it) {
      if (warp_aborted(abort_flag)) break;
      const int s = it % S;
      if (it >= S && !warp_wait(&empty[s], ((it / S) - 1) & 1, p.err)) {
        *abort_flag = 1;
        break;
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[s], b_bytes);
        tma_load_2d(sB + s * b_bytes, &xmap, kb0 * 256 + it * kBK, m0, &full[s]);
      }
      __syncwarp();
      ++n_b;
    }
    for (int s = 0; s < S; ++s) {
      // (after an abort the slot's phase may lack the dequantisation arrivals: the bounded
      // wait then gives up, long after the TMA bytes have landed)
      const int cnt = n_b > s ? (n_b - s + S - 1) / S : 0;
      if (cnt) warp_wait(&full[s], (cnt - 1) & 1, p.err);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      for (int it = 0; it < n_chunks; ++it) {
        if (*abort_flag) break;
        const int sa = it % S, sb = sa;
        if (!mbar_wait_bounded(&full[sa], (uint32_t)(it / S) & 1u, p.err, kDevErrTcWait)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_addr(sA + sa * kABytes), b0 = smem_addr(sB + sb * b_bytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          umma_bf16(tmem, sw128_desc(a0 + 32 * kk), sw128_desc(b0 + 32 * kk), p.idesc,
                    (it | kk) != 0);
        umma_commit(&empty[sa]);
      }
      umma_commit(acc_full);
    }
    __syncwarp();
  } else {
    // ---------------- dequantisation: a super-block per iteration, in two halves of two
    // chunks; warps 3-6 produce K positions [0, 32) of every chunk, warps 7-10 [32, 64)
    const int t = threadIdx.x - 96;
    const int h = t >> 7, r = t & 127;
    if (h == 0)
      dequant_rows<QT, 0>(p, r, n0, kb0, kb1 - kb0, sA, sRaw, raw_stage_bytes, full, empty,
                          raw_full, raw_empty, abort_flag);
    else
      dequant_rows<QT, 1>(p, r, n0, kb0, kb1 - kb0, sA, sRaw, raw_stage_bytes, full, empty,
                          raw_full, raw_empty, abort_flag);

    // ---------------- epilogue: TMEM -> registers -> Y (one split) or the CTA's partial
    // tile in shared memory (split-K, summed across the cluster below)
    const bool got_acc = warp_wait(acc_full, 0, p.err);
    const bool have_acc = got_acc && !warp_aborted(abort_flag);
    tc_fence_after();
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int n = n0 + row;
    const int half = (warp - 3) >> 2;
    const int cw = p.tn >> 1;
    float* part = reinterpret_cast<float*>(smem);  // [tn][128], over the drained rings
    if (have_acc) {
      for (int c = half * cw; c < (half + 1) * cw; c += 8) {
        uint32_t v[8];
        tmem_ld8(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c, v);
        if (p.splits == 1) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int m = m0 + c + i;
            if (m < p.M && n < p.N) {
              const size_t o = (size_t)m * p.N + n;
              const float r = p.residual ? p.residual[o] : 0.f;
              p.y[o] = __uint_as_float(v[i]) + r;
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) part[(c + i) * kBM + row] = __uint_as_float(v[i]);
        }
      }
    }
  }

  tc_fence_before();
  if (p.splits > 1) {
    // Split-K: the S CTAs of a tile form one cluster (ranks = blockIdx.z). After every
    // partial tile is in shared memory, CTA c sums token columns [c*per, (c+1)*per) of all
    // S partial tiles over distributed shared memory, in rank order (deterministic), and
    // writes them to Y; the second cluster barrier keeps every tile alive until all reads
    // are done.
    cluster_sync();
    if (warp >= 3) {
      const int t = threadIdx.x - 96;
      const int per = (p.tn + p.splits - 1) / p.splits;
      const int j0 = z * per, j1 = min(p.tn, j0 + per);
      const float* part = reinterpret_cast<const float*>(smem);
      for (int idx = t; idx < (j1 - j0) * (kBM / 4); idx += kDqThreads) {
        const int j = j0 + idx / (kBM / 4), r4 = (idx % (kBM / 4)) * 4;
        const uint32_t la = smem_addr(part + j * kBM + r4);
        float4 acc = ld_dsmem_f4(la, 0);
        for (int s = 1; s < p.splits; ++s) {
          const float4 v = ld_dsmem_f4(la, (uint32_t)s);
          acc.x += v.x;
          acc.y += v.y;
          acc.z += v.z;
          acc.w += v.w;
        }
        const int m = m0 + j, nn = n0 + r4;
        if (m < p.M) {
          float* dst = p.y + (size_t)m * p.N + nn;
          const float* res = p.residual ? p.residual + (size_t)m * p.N + nn : nullptr;
          if ((p.N & 3) == 0 && nn + 3 < p.N) {
            if (res) {
              const float4 r4 = *reinterpret_cast<const float4*>(res);
              acc.x += r4.x;
              acc.y += r4.y;
              acc.z += r4.z;
              acc.w += r4.w;
            }
            *reinterpret_cast<float4*>(dst) = acc;
          } else {
            const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
            for (int e = 0; e < 4 && nn + e < p.N; ++e) dst[e] = a4[e] + (res ? res[e] : 0.f);
          }
        }
      }
    }
    cluster_sync();
  } else {
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, (uint32_t)p.tmem_cols);
  }
}

// ---- host side ----------------------------------------------------------------------

template <int QT>
cudaError_t launch_t(const LaunchEnv& env, const TcPlan& pl, const void* w, const uint16_t* x,
                     float* y, int M, int K, int N, const float* residual) {
  CUtensorMap map, wmap;
  if (!encode_2d(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)K, (uint64_t)M,
                 (uint64_t)K * 2, (uint32_t)kBK, (uint32_t)pl.tn, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  const long long row_bytes = (long long)(K / 256) * KQ<QT>::kBlockBytes;
  memset(&wmap, 0, sizeof wmap);
  if (pl.raw_tma &&
      !encode_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT64, w, (uint64_t)row_bytes / 8, (uint64_t)N,
                 (uint64_t)row_bytes, (uint32_t)raw_slot_bytes(QT, pl.kbs) / 8, (uint32_t)kBM,
                 CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;

  TcParams p{};
  p.w = static_cast<const uint8_t*>(w);
  p.bb = KQ<QT>::kBlockBytes;
  p.nb = K / 256;
  p.row_bytes = (long long)p.nb * p.bb;
  p.w_end = p.w + p.row_bytes * N;
  p.y = y;
  p.residual = residual;
  p.M = M;
  p.K = K;
  p.N = N;
  p.tn = pl.tn;
  p.splits = pl.splits;
  p.stages = pl.stages;
  p.slot = raw_slot_bytes(QT, pl.kbs);
  p.kbs = pl.kbs;
  p.tmem_cols = pl.tmem_cols;
  p.n_tiles = pl.n_tiles;
  p.off_b = (uint32_t)(pl.stages * kABytes);
  p.off_raw = p.off_b + (uint32_t)(pl.stages * pl.tn * 128);
  p.raw_stages = pl.raw_stages;
  p.raw_tma = pl.raw_tma;
  p.off_bar = p.off_raw + (uint32_t)(pl.raw_stages * kBM * p.slot);
  // instruction descriptor: f32 accumulator (bits 4-5 = 1), A and B bf16 (bits 7-9 and
  // 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 (bits 17-22), M >> 4 (bits 24-28)
  p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(pl.tn >> 3) << 17) |
            ((uint32_t)(kBM >> 4) << 24);
  p.err = env.d_err;

  auto kern = gemm_kq_tc_kernel<QT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.n_tiles, pl.m_tiles, pl.splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = env.stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = pl.splits;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (pl.splits > 1) {
    // clusters are placed per GPC: the plan's split count can need a second wave of
    // clusters (e.g. 24 tiles x 6 splits on 22 resident clusters of 6); take the split
    // count with the fewest waves x K-blocks per CTA
    const int s = pick_splits((const void*)kern, cfg, pl.n_tiles * pl.m_tiles, K / 256, pl.splits);
    p.splits = s;
    cfg.gridDim.z = s;
    attr[0].val.clusterDim.z = s;
  }
  cfg.numAttrs = env.pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, map, wmap, p);
}

}  // namespace

bool plan_gemm_kq_tc(int qtype, int M, int K, int N, int sm_count, TcPlan* pl) {
  if (M < 16 || K < 256 || K % 256 || N < 1 || kq_block_bytes(qtype) == 0) return false;
  TcPlan r{};
  r.m_tiles = (M + 255) / 256;
  r.tn = ((M + r.m_tiles - 1) / r.m_tiles + 15) / 16 * 16;
  r.n_tiles = (N + kBM - 1) / kBM;
  r.tmem_cols = next_pow2_cols(r.tn);
  // the raw ring is one 2-D TMA box per stage when every row starts 16-byte aligned
  // (Q4_K, Q5_K; Q6_K when K/256 is a multiple of 8), else one bulk copy per row
  r.raw_tma = ((long long)(K / 256) * kq_block_bytes(qtype)) % 16 == 0;
  // Shared memory: the A/X ring (3-4 slots of 16 KB + tn x 128 B) and a raw ring of 2+
  // stages of `kbs` super-blocks per row (wider TMA rows stream faster).
  const int per_stage = kABytes + r.tn * 128;
  const int fixed = 1024 + 512;
  r.stages = r.tn > 128 ? 3 : 4;
  r.kbs = 1;
  for (int kbs = kMaxKbs; kbs > 1; kbs >>= 1)
    if (fixed + r.stages * per_stage + 2 * kBM * raw_slot_bytes(qtype, kbs) <= kSmemBudget) {
      r.kbs = kbs;
      break;
    }
  const int raw_stage = kBM * raw_slot_bytes(qtype, r.kbs);
  if (fixed + r.stages * per_stage + 2 * raw_stage > kSmemBudget) return false;
  r.raw_stages = (kSmemBudget - fixed - r.stages * per_stage) / raw_stage;
  if (r.raw_stages > kMaxRawStages) r.raw_stages = kMaxRawStages;
  const int rings = r.stages * per_stage + r.raw_stages * raw_stage;
  r.smem = fixed + rings;
  // one CTA per SM (the launch bounds and the TMEM columns assume it)
  if (r.smem < kSmemBudget / 2 + 1024) r.smem = kSmemBudget / 2 + 1024;
  // split-K when the tile grid leaves SMs idle: a cluster of up to 8 CTAs per tile, each
  // CTA at least 2 super-blocks deep; the partial tile (tn x 128 f32) reuses the drained
  // A/B and raw rings
  const int nb = K / 256;
  const int base = r.n_tiles * r.m_tiles;
  int splits = sm_count > 0 ? sm_count / base : 1;
  if (splits > kMaxSplits) splits = kMaxSplits;
  if (splits > nb / 2) splits = nb / 2;
  if (splits < 1) splits = 1;
  if (splits > 1 && r.tn * kBM * 4 > rings) splits = 1;
  r.splits = splits;
  *pl = r;
  return true;
}

cudaError_t launch_gemm_kq_tc(const LaunchEnv& env, int qtype, const void* w,
                              const uint16_t* x_bf16, float* y, int M, int K, int N,
                              const TcPlan& pl, const float* residual) {
  switch (qtype) {
    case RRR_Q4_K: return launch_t<RRR_Q4_K>(env, pl, w, x_bf16, y, M, K, N, residual);
    case RRR_Q5_K: return launch_t<RRR_Q5_K>(env, pl, w, x_bf16, y, M, K, N, residual);
    case RRR_Q6_K: return launch_t<RRR_Q6_K>(env, pl, w, x_bf16, y, M, K, N, residual);
    default: return cudaErrorNotSupported;
  }
}

}  // namespace rrr
