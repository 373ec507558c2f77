// gemm_kq_i8.cu — kernel (2), small batches on the integer tensor-core path:
// Y[M,N] = X[M,K] · W[N,K]^T for 1 <= M <= 64 tokens, W raw GGUF Q4_K / Q5_K / Q6_K
// super-blocks, X bf16, Y f32 (the `matmul_gpuq{4,5,6}_batch` dispatches of the batched
// prefill, src/model/phi4.rs:1257-1268, 1346-1357, 1380-1391).
//
// Formulation: the weights are never dequantised. The raw quants are the A operand of
// integer MMAs (u8: Q4_K / Q5_K q in 0..31; s8: Q6_K as 4*(q - 32)), X enters as int8
// digits, and the per-row scales are applied to the s32 results:
//  * X preparation (xdig_kernel, one warp per token and super-block of 256 elements):
//    T = round(x * 2^(14-E)) with 2^E > max|x| of the block, |T| <= 16383, split into two
//    int8 digits T = 128*hi + lo (lo in 0..127); xs = 2^(E-14). |x - xs*T| <= xs/2 =
//    max|x| * 2^-15 (bf16 elements within 2^-7 of the block maximum are exact). Also the
//    sub-block sums xs * sum(T) over 32 elements (the Q4_K / Q5_K min terms).
//  * One CTA = one tile of 16*w weight rows (w = 4..16 consumer warps, the height and the
//    K split chosen per shape by choose_tile) x 16 tokens over a range of K super-blocks
//    (split-K across a thread-block cluster when the tile grid is smaller than the GPU).
//    More than 16 tokens take more token tiles: the tiles of one row tile are neighbours
//    in the grid, so HBM delivers each weight once and L2 the other times, and the
//    registers stay at one tile's sums. Warp 0 streams, per stage of kbs super-blocks, one
//    2-D TMA box of the raw blocks of the tile's rows, the digit rows of the stage (2*kbs
//    boxes of 128 k x 32 digit rows, 128-byte swizzle) and the stage's scales and sums (one
//    bulk copy). The weight boxes of the first stages go out before the grid dependency
//    wait (weights are constant); everything that depends on X after it.
//  * Warps 1..w own 16 rows each (one m16 tile). Q4_K / Q5_K: per 32-weight sub-block one
//    mma.sync.m16n8k32 (u8 x s8 -> s32) per 8 digit columns (4 tokens x 2 digits), the
//    A fragment built once from the raw bytes (nibble mask, Q5_K fifth bit) and reused
//    over every token; the 6-bit sub-block scale multiplies the s32 result (integer
//    multiply-add); per super-block d * xs * (128 * S_hi + S_lo) - dmin * sum(m * sums)
//    in f32. Q6_K: its scales cover 16 weights, so mma.sync.m16n8k16 (s8 x s8) per
//    16-weight group, the signed int8 scale by integer multiply-add, d/4 * xs * (...) per
//    super-block. B fragments come from the swizzled digit boxes with ldmatrix.
// Epilogue as the bf16 small-batch kernel: the accumulators go to a shared-memory tile
// [token][row] (over the drained ring), the CTAs of a cluster sum their partial tiles over
// distributed shared memory in split order (deterministic) and store Y (+ residual).
// Every mbarrier wait is bounded (about one second) and reports through the context's
// device error flag.
//
// Accuracy: the weights are exact; the only rounding of the inputs is the digit
// representation of x (above), then f32 accumulation: results are within the tensor-core
// tolerance (1e-2 relative L2) of the f32 reference with a wide margin, not bit-exact.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <string.h>

#include "internal.h"
#include "kquant.cuh"
#include "rrr_common.cuh"
#include "tile_common.cuh"

namespace rrr {
namespace {

constexpr int kMaxRows = 256;                  // weight rows per tile (at most)
constexpr int kMT = 1;                         // m16 tiles per consumer warp
constexpr int kWR = 16 * kMT;                  // rows per consumer warp
constexpr int kMaxCWarps = kMaxRows / kWR;     // consumer warps (at most)
constexpr int kThreads = (kMaxCWarps + 1) * 32;  // launch bound: + the producer warp
constexpr int kTileN = 16;                     // tokens per tile (larger M: more tiles)
constexpr int kMaxTn = 64;
constexpr int kMaxSplits = 8;                  // portable cluster size
constexpr int kSmemBudget = 232448;            // 227 KB opt-in maximum on sm_100

struct I8Params {
  float* y;
  const float* residual;  // optional [M, N] f32 added in the epilogue (may equal y)
  const float* aux;       // [token tile][nb][16 scales | 16 x 8 sub-block sums] f32
  int M, N, nb, bb;       // nb super-blocks per row, bb bytes per super-block
  int splits, stages, kbs, pitch;
  int cwarps, rows;       // consumer warps and weight rows of a tile (rows = 16 * cwarps)
  uint32_t raw_bytes, box_bytes, aux_off, stage_bytes;  // raw part, one digit box, aux offset, stage
  uint32_t wbox_bytes;    // bytes of the weight box (rows x pitch; the raw part is padded)
  int* err;
};

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                            uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}

// D = A (16x32 u8) * B (32x8 s8), s32.
__device__ __forceinline__ void mma_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
// D = A (16x16 s8) * B (16x8 s8), s32.
__device__ __forceinline__ void mma_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
      "{%7,%7,%7,%7};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}

// Byte i of w, zero-extended / sign-extended (one permute).
__device__ __forceinline__ int ubyte(uint32_t w, int i) {
  return (int)__byte_perm(w, 0u, 0x4440u | (uint32_t)i);
}
__device__ __forceinline__ int sbyte_ext(uint32_t w, int i) {
  const uint32_t sel = (uint32_t)i | ((uint32_t)(i | 8) << 4) | ((uint32_t)(i | 8) << 8) |
                       ((uint32_t)(i | 8) << 12);
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(w), "r"(0u), "r"(sel));
  return (int)r;
}
// qh bit s of each byte moved to bit 4.
__device__ __forceinline__ uint32_t bit4_of(uint32_t x, int s) {
  return (s <= 4 ? (x << (4 - s)) : (x >> (s - 4))) & 0x10101010u;
}
// 32-bit word at byte offset p of a block that starts MIS bytes (0 or 2) past a 4-byte
// boundary (MIS uniform over the warp).
template <int MIS>
__device__ __forceinline__ uint32_t ldw(const uint8_t* p) {
  if (MIS == 0) return *reinterpret_cast<const uint32_t*>(p);
  const uint32_t* q = reinterpret_cast<const uint32_t*>(p - 2);
  return __byte_perm(q[0], q[1], 0x5432);
}
// Q6_K group j (0..3) of a (ql0, ql1, qh) word triple as signed bytes 4*(q - 32):
// q = nibble (j >> 1) of ql_(j & 1) | qh bits 2j, 2j+1 << 4 (phi4.rs:456-475).
__device__ __forceinline__ uint32_t q6_s8x4(uint32_t ql0, uint32_t ql1, uint32_t qh, int j) {
  const uint32_t ql = (j & 1) ? ql1 : ql0;
  const uint32_t lo = ((j >> 1) ? (ql >> 2) : (ql << 2)) & 0x3C3C3C3Cu;
  const uint32_t hi = (qh << (6 - 2 * j)) & 0xC0C0C0C0u;
  return (lo | hi) ^ 0x80808080u;
}

// Address of this lane's ldmatrix row: digit row `row` (0 .. 31), 16-byte chunk `chk`
// of a 128-byte-swizzled box at shared address `box`.
__device__ __forceinline__ uint32_t dig_addr(uint32_t box, int row, int chk) {
  return box + sw128_off(row, chk);
}

// ---- one super-block of a consumer warp: rows 16mt + g and 16mt + g + 8 (mt < MT) of its
// 16*MT; token tiles H0 .. H0+NTH-1 (4 tokens x 2 digits each, NTH even). rowg points at
// row g's block; acc[mt][nt][r] += the row's dot product with token 4nt + t.

template <int QT, int MT, int NT, int H0, int NTH>
__device__ __forceinline__ void sb_q45(const uint8_t* rowg, int pitch, uint32_t dbox,
                                       uint32_t box_bytes, const float* ax, int tn, int t,
                                       int lane, float (&acc)[MT][NT][2]) {
  constexpr int QS = (QT == RRR_Q4_K) ? 16 : 48;
  // 6-bit scales of sub-blocks 0-3 / 4-7 of each row (phi4.rs:492-498)
  uint32_t s03[MT][2], s47[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const uint4 h = *reinterpret_cast<const uint4*>(rowg + (16 * mt + 8 * r) * pitch);
      s03[mt][r] = h.y & 0x3F3F3F3Fu;
      s47[mt][r] = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    }
  // ldmatrix roles: matrix mi = lane / 8 -> token tile 2np + (mi >> 1), chunk half mi & 1
  const int lrow = 8 * ((lane >> 3) >> 1) + (lane & 7), lchk = (lane >> 3) & 1;
  int ia[MT][NTH][4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    // bytes 4t.. and 16+4t.. of qs group c; Q5_K fifth bits: qh[l] bit s (phi4.rs:530-538)
    uint32_t wl[MT][2], wh[MT][2], qa[MT][2], qb[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const uint8_t* b = rowg + (16 * mt + 8 * r) * pitch;
        wl[mt][r] = *reinterpret_cast<const uint32_t*>(b + QS + 32 * c + 4 * t);
        wh[mt][r] = *reinterpret_cast<const uint32_t*>(b + QS + 32 * c + 16 + 4 * t);
        qa[mt][r] = qb[mt][r] = 0u;
        if (QT == RRR_Q5_K) {
          qa[mt][r] = *reinterpret_cast<const uint32_t*>(b + 16 + 4 * t);
          qb[mt][r] = *reinterpret_cast<const uint32_t*>(b + 32 + 4 * t);
        }
      }
#pragma unroll
    for (int hs = 0; hs < 2; ++hs) {
      const int s = 2 * c + hs;  // sub-block: low nibbles of qs group c, then high
      uint32_t a[MT][4];
      int sc[MT][2];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        a[mt][0] = (hs ? (wl[mt][0] >> 4) : wl[mt][0]) & 0x0F0F0F0Fu;
        a[mt][1] = (hs ? (wl[mt][1] >> 4) : wl[mt][1]) & 0x0F0F0F0Fu;
        a[mt][2] = (hs ? (wh[mt][0] >> 4) : wh[mt][0]) & 0x0F0F0F0Fu;
        a[mt][3] = (hs ? (wh[mt][1] >> 4) : wh[mt][1]) & 0x0F0F0F0Fu;
        if (QT == RRR_Q5_K) {
          a[mt][0] |= bit4_of(qa[mt][0], s);
          a[mt][1] |= bit4_of(qa[mt][1], s);
          a[mt][2] |= bit4_of(qb[mt][0], s);
          a[mt][3] |= bit4_of(qb[mt][1], s);
        }
        sc[mt][0] = ubyte(s < 4 ? s03[mt][0] : s47[mt][0], s & 3);
        sc[mt][1] = ubyte(s < 4 ? s03[mt][1] : s47[mt][1], s & 3);
      }
      const uint32_t box = dbox + (uint32_t)(s >> 2) * box_bytes;
#pragma unroll
      for (int np = 0; np < NTH / 2; ++np) {
        uint32_t r0, r1, r2, r3;
        ldmatrix_x4(dig_addr(box, 8 * (H0 + 2 * np) + lrow, 2 * (s & 3) + lchk), r0, r1, r2, r3);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          int d[4], e[4];
          mma_k32(d, a[mt][0], a[mt][1], a[mt][2], a[mt][3], r0, r1);
          mma_k32(e, a[mt][0], a[mt][1], a[mt][2], a[mt][3], r2, r3);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int f = sc[mt][i >> 1];
            ia[mt][2 * np][i] = (s == 0 ? 0 : ia[mt][2 * np][i]) + f * d[i];
            ia[mt][2 * np + 1][i] = (s == 0 ? 0 : ia[mt][2 * np + 1][i]) + f * e[i];
          }
        }
      }
    }
  }
  // f32 per super-block: d * xs * (128 S_hi + S_lo) - dmin * sum_s m_s * sums_s (the header
  // words are read again here: only the scale words were kept through the MMA loop)
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const uint4 h = *reinterpret_cast<const uint4*>(rowg + (16 * mt + 8 * r) * pitch);
      const float dd = f16_bits_to_f32(h.x & 0xFFFFu), dm = f16_bits_to_f32(h.x >> 16);
      const uint32_t m03 = h.z & 0x3F3F3F3Fu, m47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
      float mf[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) mf[q] = (float)ubyte(q < 4 ? m03 : m47, q & 3);
#pragma unroll
      for (int j = 0; j < NTH; ++j) {
        const int tok = 4 * (H0 + j) + t;
        const float xs = ax[tok];
        const float4 sa = *reinterpret_cast<const float4*>(ax + tn + tok * 8);
        const float4 sb = *reinterpret_cast<const float4*>(ax + tn + tok * 8 + 4);
        float m = mf[0] * sa.x;
        m = fmaf(mf[1], sa.y, m);
        m = fmaf(mf[2], sa.z, m);
        m = fmaf(mf[3], sa.w, m);
        m = fmaf(mf[4], sb.x, m);
        m = fmaf(mf[5], sb.y, m);
        m = fmaf(mf[6], sb.z, m);
        m = fmaf(mf[7], sb.w, m);
        const float v = fmaf(128.f, (float)ia[mt][j][2 * r + 1], (float)ia[mt][j][2 * r]);
        acc[mt][H0 + j][r] += fmaf(dd * xs, v, -dm * m);
      }
    }
}

template <int MT, int NT, int H0, int NTH, int MIS>
__device__ __forceinline__ void sb_q6(const uint8_t* rowg, int pitch, uint32_t dbox,
                                      uint32_t box_bytes, const float* ax, int t, int lane,
                                      float (&acc)[MT][NT][2]) {
  // ldmatrix roles: matrix mi = lane / 8 -> token tile q + mi (x4) or q + (mi & 1) (x2)
  const int lrow4 = lane, lrow2 = lane & 15;
  int ia[MT][NTH][4];
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    // int8 scales 8hh .. 8hh+7 of each row (bytes 192 + 8hh ..)
    uint32_t sw[MT][2][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const uint8_t* b = rowg + (16 * mt + 8 * r) * pitch;
        sw[mt][r][0] = ldw<MIS>(b + 192 + 8 * hh);
        sw[mt][r][1] = ldw<MIS>(b + 196 + 8 * hh);
      }
#pragma unroll
    for (int lh = 0; lh < 2; ++lh) {
      const int pq = 64 * hh + 16 * lh + 4 * t, ph = 128 + 32 * hh + 16 * lh + 4 * t;
      uint32_t x0[MT][2], x1[MT][2], xh[MT][2];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const uint8_t* b = rowg + (16 * mt + 8 * r) * pitch;
          x0[mt][r] = ldw<MIS>(b + pq);
          x1[mt][r] = ldw<MIS>(b + pq + 32);
          xh[mt][r] = ldw<MIS>(b + ph);
        }
      const uint32_t box = dbox + (uint32_t)hh * box_bytes;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int il = 2 * j + lh;  // scale index within the half = 16-byte chunk of the box
        uint32_t a[MT][2];
        int sc[MT][2];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            a[mt][r] = q6_s8x4(x0[mt][r], x1[mt][r], xh[mt][r], j);
            sc[mt][r] = sbyte_ext(sw[mt][r][il >> 2], il & 3);
          }
        const bool first = (hh == 0 && lh == 0 && j == 0);
#pragma unroll
        for (int q = 0; q < NTH; q += 4) {
          uint32_t rb[4] = {0u, 0u, 0u, 0u};
          if (q + 4 <= NTH)
            ldmatrix_x4(dig_addr(box, 8 * (H0 + q) + lrow4, il), rb[0], rb[1], rb[2], rb[3]);
          else
            ldmatrix_x2(dig_addr(box, 8 * (H0 + q) + lrow2, il), rb[0], rb[1]);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (q + u >= NTH) break;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              int d[4];
              mma_k16(d, a[mt][0], a[mt][1], rb[u]);
#pragma unroll
              for (int i = 0; i < 4; ++i)
                ia[mt][q + u][i] = (first ? 0 : ia[mt][q + u][i]) + sc[mt][i >> 1] * d[i];
            }
          }
        }
      }
    }
  }
  // A carried 4 * (q - 32): d / 4 * xs * (128 S_hi + S_lo)
  float dd[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int r = 0; r < 2; ++r)
      dd[mt][r] = 0.25f * f16_bits_to_f32(ldw<MIS>(rowg + (16 * mt + 8 * r) * pitch + 208) & 0xFFFFu);
#pragma unroll
  for (int j = 0; j < NTH; ++j) {
    const float xs = ax[4 * (H0 + j) + t];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float v = fmaf(128.f, (float)ia[mt][j][2 * r + 1], (float)ia[mt][j][2 * r]);
        acc[mt][H0 + j][r] = fmaf(dd[mt][r] * xs, v, acc[mt][H0 + j][r]);
      }
  }
}

// One super-block of the warp's rows against the tile's 16 tokens (4 token tiles).
template <int QT>
__device__ __forceinline__ void superblock(const uint8_t* rowg, int pitch, uint32_t dbox,
                                           uint32_t box_bytes, const float* ax, int t, int lane,
                                           int mis, float (&acc)[kMT][kTileN / 4][2]) {
  constexpr int NT = kTileN / 4;
  if constexpr (QT == RRR_Q6_K) {
    if (mis)
      sb_q6<kMT, NT, 0, NT, 2>(rowg, pitch, dbox, box_bytes, ax, t, lane, acc);
    else
      sb_q6<kMT, NT, 0, NT, 0>(rowg, pitch, dbox, box_bytes, ax, t, lane, acc);
  } else {
    sb_q45<QT, kMT, NT, 0, NT>(rowg, pitch, dbox, box_bytes, ax, kTileN, t, lane, acc);
  }
}

// ---- the kernels --------------------------------------------------------------------

// X preparation: one warp per (super-block, token) of [nb][tn] (tn = M rounded up to the
// token tile); tokens >= M get zero scale and sums (their digit rows are the TMA's zero
// fill past row 2M).
__global__ void __launch_bounds__(256) xdig_kernel(const uint16_t* __restrict__ x, int M, int K,
                                                   int tn, int8_t* __restrict__ dig,
                                                   float* __restrict__ aux) {
  // dependents may be scheduled now; X (written by the previous kernel) is read and the
  // digits (read by the previous GEMM) are written only after it has completed
  pdl_launch_dependents();
  pdl_wait();
  const int wid = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int nb = K / 256;
  if (wid >= nb * tn) return;
  const int kb = wid / tn, tok = wid % tn;
  // this token's tile block of the scales and sums, and its index inside
  float* ab = aux + ((size_t)(tok / kTileN) * nb + kb) * (kTileN * 9);
  const int tt = tok % kTileN;
  if (tok >= M) {
    if (lane == 0) ab[tt] = 0.f;
    if (lane < 8) ab[kTileN + tt * 8 + lane] = 0.f;
    return;
  }
  const uint4 raw = *reinterpret_cast<const uint4*>(x + (size_t)tok * K + kb * 256 + lane * 8);
  const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
  float v[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(wv[i] << 16);
    v[2 * i + 1] = __uint_as_float(wv[i] & 0xFFFF0000u);
  }
  uint32_t mb = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) mb = max(mb, __float_as_uint(v[i]) & 0x7FFFFFFFu);
  mb = __reduce_max_sync(0xffffffffu, mb);
  int T[8];
  float xs = 0.f;
  if (mb == 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) T[i] = 0;
  } else {
    // 2^E > max|x| with E = floor(log2 max|x|) + 1 (a subnormal maximum counts as 2^-127)
    const int E = (int)(mb >> 23) - 126;
    const int p = 14 - E, p1 = min(p, 127), p2 = p - p1;  // x * 2^p in two exact steps
    const float s1 = __uint_as_float((uint32_t)(p1 + 127) << 23);
    const float s2 = __uint_as_float((uint32_t)(p2 + 127) << 23);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int q = __float2int_rn(v[i] * s1 * s2);
      T[i] = max(-16383, min(16383, q));
    }
    const int e = E - 14;  // xs = 2^e, e >= -140: below 2^-126 as 2^(e+64) * 2^-64
    xs = e >= -126 ? __uint_as_float((uint32_t)(e + 127) << 23)
                   : __uint_as_float((uint32_t)(e + 64 + 127) << 23) * 5.42101086242752217e-20f;
  }
  uint32_t lo[2] = {0u, 0u}, hi[2] = {0u, 0u};
  int sum = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int h = T[i] >> 7, l = T[i] & 127;
    lo[i >> 2] |= (uint32_t)l << (8 * (i & 3));
    hi[i >> 2] |= ((uint32_t)h & 0xFFu) << (8 * (i & 3));
    sum += T[i];
  }
  int8_t* row = dig + (size_t)(2 * tok) * K + kb * 256 + lane * 8;
  *reinterpret_cast<uint2*>(row) = make_uint2(lo[0], lo[1]);
  *reinterpret_cast<uint2*>(row + K) = make_uint2(hi[0], hi[1]);
  sum += __shfl_xor_sync(0xffffffffu, sum, 1);
  sum += __shfl_xor_sync(0xffffffffu, sum, 2);
  if ((lane & 3) == 0) ab[kTileN + tt * 8 + (lane >> 2)] = (float)sum * xs;
  if (lane == 0) ab[tt] = xs;
}

template <int QT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kq_i8_kernel(const __grid_constant__ CUtensorMap dmap,
                      const __grid_constant__ CUtensorMap wmap, const I8Params p) {
  constexpr int TN = kTileN;
  constexpr int NT = TN / 4;  // token tiles of 8 digit columns
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = smem_dyn + ((1024u - (smem_addr(smem_dyn) & 1023u)) & 1023u);
  const int S = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * p.stage_bytes);
  uint64_t* empty = full + S;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + S);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the token tiles of one row tile are neighbours in the grid (x), so they read its
  // weights from L2 at about the same time
  const int m0 = blockIdx.x * TN, n0 = blockIdx.y * p.rows, z = blockIdx.z;
  const int pstride = p.rows + 4;  // floats per token row of the partial tile
  const int kb0 = (int)((long long)z * p.nb / p.splits);
  const int kb1 = (int)((long long)(z + 1) * p.nb / p.splits);
  const int n_blk = kb1 - kb0;
  const int n_st = (n_blk + p.kbs - 1) / p.kbs;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], p.cwarps);
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == 0) {
    // ---------------- producer
    auto x_part = [&](int st) {  // digit boxes and scales/sums of stage st
      const int s = st % S;
      const int kb = kb0 + st * p.kbs;
      const int nk = min(p.kbs, kb1 - kb);
      uint8_t* dst = smem + (size_t)s * p.stage_bytes;
      for (int i = 0; i < 2 * nk; ++i)
        tma_load_2d(dst + p.raw_bytes + (uint32_t)i * p.box_bytes, &dmap, kb * 256 + 128 * i, m0 * 2,
                    &full[s]);
      bulk_g2s(dst + p.aux_off, p.aux + ((size_t)blockIdx.x * p.nb + kb) * (TN * 9),
               (uint32_t)(nk * TN * 36), &full[s]);
    };
    auto w_part = [&](int st) {  // expected bytes of the whole stage, then the weight box
      const int s = st % S;
      const int kb = kb0 + st * p.kbs;
      const int nk = min(p.kbs, kb1 - kb);
      uint8_t* dst = smem + (size_t)s * p.stage_bytes;
      mbar_arrive_expect_tx(&full[s], p.wbox_bytes + (uint32_t)(2 * nk) * p.box_bytes + (uint32_t)(nk * TN * 36));
      tma_load_2d(dst, &wmap, (int)(((long long)kb * p.bb & ~15ll) >> 3), n0, &full[s]);
    };
    const int pre = min(S, n_st);
    if (lane == 0)
      for (int st = 0; st < pre; ++st) w_part(st);
    pdl_wait();
    if (lane == 0)
      for (int st = 0; st < pre; ++st) x_part(st);
    __syncwarp();
    int issued = pre;
    for (int st = pre; st < n_st; ++st) {
      if (warp_aborted(abort_flag)) break;
      const int s = st % S;
      if (!warp_wait(&empty[s], ((st / S) - 1) & 1, p.err)) {
        *abort_flag = 1;
        break;
      }
      if (lane == 0) {
        w_part(st);
        x_part(st);
      }
      __syncwarp();
      ++issued;
    }
    // copies still in flight (only after an abort) must land before the CTA exits
    for (int s = 0; s < S; ++s) {
      const int cnt = issued > s ? (issued - s + S - 1) / S : 0;
      if (cnt) warp_wait(&full[s], (cnt - 1) & 1, p.err);
    }
  } else {
    // ---------------- consumers: warp cw owns rows kWR*cw .. kWR*cw + kWR-1
    pdl_wait();
    const int cw = warp - 1;
    const int g = lane >> 2, t = lane & 3;
    float acc[kMT][NT][2];
#pragma unroll
    for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
      for (int j = 0; j < NT; ++j) acc[mt][j][0] = acc[mt][j][1] = 0.f;
    for (int st = 0; st < n_st; ++st) {
      if (warp_aborted(abort_flag)) break;
      const int s = st % S;
      if (!warp_wait(&full[s], (uint32_t)(st / S) & 1u, p.err)) {
        *abort_flag = 1;
        break;
      }
      const uint8_t* stage = smem + (size_t)s * p.stage_bytes;
      const int kb = kb0 + st * p.kbs;
      const int nk = min(p.kbs, kb1 - kb);
      const int env = (int)(((long long)kb * p.bb) & 15);
      const float* axs = reinterpret_cast<const float*>(stage + p.aux_off);
#pragma unroll 1
      for (int kk = 0; kk < nk; ++kk) {
        const uint8_t* rowg = stage + (kWR * cw + g) * p.pitch + env + kk * p.bb;
        const uint32_t dbox = smem_addr(stage + p.raw_bytes) + (uint32_t)(2 * kk) * p.box_bytes;
        superblock<QT>(rowg, p.pitch, dbox, p.box_bytes, axs + kk * TN * 9, t, lane,
                       (env + kk * p.bb) & 2, acc);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    // all stages consumed by every consumer before the ring is reused for the partial tile
    named_barrier(1, p.cwarps * 32);
    float* part = reinterpret_cast<float*>(smem);  // [TN][pstride]
#pragma unroll
    for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const int tok = 4 * j + t;
        part[tok * pstride + kWR * cw + 16 * mt + g] = acc[mt][j][0];
        part[tok * pstride + kWR * cw + 16 * mt + g + 8] = acc[mt][j][1];
      }
  }

  // ---------------- sum the partial tiles of the cluster (split order) and store Y
  __syncthreads();
  if (p.splits > 1) cluster_sync();
  const bool ok = !*abort_flag;
  if (ok && threadIdx.x >= 32) {
    const int tid = threadIdx.x - 32;
    const int per = (TN + p.splits - 1) / p.splits;
    const int j0 = z * per, j1 = min(TN, j0 + per);
    const float* part = reinterpret_cast<const float*>(smem);
    const int r4n = p.rows / 4;
    for (int idx = tid; idx < (j1 - j0) * r4n; idx += p.cwarps * 32) {
      const int j = j0 + idx / r4n, r4 = (idx % r4n) * 4;
      const uint32_t la = smem_addr(part + j * pstride + r4);
      float4 v = ld_dsmem_f4(la, 0);
      for (int s2 = 1; s2 < p.splits; ++s2) {
        const float4 u = ld_dsmem_f4(la, (uint32_t)s2);
        v.x += u.x;
        v.y += u.y;
        v.z += u.z;
        v.w += u.w;
      }
      const int m = m0 + j, n = n0 + r4;
      if (m < p.M && n < p.N) {
        float* dst = p.y + (size_t)m * p.N + n;
        const float* res = p.residual ? p.residual + (size_t)m * p.N + n : nullptr;
        if ((p.N & 3) == 0 && n + 3 < p.N) {
          if (res) {
            const float4 q = *reinterpret_cast<const float4*>(res);
            v.x += q.x;
            v.y += q.y;
            v.z += q.z;
            v.w += q.w;
          }
          *reinterpret_cast<float4*>(dst) = v;
        } else {
          const float a4[4] = {v.x, v.y, v.z, v.w};
          for (int e = 0; e < 4 && n + e < p.N; ++e) dst[e] = a4[e] + (res ? res[e] : 0.f);
        }
      }
    }
  }
  if (p.splits > 1) cluster_sync();
}

// ---- host side ----------------------------------------------------------------------

// Stage layout: raw [rows][pitch] (box of kbs super-blocks + envelope, pitch an odd number
// of 16-byte units) padded to 1024 bytes (the digit boxes after it use the 128-byte
// swizzle, whose pattern is anchored at 1024-byte boundaries), digits [2*kbs boxes][32
// rows][128 B], then the scales and sums [kbs][16 x 9] f32; the stage rounded to 1024 bytes.
int raw_part_bytes(int qtype, int kbs, int rows) {
  return (rows * raw_slot_bytes(qtype, kbs) + 1023) & ~1023;
}
int stage_bytes_i8(int qtype, int kbs, int rows) {
  const int b = raw_part_bytes(qtype, kbs, rows) + 2 * kbs * (2 * kTileN * 128) + kbs * kTileN * 36;
  return (b + 1023) & ~1023;
}

// Ring of one tile shape: super-blocks per stage and stages (0: does not fit).
struct Ring {
  int kbs, stages, smem;
};
Ring ring_for(int qtype, int rows) {
  const int fixed = 1024 + 256;
  for (int kbs = 2; kbs >= 1; --kbs) {
    const int sb = stage_bytes_i8(qtype, kbs, rows);
    int st = (kSmemBudget - fixed) / sb;
    if (st > 4) st = 4;
    if (st >= 3 || (kbs == 1 && st >= 2)) {
      // the partial tile [16][rows + 4] f32 reuses the ring
      if (kTileN * (rows + 4) * 4 > st * sb) return Ring{0, 0, 0};
      return Ring{kbs, st, fixed + st * sb};
    }
  }
  return Ring{0, 0, 0};
}

template <int QT>
cudaError_t launch_q(const LaunchEnv& env, const I8Plan& pl, const void* w, const uint16_t* x,
                     float* y, int M, int K, int N, const float* residual, void* scratch) {
  const int nb = K / 256;
  const int tn = pl.m_tiles * kTileN;
  int8_t* dig = reinterpret_cast<int8_t*>(scratch);
  float* aux = reinterpret_cast<float*>(reinterpret_cast<char*>(scratch) + i8_digit_bytes(K));
  auto kern = gemm_kq_i8_kernel<QT>;
  // Tile shape: rows per CTA (16 per consumer warp) and K splits (choose_tile).
  const int qi = QT - RRR_Q4_K;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = env.stream;
  // the choice per (device, N, K, token tiles), made once
  struct Choice {
    int dev, N, nb, mt, cw, s;
    Ring ring;
  };
  static thread_local Choice chosen[3][16];
  static thread_local int n_chosen[3] = {0, 0, 0};
  int dev = 0;
  cudaGetDevice(&dev);
  int best_cw = 0, best_s = 1;
  Ring best_ring{0, 0, 0};
  for (int i = 0; i < n_chosen[qi]; ++i) {
    const Choice& c = chosen[qi][i];
    if (c.dev == dev && c.N == N && c.nb == nb && c.mt == pl.m_tiles) {
      best_cw = c.cw;
      best_s = c.s;
      best_ring = c.ring;
    }
  }
  if (best_cw == 0) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget);
    if (e != cudaSuccess) return e;
    TileCand cand[kMaxCWarps];
    Ring rings[kMaxCWarps];
    int cws[kMaxCWarps], nc = 0;
    for (int cw = kMaxCWarps; cw >= 4; --cw) {
      const Ring rg = ring_for(QT, cw * kWR);
      if (rg.stages == 0) continue;
      cand[nc] = TileCand{cw * kWR, (cw + 1) * 32, rg.smem};
      rings[nc] = rg;
      cws[nc++] = cw;
    }
    int sp = 1;
    const int i = choose_tile((const void*)kern, env.stream, cand, nc, N, pl.m_tiles, nb,
                              std::min(kMaxSplits, std::max(1, nb / 2)), env.sm_count, &sp);
    if (i < 0) return cudaErrorInvalidConfiguration;
    best_cw = cws[i];
    best_s = sp;
    best_ring = rings[i];
    Choice c{dev, N, nb, pl.m_tiles, best_cw, best_s, best_ring};
    if (n_chosen[qi] < 16) chosen[qi][n_chosen[qi]++] = c;
    else chosen[qi][(N + nb) % 16] = c;
  }
  const int rows = best_cw * kWR;
  CUtensorMap dmap, wmap;
  // digit rows [2M][K] bytes; rows of tokens past M are the copy's zero fill
  if (!encode_2d(&dmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, dig, (uint64_t)K, (uint64_t)(2 * M),
                 (uint64_t)K, 128u, (uint32_t)(2 * kTileN), CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  const long long row_bytes = (long long)nb * KQ<QT>::kBlockBytes;
  const int pitch = raw_slot_bytes(QT, best_ring.kbs);
  if (!encode_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT64, w, (uint64_t)row_bytes / 8, (uint64_t)N,
                 (uint64_t)row_bytes, (uint32_t)pitch / 8, (uint32_t)rows, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  // the digits first (one warp per super-block and token)
  const int warps = nb * tn;
  cudaError_t e = rrr_launch_pdl(xdig_kernel, dim3((warps + 7) / 8), dim3(256), 0, env.stream, env.pdl,
                                 x, M, K, tn, dig, aux);
  if (e != cudaSuccess) return e;
  I8Params p{};
  p.y = y;
  p.residual = residual;
  p.aux = aux;
  p.M = M;
  p.N = N;
  p.nb = nb;
  p.bb = KQ<QT>::kBlockBytes;
  p.splits = best_s;
  p.stages = best_ring.stages;
  p.kbs = best_ring.kbs;
  p.pitch = pitch;
  p.cwarps = best_cw;
  p.rows = rows;
  p.raw_bytes = (uint32_t)raw_part_bytes(QT, best_ring.kbs, rows);
  p.wbox_bytes = (uint32_t)(rows * pitch);
  p.box_bytes = (uint32_t)(2 * kTileN * 128);
  p.aux_off = p.raw_bytes + (uint32_t)(2 * best_ring.kbs) * p.box_bytes;
  p.stage_bytes = (uint32_t)stage_bytes_i8(QT, best_ring.kbs, rows);
  p.err = env.d_err;
  cfg.gridDim = dim3(pl.m_tiles, (N + rows - 1) / rows, best_s);
  cfg.blockDim = dim3((best_cw + 1) * 32);
  cfg.dynamicSmemBytes = best_ring.smem;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = best_s;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = env.pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, dmap, wmap, p);
}

}  // namespace

size_t i8_digit_bytes(int K) { return (size_t)2 * kMaxTn * K; }
size_t i8_scratch_bytes(int K) {
  return i8_digit_bytes(K) + (size_t)(K / 256) * kMaxTn * 9 * sizeof(float);
}

bool plan_gemm_kq_i8(int qtype, int M, int K, int N, int sm_count, I8Plan* pl) {
  const int bb = kq_block_bytes(qtype);
  if (M < 1 || M > kMaxTn || K < 256 || K % 256 || K > kGemvMaxK || N < 1 || bb == 0) return false;
  // the raw stage is one TMA box: every row must start 16-byte aligned
  if (((long long)(K / 256) * bb) % 16 != 0) return false;
  I8Plan r{};
  r.tn = kTileN;
  r.m_tiles = (M + kTileN - 1) / kTileN;
  // the tile rows and split count are chosen at launch, from the kernel's cluster occupancy
  r.n_tiles = 0;
  r.splits = 0;
  const Ring rg = ring_for(qtype, kMaxRows);
  if (rg.stages == 0) return false;
  r.stages = rg.stages;
  r.kbs = rg.kbs;
  r.smem = rg.smem;
  (void)sm_count;
  *pl = r;
  return true;
}

cudaError_t launch_gemm_kq_i8(const LaunchEnv& env, int qtype, const void* w,
                              const uint16_t* x_bf16, float* y, int M, int K, int N,
                              const I8Plan& pl, const float* residual, void* scratch) {
  switch (qtype) {
    case RRR_Q4_K: return launch_q<RRR_Q4_K>(env, pl, w, x_bf16, y, M, K, N, residual, scratch);
    case RRR_Q5_K: return launch_q<RRR_Q5_K>(env, pl, w, x_bf16, y, M, K, N, residual, scratch);
    case RRR_Q6_K: return launch_q<RRR_Q6_K>(env, pl, w, x_bf16, y, M, K, N, residual, scratch);
    default: return cudaErrorNotSupported;
  }
}

}  // namespace rrr
