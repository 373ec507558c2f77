// gemv_kq.cu — kernel (1): fused raw-block K-quant GEMV, y = W x (+ residual), for the
// Q4_K / Q5_K / Q6_K super-blocks GGUF stores (reference: gpu_matmul_kquant and the
// matmul_q{4,5,6}k dispatches, src/model/phi4.rs:631-658, 1081-1096; element formats
// phi4.rs:444-542).
//
// Design (sm_100a, HBM-bound):
//  * One CTA = 1 producer warp + NW consumer warps. The producer streams 16-row tiles of
//    raw blocks (K split into chunks of kc blocks) with 1-D bulk copies (cp.async.bulk,
//    mbarrier complete_tx) into a ring of shared-memory stages; consumers free a stage
//    through an "empty" mbarrier. Every wait is bounded (%globaltimer) and reports
//    through the context's error flag instead of hanging.
//  * x is decomposed once per CTA into three int8 "digits" per element against a per-
//    256-element scale xs: x ~= xs*(d0 + d1/2^7 + d2/2^14), |error| <= xs*2^-15 (about
//    f32 precision). The per-sub-block sums sum_j q_j*x_j then come from exact int8
//    tensor-core dot products (mma.sync m16n8k32, u8 quants x s8 digits, int32
//    accumulate): a 16-row x 32-weight tile per instruction, digits of two scale groups
//    in columns 0-2 and 3-5. Scales are applied by integer multiply-add per sub-block,
//    d/dmin in f32 once per block. This keeps the CUDA-core work near one instruction
//    per weight so the kernel stays memory-bound. Dequantised weights are never
//    materialised; the bit-exact dequantisation is rrr_dequant_kq (dequant.cu).
//  * Tile epilogue: shuffle reduction over the 4 lanes that share a row, then a
//    deterministic sum over warps through shared memory, + residual, store.
//  * Programmatic dependent launch: the producer starts streaming weights before
//    griddepcontrol.wait; x is read and y written only after it.
#include <algorithm>

#include "internal.h"
#include "kquant.cuh"

namespace rrr {
namespace {

constexpr int kTileRows = 16;
constexpr int kNW = 4;  // consumer warps per CTA
constexpr int kXBf16 = 100;  // internal prologue mode: x is bf16 (batched fallback)

struct GemvParams {
  const uint8_t* w;
  const float* x;
  const uint16_t* xb;  // bf16 input (internal mode kXBf16)
  float* y;
  const float* residual;
  const float* gamma;
  float eps;
  int mode, n_q, n_kv, hd;
  int K, N, nb;
  long long row_bytes, total_bytes;
  int kc, n_chunks, n_tiles;
  int row_stride, stage_bytes, nstages;
  int dig_stride;
  int off_bars, off_dig, off_xscale, off_xsum, off_red, off_misc;
  int* err;
};

__device__ __forceinline__ void mma_u8s8(int& d0, int& d1, int& d2, int& d3, uint32_t a0,
                                         uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d0), "+r"(d1), "+r"(d2), "+r"(d3)
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Weight of B column c (digit c % 3 of scale group c / 3); columns 6 and 7 are unused.
__device__ __forceinline__ float digit_weight(int c) {
  return c >= 6 ? 0.f : (c % 3 == 0 ? 1.f : (c % 3 == 1 ? (1.f / 128.f) : (1.f / 16384.f)));
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xFFu; }

// ---------------------------------------------------------------- Q4_K block
// Rows g and g+8 of the tile, block `kb` of the row. MMA (pair p, half h) covers qs
// bytes 32p + 8*tig + 4h .. +3 of both rows: low nibbles = sub 2p (group A, slots 0-15),
// high nibbles taken as (byte & 0xF0) = 16*q = sub 2p+1 (group B, slots 16-31).
__device__ __forceinline__ void block_q4k(const uint8_t* b0, const uint8_t* b1, int kb,
                                          const int8_t* dig, int ds, const float* xscale,
                                          const float* xsum, int g, int tig, float& acc0,
                                          float& acc1) {
  const uint4 h0 = *reinterpret_cast<const uint4*>(b0);
  const uint4 h1 = *reinterpret_cast<const uint4*>(b1);
  const float d_0 = f16_bits_to_f32(h0.x & 0xFFFFu), dm_0 = f16_bits_to_f32(h0.x >> 16);
  const float d_1 = f16_bits_to_f32(h1.x & 0xFFFFu), dm_1 = f16_bits_to_f32(h1.x >> 16);
  const uint32_t sc03_0 = h0.y & 0x3F3F3F3Fu, m03_0 = h0.z & 0x3F3F3F3Fu;
  const uint32_t sc47_0 = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
  const uint32_t m47_0 = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
  const uint32_t sc03_1 = h1.y & 0x3F3F3F3Fu, m03_1 = h1.z & 0x3F3F3F3Fu;
  const uint32_t sc47_1 = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
  const uint32_t m47_1 = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);

  const int n = g;  // B column supplied by this lane
  const bool nA = n < 3, nB = (n >= 3) && (n < 6);
  const int8_t* dp = dig + (n < 6 ? (n % 3) * ds : 0) + kb * 256 + 8 * tig + (nB ? 32 : 0);
  const bool c0B = (2 * tig) >= 3, c1B = (2 * tig + 1) >= 3;
  int i00 = 0, i01 = 0, i10 = 0, i11 = 0;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint2 w = *reinterpret_cast<const uint2*>(b0 + 16 + 32 * p + 8 * tig);
    const uint2 v = *reinterpret_cast<const uint2*>(b1 + 16 + 32 * p + 8 * tig);
    uint2 bb = make_uint2(0u, 0u);
    if (nA || nB) bb = *reinterpret_cast<const uint2*>(dp + 64 * p);
    int D0 = 0, D1 = 0, D2 = 0, D3 = 0;
    mma_u8s8(D0, D1, D2, D3, w.x & 0x0F0F0F0Fu, v.x & 0x0F0F0F0Fu, w.x & 0xF0F0F0F0u,
             v.x & 0xF0F0F0F0u, nA ? bb.x : 0u, nB ? bb.x : 0u);
    mma_u8s8(D0, D1, D2, D3, w.y & 0x0F0F0F0Fu, v.y & 0x0F0F0F0Fu, w.y & 0xF0F0F0F0u,
             v.y & 0xF0F0F0F0u, nA ? bb.y : 0u, nB ? bb.y : 0u);
    const int sa = 2 * p, sb = 2 * p + 1;
    const int sA0 = 16 * (int)byte_of(sa < 4 ? sc03_0 : sc47_0, sa & 3);
    const int sB0 = (int)byte_of(sb < 4 ? sc03_0 : sc47_0, sb & 3);
    const int sA1 = 16 * (int)byte_of(sa < 4 ? sc03_1 : sc47_1, sa & 3);
    const int sB1 = (int)byte_of(sb < 4 ? sc03_1 : sc47_1, sb & 3);
    i00 += (c0B ? sB0 : sA0) * D0;
    i01 += (c1B ? sB0 : sA0) * D1;
    i10 += (c0B ? sB1 : sA1) * D2;
    i11 += (c1B ? sB1 : sA1) * D3;
  }
  const float xs = xscale[kb];
  const float w0 = digit_weight(2 * tig) * (1.f / 16.f), w1 = digit_weight(2 * tig + 1) * (1.f / 16.f);
  const float v0 = (float)i00 * w0 + (float)i01 * w1;
  const float v1 = (float)i10 * w0 + (float)i11 * w1;
  // min term of sub-blocks 2*tig and 2*tig+1: dmin * (m_a*S_a + m_b*S_b)
  const float* xsb = xsum + kb * 16 + 4 * tig;
  const float Sa = xsb[0] + xsb[1], Sb = xsb[2] + xsb[3];
  const int sh = 16 * (tig & 1);
  const uint32_t mw0 = tig < 2 ? m03_0 : m47_0, mw1 = tig < 2 ? m03_1 : m47_1;
  const float ma0 = (float)((mw0 >> sh) & 0xFFu), mb0 = (float)((mw0 >> (sh + 8)) & 0xFFu);
  const float ma1 = (float)((mw1 >> sh) & 0xFFu), mb1 = (float)((mw1 >> (sh + 8)) & 0xFFu);
  acc0 += d_0 * xs * v0 - dm_0 * (ma0 * Sa + mb0 * Sb);
  acc1 += d_1 * xs * v1 - dm_1 * (ma1 * Sa + mb1 * Sb);
}

// qh bit `s` of each byte moved to bit 4.
__device__ __forceinline__ uint32_t qh_bit4(uint32_t x, int s) {
  return (s <= 4 ? (x << (4 - s)) : (x >> (s - 4))) & 0x10101010u;
}

// ---------------------------------------------------------------- Q5_K block
__device__ __forceinline__ void block_q5k(const uint8_t* b0, const uint8_t* b1, int kb,
                                          const int8_t* dig, int ds, const float* xscale,
                                          const float* xsum, int g, int tig, float& acc0,
                                          float& acc1) {
  const uint4 h0 = *reinterpret_cast<const uint4*>(b0);
  const uint4 h1 = *reinterpret_cast<const uint4*>(b1);
  const float d_0 = f16_bits_to_f32(h0.x & 0xFFFFu), dm_0 = f16_bits_to_f32(h0.x >> 16);
  const float d_1 = f16_bits_to_f32(h1.x & 0xFFFFu), dm_1 = f16_bits_to_f32(h1.x >> 16);
  const uint32_t sc03_0 = h0.y & 0x3F3F3F3Fu, m03_0 = h0.z & 0x3F3F3F3Fu;
  const uint32_t sc47_0 = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
  const uint32_t m47_0 = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
  const uint32_t sc03_1 = h1.y & 0x3F3F3F3Fu, m03_1 = h1.z & 0x3F3F3F3Fu;
  const uint32_t sc47_1 = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
  const uint32_t m47_1 = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
  const uint2 qh0 = *reinterpret_cast<const uint2*>(b0 + 16 + 8 * tig);
  const uint2 qh1 = *reinterpret_cast<const uint2*>(b1 + 16 + 8 * tig);

  const int n = g;
  const bool nA = n < 3, nB = (n >= 3) && (n < 6);
  const int8_t* dp = dig + (n < 6 ? (n % 3) * ds : 0) + kb * 256 + 8 * tig + (nB ? 32 : 0);
  const bool c0B = (2 * tig) >= 3, c1B = (2 * tig + 1) >= 3;
  int i00 = 0, i01 = 0, i10 = 0, i11 = 0;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint2 w = *reinterpret_cast<const uint2*>(b0 + 48 + 32 * p + 8 * tig);
    const uint2 v = *reinterpret_cast<const uint2*>(b1 + 48 + 32 * p + 8 * tig);
    uint2 bb = make_uint2(0u, 0u);
    if (nA || nB) bb = *reinterpret_cast<const uint2*>(dp + 64 * p);
    const int sa = 2 * p, sb = 2 * p + 1;
    int D0 = 0, D1 = 0, D2 = 0, D3 = 0;
    mma_u8s8(D0, D1, D2, D3, (w.x & 0x0F0F0F0Fu) | qh_bit4(qh0.x, sa),
             (v.x & 0x0F0F0F0Fu) | qh_bit4(qh1.x, sa),
             ((w.x >> 4) & 0x0F0F0F0Fu) | qh_bit4(qh0.x, sb),
             ((v.x >> 4) & 0x0F0F0F0Fu) | qh_bit4(qh1.x, sb), nA ? bb.x : 0u, nB ? bb.x : 0u);
    mma_u8s8(D0, D1, D2, D3, (w.y & 0x0F0F0F0Fu) | qh_bit4(qh0.y, sa),
             (v.y & 0x0F0F0F0Fu) | qh_bit4(qh1.y, sa),
             ((w.y >> 4) & 0x0F0F0F0Fu) | qh_bit4(qh0.y, sb),
             ((v.y >> 4) & 0x0F0F0F0Fu) | qh_bit4(qh1.y, sb), nA ? bb.y : 0u, nB ? bb.y : 0u);
    const int sA0 = (int)byte_of(sa < 4 ? sc03_0 : sc47_0, sa & 3);
    const int sB0 = (int)byte_of(sb < 4 ? sc03_0 : sc47_0, sb & 3);
    const int sA1 = (int)byte_of(sa < 4 ? sc03_1 : sc47_1, sa & 3);
    const int sB1 = (int)byte_of(sb < 4 ? sc03_1 : sc47_1, sb & 3);
    i00 += (c0B ? sB0 : sA0) * D0;
    i01 += (c1B ? sB0 : sA0) * D1;
    i10 += (c0B ? sB1 : sA1) * D2;
    i11 += (c1B ? sB1 : sA1) * D3;
  }
  const float xs = xscale[kb];
  const float w0 = digit_weight(2 * tig), w1 = digit_weight(2 * tig + 1);
  const float v0 = (float)i00 * w0 + (float)i01 * w1;
  const float v1 = (float)i10 * w0 + (float)i11 * w1;
  const float* xsb = xsum + kb * 16 + 4 * tig;
  const float Sa = xsb[0] + xsb[1], Sb = xsb[2] + xsb[3];
  const int sh = 16 * (tig & 1);
  const uint32_t mw0 = tig < 2 ? m03_0 : m47_0, mw1 = tig < 2 ? m03_1 : m47_1;
  const float ma0 = (float)((mw0 >> sh) & 0xFFu), mb0 = (float)((mw0 >> (sh + 8)) & 0xFFu);
  const float ma1 = (float)((mw1 >> sh) & 0xFFu), mb1 = (float)((mw1 >> (sh + 8)) & 0xFFu);
  acc0 += d_0 * xs * v0 - dm_0 * (ma0 * Sa + mb0 * Sb);
  acc1 += d_1 * xs * v1 - dm_1 * (ma1 * Sa + mb1 * Sb);
}

// 32-bit load from a shared-memory byte address that is 4-byte or 2-byte aligned.
template <bool ALIGNED>
__device__ __forceinline__ uint32_t ldw(const uint8_t* p) {
  if (ALIGNED) return *reinterpret_cast<const uint32_t*>(p);
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* q = reinterpret_cast<const uint32_t*>(a & ~static_cast<uintptr_t>(3));
  return __byte_perm(q[0], q[1], (a & 2) ? 0x5432 : 0x3210);
}

__device__ __forceinline__ int sbyte(uint32_t w, int i) { return (int)(int8_t)(w >> (8 * i)); }

// Q6_K bits of element group (k): nibble (k>>1) of the ql word | 2 qh bits (2k) << 4.
__device__ __forceinline__ uint32_t q6_bytes(uint32_t ql, uint32_t qh, int k) {
  const uint32_t lo = (k >> 1) ? ((ql >> 4) & 0x0F0F0F0Fu) : (ql & 0x0F0F0F0Fu);
  const uint32_t hi = (k <= 2 ? (qh << (4 - 2 * k)) : (qh >> (2 * k - 4))) & 0x30303030u;
  return lo | hi;
}

// ---------------------------------------------------------------- Q6_K block
// MMA (g, k) covers elements g*128 + 32k + l of rows g and g+8: group A = l in [0,16)
// (scale g*8+2k), group B = l in [16,32) (scale g*8+2k+1); lane tig holds l = 4tig+i
// (A) and 16+4tig+i (B). q is taken unsigned (0..63); the -32 offset is applied in f32
// with the 16-element sums of x.
template <bool AL>
__device__ __forceinline__ void block_q6k(const uint8_t* b0, const uint8_t* b1, int kb,
                                          const int8_t* dig, int ds, const float* xscale,
                                          const float* xsum, int g, int tig, float& acc0,
                                          float& acc1) {
  const float d_0 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(b0 + 208));
  const float d_1 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(b1 + 208));
  uint32_t sw0[4], sw1[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    sw0[i] = ldw<AL>(b0 + 192 + 4 * i);
    sw1[i] = ldw<AL>(b1 + 192 + 4 * i);
  }
  const int n = g;
  const bool nA = n < 3, nB = (n >= 3) && (n < 6);
  const int8_t* dp = dig + (n < 6 ? (n % 3) * ds : 0) + kb * 256 + 4 * tig + (nB ? 16 : 0);
  const bool c0B = (2 * tig) >= 3, c1B = (2 * tig + 1) >= 3;
  int i00 = 0, i01 = 0, i10 = 0, i11 = 0;
#pragma unroll
  for (int hg = 0; hg < 2; ++hg) {
    const uint8_t* p0 = b0 + hg * 64 + 4 * tig;
    const uint8_t* p1 = b1 + hg * 64 + 4 * tig;
    const uint32_t qlA0_0 = ldw<AL>(p0), qlB0_0 = ldw<AL>(p0 + 16);
    const uint32_t qlA1_0 = ldw<AL>(p0 + 32), qlB1_0 = ldw<AL>(p0 + 48);
    const uint32_t qlA0_1 = ldw<AL>(p1), qlB0_1 = ldw<AL>(p1 + 16);
    const uint32_t qlA1_1 = ldw<AL>(p1 + 32), qlB1_1 = ldw<AL>(p1 + 48);
    const uint8_t* h0p = b0 + 128 + hg * 32 + 4 * tig;
    const uint8_t* h1p = b1 + 128 + hg * 32 + 4 * tig;
    const uint32_t qhA_0 = ldw<AL>(h0p), qhB_0 = ldw<AL>(h0p + 16);
    const uint32_t qhA_1 = ldw<AL>(h1p), qhB_1 = ldw<AL>(h1p + 16);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t qlA_0 = (k & 1) ? qlA1_0 : qlA0_0, qlB_0 = (k & 1) ? qlB1_0 : qlB0_0;
      const uint32_t qlA_1 = (k & 1) ? qlA1_1 : qlA0_1, qlB_1 = (k & 1) ? qlB1_1 : qlB0_1;
      const int8_t* dk = dp + hg * 128 + 32 * k;
      const uint32_t bv = (nA || nB) ? *reinterpret_cast<const uint32_t*>(dk) : 0u;
      int D0 = 0, D1 = 0, D2 = 0, D3 = 0;
      mma_u8s8(D0, D1, D2, D3, q6_bytes(qlA_0, qhA_0, k), q6_bytes(qlA_1, qhA_1, k),
               q6_bytes(qlB_0, qhB_0, k), q6_bytes(qlB_1, qhB_1, k), nA ? bv : 0u,
               nB ? bv : 0u);
      const int ga = hg * 8 + 2 * k, gb = ga + 1;
      const int sA0 = sbyte(sw0[ga >> 2], ga & 3), sB0 = sbyte(sw0[gb >> 2], gb & 3);
      const int sA1 = sbyte(sw1[ga >> 2], ga & 3), sB1 = sbyte(sw1[gb >> 2], gb & 3);
      i00 += (c0B ? sB0 : sA0) * D0;
      i01 += (c1B ? sB0 : sA0) * D1;
      i10 += (c0B ? sB1 : sA1) * D2;
      i11 += (c1B ? sB1 : sA1) * D3;
    }
  }
  const float xs = xscale[kb];
  const float w0 = digit_weight(2 * tig), w1 = digit_weight(2 * tig + 1);
  const float v0 = (float)i00 * w0 + (float)i01 * w1;
  const float v1 = (float)i10 * w0 + (float)i11 * w1;
  // -32 offset: sum over scale groups 4tig..4tig+3 of scale * (16-element sum of x)
  const float* xg = xsum + kb * 16 + 4 * tig;
  const uint32_t s0 = tig == 0 ? sw0[0] : tig == 1 ? sw0[1] : tig == 2 ? sw0[2] : sw0[3];
  const uint32_t s1 = tig == 0 ? sw1[0] : tig == 1 ? sw1[1] : tig == 2 ? sw1[2] : sw1[3];
  float o0 = 0.f, o1 = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    o0 += (float)sbyte(s0, i) * xg[i];
    o1 += (float)sbyte(s1, i) * xg[i];
  }
  acc0 += d_0 * (xs * v0 - 32.f * o0);
  acc1 += d_1 * (xs * v1 - 32.f * o1);
}

// ---------------------------------------------------------------- x preparation
// Eight consecutive GEMV inputs starting at k0 (a multiple of 8), after the prologue.
__device__ __forceinline__ void load_input8(const GemvParams& p, int k0, float inv_rms,
                                            float v[8]) {
  if (p.mode == kXBf16) {
    const uint4 r = *reinterpret_cast<const uint4*>(p.xb + k0);
    const uint32_t u[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(u[i] << 16);
      v[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
    }
    return;
  }
  if (p.mode == RRR_X_GQA_V) {
    const int hpk = p.n_q / p.n_kv;
    const int head = k0 / p.hd, e = k0 % p.hd;
    k0 = p.n_q * p.hd + p.n_kv * p.hd + (head / hpk) * p.hd + e;
  }
  const float4 a = *reinterpret_cast<const float4*>(p.x + k0);
  const float4 b = *reinterpret_cast<const float4*>(p.x + k0 + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  if (p.mode == RRR_X_RMSNORM) {
    const float4 ga = *reinterpret_cast<const float4*>(p.gamma + k0);
    const float4 gb = *reinterpret_cast<const float4*>(p.gamma + k0 + 4);
    const float gg[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fmul_rn(gg[i], v[i]), inv_rms);
  } else if (p.mode == RRR_X_SILU_GATE) {
    const float4 ua = *reinterpret_cast<const float4*>(p.x + p.K + k0);
    const float4 ub = *reinterpret_cast<const float4*>(p.x + p.K + k0 + 4);
    const float uu[8] = {ua.x, ua.y, ua.z, ua.w, ub.x, ub.y, ub.z, ub.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float s = __fdiv_rn(v[i], __fadd_rn(1.0f, expf(-v[i])));
      v[i] = __fmul_rn(s, uu[i]);
    }
  }
}

__device__ void prepare_x(const GemvParams& p, int8_t* dig, float* xscale, float* xsum,
                          float* misc, int warp, int lane) {
  const int NT = kNW * 32, t = warp * 32 + lane;
  float inv_rms = 1.f;
  if (p.mode == RRR_X_RMSNORM) {
    float ss = 0.f;
    for (int k4 = t; k4 < p.K / 4; k4 += NT) {
      const float4 v = reinterpret_cast<const float4*>(p.x)[k4];
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    ss = warp_sum(ss);
    if (lane == 0) misc[warp] = ss;
    named_barrier(1, NT);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kNW; ++w) tot += misc[w];
    inv_rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)p.K), p.eps)));
  }
  for (int b = warp; b < p.nb; b += kNW) {
    const int k0 = b * 256 + lane * 8;
    float v[8];
    load_input8(p, k0, inv_rms, v);
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(v[i]));
    m = warp_max(m);
    const float inv = m > 0.f ? 127.f / m : 0.f;
    uint32_t q[3][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}};
    float s8 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float t0 = v[i] * inv;
      const float r0 = rintf(t0);
      const float t1 = (t0 - r0) * 128.f;
      const float r1 = rintf(t1);
      const float r2 = rintf((t1 - r1) * 128.f);
      q[0][i >> 2] |= ((uint32_t)(int)r0 & 0xFFu) << (8 * (i & 3));
      q[1][i >> 2] |= ((uint32_t)(int)r1 & 0xFFu) << (8 * (i & 3));
      q[2][i >> 2] |= ((uint32_t)(int)r2 & 0xFFu) << (8 * (i & 3));
      s8 += v[i];
    }
#pragma unroll
    for (int dgt = 0; dgt < 3; ++dgt)
      *reinterpret_cast<uint2*>(dig + dgt * p.dig_stride + k0) = make_uint2(q[dgt][0], q[dgt][1]);
    const float s16 = s8 + __shfl_xor_sync(0xffffffffu, s8, 1);
    if ((lane & 1) == 0) xsum[b * 16 + (lane >> 1)] = s16;
    if (lane == 0) xscale[b] = m * (1.f / 127.f);
  }
}

// ---------------------------------------------------------------- the kernel
template <int QT>
__global__ void __launch_bounds__((kNW + 1) * 32) gemv_kq_kernel(const GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int BB = KQ<QT>::kBlockBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_bars);
  uint64_t* empty = full + p.nstages;
  int8_t* dig = reinterpret_cast<int8_t*>(smem + p.off_dig);
  float* xscale = reinterpret_cast<float*>(smem + p.off_xscale);
  float* xsum = reinterpret_cast<float*>(smem + p.off_xsum);
  float* red = reinterpret_cast<float*>(smem + p.off_red);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + p.off_misc);
  float* misc = reinterpret_cast<float*>(smem + p.off_misc + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.nstages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kNW);
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kNW) {
    // ------------------------------------------------------------ producer warp
    const long long floor_total = p.total_bytes & ~15ll;
    int it = 0, issued = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.n_tiles && ok; tile += gridDim.x) {
      const int rows = min(kTileRows, p.N - tile * kTileRows);
      for (int c = 0; c < p.n_chunks && ok; ++c, ++it) {
        const int s = it % p.nstages;
        const uint32_t ph = (uint32_t)(it / p.nstages) & 1u;
        if (it >= p.nstages) {
          int w = 1;
          if (lane == 0) {
            w = mbar_wait_bounded(&empty[s], ph ^ 1u, p.err, kDevErrEmptyTimeout) ? 1 : 0;
            if (!w) *abort_flag = 1;
          }
          w = __shfl_sync(0xffffffffu, w, 0);
          if (!w || *abort_flag) { ok = false; break; }
        }
        const int kb0 = c * p.kc;
        const int kcount = min(p.kc, p.nb - kb0);
        const long long chunk = (long long)kcount * BB;
        uint8_t* stage = smem + (size_t)s * p.stage_bytes;
        long long a0 = 0, a1 = 0;
        uint32_t tx = 0;
        if (lane < rows) {
          const long long start = (long long)(tile * kTileRows + lane) * p.row_bytes + (long long)kb0 * BB;
          const long long end = start + chunk;
          a0 = start & ~15ll;
          a1 = min((end + 15) & ~15ll, floor_total);
          if (a1 < a0) a1 = a0;
          tx = (uint32_t)(a1 - a0);
          // bytes after the last whole 16-B granule of the buffer: plain loads
          for (long long q = max(a1, start); q < end; ++q)
            stage[lane * p.row_stride + (int)(q - a0)] = p.w[q];
        }
        uint32_t tot = tx;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
        __syncwarp();
        if (lane == 0) mbar_arrive_expect_tx(&full[s], tot);
        __syncwarp();
        if (tx > 0) bulk_g2s(stage + lane * p.row_stride, p.w + a0, tx, &full[s]);
        ++issued;
      }
    }
    // No copy may still be in flight when the CTA exits.
    if (lane == 0) {
      const int first = issued > p.nstages ? issued - p.nstages : 0;
      for (int i = first; i < issued; ++i)
        mbar_wait_bounded(&full[i % p.nstages], (uint32_t)(i / p.nstages) & 1u, p.err,
                          kDevErrDrainTimeout);
    }
    return;
  }

  // -------------------------------------------------------------- consumer warps
  pdl_wait();
  prepare_x(p, dig, xscale, xsum, misc, warp, lane);
  named_barrier(1, kNW * 32);

  const int g = lane >> 2, tig = lane & 3;
  int it = 0, par = 0;
  for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
    const int rows = min(kTileRows, p.N - tile * kTileRows);
    float acc0 = 0.f, acc1 = 0.f;
    for (int c = 0; c < p.n_chunks; ++c, ++it) {
      const int s = it % p.nstages;
      const uint32_t ph = (uint32_t)(it / p.nstages) & 1u;
      bool have = (*abort_flag == 0);
      if (have) {
        have = mbar_wait_bounded(&full[s], ph, p.err, kDevErrFullTimeout);
        if (!have) *abort_flag = 1;
      }
      if (!have) continue;
      const int kb0 = c * p.kc;
      const int kcount = min(p.kc, p.nb - kb0);
      const uint8_t* stage = smem + (size_t)s * p.stage_bytes;
      const long long base = (long long)tile * kTileRows * p.row_bytes + (long long)kb0 * BB;
      const int off0 = (int)((base + (long long)g * p.row_bytes) & 15);
      const int off1 = (int)((base + (long long)(g + 8) * p.row_bytes) & 15);
      const uint8_t* r0 = stage + g * p.row_stride + off0;
      const uint8_t* r1 = stage + (g + 8) * p.row_stride + off1;
      for (int bi = warp; bi < kcount; bi += kNW) {
        const uint8_t* q0 = r0 + bi * BB;
        const uint8_t* q1 = r1 + bi * BB;
        if constexpr (QT == RRR_Q4_K) {
          block_q4k(q0, q1, kb0 + bi, dig, p.dig_stride, xscale, xsum, g, tig, acc0, acc1);
        } else if constexpr (QT == RRR_Q5_K) {
          block_q5k(q0, q1, kb0 + bi, dig, p.dig_stride, xscale, xsum, g, tig, acc0, acc1);
        } else {
          const bool al = __all_sync(0xffffffffu, (((uintptr_t)q0 | (uintptr_t)q1) & 3) == 0);
          if (al)
            block_q6k<true>(q0, q1, kb0 + bi, dig, p.dig_stride, xscale, xsum, g, tig, acc0, acc1);
          else
            block_q6k<false>(q0, q1, kb0 + bi, dig, p.dig_stride, xscale, xsum, g, tig, acc0, acc1);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
    float* rb = red + par * kNW * kTileRows;
    if (tig == 0) {
      rb[warp * kTileRows + g] = acc0;
      rb[warp * kTileRows + g + 8] = acc1;
    }
    named_barrier(1, kNW * 32);
    if (threadIdx.x < rows && *abort_flag == 0) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kNW; ++w) v += rb[w * kTileRows + threadIdx.x];
      const int row = tile * kTileRows + threadIdx.x;
      if (p.residual) v = p.residual[row] + v;
      p.y[row] = v;
    }
    par ^= 1;
  }
}

template <int QT>
cudaError_t launch_t(const LaunchEnv& env, GemvParams& p) {
  constexpr int BB = KQ<QT>::kBlockBytes;
  const int kc_max = (QT == RRR_Q6_K) ? 8 : 12;
  const int n_ch = (p.nb + kc_max - 1) / kc_max;
  p.kc = (p.nb + n_ch - 1) / n_ch;
  p.n_chunks = (p.nb + p.kc - 1) / p.kc;
  p.n_tiles = (p.N + kTileRows - 1) / kTileRows;
  const int chunk = p.kc * BB;
  p.row_stride = ((chunk + 32 + 127) / 128) * 128 + (QT == RRR_Q6_K ? 16 : 32);
  p.stage_bytes = kTileRows * p.row_stride;
  p.nstages = 2;
  p.dig_stride = p.K + 96;
  int off = p.nstages * p.stage_bytes;
  p.off_bars = off;          off += 2 * p.nstages * 8;
  p.off_dig = off;           off += 3 * p.dig_stride;
  off = (off + 15) & ~15;
  p.off_xscale = off;        off += p.nb * 4;
  p.off_xsum = off;          off += (p.K / 16) * 4;
  p.off_red = off;           off += 2 * kNW * kTileRows * 4;
  p.off_misc = off;          off += 16 + kNW * 4;
  const int smem = (off + 127) & ~127;

  static unsigned long long configured = 0;  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured & (1ull << (dev & 63)))) {
    cudaError_t e = cudaFuncSetAttribute(gemv_kq_kernel<QT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    configured |= 1ull << (dev & 63);
  }
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_kq_kernel<QT>,
                                                                (kNW + 1) * 32, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  const int grid = std::min(p.n_tiles, per_sm * env.sm_count);
  return rrr_launch_pdl(gemv_kq_kernel<QT>, dim3(grid), dim3((kNW + 1) * 32), smem,
                        env.stream, env.pdl, p);
}

// ---------------------------------------------------------------- layout self-test
// m16n8k32 u8 x s8 -> s32 through mma_u8s8 with A[r][k] = (r*7 + k*3) & 0xFF,
// B[k][n] = ((k*5 + n*11) & 0xFF) - 128, against the expected products.
__global__ void mma_selftest_kernel(int* ok) {
  const int lane = threadIdx.x, g = lane >> 2, tig = lane & 3;
  auto A = [](int r, int k) -> uint32_t { return (uint32_t)((r * 7 + k * 3) & 0xFF); };
  auto B = [](int k, int n) -> int { return ((k * 5 + n * 11) & 0xFF) - 128; };
  uint32_t a[4] = {0, 0, 0, 0}, b[2] = {0, 0};
  for (int i = 0; i < 4; ++i) {
    a[0] |= A(g, 4 * tig + i) << (8 * i);
    a[1] |= A(g + 8, 4 * tig + i) << (8 * i);
    a[2] |= A(g, 16 + 4 * tig + i) << (8 * i);
    a[3] |= A(g + 8, 16 + 4 * tig + i) << (8 * i);
    b[0] |= ((uint32_t)B(4 * tig + i, g) & 0xFFu) << (8 * i);
    b[1] |= ((uint32_t)B(16 + 4 * tig + i, g) & 0xFFu) << (8 * i);
  }
  int d[4] = {0, 0, 0, 0};
  mma_u8s8(d[0], d[1], d[2], d[3], a[0], a[1], a[2], a[3], b[0], b[1]);
  int good = 1;
  for (int i = 0; i < 4; ++i) {
    const int r = g + (i >= 2 ? 8 : 0), n = 2 * tig + (i & 1);
    int ref = 0;
    for (int k = 0; k < 32; ++k) ref += (int)A(r, k) * B(k, n);
    if (ref != d[i]) good = 0;
  }
  good = __all_sync(0xffffffffu, good);
  if (lane == 0) *ok = good;
}

}  // namespace

cudaError_t launch_gemv_kq(const LaunchEnv& env, int qtype, const void* w, const float* x,
                           float* y, int K, int N, const float* residual,
                           const rrr_gemv_prologue* pro) {
  GemvParams p = {};
  p.w = static_cast<const uint8_t*>(w);
  p.x = x;
  p.y = y;
  p.residual = residual;
  p.mode = pro ? pro->mode : RRR_X_PLAIN;
  p.gamma = pro ? pro->gamma : nullptr;
  p.eps = pro ? pro->eps : 0.f;
  p.n_q = pro ? pro->n_q_heads : 0;
  p.n_kv = pro ? pro->n_kv_heads : 0;
  p.hd = pro ? pro->head_dim : 0;
  p.K = K;
  p.N = N;
  p.nb = K / 256;
  p.row_bytes = (long long)p.nb * kq_block_bytes(qtype);
  p.total_bytes = p.row_bytes * N;
  p.err = env.d_err;
  switch (qtype) {
    case RRR_Q4_K: return launch_t<RRR_Q4_K>(env, p);
    case RRR_Q5_K: return launch_t<RRR_Q5_K>(env, p);
    case RRR_Q6_K: return launch_t<RRR_Q6_K>(env, p);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemv_kq_bf16(const LaunchEnv& env, int qtype, const void* w,
                                const uint16_t* x, float* y, int K, int N) {
  GemvParams p = {};
  p.w = static_cast<const uint8_t*>(w);
  p.xb = x;
  p.y = y;
  p.mode = kXBf16;
  p.K = K;
  p.N = N;
  p.nb = K / 256;
  p.row_bytes = (long long)p.nb * kq_block_bytes(qtype);
  p.total_bytes = p.row_bytes * N;
  p.err = env.d_err;
  switch (qtype) {
    case RRR_Q4_K: return launch_t<RRR_Q4_K>(env, p);
    case RRR_Q5_K: return launch_t<RRR_Q5_K>(env, p);
    case RRR_Q6_K: return launch_t<RRR_Q6_K>(env, p);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_mma_selftest(const LaunchEnv& env, int* d_ok) {
  mma_selftest_kernel<<<1, 32, 0, env.stream>>>(d_ok);
  return cudaGetLastError();
}

}  // namespace rrr
