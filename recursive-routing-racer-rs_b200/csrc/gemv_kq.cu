// gemv_kq.cu — kernel (1): fused raw-block K-quant GEMV, y = W x (+ residual), for the
// Q4_K / Q5_K / Q6_K super-blocks GGUF stores (reference: gpu_matmul_kquant and the
// matmul_q{4,5,6}k dispatches, src/model/phi4.rs:631-658, 1081-1096; element formats
// phi4.rs:444-542).
//
// Design (sm_100a, HBM-bound):
//  * One CTA = 1 producer warp + 8 consumer warps, two CTAs per SM. The producer streams 16-row tiles of raw blocks (K
//    split into chunks of kc blocks) with 1-D bulk copies (cp.async.bulk, mbarrier
//    complete_tx) into a ring of shared-memory stages; consumers free a stage through an
//    "empty" mbarrier. Every wait is bounded (%globaltimer) and reports through the
//    context's error flag instead of hanging.
//  * x is decomposed once per CTA into four int8 "digits" per element against a per-
//    256-element power-of-two scale xs = 2^(E-20), E = floor(log2 max|x|):
//    x ~= xs*(d0 + 256*d1 + 65536*d2 + d3/128), |error| <= xs/256 <= max|x|*2^-28
//    (elements within 1/16 of the block maximum are represented exactly). The per-scale-
//    group sums sum_j q_j*x_j then come from exact integer tensor-core dot products
//    (mma.sync m16n8k32, u8 quants x s8 digits, s32 accumulate): a 16-row x 32-weight
//    tile per instruction, the digits of two scale groups in B columns 0-3 and 4-7.
//    Scales are applied by integer multiply-add per
//    group, d / dmin in f32 once per half block. The CUDA cores do about one instruction
//    per weight, so the kernel stays memory-bound. Dequantised weights are never
//    materialised; the bit-exact dequantisation is rrr_dequant_kq (kernels.cu).
//  * Work items are whole blocks (256 weights of 16 rows); the warp that takes the first
//    block rotates from stage to stage so that the blocks of a stage (12 for K = 3072,
//    8 for Q6_K K = 8192) spread evenly over the warps.
//  * Tile epilogue: shuffle reduction over the 4 lanes that share a row, then a
//    deterministic sum over warps through shared memory, + residual, store. The SwiGLU
//    output mode pairs gate row tile t with up row tile t (rows F + 16t ...) in one CTA
//    and stores silu(gate) * up (the `silu_gate` shader, phi4.rs:1368-1373, fused).
//  * Programmatic dependent launch: the producer starts streaming weights before
//    griddepcontrol.wait; x is read and y written only after it.
//  * Tensor-parallel step on peer memory (GemvFuse): the RMSNORM prologue can take its input
//    as the rank-order sum of the G ranks' tagged partial rows (the all-reduce of the
//    previous O-projection / down, waited for word by word), and the plain epilogue can push
//    each finished row, tagged, to every rank instead of storing it: the exchange kernels
//    between the GEMVs disappear.
#include <algorithm>
#include <cstdlib>

#include "internal.h"
#include "kquant.cuh"

namespace rrr {
namespace {

constexpr int kTileRows = 16;
constexpr int kNW = 8;                  // consumer warps per group
constexpr int kGroups = 2;              // producer + consumer groups per CTA; they share the
                                        // x digits, which are prepared once per CTA
constexpr int kThreads = kGroups * (kNW + 1) * 32;
constexpr int kMinCtas = 2 / kGroups;   // CTAs per SM
constexpr int kXBf16 = 100;             // internal prologue mode: x is bf16 (batched path)
constexpr int kSmemBudget = 113 * 1024 * kGroups;  // 226 KB per SM
constexpr int kMaxStages = 6;
constexpr int kSlots = 8;               // row-tile reduction slots (> stages + 1)

struct GemvParams {
  const uint8_t* w;
  const float* x;
  const uint16_t* xb;  // bf16 input (mode kXBf16)
  float* y;
  const float* residual;
  const float* gamma;
  float eps;
  int mode, out_mode, n_q, n_kv, hd, k_off;
  int K, N, nb;        // N: weight rows
  long long row_bytes, total_bytes;
  int kc, n_chunks, n_tiles, half_rows;
  int row_stride, stage_bytes, nstages, dig_stride;
  int off_bars, off_dig, off_xscale, off_xsum, off_red, off_gate, off_misc;
  int* err;
  // fused tensor-parallel exchange (GemvFuse; G = 0: off)
  const unsigned long long* sum_in;
  float* h_out;
  unsigned long long* push[kMaxTpRanks];
  int G;
  const unsigned* epoch;
  int x_early;  // prepare x before the grid dependency wait (x not written by overlapping kernels)
  // timeline records of this launch (rrr_set_trace; null: off): 8 u64 per CTA
  unsigned long long* trace;
  unsigned long long trace_tag;  // launch sequence number << 16
};

__device__ __forceinline__ void mma_u8s8(int& d0, int& d1, int& d2, int& d3, uint32_t a0,
                                         uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d0), "+r"(d1), "+r"(d2), "+r"(d3)
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// First MMA of an accumulation chain (C = 0).
__device__ __forceinline__ void mma_u8s8_z(int& d0, int& d1, int& d2, int& d3, uint32_t a0,
                                           uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                           uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// prmt selector of byte i of a word, sign-extended to 32 bits (selector nibbles with bit 3
// set replicate the sign of the selected byte). __byte_perm ignores that bit, so the
// permute is issued as prmt.b32 directly (byte_sext).
__host__ __device__ constexpr uint32_t sext_sel(int i) {
  return (uint32_t)i | ((uint32_t)(i | 8) << 4) | ((uint32_t)(i | 8) << 8) | ((uint32_t)(i | 8) << 12);
}
__device__ __forceinline__ int byte_sext(uint32_t w, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(w), "r"(0u), "r"(sel));
  return (int)r;
}

// Lane roles inside an MMA tile: rows g and g+8 of the A operand; B column n = g carries
// digit n of scale group A (n = 0..3) or digit n-4 of group B (n = 4..7); the lane's D
// columns 2*tig, 2*tig+1 therefore belong to a single group (hb = tig >> 1), so one scale
// per row applies to both.
struct Lane {
  int g, tig, hb;
  uint32_t mA, mB;  // masks selecting which half of a compact B fragment this lane fills
  int dsel;         // digit supplied in B column g (compact layout)
  int frag_off;     // byte offset of this lane's B fragment inside a pair (fragment layout)
  float w0, w1;     // f32 weights of the lane's two D columns
  uint32_t msel0, msel1;  // byte permutes placing min byte 2(tig&1) / +1 under 2^23's exponent
  uint32_t ssel;  // byte permute extracting scale byte hb (zero-extended); + 2: byte 2 + hb
};

__device__ __forceinline__ Lane make_lane(int lane, bool q4) {
  Lane L;
  L.g = lane >> 2;
  L.tig = lane & 3;
  L.hb = L.tig >> 1;
  L.msel0 = 0x7440u | (uint32_t)(2 * (L.tig & 1));
  L.msel1 = 0x7440u | (uint32_t)(2 * (L.tig & 1) + 1);
  L.ssel = 0x4440u | (uint32_t)L.hb;
  L.mA = L.g < 4 ? 0xFFFFFFFFu : 0u;
  L.mB = L.g >= 4 ? 0xFFFFFFFFu : 0u;
  L.dsel = L.g & 3;
  L.frag_off = (L.g * 4 + L.tig) * 16;
  // columns: tig 0 -> (d0, d1), tig 1 -> (d2, d3), tig 2 -> (d0, d1), tig 3 -> (d2, d3)
  const float scale = (q4 && L.hb) ? (1.f / 16.f) : 1.f;  // Q4_K high nibbles enter x16
  L.w0 = ((L.tig & 1) ? 65536.f : 1.f) * scale;
  L.w1 = ((L.tig & 1) ? (1.f / 128.f) : 256.f) * scale;
  return L;
}

// Exact float of byte (sel & 3) of w: one permute puts the byte under the exponent of
// 2^23 (0x4B000000), one subtraction removes it (sel = 0x7440 | byte index).
__device__ __forceinline__ float byte_u2f(uint32_t w, uint32_t sel) {
  return __fsub_rn(__uint_as_float(__byte_perm(w, 0x4B000000u, sel)), 8388608.0f);
}

// qh bit `s` of each byte moved to bit 4.
__device__ __forceinline__ uint32_t qh_bit4(uint32_t x, int s) {
  return (s <= 4 ? (x << (4 - s)) : (x >> (s - 4))) & 0x10101010u;
}

// B fragments of one sub-block pair (64 x elements) for the two MMAs of the pair:
// (b0, b1) of MMA 1 and (b0, b1) of MMA 2. FRAG: read ready-made from the per-lane
// fragment layout (one 16-byte load); otherwise from the compact digit rows with masks.
template <bool FRAG>
__device__ __forceinline__ uint4 load_bfrag(const int8_t* dig, int ds, int pair, const Lane& L) {
  if (FRAG) return *reinterpret_cast<const uint4*>(dig + pair * 512 + L.frag_off);
  const uint2 bb = *reinterpret_cast<const uint2*>(dig + L.dsel * ds + pair * 64 + 8 * L.tig +
                                                   (L.mB ? 32 : 0));
  return make_uint4(bb.x & L.mA, bb.x & L.mB, bb.y & L.mA, bb.y & L.mB);
}

// One Q4_K / Q5_K block (256 weights) of rows g and g+8. MMA (pair p, half-word h) covers
// qs bytes 32p + 8*tig + 4h .. +3 of both rows: low nibbles = sub 2p (group A, k-slots
// 0-15), high nibbles = sub 2p+1 (group B, k-slots 16-31). For Q4_K the high nibbles
// enter as (byte & 0xF0) = 16*q (no shift). Scale / min unpacking follows phi4.rs:492-498
// four sub-blocks per 32-bit word; the integer scale of each pair is applied to the s32
// sums by multiply-add, d and dmin once per block in f32.
template <int QT, bool FRAG>
__device__ __forceinline__ void block_q45(const uint8_t* b0, const uint8_t* b1, int kb,
                                          const int8_t* dig, int ds, const float* xscale,
                                          const float* xsum32, const Lane& L, float& acc0,
                                          float& acc1) {
  constexpr int QS = (QT == RRR_Q4_K) ? 16 : 48;
  const uint4 h0 = *reinterpret_cast<const uint4*>(b0);
  const uint4 h1 = *reinterpret_cast<const uint4*>(b1);
  // this lane's group (sub 2p + hb): byte 2*(p&1) + hb of the packed word of subs 0-3 / 4-7
  const uint32_t s03_0 = h0.y & 0x3F3F3F3Fu;
  const uint32_t s47_0 = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
  const uint32_t s03_1 = h1.y & 0x3F3F3F3Fu;
  const uint32_t s47_1 = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
  uint2 qh0 = make_uint2(0u, 0u), qh1 = make_uint2(0u, 0u);
  if (QT == RRR_Q5_K) {
    qh0 = *reinterpret_cast<const uint2*>(b0 + 16 + 8 * L.tig);
    qh1 = *reinterpret_cast<const uint2*>(b1 + 16 + 8 * L.tig);
  }
  int i00 = 0, i01 = 0, i10 = 0, i11 = 0;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint2 w = *reinterpret_cast<const uint2*>(b0 + QS + 32 * p + 8 * L.tig);
    const uint2 v = *reinterpret_cast<const uint2*>(b1 + QS + 32 * p + 8 * L.tig);
    const uint4 bf = load_bfrag<FRAG>(dig, ds, kb * 4 + p, L);
    int D0, D1, D2, D3;
    if (QT == RRR_Q4_K) {
      mma_u8s8_z(D0, D1, D2, D3, w.x & 0x0F0F0F0Fu, v.x & 0x0F0F0F0Fu, w.x & 0xF0F0F0F0u,
                 v.x & 0xF0F0F0F0u, bf.x, bf.y);
      mma_u8s8(D0, D1, D2, D3, w.y & 0x0F0F0F0Fu, v.y & 0x0F0F0F0Fu, w.y & 0xF0F0F0F0u,
               v.y & 0xF0F0F0F0u, bf.z, bf.w);
    } else {
      const int sa = 2 * p, sb = 2 * p + 1;
      mma_u8s8_z(D0, D1, D2, D3, (w.x & 0x0F0F0F0Fu) | qh_bit4(qh0.x, sa),
                 (v.x & 0x0F0F0F0Fu) | qh_bit4(qh1.x, sa),
                 ((w.x >> 4) & 0x0F0F0F0Fu) | qh_bit4(qh0.x, sb),
                 ((v.x >> 4) & 0x0F0F0F0Fu) | qh_bit4(qh1.x, sb), bf.x, bf.y);
      mma_u8s8(D0, D1, D2, D3, (w.y & 0x0F0F0F0Fu) | qh_bit4(qh0.y, sa),
               (v.y & 0x0F0F0F0Fu) | qh_bit4(qh1.y, sa),
               ((w.y >> 4) & 0x0F0F0F0Fu) | qh_bit4(qh0.y, sb),
               ((v.y >> 4) & 0x0F0F0F0Fu) | qh_bit4(qh1.y, sb), bf.z, bf.w);
    }
    const uint32_t ssel = L.ssel + ((p & 1) ? 2u : 0u);
    const int r0 = (int)__byte_perm(p < 2 ? s03_0 : s47_0, 0u, ssel);
    const int r1 = (int)__byte_perm(p < 2 ? s03_1 : s47_1, 0u, ssel);
    i00 += r0 * D0;
    i01 += r0 * D1;
    i10 += r1 * D2;
    i11 += r1 * D3;
  }
  const float xs = xscale[kb];
  const float d0 = f16_bits_to_f32(h0.x & 0xFFFFu), d1 = f16_bits_to_f32(h1.x & 0xFFFFu);
  const float dm0 = f16_bits_to_f32(h0.x >> 16), dm1 = f16_bits_to_f32(h1.x >> 16);
  // min term of sub-blocks 2*tig, 2*tig+1 (bytes 2(tig&1), +1 of the mins of subs 0-3 /
  // 4-7): dmin * (m_a * S_a + m_b * S_b), S = sum of x over the sub-block
  const uint32_t mw0 = L.tig < 2 ? (h0.z & 0x3F3F3F3Fu)
                                 : (((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u));
  const uint32_t mw1 = L.tig < 2 ? (h1.z & 0x3F3F3F3Fu)
                                 : (((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u));
  const float2 S = *reinterpret_cast<const float2*>(xsum32 + kb * 8 + 2 * L.tig);
  const float mt0 = byte_u2f(mw0, L.msel0) * S.x + byte_u2f(mw0, L.msel1) * S.y;
  const float mt1 = byte_u2f(mw1, L.msel0) * S.x + byte_u2f(mw1, L.msel1) * S.y;
  acc0 += d0 * xs * ((float)i00 * L.w0 + (float)i01 * L.w1) - dm0 * mt0;
  acc1 += d1 * xs * ((float)i10 * L.w0 + (float)i11 * L.w1) - dm1 * mt1;
}

// 32-bit load from a shared-memory byte address p with p % 4 == MIS for MIS = 0 or 2
// (Q6_K blocks of 210 bytes start 4-byte aligned or 2 bytes past; rows and chunks start
// at even offsets), or, MIS = 1, either of the two per lane.
template <int MIS>
__device__ __forceinline__ uint32_t ldw(const uint8_t* p) {
  if (MIS == 0) return *reinterpret_cast<const uint32_t*>(p);
  if (MIS == 2) {  // two bytes past a 4-byte boundary (every lane of the warp)
    const uint32_t* q = reinterpret_cast<const uint32_t*>(p - 2);
    return __byte_perm(q[0], q[1], 0x5432);
  }
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* q = reinterpret_cast<const uint32_t*>(a & ~static_cast<uintptr_t>(3));
  return __byte_perm(q[0], q[1], (a & 2) ? 0x5432 : 0x3210);
}

// The same for lanes whose blocks start at different offsets mod 4 (0 or 2): the aligned
// base and the permute selector are taken once per block (b = block start of this lane).
struct LaneWords {
  const uint8_t* base;  // b rounded down to 4 bytes
  uint32_t sel;         // byte permute of two aligned words
  __device__ __forceinline__ explicit LaneWords(const uint8_t* b)
      : base(b - (reinterpret_cast<uintptr_t>(b) & 2)),
        sel((reinterpret_cast<uintptr_t>(b) & 2) ? 0x5432u : 0x3210u) {}
  // word at byte offset off (a multiple of 4) of the block
  __device__ __forceinline__ uint32_t operator()(int off) const {
    const uint32_t* q = reinterpret_cast<const uint32_t*>(base + off);
    return __byte_perm(q[0], q[1], sel);
  }
};

__device__ __forceinline__ int sbyte(uint32_t w, int i) { return (int)(int8_t)(w >> (8 * i)); }

// Q6_K bits of element group k: nibble (k>>1) of the ql word | 2 qh bits (2k) << 4.
__device__ __forceinline__ uint32_t q6_bytes(uint32_t ql, uint32_t qh, int k) {
  const uint32_t lo = (k >> 1) ? ((ql >> 4) & 0x0F0F0F0Fu) : (ql & 0x0F0F0F0Fu);
  const uint32_t hi = (k <= 2 ? (qh << (4 - 2 * k)) : (qh >> (2 * k - 4))) & 0x30303030u;
  return lo | hi;
}

// One Q6_K block of rows g and g+8. MMA (hg, k) covers elements hg*128 + 32k + l: group
// A = l in [0,16) (scale hg*8+2k), group B = l in [16,32) (scale hg*8+2k+1); lane tig
// holds l = 4tig+i (A) and 16+4tig+i (B) (element layout of phi4.rs:456-475). q is taken
// unsigned (0..63); the -32 offset is applied in f32 with the 16-element sums of x.
template <int AL>
__device__ __forceinline__ void block_q6(const uint8_t* b0, const uint8_t* b1, int kb,
                                         const int8_t* dig, int ds, const float* xscale,
                                         const float* xsum, const Lane& L, float& acc0,
                                         float& acc1) {
  // word readers of this lane's two rows (AL 1: per-lane base and selector, once)
  const LaneWords lw0(b0), lw1(b1);
  auto W0 = [&](int off) { return AL == 1 ? lw0(off) : ldw<AL>(b0 + off); };
  auto W1 = [&](int off) { return AL == 1 ? lw1(off) : ldw<AL>(b1 + off); };
  uint32_t sw0[4], sw1[4];
  if (AL == 2) {
    // the 16 scale bytes as five aligned words shifted by two bytes
    const uint32_t* q0 = reinterpret_cast<const uint32_t*>(b0 + 190);
    const uint32_t* q1 = reinterpret_cast<const uint32_t*>(b1 + 190);
    uint32_t w0[5], w1[5];
#pragma unroll
    for (int i = 0; i < 5; ++i) {
      w0[i] = q0[i];
      w1[i] = q1[i];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      sw0[i] = __byte_perm(w0[i], w0[i + 1], 0x5432);
      sw1[i] = __byte_perm(w1[i], w1[i + 1], 0x5432);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      sw0[i] = W0(192 + 4 * i);
      sw1[i] = W1(192 + 4 * i);
    }
  }
  const int8_t* dp = dig + L.dsel * ds + kb * 256 + 4 * L.tig + (L.mB ? 16 : 0);
  int i00 = 0, i01 = 0, i10 = 0, i11 = 0;
#pragma unroll
  for (int hg = 0; hg < 2; ++hg) {
    const int pq = hg * 64 + 4 * L.tig, ph = 128 + hg * 32 + 4 * L.tig;
    const uint32_t qlA0_0 = W0(pq), qlB0_0 = W0(pq + 16);
    const uint32_t qlA1_0 = W0(pq + 32), qlB1_0 = W0(pq + 48);
    const uint32_t qlA0_1 = W1(pq), qlB0_1 = W1(pq + 16);
    const uint32_t qlA1_1 = W1(pq + 32), qlB1_1 = W1(pq + 48);
    const uint32_t qhA_0 = W0(ph), qhB_0 = W0(ph + 16);
    const uint32_t qhA_1 = W1(ph), qhB_1 = W1(ph + 16);
    // this lane's scale group of MMA k: byte 2*(k&1) + hb of word 2hg + (k >> 1)
    const uint32_t tA0 = sw0[2 * hg] >> (8 * L.hb), tB0 = sw0[2 * hg + 1] >> (8 * L.hb);
    const uint32_t tA1 = sw1[2 * hg] >> (8 * L.hb), tB1 = sw1[2 * hg + 1] >> (8 * L.hb);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t qlA_0 = (k & 1) ? qlA1_0 : qlA0_0, qlB_0 = (k & 1) ? qlB1_0 : qlB0_0;
      const uint32_t qlA_1 = (k & 1) ? qlA1_1 : qlA0_1, qlB_1 = (k & 1) ? qlB1_1 : qlB0_1;
      const uint32_t bv = *reinterpret_cast<const uint32_t*>(dp + hg * 128 + 32 * k);
      int D0, D1, D2, D3;
      mma_u8s8_z(D0, D1, D2, D3, q6_bytes(qlA_0, qhA_0, k), q6_bytes(qlA_1, qhA_1, k),
                 q6_bytes(qlB_0, qhB_0, k), q6_bytes(qlB_1, qhB_1, k), bv & L.mA, bv & L.mB);
      constexpr uint32_t qsel0 = sext_sel(0), qsel2 = sext_sel(2);
      const uint32_t qsel = (k & 1) ? qsel2 : qsel0;
      const int sc0 = byte_sext(k < 2 ? tA0 : tB0, qsel);
      const int sc1 = byte_sext(k < 2 ? tA1 : tB1, qsel);
      i00 += sc0 * D0;
      i01 += sc0 * D1;
      i10 += sc1 * D2;
      i11 += sc1 * D3;
    }
  }
  const float xs = xscale[kb];
  const float d_0 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(b0 + 208));
  const float d_1 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(b1 + 208));
  // -32 offset: scale groups 4tig .. 4tig+3 (bytes of word tig)
  const float4 xg = *reinterpret_cast<const float4*>(xsum + kb * 16 + 4 * L.tig);
  const uint32_t t0 = L.tig == 0 ? sw0[0] : L.tig == 1 ? sw0[1] : L.tig == 2 ? sw0[2] : sw0[3];
  const uint32_t t1 = L.tig == 0 ? sw1[0] : L.tig == 1 ? sw1[1] : L.tig == 2 ? sw1[2] : sw1[3];
  const float o0 = (float)sbyte(t0, 0) * xg.x + (float)sbyte(t0, 1) * xg.y +
                   (float)sbyte(t0, 2) * xg.z + (float)sbyte(t0, 3) * xg.w;
  const float o1 = (float)sbyte(t1, 0) * xg.x + (float)sbyte(t1, 1) * xg.y +
                   (float)sbyte(t1, 2) * xg.z + (float)sbyte(t1, 3) * xg.w;
  acc0 += d_0 * (xs * ((float)i00 * L.w0 + (float)i01 * L.w1) - 32.f * o0);
  acc1 += d_1 * (xs * ((float)i10 * L.w0 + (float)i11 * L.w1) - 32.f * o1);
}

// ---------------------------------------------------------------- x preparation
// Raw inputs of elements k0 .. k0+7 (k0 a multiple of 8): v = x (after the GQA index map
// or bf16 widening, or the sum of the ranks' tagged rows of epoch `tag` under GemvFuse), a =
// gamma (RMSNORM) or up (SILU_GATE). `ok` turns false when a tagged word never arrived.
__device__ __forceinline__ void load_raw8(const GemvParams& p, int k0, float v[8], float a[8],
                                          unsigned tag, bool& ok) {
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
  int kx = k0;
  if (p.mode == RRR_X_GQA_V) {
    const int kh = k0 - p.k_off;  // outside the heads' window the input is 0
    if (kh < 0 || kh >= p.n_q * p.hd) {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.f;
      return;
    }
    const int hpk = p.n_q / p.n_kv;
    const int head = kh / p.hd, e = kh % p.hd;
    kx = p.n_q * p.hd + p.n_kv * p.hd + (head / hpk) * p.hd + e;
  }
  if (p.sum_in) {
    // rank order, like the exchange kernel's all-reduce: the same bits on every rank
    for (int r = 0; r < p.G; ++r) {
      const unsigned long long* src = p.sum_in + (size_t)r * p.K + k0;
      unsigned long long w[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) ld_relaxed_sys_v2_u64(src + 2 * i, w[2 * i], w[2 * i + 1]);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float f = __uint_as_float((unsigned)wait_tagged(src + i, w[i], tag, ok, p.err));
        v[i] = r == 0 ? f : v[i] + f;
      }
    }
    if (p.h_out && blockIdx.x == 0) {
      *reinterpret_cast<float4*>(p.h_out + k0) = make_float4(v[0], v[1], v[2], v[3]);
      *reinterpret_cast<float4*>(p.h_out + k0 + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
  } else {
    const float4 x0 = *reinterpret_cast<const float4*>(p.x + kx);
    const float4 x1 = *reinterpret_cast<const float4*>(p.x + kx + 4);
    v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w;
    v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
  }
  const float* aux = p.mode == RRR_X_RMSNORM ? p.gamma + k0
                     : p.mode == RRR_X_SILU_GATE ? p.x + p.K + k0 : nullptr;
  if (aux) {
    const float4 a0 = *reinterpret_cast<const float4*>(aux);
    const float4 a1 = *reinterpret_cast<const float4*>(aux + 4);
    a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
    a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
  }
}

// The GEMV input from the raw values, before the RMS factor: gamma*x for RMSNORM (the
// factor 1/rms of rms_norm(x)*gamma = (gamma*x)*inv, phi4.rs:598, is applied to the finished
// row sums, since every output is linear in the input); silu(g)*u = g/(1+e^-g)*u for
// SILU_GATE (phi4.rs:1368-1373). Returns sum(x^2) of the raw values for RMSNORM.
__device__ __forceinline__ float finish8(const GemvParams& p, float v[8], const float a[8]) {
  float ss = 0.f;
  if (p.mode == RRR_X_RMSNORM) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      ss = fmaf(v[i], v[i], ss);
      v[i] = __fmul_rn(a[i], v[i]);
    }
  } else if (p.mode == RRR_X_SILU_GATE) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      v[i] = __fmul_rn(__fdiv_rn(v[i], __fadd_rn(1.0f, expf(-v[i]))), a[i]);
  }
  return ss;
}

// Byte `i` of four words, packed (a.bi, b.bi, c.bi, d.bi).
template <int I>
__device__ __forceinline__ uint32_t gather_byte(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  constexpr uint32_t sel = (uint32_t)I | ((uint32_t)(I + 4) << 4);  // (x.bI, y.bI) in bytes 0, 1
  return __byte_perm(__byte_perm(a, b, sel), __byte_perm(c, d, sel), 0x5410);
}

// Digits, block scales and partial sums of the GEMV input, in one pass over x: warp w
// handles blocks w, w+8, ..., loading up to kPrepGroup blocks at once (one L2 round trip per
// group while the weight stream loads the memory system). The digits quantise gamma*x per
// 256-block (the RMS factor is applied to the finished row sums instead); misc[warp]
// receives the warp's sum of x^2 (RMSNORM) for that factor.
constexpr int kPrepGroup = 2;

template <bool FRAG>
__device__ __forceinline__ void prepare_x(const GemvParams& p, int8_t* dig, float* xscale, float* xsum,
                          float* misc, int warp, int lane, unsigned tag, bool& ok) {
  constexpr int NPW = kGroups * kNW;  // every consumer warp of the CTA takes part
  float ssq = 0.f;
  for (int bg = warp; bg < p.nb; bg += kPrepGroup * NPW) {
    // the group's blocks bg, bg+8, ...: loads first, then each step for all blocks at once
    // (independent shuffle chains interleave)
    float vg[kPrepGroup][8], ag[kPrepGroup][8];
    const int ng = min(kPrepGroup, (p.nb - bg + NPW - 1) / NPW);
#pragma unroll
    for (int g = 0; g < kPrepGroup; ++g)
      if (g < ng) load_raw8(p, (bg + g * NPW) * 256 + lane * 8, vg[g], ag[g], tag, ok);
    float m[kPrepGroup], s8[kPrepGroup];
#pragma unroll
    for (int g = 0; g < kPrepGroup; ++g) {
      m[g] = 0.f;
      s8[g] = 0.f;
      if (g < ng) {
        ssq += finish8(p, vg[g], ag[g]);
        const float* v = vg[g];
        // max |v| as a tree (NaN ignored as by the sequential fmaxf from 0)
        const float a = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
        const float b = fmaxf(fmaxf(fabsf(v[4]), fabsf(v[5])), fmaxf(fabsf(v[6]), fabsf(v[7])));
        m[g] = fmaxf(fmaxf(a, b), 0.f);
#pragma unroll
        for (int i = 0; i < 8; ++i) s8[g] += v[i];
      }
    }
    // the block maximum over the warp in one integer reduction: non-negative floats order
    // like their bit patterns
#pragma unroll
    for (int g = 0; g < kPrepGroup; ++g)
      m[g] = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m[g])));
    float s16[kPrepGroup], s32[kPrepGroup];
#pragma unroll
    for (int g = 0; g < kPrepGroup; ++g) s16[g] = s8[g] + __shfl_xor_sync(0xffffffffu, s8[g], 1);
#pragma unroll
    for (int g = 0; g < kPrepGroup; ++g) s32[g] = s16[g] + __shfl_xor_sync(0xffffffffu, s16[g], 2);
#pragma unroll
    for (int g = 0; g < kPrepGroup; ++g) {
      if (g >= ng) break;
      const int b = bg + g * NPW;
      const float* v = vg[g];
      // Block scale xs = 2^(E-20) with E = floor(log2 max) (from the exponent field; E
      // is clamped to >= -100 so that 1/xs stays finite, which only coarsens blocks whose
      // maximum is below 2^-100), so |v| / xs < 2^21. T = round(v / xs) comes out of one
      // FMA with the magic number 1.5*2^23 + 0x8080: the result lies in [2^23, 2^24), so its
      // mantissa holds T + 0x8080 + 2^22 exactly, and bytes 0, 1, 2 of the float are the
      // base-256 digits b0, b1 (unsigned) and b2 (7 bits) of T + 0x8080 + 2^22. The signed
      // digits are d0 = b0 - 128, d1 = b1 - 128 (a flip of bit 7), d2 = b2 - 64, so that
      // T = d0 + 256*d1 + 65536*d2 with d0, d1 in [-128, 127] and d2 in [-32, 32]. The
      // remainder v/xs - T (exact in f32, |.| <= 1/2) gives d3 = round(128 * remainder) in
      // [-64, 64] from a second magic FMA (byte 0, offset 128).
      const int E = max((int)((__float_as_uint(m[g]) >> 23) & 0xFFu) - 127, -100);
      const float up = __uint_as_float((uint32_t)(127 + 20 - E) << 23);  // 1/xs = 2^(20-E)
      constexpr float kMagicHi = 12615808.0f;  // 1.5*2^23 + 0x8080
      constexpr float kMagicLo = 12583040.0f;  // 1.5*2^23 + 128
      uint32_t hi[8], lo[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float a = __fmaf_rn(v[i], up, kMagicHi);
        const float r = __fmaf_rn(v[i], up, -__fsub_rn(a, kMagicHi));
        hi[i] = __float_as_uint(a);
        lo[i] = __float_as_uint(__fmaf_rn(r, 128.f, kMagicLo));
      }
      // digit rows of elements 0-3 (m1) and 4-7 (m2)
      auto d2fix = [](uint32_t w) { return ((w | 0x80808080u) - 0x40404040u) ^ 0x80808080u; };
      const uint32_t m1[4] = {gather_byte<0>(hi[0], hi[1], hi[2], hi[3]) ^ 0x80808080u,
                              gather_byte<1>(hi[0], hi[1], hi[2], hi[3]) ^ 0x80808080u,
                              d2fix(gather_byte<2>(hi[0], hi[1], hi[2], hi[3])),
                              gather_byte<0>(lo[0], lo[1], lo[2], lo[3]) ^ 0x80808080u};
      const uint32_t m2[4] = {gather_byte<0>(hi[4], hi[5], hi[6], hi[7]) ^ 0x80808080u,
                              gather_byte<1>(hi[4], hi[5], hi[6], hi[7]) ^ 0x80808080u,
                              d2fix(gather_byte<2>(hi[4], hi[5], hi[6], hi[7])),
                              gather_byte<0>(lo[4], lo[5], lo[6], lo[7]) ^ 0x80808080u};
      if (FRAG) {
        // per-lane B fragments: pair P = 4b + lane/8, group (lane>>2)&1, tig = lane&3;
        // column n of the pair at n*64 + tig*16 holds (b0, b1) of MMA 1 and MMA 2
        const int grp = (lane >> 2) & 1;
        uint8_t* fb = reinterpret_cast<uint8_t*>(dig) + (b * 4 + (lane >> 3)) * 512 + (lane & 3) * 16;
#pragma unroll
        for (int dgt = 0; dgt < 4; ++dgt)
          *reinterpret_cast<uint4*>(fb + (grp * 4 + dgt) * 64) =
              grp ? make_uint4(0u, m1[dgt], 0u, m2[dgt]) : make_uint4(m1[dgt], 0u, m2[dgt], 0u);
      } else {
        const int k0 = b * 256 + lane * 8;
#pragma unroll
        for (int dgt = 0; dgt < 4; ++dgt)
          *reinterpret_cast<uint2*>(dig + dgt * p.dig_stride + k0) = make_uint2(m1[dgt], m2[dgt]);
      }
      if ((lane & 1) == 0) xsum[b * 16 + (lane >> 1)] = s16[g];
      if ((lane & 3) == 0) xsum[p.K / 16 + b * 8 + (lane >> 2)] = s32[g];
      if (lane == 0) xscale[b] = m[g] > 0.f ? __uint_as_float((uint32_t)(127 + E - 20) << 23) : 0.f;
    }
  }
  if (p.mode == RRR_X_RMSNORM) {
    ssq = warp_sum(ssq);
    if (lane == 0) misc[warp] = ssq;
  }
}

// 1/rms of the RMSNORM input from the warps' sums of x^2 (after the barrier that follows
// prepare_x), 1 otherwise: 1 / sqrt(mean(x^2) + eps) (phi4.rs:593-599).
__device__ __forceinline__ float row_scale(const GemvParams& p, const float* misc) {
  if (p.mode != RRR_X_RMSNORM) return 1.f;
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kGroups * kNW; ++w) tot += misc[w];
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)p.K), p.eps)));
}

// Row tile j (0 = gate / plain, 1 = up) of work tile wt: first weight row and row count.
__device__ __forceinline__ int tile_row0(const GemvParams& p, int wt, int j) {
  return (j ? p.half_rows : 0) + wt * kTileRows;
}
__device__ __forceinline__ int tile_rows(const GemvParams& p, int wt) {
  const int lim = p.out_mode ? p.half_rows : p.N;
  return min(kTileRows, lim - wt * kTileRows);
}

// ---------------------------------------------------------------- per-GEMV pipelines
// A group's position in its ring.
struct RingPos {
  int s = 0;          // stage index
  uint32_t ph = 0;    // phase parity of stage s
  int issued = 0;     // producer: stages issued so far
  int ts = 0, ss = 0; // consumers: row-tile and stage sequence numbers
};

// One producer / consumer group's shared memory (the ring and the tile reductions are the
// group's; the x digits and sums are the CTA's).
struct GroupSmem {
  uint64_t* full;
  uint64_t* empty;
  uint8_t* ring;
  int8_t* dig;
  float* xscale;
  float* xsum;
  float* misc;
  float* red;
  float* gate;
  int* cnt;
  volatile int* abort_flag;
  int nstages, stage_bytes;
};

__device__ __forceinline__ GroupSmem group_smem(uint8_t* smem, const GemvParams& p, int grp) {
  GroupSmem g;
  g.full = reinterpret_cast<uint64_t*>(smem + p.off_bars) + grp * 2 * p.nstages;
  g.empty = g.full + p.nstages;
  g.ring = smem + (size_t)grp * p.nstages * p.stage_bytes;
  g.dig = reinterpret_cast<int8_t*>(smem + p.off_dig);
  g.xscale = reinterpret_cast<float*>(smem + p.off_xscale);
  g.xsum = reinterpret_cast<float*>(smem + p.off_xsum);
  g.misc = reinterpret_cast<float*>(smem + p.off_misc + 16);
  g.red = reinterpret_cast<float*>(smem + p.off_red) + grp * kSlots * kNW * kTileRows;
  g.gate = reinterpret_cast<float*>(smem + p.off_gate) + grp * kSlots * kTileRows;
  g.cnt = reinterpret_cast<int*>(smem + p.off_misc + 16 + kGroups * kNW * 4) + grp * kSlots;
  g.abort_flag = reinterpret_cast<volatile int*>(smem + p.off_misc);
  g.nstages = p.nstages;
  g.stage_bytes = p.stage_bytes;
  return g;
}

// Barrier initialisation of the CTA (thread 0): a full barrier (one arrival + bytes) and an
// empty barrier (kNW consumer warps) per stage and group.
__device__ __forceinline__ void init_cta_smem(uint8_t* smem, const GemvParams& p) {
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_bars);
  for (int g = 0; g < kGroups; ++g)
    for (int s = 0; s < p.nstages; ++s) {
      mbar_init(&bars[g * 2 * p.nstages + s], 1);
      mbar_init(&bars[g * 2 * p.nstages + p.nstages + s], kNW);
    }
  *reinterpret_cast<volatile int*>(smem + p.off_misc) = 0;
  int* cnt0 = reinterpret_cast<int*>(smem + p.off_misc + 16 + kGroups * kNW * 4);
  for (int i = 0; i < kGroups * kSlots; ++i) cnt0[i] = 0;
  fence_mbarrier_init();
}

// Producer warp: streams the group's row tiles of one GEMV (tiles vb, vb + vstride, ...)
// into the ring, chunk by chunk, each row of a chunk as one 1-D bulk copy. Returns false
// when the CTA aborted (a bounded wait ran out). limit_scale stretches its waits for free
// stages (consumers that wait for other ranks' rows or other CTAs wait longer first).
template <int QT>
__device__ __forceinline__ bool produce_item(const GemvParams& p, const GroupSmem& g, int vb, int vstride, int lane,
                             RingPos& rp, uint32_t limit_scale) {
  constexpr int BB = KQ<QT>::kBlockBytes;
  const int n_sub = p.out_mode ? 2 : 1;
  const long long floor_total = p.total_bytes & ~15ll;
  for (int wt = vb; wt < p.n_tiles; wt += vstride) {
    const int rows = tile_rows(p, wt);
    for (int j = 0; j < n_sub; ++j) {
      const int row0 = tile_row0(p, wt, j);
      for (int c = 0; c < p.n_chunks; ++c) {
        if (rp.issued >= g.nstages) {
          int w = 1;
          if (lane == 0) {
            w = mbar_wait_bounded(&g.empty[rp.s], rp.ph ^ 1u, p.err, kDevErrEmptyTimeout,
                                  limit_scale) ? 1 : 0;
            if (!w) *g.abort_flag = 1;
          }
          w = __shfl_sync(0xffffffffu, w, 0);
          if (!w || *g.abort_flag) return false;
        }
        const int kb0 = c * p.kc;
        const int kcount = min(p.kc, p.nb - kb0);
        const long long chunk = (long long)kcount * BB;
        uint8_t* stage = g.ring + (size_t)rp.s * g.stage_bytes;
        long long a0 = 0, a1 = 0;
        uint32_t tx = 0;
        if (lane < rows) {
          const long long start = (long long)(row0 + lane) * p.row_bytes + (long long)kb0 * BB;
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
        if (lane == 0) mbar_arrive_expect_tx(&g.full[rp.s], tot);
        __syncwarp();
        if (tx > 0) bulk_g2s(stage + lane * p.row_stride, p.w + a0, tx, &g.full[rp.s]);
        ++rp.issued;
        if (++rp.s == g.nstages) {
          rp.s = 0;
          rp.ph ^= 1u;
        }
      }
    }
  }
  return true;
}

// No copy may still be in flight when the CTA exits: the producer waits for the last
// stages it issued (the earlier ones were consumed).
__device__ __forceinline__ void drain_ring(const GroupSmem& g, const RingPos& rp, int lane, int* err) {
  if (lane != 0) return;
  const int first = rp.issued > g.nstages ? rp.issued - g.nstages : 0;
  for (int i = first; i < rp.issued; ++i)
    mbar_wait_bounded(&g.full[i % g.nstages], (uint32_t)(i / g.nstages) & 1u, err,
                      kDevErrDrainTimeout);
}

// Consumer warps of a group: the row tiles of one GEMV from the ring (x digits prepared),
// each tile's warp sums reduced by the last warp to finish it, which stores the rows (y,
// + residual; silu(gate) * up; or the tagged push to every rank).
template <int QT, bool FRAG>
__device__ __forceinline__ void consume_item(const GemvParams& p, const GroupSmem& g, int vb, int vstride, int cw,
                             int lane, float inv_rms, unsigned tag, bool feed, RingPos& rp) {
  constexpr int BB = KQ<QT>::kBlockBytes;
  const Lane L = make_lane(lane, QT == RRR_Q4_K);
  const int n_sub = p.out_mode ? 2 : 1;
  const float* xsum32 = g.xsum + p.K / 16;
  // Byte offset mod 16 of a chunk start inside its 16-byte granule (only Q6_K rows and
  // chunks can start unaligned); 32-bit arithmetic on the residues.
  const int rb16 = (int)(p.row_bytes & 15), cb16 = (p.kc * BB) & 15;
  for (int wt = vb; wt < p.n_tiles; wt += vstride) {
    const int rows = tile_rows(p, wt);
    for (int j = 0; j < n_sub; ++j, ++rp.ts) {
      const int row0 = tile_row0(p, wt, j);
      float acc0 = 0.f, acc1 = 0.f;
      for (int c = 0; c < p.n_chunks; ++c) {
        const int cs = rp.s;
        const uint32_t cph = rp.ph;
        if (++rp.s == g.nstages) {
          rp.s = 0;
          rp.ph ^= 1u;
        }
        bool have = (*g.abort_flag == 0);
        if (have) {
          have = mbar_wait_bounded(&g.full[cs], cph, p.err, kDevErrFullTimeout);
          if (!have) *g.abort_flag = 1;
        }
        if (!have) continue;
        const int kb0 = c * p.kc;
        const int items = min(p.kc, p.nb - kb0);
        const uint8_t* stage = g.ring + cs * g.stage_bytes;
        int off0 = 0, off1 = 0;
        if (QT == RRR_Q6_K) {
          off0 = ((row0 + L.g) * rb16 + c * cb16) & 15;
          off1 = ((row0 + L.g + 8) * rb16 + c * cb16) & 15;
        }
        const uint8_t* r0 = stage + L.g * p.row_stride + off0;
        const uint8_t* r1 = stage + (L.g + 8) * p.row_stride + off1;
        // Whole blocks are the work items; the warp that starts the list rotates from
        // stage to stage so leftover blocks (12 per stage for K = 3072) spread over warps.
        const int w0 = (cw + rp.ss * items) % kNW;
        ++rp.ss;
        for (int bi = w0; bi < items; bi += kNW) {
          const uint8_t* q0 = r0 + bi * BB;
          const uint8_t* q1 = r1 + bi * BB;
          if constexpr (QT == RRR_Q6_K) {
            const bool al = __all_sync(0xffffffffu, (((uintptr_t)q0 | (uintptr_t)q1) & 3) == 0);
            const bool m2 = __all_sync(0xffffffffu, ((uintptr_t)q0 & 3) == 2 && ((uintptr_t)q1 & 3) == 2);
            if (al)
              block_q6<0>(q0, q1, kb0 + bi, g.dig, p.dig_stride, g.xscale, g.xsum, L, acc0, acc1);
            else if (m2)
              block_q6<2>(q0, q1, kb0 + bi, g.dig, p.dig_stride, g.xscale, g.xsum, L, acc0, acc1);
            else
              block_q6<1>(q0, q1, kb0 + bi, g.dig, p.dig_stride, g.xscale, g.xsum, L, acc0, acc1);
          } else {
            block_q45<QT, FRAG>(q0, q1, kb0 + bi, g.dig, p.dig_stride, g.xscale, xsum32, L, acc0, acc1);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&g.empty[cs]);
      }
      // Row sums of this warp (over the 4 lanes of a row), parked in slot ts % kSlots; the
      // last warp to finish the tile (shared counter) adds the warps' sums in warp order
      // and stores the rows: no CTA-wide barrier, warps run ahead into the next tile.
      acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
      acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
      acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
      acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
      const int slot = rp.ts % kSlots;
      float* rb = g.red + slot * kNW * kTileRows;
      if (L.tig == 0) {
        rb[cw * kTileRows + L.g] = acc0;
        rb[cw * kTileRows + L.g + 8] = acc1;
      }
      __syncwarp();
      int last = 0;
      if (lane == 0) {
        __threadfence_block();
        last = atomicAdd(&g.cnt[slot], 1) == kNW - 1;
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last) {
        __threadfence_block();
        if (lane < rows && *g.abort_flag == 0) {
          float v = 0.f;
#pragma unroll
          for (int w = 0; w < kNW; ++w) v += rb[w * kTileRows + lane];
          v *= inv_rms;
          if (p.out_mode == 0) {
            const int row = row0 + lane;
            if (p.residual) v = p.residual[row] + v;
            if (!p.push[0]) {
              p.y[row] = v;
            } else if (feed) {
              const unsigned long long wv = ((unsigned long long)tag << 32) | __float_as_uint(v);
#pragma unroll
              for (int r = 0; r < kMaxTpRanks; ++r)
                if (r < p.G) st_relaxed_sys_u64(p.push[r] + row, wv);
            }
          } else if (j == 0) {
            g.gate[slot * kTileRows + lane] = v;
          } else {
            // gate of this work tile was finalised (by some warp) before every warp
            // arrived here
            const float gv = g.gate[((rp.ts - 1) % kSlots) * kTileRows + lane];
            const float sg = __fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv)));
            p.y[wt * kTileRows + lane] = __fmul_rn(sg, v);
          }
        }
        __syncwarp();
        if (lane == 0) g.cnt[slot] = 0;
      }
    }
  }
}

// Consumers: the GEMV input of one GEMV (digits, scales, sums; the ranks' rows summed under
// GemvFuse), then the row scale of its RMSNorm. All consumer warps of the CTA take part.
template <bool FRAG>
__device__ __forceinline__ float prepare_item(const GemvParams& p, const GroupSmem& g, int warp,
                                              int lane, unsigned tag) {
  bool xok = true;
  prepare_x<FRAG>(p, g.dig, g.xscale, g.xsum, g.misc, warp, lane, tag, xok);
  named_barrier(1, kGroups * kNW * 32);
  return row_scale(p, g.misc);
}

// ---------------------------------------------------------------- the kernel
template <int QT, bool FRAG>
__global__ void __launch_bounds__(kThreads, kMinCtas) gemv_kq_kernel(const GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // warps [0, kGroups*kNW): consumers of group warp / kNW; then one producer per group
  const bool producer = warp >= kGroups * kNW;
  const int grp = producer ? warp - kGroups * kNW : warp / kNW;
  const GroupSmem g = group_smem(smem, p, grp);
  // this group's tiles: vb, vb + vstride, ...: group 0 of every CTA first, so that with
  // fewer tiles than groups every SM still gets work
  const int vb = grp * gridDim.x + blockIdx.x, vstride = gridDim.x * kGroups;

  unsigned long long* const tr = p.trace ? p.trace + 8 * (size_t)blockIdx.x : nullptr;
  if (tr && threadIdx.x == 0) tr[0] = globaltimer_ns();
  if (threadIdx.x == 0) init_cta_smem(smem, p);
  __syncthreads();
  pdl_launch_dependents();

  RingPos rp;
  if (producer) {
    // First the GEMV input (and gamma) into L2, ahead of this CTA's weight stream: the
    // consumers read it after the preceding grid has finished, by which time the weight
    // copies of every CTA fill the memory queues.
    if (lane == 0) {
      const uint32_t xb = p.mode == kXBf16 ? (uint32_t)p.K * 2
                          : p.mode == RRR_X_SILU_GATE ? (uint32_t)p.K * 8
                          : p.mode == RRR_X_GQA_V ? (uint32_t)(p.n_kv * p.hd) * 4 : (uint32_t)p.K * 4;
      const void* xs = p.mode == kXBf16 ? (const void*)p.xb
                       : p.mode == RRR_X_GQA_V ? (const void*)(p.x + (p.n_q + p.n_kv) * p.hd)
                       : (const void*)p.x;
      if (!p.sum_in)  // (the ranks' rows arrive while this kernel waits for them)
        for (uint32_t o = 0; o < xb; o += 16384) bulk_prefetch_l2((const char*)xs + o, min(16384u, xb - o));
      if (p.mode == RRR_X_RMSNORM)
        for (uint32_t o = 0; o < (uint32_t)p.K * 4; o += 16384)
          bulk_prefetch_l2((const char*)p.gamma + o, min(16384u, (uint32_t)p.K * 4 - o));
    }
    // (consumers that wait for the ranks' rows first get twice the limit, so that a
    // missing rank is reported as such)
    if (tr && grp == 0 && lane == 0) tr[1] = globaltimer_ns();
    produce_item<QT>(p, g, vb, vstride, lane, rp, p.sum_in ? 2u : 1u);
    if (tr && grp == 0 && lane == 0) tr[5] = globaltimer_ns();
    drain_ring(g, rp, lane, p.err);
    return;
  }

  // An input that no overlapping kernel writes (x_early) is prepared while the preceding
  // grid drains; otherwise after the grid dependency wait. One copy of the preparation code
  // either way: only the wait moves.
  if (!p.x_early) {
    pdl_wait();
    if (tr && threadIdx.x == 0) tr[2] = globaltimer_ns();
  }
  // fused exchange (never x_early): this step's epoch
  const unsigned tag = p.G ? *p.epoch + 1u : 0u;
  const float inv_rms = prepare_item<FRAG>(p, g, warp, lane, tag);
  if (tr && threadIdx.x == 0) tr[3] = globaltimer_ns();
  if (p.x_early) {
    pdl_wait();
    if (tr && threadIdx.x == 0) tr[2] = globaltimer_ns();
  }
  // whether this rank still feeds its peers (no error recorded by an earlier kernel, e.g. a
  // wait that ran out)
  const bool feed = p.push[0] && *reinterpret_cast<volatile int*>(p.err) == 0;
  consume_item<QT, FRAG>(p, g, vb, vstride, warp % kNW, lane, inv_rms, tag, feed, rp);
  if (tr) {
    named_barrier(1, kGroups * kNW * 32);
    if (threadIdx.x == 0) {
      tr[4] = globaltimer_ns();
      tr[6] = ((unsigned long long)QT << 56) | ((unsigned long long)p.K << 28) | (unsigned long long)p.N;
      tr[7] = p.trace_tag | blockIdx.x;
    }
  }
}

// Shared-memory layout of one launch. FRAG: the x digits are stored as ready-made per-lane
// B fragments (8 bytes per element; Q4_K / Q5_K) instead of three compact digit rows.
template <int QT>
int plan_layout(GemvParams& p, bool frag) {
  constexpr int BB = KQ<QT>::kBlockBytes;
  const int chunk = p.kc * BB;
  const bool aligned16 = (p.row_bytes % 16 == 0) && (chunk % 16 == 0);
  // Stage row stride: room for the chunk plus the 16-byte rounding of unaligned chunk
  // starts, padded so that rows fall in distinct shared-memory banks (the Q4_K/Q5_K
  // 8-byte reads of 4 rows, the Q6_K 4-byte reads of 8 rows).
  const int need = chunk + (aligned16 ? 0 : 30);
  const int target = (QT == RRR_Q6_K) ? 16 : 96;
  int rs = (need / 128) * 128 + target;
  if (rs < need) rs += 128;
  p.row_stride = rs;
  p.stage_bytes = kTileRows * p.row_stride;
  p.dig_stride = p.K + 96;
  const int dig_bytes = frag ? p.K * 8 : 4 * p.dig_stride;
  int fixed = kGroups * 2 * kMaxStages * 8 + dig_bytes + 16;
  fixed += p.nb * 4 + 16 + (p.K / 16) * 4 + (p.K / 32) * 4;  // xscale, xsum16, xsum32
  fixed += kGroups * kSlots * kNW * kTileRows * 4;            // red
  fixed += kGroups * kSlots * kTileRows * 4 + 16 + kGroups * kNW * 4 + kGroups * kSlots * 4 + 64;
  p.nstages = std::max(2, std::min(kMaxStages, (kSmemBudget - fixed) / (kGroups * p.stage_bytes)));
  int off = kGroups * p.nstages * p.stage_bytes;
  p.off_bars = off;          off += kGroups * 2 * p.nstages * 8;
  off = (off + 15) & ~15;
  p.off_dig = off;           off += dig_bytes;
  off = (off + 15) & ~15;
  p.off_xscale = off;        off += p.nb * 4;
  off = (off + 15) & ~15;
  p.off_xsum = off;          off += (p.K / 16) * 4 + (p.K / 32) * 4;  // xsum16, xsum32
  p.off_red = off;           off += kGroups * kSlots * kNW * kTileRows * 4;
  p.off_gate = off;          off += kGroups * kSlots * kTileRows * 4;
  p.off_misc = off;          off += 16 + kGroups * kNW * 4 + kGroups * kSlots * 4;
  return (off + 127) & ~127;
}

struct OccEntry {
  const void* fn;
  int dev, smem, per_sm;
};

template <int QT, bool FRAG>
cudaError_t launch_k(const LaunchEnv& env, const GemvParams& p, int smem) {
  auto kern = gemv_kq_kernel<QT, FRAG>;
  // Kernel attribute and occupancy per (kernel, device, shared-memory size), computed once:
  // the launch path stays a single cudaLaunchKernelEx.
  static thread_local OccEntry cache[32];
  static thread_local int n_cache = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  int per_sm = 0;
  for (int i = 0; i < n_cache; ++i)
    if (cache[i].fn == (const void*)kern && cache[i].dev == dev && cache[i].smem == smem)
      per_sm = cache[i].per_sm;
  if (per_sm == 0) {
    // the attribute is per kernel: set it to the device maximum so that every layout of
    // this kernel (different K) can launch
    int optin = 0;
    cudaError_t e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    if (smem > optin) return cudaErrorInvalidConfiguration;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    if (n_cache < 32) cache[n_cache++] = OccEntry{(const void*)kern, dev, smem, per_sm};
  }
  // kMinCtas CTAs per SM (two producers and 16 consumer warps per SM); each CTA runs
  // kGroups producer/consumer groups, so it needs at least kGroups tiles to be busy
  const int grid = std::max(1, std::min(p.n_tiles, std::min(per_sm, kMinCtas) * env.sm_count));
  GemvParams q = p;
  if (env.trace && grid <= env.trace_cap) {
    if (*env.trace_next + grid > env.trace_cap) *env.trace_next = 0;
    q.trace = env.trace + 8 * (size_t)*env.trace_next;
    q.trace_tag = (unsigned long long)(*env.trace_seq)++ << 16;
    *env.trace_next += grid;
  }
  return rrr_launch_pdl(kern, dim3(grid), dim3(kThreads), smem, env.stream, env.pdl, q);
}

template <int QT>
cudaError_t launch_t(const LaunchEnv& env, GemvParams& p) {
  const int kc_max = (QT == RRR_Q6_K) ? 8 : 12;
  const int n_ch = (p.nb + kc_max - 1) / kc_max;
  p.kc = (p.nb + n_ch - 1) / n_ch;
  p.n_chunks = (p.nb + p.kc - 1) / p.kc;
  p.half_rows = p.out_mode ? p.N / 2 : 0;
  const int lim = p.out_mode ? p.half_rows : p.N;
  p.n_tiles = (lim + kTileRows - 1) / kTileRows;
  if constexpr (QT != RRR_Q6_K) {
    // fragment layout when three stages still fit beside it
    GemvParams q = p;
    const int smem = plan_layout<QT>(q, true);
    if (q.nstages >= 3 || (QT == RRR_Q5_K && q.nstages >= 2 && p.K <= 4096)) {
      p = q;
      return launch_k<QT, true>(env, p, smem);
    }
  }
  const int smem = plan_layout<QT>(p, false);
  return launch_k<QT, false>(env, p, smem);
}

cudaError_t launch_any(const LaunchEnv& env, int qtype, GemvParams& p) {
  p.nb = p.K / 256;
  p.row_bytes = (long long)p.nb * kq_block_bytes(qtype);
  p.total_bytes = p.row_bytes * p.N;
  p.err = env.d_err;
  switch (qtype) {
    case RRR_Q4_K: return launch_t<RRR_Q4_K>(env, p);
    case RRR_Q5_K: return launch_t<RRR_Q5_K>(env, p);
    case RRR_Q6_K: return launch_t<RRR_Q6_K>(env, p);
    default: return cudaErrorInvalidValue;
  }
}

// ---------------------------------------------------------------- launch parameters (host)
// The kernel parameters of one GEMV from its description (shapes and layout follow).
void fill_params(GemvParams& p, const GemvDesc& d) {
  p.w = static_cast<const uint8_t*>(d.w);
  p.x = d.x;
  p.y = d.y;
  p.residual = d.swiglu ? nullptr : d.residual;
  p.out_mode = d.swiglu ? 1 : 0;
  p.mode = d.pro.mode;
  p.gamma = d.pro.gamma;
  p.eps = d.pro.eps;
  p.n_q = d.pro.n_q_heads;
  p.n_kv = d.pro.n_kv_heads;
  p.hd = d.pro.head_dim;
  p.k_off = d.pro.mode == RRR_X_GQA_V ? d.pro.k_offset : 0;
  p.K = d.K;
  p.N = d.swiglu ? 2 * d.N : d.N;
  // (the ranks' rows of a fused exchange arrive during the grid, never early)
  p.x_early = d.x_early && d.fuse.G < 1 ? 1 : 0;
  if (d.fuse.G >= 1) {
    p.sum_in = d.fuse.sum_in;
    p.h_out = d.fuse.h_out;
    for (int r = 0; r < kMaxTpRanks; ++r) p.push[r] = r < d.fuse.G ? d.fuse.push[r] : nullptr;
    p.G = d.fuse.G;
    p.epoch = d.fuse.epoch;
  }
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
                           const rrr_gemv_prologue* pro, const GemvFuse* fuse, bool x_early) {
  GemvDesc d;
  d.qtype = qtype;
  d.w = w;
  d.x = x;
  d.y = y;
  d.K = K;
  d.N = N;
  d.residual = residual;
  if (pro) d.pro = *pro;
  if (fuse) d.fuse = *fuse;
  d.x_early = x_early;
  GemvParams p = {};
  fill_params(p, d);
  return launch_any(env, qtype, p);
}

cudaError_t launch_gemv_kq_swiglu(const LaunchEnv& env, int qtype, const void* w,
                                  const float* x, float* y, int K, int F,
                                  const rrr_gemv_prologue* pro, const GemvFuse* fuse) {
  GemvDesc d;
  d.qtype = qtype;
  d.w = w;
  d.x = x;
  d.y = y;
  d.K = K;
  d.N = F;
  d.swiglu = true;
  if (pro) d.pro = *pro;
  if (fuse) d.fuse = *fuse;
  GemvParams p = {};
  fill_params(p, d);
  return launch_any(env, qtype, p);
}

cudaError_t launch_gemv_kq_bf16(const LaunchEnv& env, int qtype, const void* w,
                                const uint16_t* x, float* y, int K, int N,
                                const float* residual) {
  GemvParams p = {};
  p.w = static_cast<const uint8_t*>(w);
  p.xb = x;
  p.y = y;
  p.residual = residual;
  p.mode = kXBf16;
  p.K = K;
  p.N = N;
  return launch_any(env, qtype, p);
}

cudaError_t launch_mma_selftest(const LaunchEnv& env, int* d_ok) {
  mma_selftest_kernel<<<1, 32, 0, env.stream>>>(d_ok);
  return cudaGetLastError();
}

}  // namespace rrr
