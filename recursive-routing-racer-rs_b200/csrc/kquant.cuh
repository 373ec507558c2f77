// kquant.cuh — GGUF K-quant super-block formats (Q4_K 144 B, Q5_K 176 B, Q6_K 210 B per
// 256 weights) and their bit-exact element dequantisation, as the reference defines them
// in src/model/phi4.rs:444-542 (dequant_q6_k / dequant_q4_k / dequant_q5_k).
#pragma once
#include <stdint.h>

#include "rrr_common.cuh"

namespace rrr {

template <int QT> struct KQ;
template <> struct KQ<RRR_Q4_K> { static constexpr int kBlockBytes = 144; };
template <> struct KQ<RRR_Q5_K> { static constexpr int kBlockBytes = 176; };
template <> struct KQ<RRR_Q6_K> { static constexpr int kBlockBytes = 210; };

__host__ __device__ inline int kq_block_bytes(int qtype) {
  return qtype == RRR_Q4_K ? 144 : qtype == RRR_Q5_K ? 176 : qtype == RRR_Q6_K ? 210 : 0;
}

// The 6-bit scale / min pair of sub-block `sub` (0..7) from the 12 packed bytes of a
// Q4_K / Q5_K block (phi4.rs:492-498, 522-528).
__device__ __forceinline__ void kq_scale_min(const uint8_t* sc, int sub, uint32_t& sv,
                                             uint32_t& mv) {
  if (sub < 4) {
    sv = sc[sub] & 0x3Fu;
    mv = sc[sub + 4] & 0x3Fu;
  } else {
    const int i = sub - 4;
    sv = (sc[8 + i] & 0x0Fu) | ((uint32_t)(sc[i] >> 6) << 4);
    mv = (uint32_t)(sc[8 + i] >> 4) | ((uint32_t)(sc[4 + i] >> 6) << 4);
  }
}

__device__ __forceinline__ uint32_t rd16(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8);
}

// Element e (0..255) of one block, with the reference's exact operation order and no
// FMA contraction (__fmul_rn / __fsub_rn are never fused).
template <int QT>
__device__ __forceinline__ float kq_dequant_elem(const uint8_t* b, int e);

// Q4_K: out = q * (d*sv) - (dmin*mv); element sub*32+j takes nibble (sub&1) of
// qs[(sub/2)*32+j] (phi4.rs:481-510).
template <>
__device__ __forceinline__ float kq_dequant_elem<RRR_Q4_K>(const uint8_t* b, int e) {
  const float d = f16_bits_to_f32(rd16(b)), dmin = f16_bits_to_f32(rd16(b + 2));
  const int sub = e >> 5, j = e & 31;
  uint32_t sv, mv;
  kq_scale_min(b + 4, sub, sv, mv);
  const float s = __fmul_rn(d, (float)sv), m = __fmul_rn(dmin, (float)mv);
  const uint8_t qb = b[16 + (sub >> 1) * 32 + j];
  const uint32_t qi = (sub & 1) ? (qb >> 4) : (qb & 0xFu);
  return __fsub_rn(__fmul_rn((float)qi, s), m);
}

// Q5_K: 5-bit q = nibble | ((qh[j] >> sub) & 1) << 4 (phi4.rs:512-542).
template <>
__device__ __forceinline__ float kq_dequant_elem<RRR_Q5_K>(const uint8_t* b, int e) {
  const float d = f16_bits_to_f32(rd16(b)), dmin = f16_bits_to_f32(rd16(b + 2));
  const int sub = e >> 5, j = e & 31;
  uint32_t sv, mv;
  kq_scale_min(b + 4, sub, sv, mv);
  const float s = __fmul_rn(d, (float)sv), m = __fmul_rn(dmin, (float)mv);
  const uint8_t qb = b[48 + (sub >> 1) * 32 + j];
  const uint32_t lo = (sub & 1) ? (qb >> 4) : (qb & 0xFu);
  const uint32_t qi = lo | (((uint32_t)(b[16 + j] >> sub) & 1u) << 4);
  return __fsub_rn(__fmul_rn((float)qi, s), m);
}

// Q6_K: element g*128 + 32k + l; q = (ql nibble | qh 2 bits << 4) - 32 with ql byte
// g*64 + 32(k&1) + l (nibble k>>1) and qh byte g*32 + l (bits 2k); scale index e/16
// (= g*8 + l/16 + 2k, phi4.rs:463); out = (d * scale) * q (phi4.rs:444-479).
template <>
__device__ __forceinline__ float kq_dequant_elem<RRR_Q6_K>(const uint8_t* b, int e) {
  const float d = f16_bits_to_f32(rd16(b + 208));
  const int g = e >> 7, k = (e >> 5) & 3, l = e & 31;
  const uint8_t qlb = b[g * 64 + 32 * (k & 1) + l];
  const uint32_t lo = (k >> 1) ? (qlb >> 4) : (qlb & 0xFu);
  const uint32_t hi = (b[128 + g * 32 + l] >> (2 * k)) & 3u;
  const int q = (int)(lo | (hi << 4)) - 32;
  const int8_t sc = (int8_t)b[192 + (e >> 4)];
  return __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
}

}  // namespace rrr
