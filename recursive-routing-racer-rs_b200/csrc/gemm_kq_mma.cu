// gemm_kq_mma.cu — kernel (2), small batches: Y[M,N] = X[M,K] · W[N,K]^T for 16 <= M <= 64
// tokens, W raw GGUF Q4_K / Q5_K / Q6_K super-blocks, X bf16, Y f32, on the register-level
// tensor-core path (mma.sync.m16n8k16, bf16 x bf16 -> f32). Same call sites as
// gemm_kq_tc.cu (the `matmul_gpuq{4,5,6}_batch` dispatches of the batched prefill,
// src/model/phi4.rs:1257-1268, 1346-1357, 1380-1391).
//
// Why a second kernel: with M <= 64 tokens the tcgen05 path spends ~100 cycles of its single
// issuing thread per MMA, wait and commit and stays near 33 us for a 28 MB weight matrix,
// while the work is one pass over the weights. Here every warp dequantises and multiplies
// its own rows: the weights go from shared memory straight into A fragments in registers
// (no dequantised tile is stored), all eight warps issue tensor-core instructions, and the
// kernel runs at the weight stream or the mma.sync rate (measured ~550 TFLOP/s bf16 on
// B200), whichever is lower.
//
// One CTA = one tile of up to 256 weight rows x TN tokens (TN = M rounded up to 16; the
// tile height and the K split chosen per shape by choose_tile) over a range of K
// super-blocks (split-K across a thread-block cluster when the tile grid is smaller than
// the GPU):
//   warp 0     producer: per stage of `kbs` super-blocks, one 2-D TMA box of the raw
//              blocks of the tile's rows (16-byte-aligned envelope, zero fill past the row
//              end and past N) and 4*kbs TMA boxes of X (64 k x TN tokens, 128-byte
//              swizzle) into a ring, all on the stage's full barrier;
//   consumers  16 rows each (one m16 tile, TN <= 32) or 32 rows (two m16 tiles sharing
//              each B fragment, TN 48 and 64): per 64-wide K chunk, the lane's A fragments
//              (rows g, g+8; k 2t, 2t+1, 2t+8, 2t+9 of each 16-k step) are built from the
//              raw bytes with the packed exact-offset dequantisation (q*a - b as one
//              f32x2 FMA on 2^23 + 65536 q, one cvt to bf16x2), B fragments come from the
//              swizzled X tile with ldmatrix, and the f32 accumulators stay in registers.
// Epilogue: the accumulators go to a shared-memory tile [token][row] (over the drained
// ring); the CTAs of a cluster sum their partial tiles over distributed shared memory in
// split order (deterministic) and store Y (+ residual) with coalesced 16-byte stores.
// Every mbarrier wait is bounded (about one second) and reports through the context's
// device error flag.
//
// Dequantised weights are rounded once to bf16 (the MMA operand type): results are within
// the tensor-core tolerance (1e-2 relative L2), not bit-exact.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <string.h>

#include "internal.h"
#include "kquant.cuh"
#include "rrr_common.cuh"
#include "tile_common.cuh"

namespace rrr {
namespace {

constexpr int kMaxRows = 256;         // weight rows per tile (at most; chosen per shape)
// MT m16 tiles per consumer warp: 16 / MT consumer warps cover the 256 rows (MT = 1 for
// TN <= 32: twice the warps to hide latency; MT = 2 for larger TN: half the X reads)
template <int MT> constexpr int cwarps() { return 16 / MT; }
template <int MT> constexpr int threads_for() { return (cwarps<MT>() + 1) * 32; }
constexpr int kMaxTn = 64;
constexpr int kMaxSplits = 8;         // portable cluster size
constexpr int kSmemBudget = 232448;   // 227 KB opt-in maximum on sm_100

struct MmaParams {
  float* y;
  const float* residual;  // optional [M, N] f32 added in the epilogue (may equal y)
  int M, N, nb, bb;       // nb super-blocks per row, bb bytes per super-block
  int tn, splits, stages, kbs, pitch;
  uint32_t raw_bytes, stage_bytes;  // raw part of a stage (padded to 1024 bytes), whole stage
  uint32_t wbox_bytes;              // bytes of the weight box (rows x pitch)
  uint32_t off_tab;                 // scale table [kbs][rows][subs + 1] float2
  int cwarps, rows;                 // consumer warps and weight rows of a tile
  int* err;
};

__device__ __forceinline__ uint32_t lds_u16(const uint8_t* p) {
  return *reinterpret_cast<const uint16_t*>(p);
}
// Bytes 2t, 2t+1, 2t+8, 2t+9 of a 16-byte run (2-byte aligned) as one word: the k values
// of the lane's A-fragment registers (k = 2t, 2t+1 | 2t+8, 2t+9) of one 16-k step.
__device__ __forceinline__ uint32_t frag_bytes(const uint8_t* run, int t) {
  return lds_u16(run + 2 * t) | (lds_u16(run + 2 * t + 8) << 16);
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                            uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// ---- A fragments of one row for one 64-wide K chunk: out[ks][0] = k 2t, 2t+1 and
// out[ks][1] = k 2t+8, 2t+9 of 16-k step ks (bf16x2 words).
template <int QT> struct MmaDq;

// Q4_K: chunk c = qs group c (bytes 16 + 32c ..): low nibbles = sub-block 2c (steps 0, 1:
// bytes 0-15, 16-31), high nibbles = sub-block 2c+1 (steps 2, 3); value q*(d*sc) - dmin*m
// (phi4.rs:481-510).
template <> struct MmaDq<RRR_Q4_K> {
  static constexpr int kSubs = 8;
  struct Row {};
  static __device__ __forceinline__ Row row(const uint8_t*, int) { return Row{}; }
  // (a / 65536, -(128 a + b)) of every sub-block: a = d*sc, b = dmin*m (phi4.rs:492-498)
  static __device__ __forceinline__ void table_row(const uint8_t* blk, float2* tab) {
    const uint4 hd = *reinterpret_cast<const uint4*>(blk);
    const float d = f16_bits_to_f32(hd.x & 0xFFFFu), dmin = f16_bits_to_f32(hd.x >> 16);
#pragma unroll
    for (int sb = 0; sb < 8; ++sb) {
      float sv, mv;
      scale_min_w(hd.y, hd.z, hd.w, sb, sv, mv);
      const RunScale r = run_scale(d * sv, dmin * mv);
      tab[sb] = make_float2(r.a.x, r.c.x);
    }
  }
  static __device__ __forceinline__ void chunk(const uint8_t* blk, const Row&, const float2* tab,
                                               int c, int t, uint32_t (&out)[4][2]) {
    const uint8_t* run = blk + 16 + 32 * c;
    const uint32_t v01 = frag_bytes(run, t), v23 = frag_bytes(run + 16, t);
    const float2 t0 = tab[2 * c], t1 = tab[2 * c + 1];
    const RunScale s0{make_float2(t0.x, t0.x), make_float2(t0.y, t0.y)};
    const RunScale s1{make_float2(t1.x, t1.x), make_float2(t1.y, t1.y)};
    emit4(v01 & 0x0F0F0F0Fu, s0, out[0]);
    emit4(v23 & 0x0F0F0F0Fu, s0, out[1]);
    emit4((v01 >> 4) & 0x0F0F0F0Fu, s1, out[2]);
    emit4((v23 >> 4) & 0x0F0F0F0Fu, s1, out[3]);
  }
};

// Q5_K: as Q4_K with qs at byte 48 and the fifth bit, bit s of qh[l] for sub-block s
// (qh at byte 16, the same byte positions as the element's qs byte) (phi4.rs:512-542).
template <> struct MmaDq<RRR_Q5_K> {
  static constexpr int kSubs = 8;
  struct Row {
    uint32_t h01, h23;
  };
  static __device__ __forceinline__ Row row(const uint8_t* blk, int t) {
    return Row{frag_bytes(blk + 16, t), frag_bytes(blk + 32, t)};
  }
  static __device__ __forceinline__ void table_row(const uint8_t* blk, float2* tab) {
    MmaDq<RRR_Q4_K>::table_row(blk, tab);  // same header layout (phi4.rs:522-528)
  }
  static __device__ __forceinline__ uint32_t bit5(uint32_t h, int s) {
    return ((h >> s) & 0x01010101u) << 4;
  }
  static __device__ __forceinline__ void chunk(const uint8_t* blk, const Row& r, const float2* tab,
                                               int c, int t, uint32_t (&out)[4][2]) {
    const uint8_t* run = blk + 48 + 32 * c;
    const uint32_t v01 = frag_bytes(run, t), v23 = frag_bytes(run + 16, t);
    const float2 t0 = tab[2 * c], t1 = tab[2 * c + 1];
    const RunScale s0{make_float2(t0.x, t0.x), make_float2(t0.y, t0.y)};
    const RunScale s1{make_float2(t1.x, t1.x), make_float2(t1.y, t1.y)};
    emit4((v01 & 0x0F0F0F0Fu) | bit5(r.h01, 2 * c), s0, out[0]);
    emit4((v23 & 0x0F0F0F0Fu) | bit5(r.h23, 2 * c), s0, out[1]);
    emit4(((v01 >> 4) & 0x0F0F0F0Fu) | bit5(r.h01, 2 * c + 1), s1, out[2]);
    emit4(((v23 >> 4) & 0x0F0F0F0Fu) | bit5(r.h23, 2 * c + 1), s1, out[3]);
  }
};

// Q6_K: chunk c is quarter pair kq = 2(c&1), 2(c&1)+1 of half g = c/2; 16-k step (kq, h)
// holds elements g*128 + 32kq + 16h + (0..15): nibble kq/2 of ql[64g + 32(kq&1) + 16h + l],
// bits 2kq of qh[32g + 16h + l], one scale (index e/16 = 8g + 2kq + h); value
// (d*scale) * (q - 32) (phi4.rs:444-479). `blk` is 2-byte aligned.
template <> struct MmaDq<RRR_Q6_K> {
  static constexpr int kSubs = 16;
  struct Row {};
  static __device__ __forceinline__ Row row(const uint8_t*, int) { return Row{}; }
  // (a / 65536, -(160 a)) of every 16-value group: a = d * scale, offset -32 a
  static __device__ __forceinline__ void table_row(const uint8_t* blk, float2* tab) {
    const float d = f16_bits_to_f32(lds_u16(blk + 208));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t w = lds_u16(blk + 192 + 2 * i);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float a = d * (float)(int8_t)(h ? (w >> 8) : w);
        const RunScale r = run_scale(a, 32.f * a);
        tab[2 * i + h] = make_float2(r.a.x, r.c.x);
      }
    }
  }
  static __device__ __forceinline__ void chunk(const uint8_t* blk, const Row&, const float2* tab,
                                               int c, int t, uint32_t (&out)[4][2]) {
    const int g = c >> 1;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const int kq = 2 * (c & 1) + (ks >> 1), h = ks & 1;
      const uint32_t v = frag_bytes(blk + 64 * g + 32 * (kq & 1) + 16 * h, t);
      const uint32_t q = frag_bytes(blk + 128 + 32 * g + 16 * h, t);
      const uint32_t val = ((v >> (4 * (kq >> 1))) & 0x0F0F0F0Fu) | (((q >> (2 * kq)) & 0x03030303u) << 4);
      const float2 ts = tab[8 * g + 2 * kq + h];
      emit4(val, RunScale{make_float2(ts.x, ts.x), make_float2(ts.y, ts.y)}, out[ks]);
    }
  }
};

// ---- the kernel ---------------------------------------------------------------------

template <int QT, int TN, int MT>
__global__ void __launch_bounds__(threads_for<MT>(), 1)
    gemm_kq_mma_kernel(const __grid_constant__ CUtensorMap xmap,
                       const __grid_constant__ CUtensorMap wmap, const MmaParams p) {
  constexpr int NF = TN / 8;  // n fragments of 8 tokens
  constexpr int WR = 16 * MT;  // rows per consumer warp
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = smem_dyn + ((1024u - (smem_addr(smem_dyn) & 1023u)) & 1023u);
  constexpr int TS = MmaDq<QT>::kSubs + 1;  // table row stride (float2): conflict-free
  const int S = p.stages;
  float2* tab = reinterpret_cast<float2*>(smem + p.off_tab);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_tab + (size_t)p.kbs * p.rows * TS * 8);
  uint64_t* empty = full + S;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + S);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * p.rows, m0 = blockIdx.y * TN, z = blockIdx.z;
  const int pstride = p.rows + 4;  // floats per token row of the partial tile
  const int kb0 = (int)((long long)z * p.nb / p.splits);
  const int kb1 = (int)((long long)(z + 1) * p.nb / p.splits);
  const int n_blk = kb1 - kb0;
  const int n_st = (n_blk + p.kbs - 1) / p.kbs;
  const uint32_t xbox = (uint32_t)TN * 128u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], p.cwarps);
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  // Programmatic dependent launch: the next grid may be scheduled now; every global
  // access of this one (X, weights, Y, residual) comes after the previous grid's results
  // are visible.
  pdl_launch_dependents();
  pdl_wait();

  if (warp == 0) {
    // ---------------- producer
    int issued = 0;
    for (int st = 0; st < n_st; ++st) {
      if (warp_aborted(abort_flag)) break;
      const int s = st % S;
      if (st >= S && !warp_wait(&empty[s], ((st / S) - 1) & 1, p.err)) {
        *abort_flag = 1;
        break;
      }
      const int kb = kb0 + st * p.kbs;
      const int nk = min(p.kbs, kb1 - kb);
      if (lane == 0) {
        uint8_t* dst = smem + (size_t)s * p.stage_bytes;
        mbar_arrive_expect_tx(&full[s], p.wbox_bytes + (uint32_t)(4 * nk) * xbox);
        tma_load_2d(dst, &wmap, (int)(((long long)kb * p.bb & ~15ll) >> 3), n0, &full[s]);
        for (int i = 0; i < 4 * nk; ++i)
          tma_load_2d(dst + p.raw_bytes + (uint32_t)i * xbox, &xmap, kb * 256 + 64 * i, m0, &full[s]);
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
    // ---------------- consumers: warp cw owns rows 32cw .. 32cw+31
    const int cw = warp - 1;
    const int g = lane >> 2, t = lane & 3;
    float acc[MT][NF][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nf = 0; nf < NF; ++nf)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[mt][nf][i] = 0.f;
    // ldmatrix row of this lane: matrix mi = lane/8 (token half mi>>1, k chunk mi&1)
    const int lm_tok = 8 * ((lane >> 3) >> 1) + (lane & 7);
    const int lm_chk = (lane >> 3) & 1;

    // this warp's scale table: its WR rows x the stage's blocks (lane l computes row l)
    float2* wtab = tab + cw * (p.kbs * WR * TS);
    for (int st = 0; st < n_st; ++st) {
      if (warp_aborted(abort_flag)) break;
      const int s = st % S;
      if (!warp_wait(&full[s], (uint32_t)(st / S) & 1u, p.err)) {
        *abort_flag = 1;
        break;
      }
      const uint8_t* raw = smem + (size_t)s * p.stage_bytes;
      const uint32_t xs = smem_addr(raw + p.raw_bytes);
      const int kb = kb0 + st * p.kbs;
      const int nk = min(p.kbs, kb1 - kb);
      const int env = (int)(((long long)kb * p.bb) & 15);
      if (lane < WR)
        for (int kk = 0; kk < nk; ++kk)
          MmaDq<QT>::table_row(raw + (WR * cw + lane) * p.pitch + env + kk * p.bb,
                               wtab + (kk * WR + lane) * TS);
      __syncwarp();
      for (int kk = 0; kk < nk; ++kk) {
        const uint8_t* b[MT][2];
        const float2* tr[MT][2];
        typename MmaDq<QT>::Row rr[MT][2];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int rl = 16 * mt + 8 * h + g;
            b[mt][h] = raw + (WR * cw + rl) * p.pitch + env + kk * p.bb;
            tr[mt][h] = wtab + (kk * WR + rl) * TS;
            rr[mt][h] = MmaDq<QT>::row(b[mt][h], t);
          }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t a[MT][4][4];
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            uint32_t lo[4][2], hi[4][2];
            MmaDq<QT>::chunk(b[mt][0], rr[mt][0], tr[mt][0], c, t, lo);
            MmaDq<QT>::chunk(b[mt][1], rr[mt][1], tr[mt][1], c, t, hi);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              a[mt][ks][0] = lo[ks][0];
              a[mt][ks][1] = hi[ks][0];
              a[mt][ks][2] = lo[ks][1];
              a[mt][ks][3] = hi[ks][1];
            }
          }
          // X box of this chunk: 64 k x TN tokens, 128-byte swizzle
          const uint32_t box = xs + (uint32_t)(4 * kk + c) * xbox;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
            for (int np = 0; np < NF / 2; ++np) {
              uint32_t b0, b1, b2, b3;
              ldmatrix_x4(box + sw128_off(16 * np + lm_tok, 2 * ks + lm_chk), b0, b1, b2, b3);
#pragma unroll
              for (int mt = 0; mt < MT; ++mt) {
                mma_bf16(acc[mt][2 * np], a[mt][ks], b0, b1);
                mma_bf16(acc[mt][2 * np + 1], a[mt][ks], b2, b3);
              }
            }
          }
        }
      }
      __syncwarp();  // the warp's table rows are rewritten next stage
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    // all stages consumed by every consumer before the ring is reused for the partial tile
    named_barrier(1, p.cwarps * 32);
    float* part = reinterpret_cast<float*>(smem);  // [TN][pstride]
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nf = 0; nf < NF; ++nf)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = WR * cw + 16 * mt + g + 8 * (i >> 1);
          const int tok = 8 * nf + 2 * t + (i & 1);
          part[tok * pstride + row] = acc[mt][nf][i];
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

// Stage layout: raw [rows][pitch] (box of kbs super-blocks + envelope, pitch an odd
// number of 16-byte units) padded to 1024 bytes, then X [4*kbs][TN][128 B] (128-byte
// swizzle, whose pattern is anchored at 1024-byte boundaries).
int raw_part_bytes(int qtype, int kbs, int rows) {
  return (rows * raw_slot_bytes(qtype, kbs) + 1023) & ~1023;
}
int stage_bytes_for(int qtype, int kbs, int tn, int rows) {
  return raw_part_bytes(qtype, kbs, rows) + 4 * kbs * tn * 128;
}
// Scale table: (a / 65536, c) per row and scale group of the stage's super-blocks.
int table_bytes_for(int qtype, int kbs, int rows) {
  return kbs * rows * ((qtype == RRR_Q6_K ? 16 : 8) + 1) * 8;
}

// Ring of one tile shape: super-blocks per stage, stages and shared memory (stages 0: the
// shape does not fit).
struct Ring {
  int kbs, stages, smem;
};
Ring ring_for(int qtype, int tn, int rows) {
  const int fixed = 1024 + 256;
  for (int kbs = 2; kbs >= 1; --kbs) {
    const int sb = stage_bytes_for(qtype, kbs, tn, rows);
    const int tb = table_bytes_for(qtype, kbs, rows);
    int st = (kSmemBudget - fixed - tb) / sb;
    if (st > 4) st = 4;
    if (st >= 3 || (kbs == 1 && st >= 2)) {
      // the partial tile [TN][rows + 4] f32 reuses the ring
      if (tn * (rows + 4) * 4 > st * sb) return Ring{0, 0, 0};
      return Ring{kbs, st, fixed + tb + st * sb};
    }
  }
  return Ring{0, 0, 0};
}

template <int QT, int TN, int MT>
cudaError_t launch_t(const LaunchEnv& env, const MmaPlan& pl, const void* w, const uint16_t* x,
                     float* y, int M, int K, int N, const float* residual) {
  constexpr int WR = 16 * MT;
  const int nb = K / 256;
  auto kern = gemm_kq_mma_kernel<QT, TN, MT>;
  // Tile height (WR rows per consumer warp) and K splits (choose_tile), chosen once per
  // (device, shape).
  struct Choice {
    int dev, N, nb, cw, s;
    Ring ring;
  };
  static thread_local Choice chosen[16];
  static thread_local int n_chosen = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  int best_cw = 0, best_s = 1;
  Ring best_ring{0, 0, 0};
  for (int i = 0; i < n_chosen; ++i)
    if (chosen[i].dev == dev && chosen[i].N == N && chosen[i].nb == nb) {
      best_cw = chosen[i].cw;
      best_s = chosen[i].s;
      best_ring = chosen[i].ring;
    }
  cudaLaunchConfig_t cfg = {};
  cfg.stream = env.stream;
  if (best_cw == 0) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget);
    if (e != cudaSuccess) return e;
    TileCand cand[kMaxRows / 16];
    Ring rings[kMaxRows / 16];
    int cws[kMaxRows / 16], nc = 0;
    for (int cw = cwarps<MT>(); cw >= 2; --cw) {
      const Ring rg = ring_for(QT, TN, cw * WR);
      if (rg.stages == 0) continue;
      cand[nc] = TileCand{cw * WR, (cw + 1) * 32, rg.smem};
      rings[nc] = rg;
      cws[nc++] = cw;
    }
    int s = 1;
    const int i = choose_tile((const void*)kern, env.stream, cand, nc, N, pl.m_tiles, nb,
                              std::min(kMaxSplits, std::max(1, nb / 2)), env.sm_count, &s);
    if (i < 0) return cudaErrorInvalidConfiguration;
    best_cw = cws[i];
    best_s = s;
    best_ring = rings[i];
    const Choice c{dev, N, nb, best_cw, best_s, best_ring};
    if (n_chosen < 16) chosen[n_chosen++] = c;
    else chosen[(N + nb) % 16] = c;
  }
  const int rows = best_cw * WR;
  CUtensorMap xmap, wmap;
  if (!encode_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)K, (uint64_t)M,
                 (uint64_t)K * 2, 64u, (uint32_t)TN, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  const long long row_bytes = (long long)nb * KQ<QT>::kBlockBytes;
  const int pitch = raw_slot_bytes(QT, best_ring.kbs);
  if (!encode_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT64, w, (uint64_t)row_bytes / 8, (uint64_t)N,
                 (uint64_t)row_bytes, (uint32_t)pitch / 8, (uint32_t)rows, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  MmaParams p{};
  p.y = y;
  p.residual = residual;
  p.M = M;
  p.N = N;
  p.nb = nb;
  p.bb = KQ<QT>::kBlockBytes;
  p.tn = TN;
  p.splits = best_s;
  p.stages = best_ring.stages;
  p.kbs = best_ring.kbs;
  p.pitch = pitch;
  p.cwarps = best_cw;
  p.rows = rows;
  p.raw_bytes = (uint32_t)raw_part_bytes(QT, best_ring.kbs, rows);
  p.wbox_bytes = (uint32_t)(rows * pitch);
  p.stage_bytes = (uint32_t)stage_bytes_for(QT, best_ring.kbs, TN, rows);
  p.off_tab = (uint32_t)best_ring.stages * p.stage_bytes;
  p.err = env.d_err;
  cfg.gridDim = dim3((N + rows - 1) / rows, pl.m_tiles, best_s);
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
  return cudaLaunchKernelEx(&cfg, kern, xmap, wmap, p);
}

template <int QT>
cudaError_t launch_q(const LaunchEnv& env, const MmaPlan& pl, const void* w, const uint16_t* x,
                     float* y, int M, int K, int N, const float* residual) {
  switch (pl.tn) {
    case 16: return launch_t<QT, 16, 1>(env, pl, w, x, y, M, K, N, residual);
    case 32: return launch_t<QT, 32, 1>(env, pl, w, x, y, M, K, N, residual);
    case 48: return launch_t<QT, 48, 2>(env, pl, w, x, y, M, K, N, residual);
    case 64: return launch_t<QT, 64, 2>(env, pl, w, x, y, M, K, N, residual);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

bool plan_gemm_kq_mma(int qtype, int M, int K, int N, int sm_count, MmaPlan* pl) {
  const int bb = kq_block_bytes(qtype);
  if (M < 1 || M > kMaxTn || K < 256 || K % 256 || N < 1 || bb == 0) return false;
  // the raw stage is one TMA box: every row must start 16-byte aligned
  if (((long long)(K / 256) * bb) % 16 != 0) return false;
  MmaPlan r{};
  r.tn = (M + 15) / 16 * 16;  // NF = tn / 8 even: one ldmatrix.x4 covers 2 n fragments
  r.m_tiles = (M + r.tn - 1) / r.tn;
  // the tile height and the split count are chosen at launch from the kernel's cluster
  // occupancy; here only whether the tallest tile fits
  const Ring rg = ring_for(qtype, r.tn, kMaxRows);
  if (rg.stages == 0) return false;
  r.n_tiles = (N + kMaxRows - 1) / kMaxRows;
  r.kbs = rg.kbs;
  r.stages = rg.stages;
  r.smem = rg.smem;
  r.splits = 0;
  (void)sm_count;
  *pl = r;
  return true;
}

cudaError_t launch_gemm_kq_mma(const LaunchEnv& env, int qtype, const void* w,
                               const uint16_t* x_bf16, float* y, int M, int K, int N,
                               const MmaPlan& pl, const float* residual) {
  switch (qtype) {
    case RRR_Q4_K: return launch_q<RRR_Q4_K>(env, pl, w, x_bf16, y, M, K, N, residual);
    case RRR_Q5_K: return launch_q<RRR_Q5_K>(env, pl, w, x_bf16, y, M, K, N, residual);
    case RRR_Q6_K: return launch_q<RRR_Q6_K>(env, pl, w, x_bf16, y, M, K, N, residual);
    default: return cudaErrorNotSupported;
  }
}

}  // namespace rrr
