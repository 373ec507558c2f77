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
//              and coalesced f32 stores; with split-K, partial tiles go to a workspace and
//              the last CTA of a tile sums them in split order (deterministic).
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

#include <mutex>

#include "internal.h"
#include "kquant.cuh"
#include "rrr_common.cuh"

namespace rrr {
namespace {

constexpr int kBM = 128;              // weight rows per tile = MMA M = TMEM lanes
constexpr int kBK = 64;               // K per ring slot: one 128-byte swizzle row of bf16
constexpr int kThreads = 352;         // 11 warps
constexpr int kDqThreads = 256;       // warps 3..10
constexpr int kRawStages = 2;
constexpr int kABytes = kBM * kBK * 2;  // 16 KB per A slot
constexpr int kMaxStages = 4;
constexpr int kSmemBudget = 232448;   // 227 KB opt-in maximum on sm_100

// Device error codes of this kernel (kDevErr* of rrr_common.cuh are 1..3).
constexpr int kDevErrTcWait = 4;

struct TcParams {
  const uint8_t* w;
  const uint8_t* w_end;
  float* y;
  float* ws;            // split-K partial tiles [splits][M][N] (splits > 1)
  unsigned* counters;   // one per output tile, zero between launches (splits > 1)
  long long row_bytes;
  int M, K, N, nb, bb;  // nb super-blocks per row, bb bytes per super-block
  int tn, splits, stages, slot, tmem_cols, n_tiles;
  uint32_t off_b, off_raw, off_bar;  // byte offsets from the 1024-aligned smem base
  uint32_t idesc;
  int* err;
};

// ---- tcgen05 / TMA primitives -------------------------------------------------------

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, bf16 inputs, f32 accumulate; accumulate = 0 overwrites.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` when every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}
// 32 lanes x 8 consecutive 32-bit columns: thread i gets lane (base + i), columns c..c+7.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// Generic-proxy shared-memory writes become visible to the async proxy (tensor core).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 2-D TMA tile load (plain, no multicast) of box {64, TN} at (c0 = k, c1 = token).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}

// Shared-memory matrix descriptor of a K-major operand in the canonical 128-byte-swizzled
// layout: rows of 128 bytes (64 bf16 of K), 8-row groups 1024 bytes apart (stride byte
// offset), 16-byte chunk c of row r stored at chunk c ^ (r % 8). Fields: start address
// >> 4 (bits 0-13), leading byte offset >> 4 (16-29, unused for this layout: 1), stride
// byte offset >> 4 (32-45), descriptor version 1 (46-47), layout type 2 = 128-byte
// swizzle (61-63). Advancing K by 16 elements inside the 128-byte row adds 32 bytes to
// the start address.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Byte offset of 16-byte chunk c (0..7) of row r inside a 128-byte-swizzled tile.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Bounded wait by every lane of a warp; the warp agrees on the outcome.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err) {
  const bool ok = mbar_wait_bounded(bar, parity, err, kDevErrTcWait);
  return __all_sync(0xffffffffu, ok);
}

// The CTA's abort flag as one value for the whole warp (warp-collective code below must
// not diverge on it).
__device__ __forceinline__ bool warp_aborted(volatile int* flag) {
  return __any_sync(0xffffffffu, *flag != 0);
}

// ---- dequantisation of one 64-wide K chunk: 32 values per thread ---------------------
// Thread half h handles l in [16h, 16h+16) of the two 32-element runs of the chunk and
// writes the bf16 words of K positions [16h, 16h+16) to out[0..7] and
// [32+16h, 32+16h+16) to out[8..15].

// exact f32 of byte b of w (0..255), minus `bias` (the 2^23 magic-number conversion)
__device__ __forceinline__ float byte_f(uint32_t w, int b, float bias) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440 | b)) - bias;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// four bytes of w -> two bf16x2 words of (q * a - b)
__device__ __forceinline__ void emit4(uint32_t w, float a, float b, float bias, uint32_t* o) {
  o[0] = pack_bf16(fmaf(byte_f(w, 0, bias), a, -b), fmaf(byte_f(w, 1, bias), a, -b));
  o[1] = pack_bf16(fmaf(byte_f(w, 2, bias), a, -b), fmaf(byte_f(w, 3, bias), a, -b));
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xFFu; }

// 6-bit scale / min of sub-block s from the 12 scale bytes held as words s0 (bytes 0-3),
// s1 (4-7), s2 (8-11) (phi4.rs:492-498).
__device__ __forceinline__ void scale_min_w(uint32_t s0, uint32_t s1, uint32_t s2, int s,
                                            float& sv, float& mv) {
  uint32_t a, b;
  if (s < 4) {
    a = byte_of(s0, s) & 63u;
    b = byte_of(s1, s) & 63u;
  } else {
    const int i = s - 4;
    a = (byte_of(s2, i) & 15u) | ((byte_of(s0, i) >> 6) << 4);
    b = (byte_of(s2, i) >> 4) | ((byte_of(s1, i) >> 6) << 4);
  }
  sv = (float)a;
  mv = (float)b;
}

template <int QT> struct TcDq;

// Q4_K: chunk j = qs bytes [32j, 32j+32); low nibbles = sub-block 2j, high = 2j+1.
template <> struct TcDq<RRR_Q4_K> {
  static __device__ __forceinline__ void run(const uint8_t* blk, int j, int h, uint32_t* out) {
    const uint4 hd = *reinterpret_cast<const uint4*>(blk);
    const float d = f16_bits_to_f32(hd.x & 0xFFFFu), dmin = f16_bits_to_f32(hd.x >> 16);
    float s0, m0, s1, m1;
    scale_min_w(hd.y, hd.z, hd.w, 2 * j, s0, m0);
    scale_min_w(hd.y, hd.z, hd.w, 2 * j + 1, s1, m1);
    const float a0 = d * s0, b0 = dmin * m0, a1 = d * s1, b1 = dmin * m1;
    const uint4 q = *reinterpret_cast<const uint4*>(blk + 16 + 32 * j + 16 * h);
    const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      emit4(qw[i] & 0x0F0F0F0Fu, a0, b0, 8388608.f, out + 2 * i);
      emit4((qw[i] >> 4) & 0x0F0F0F0Fu, a1, b1, 8388608.f, out + 8 + 2 * i);
    }
  }
};

// Q5_K: as Q4_K plus the fifth bit: bit s of qh[l] for sub-block s (phi4.rs:512-542).
template <> struct TcDq<RRR_Q5_K> {
  static __device__ __forceinline__ void run(const uint8_t* blk, int j, int h, uint32_t* out) {
    const uint4 hd = *reinterpret_cast<const uint4*>(blk);
    const float d = f16_bits_to_f32(hd.x & 0xFFFFu), dmin = f16_bits_to_f32(hd.x >> 16);
    float s0, m0, s1, m1;
    scale_min_w(hd.y, hd.z, hd.w, 2 * j, s0, m0);
    scale_min_w(hd.y, hd.z, hd.w, 2 * j + 1, s1, m1);
    const float a0 = d * s0, b0 = dmin * m0, a1 = d * s1, b1 = dmin * m1;
    const uint4 qh = *reinterpret_cast<const uint4*>(blk + 16 + 16 * h);
    const uint4 q = *reinterpret_cast<const uint4*>(blk + 48 + 32 * j + 16 * h);
    const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
    const uint32_t hw[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo = (qw[i] & 0x0F0F0F0Fu) | (((hw[i] >> (2 * j)) & 0x01010101u) << 4);
      const uint32_t hi = ((qw[i] >> 4) & 0x0F0F0F0Fu) | (((hw[i] >> (2 * j + 1)) & 0x01010101u) << 4);
      emit4(lo, a0, b0, 8388608.f, out + 2 * i);
      emit4(hi, a1, b1, 8388608.f, out + 8 + 2 * i);
    }
  }
};

// 16 bytes at a 2-byte-aligned shared address, via aligned 32-bit loads and funnel shifts.
__device__ __forceinline__ void ld16_a2(const uint8_t* p, uint32_t (&o)[4]) {
  const uint32_t* q = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(p) & ~(uintptr_t)3);
  const uint32_t sh = (uint32_t)(reinterpret_cast<uintptr_t>(p) & 3) * 8;
  uint32_t w[5];
#pragma unroll
  for (int i = 0; i < 5; ++i) w[i] = q[i];
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = __funnelshift_r(w[i], w[i + 1], sh);
}

// Q6_K: chunk j covers half g = j/2 and runs k = 2(j%2), 2(j%2)+1 of 32 elements: run k
// takes nibble (j%2) of ql[64g + 32(k&1) + l] and bits 2k of qh[32g + l]; scale index
// e/16 = 8g + 2k + l/16; value (d*scale) * (q - 32) (phi4.rs:444-479). `blk` is only
// 2-byte aligned.
template <> struct TcDq<RRR_Q6_K> {
  static __device__ __forceinline__ void run(const uint8_t* blk, int j, int h, uint32_t* out) {
    const int g = j >> 1, jj = j & 1, kA = 2 * jj;
    uint32_t qa[4], qb[4], qh[4];
    ld16_a2(blk + 64 * g + 16 * h, qa);
    ld16_a2(blk + 64 * g + 32 + 16 * h, qb);
    ld16_a2(blk + 128 + 32 * g + 16 * h, qh);
    const float d = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(blk + 208));
    const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192 + 8 * g + 2 * kA + h);
    const float aA = d * (float)sc[0], aB = d * (float)sc[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t nA = jj ? ((qa[i] >> 4) & 0x0F0F0F0Fu) : (qa[i] & 0x0F0F0F0Fu);
      const uint32_t nB = jj ? ((qb[i] >> 4) & 0x0F0F0F0Fu) : (qb[i] & 0x0F0F0F0Fu);
      const uint32_t bA = nA | (((qh[i] >> (2 * kA)) & 0x03030303u) << 4);
      const uint32_t bB = nB | (((qh[i] >> (2 * kA + 2)) & 0x03030303u) << 4);
      emit4(bA, aA, 0.f, 8388640.f, out + 2 * i);       // (2^23 + q) - (2^23 + 32) = q - 32
      emit4(bB, aB, 0.f, 8388640.f, out + 8 + 2 * i);
    }
  }
};

// ---- the kernel ---------------------------------------------------------------------

template <int QT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kq_tc_kernel(const __grid_constant__ CUtensorMap xmap, const TcParams p) {
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) &
                                             ~(uintptr_t)1023);
  const int S = p.stages;
  uint8_t* sA = smem;
  uint8_t* sB = smem + p.off_b;
  uint8_t* sRaw = smem + p.off_raw;
  uint64_t* full_a = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  uint64_t* full_b = full_a + S;
  uint64_t* empty = full_b + S;
  uint64_t* raw_full = empty + S;
  uint64_t* raw_empty = raw_full + kRawStages;
  uint64_t* acc_full = raw_empty + kRawStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = abort_flag + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBM, m0 = blockIdx.y * p.tn, z = blockIdx.z;
  const int kb0 = (int)((long long)z * p.nb / p.splits);
  const int kb1 = (int)((long long)(z + 1) * p.nb / p.splits);
  const int n_chunks = 4 * (kb1 - kb0);
  const uint32_t b_bytes = (uint32_t)p.tn * 128u;
  const uint32_t raw_stage_bytes = (uint32_t)kBM * (uint32_t)p.slot;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_a[s], kDqThreads / 32);
      mbar_init(&full_b[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int r = 0; r < kRawStages; ++r) {
      mbar_init(&raw_full[r], 1);
      mbar_init(&raw_empty[r], kDqThreads / 32);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    *last_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, (uint32_t)p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- raw-block producer: runs up to kRawStages super-blocks ahead
    const int n_blk = kb1 - kb0;
    int n_raw = 0;
    for (int blk = 0; blk < n_blk; ++blk) {
      if (warp_aborted(abort_flag)) break;
      const int r = blk % kRawStages;
      if (blk >= kRawStages && !warp_wait(&raw_empty[r], ((blk / kRawStages) - 1) & 1, p.err)) {
        *abort_flag = 1;
        break;
      }
      uint8_t* dst_stage = sRaw + r * raw_stage_bytes;
      const long long kb = kb0 + blk;
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
          const uint8_t* end = src + p.bb;
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
    for (int r = 0; r < kRawStages; ++r) {
      const int cnt = n_raw > r ? (n_raw - r + kRawStages - 1) / kRawStages : 0;
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
        mbar_arrive_expect_tx(&full_b[s], b_bytes);
        tma_load_2d(sB + s * b_bytes, &xmap, kb0 * 256 + it * kBK, m0, &full_b[s]);
      }
      __syncwarp();
      ++n_b;
    }
    for (int s = 0; s < S; ++s) {
      const int cnt = n_b > s ? (n_b - s + S - 1) / S : 0;
      if (cnt) warp_wait(&full_b[s], (cnt - 1) & 1, p.err);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      for (int it = 0; it < n_chunks; ++it) {
        if (*abort_flag) break;
        const int s = it % S;
        const uint32_t ph = (uint32_t)(it / S) & 1u;
        if (!mbar_wait_bounded(&full_a[s], ph, p.err, kDevErrTcWait) ||
            !mbar_wait_bounded(&full_b[s], ph, p.err, kDevErrTcWait)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_addr(sA + s * kABytes), b0 = smem_addr(sB + s * b_bytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          umma_bf16(tmem, sw128_desc(a0 + 32 * kk), sw128_desc(b0 + 32 * kk), p.idesc,
                    (it | kk) != 0);
        umma_commit(&empty[s]);
      }
      umma_commit(acc_full);
    }
    __syncwarp();
  } else {
    // ---------------- dequantisation
    const int t = threadIdx.x - 96;
    const int h = t >> 7, r = t & 127;
    const bool row_ok = n0 + r < p.N;
    for (int it = 0; it < n_chunks; ++it) {
      if (warp_aborted(abort_flag)) break;
      const int blk = it >> 2, j = it & 3, rs = blk % kRawStages;
      if (j == 0 && !warp_wait(&raw_full[rs], (blk / kRawStages) & 1, p.err)) {
        *abort_flag = 1;
        break;
      }
      uint32_t out[16];
      if (row_ok) {
        const uint8_t* row = sRaw + rs * raw_stage_bytes + r * p.slot;
        const long long off = (long long)(n0 + r) * p.row_bytes + (long long)(kb0 + blk) * p.bb;
        TcDq<QT>::run(row + (reinterpret_cast<uintptr_t>(p.w + off) & 15), j, h, out);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) out[i] = 0u;
      }
      const int s = it % S;
      if (it >= S && !warp_wait(&empty[s], ((it / S) - 1) & 1, p.err)) {
        *abort_flag = 1;
        break;
      }
      uint8_t* a = sA + s * kABytes;
      const int c0 = 2 * h;
      *reinterpret_cast<uint4*>(a + sw128_off(r, c0)) = make_uint4(out[0], out[1], out[2], out[3]);
      *reinterpret_cast<uint4*>(a + sw128_off(r, c0 + 1)) = make_uint4(out[4], out[5], out[6], out[7]);
      *reinterpret_cast<uint4*>(a + sw128_off(r, c0 + 4)) = make_uint4(out[8], out[9], out[10], out[11]);
      *reinterpret_cast<uint4*>(a + sw128_off(r, c0 + 5)) = make_uint4(out[12], out[13], out[14], out[15]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full_a[s]);
      if (j == 3 && lane == 0) mbar_arrive(&raw_empty[rs]);
    }

    // ---------------- epilogue: TMEM -> registers -> global
    const bool got_acc = warp_wait(acc_full, 0, p.err);
    const bool have_acc = got_acc && !warp_aborted(abort_flag);
    tc_fence_after();
    const int q = warp & 3;
    const int n = n0 + q * 32 + lane;
    const int half = (warp - 3) >> 2;
    const int cw = p.tn >> 1;
    float* out = p.splits > 1 ? p.ws + (size_t)z * p.M * p.N : p.y;
    if (have_acc) {
      for (int c = half * cw; c < (half + 1) * cw; c += 8) {
        uint32_t v[8];
        tmem_ld8(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int m = m0 + c + i;
          if (m < p.M && n < p.N) out[(size_t)m * p.N + n] = __uint_as_float(v[i]);
        }
      }
    }
    if (p.splits > 1) {
      // the last CTA of this tile sums the partials in split order
      __threadfence();
      named_barrier(1, kDqThreads);
      const int tile = blockIdx.y * p.n_tiles + blockIdx.x;
      if (t == 0) *last_flag = atomicAdd(&p.counters[tile], 1u) == (unsigned)(p.splits - 1);
      named_barrier(1, kDqThreads);
      if (*last_flag) {
        __threadfence();
        for (int idx = t; idx < kBM * p.tn; idx += kDqThreads) {
          const int mm = m0 + idx / kBM, nn = n0 + idx % kBM;
          if (mm < p.M && nn < p.N) {
            const size_t o = (size_t)mm * p.N + nn;
            float acc = 0.f;
            for (int s = 0; s < p.splits; ++s) acc += __ldcg(p.ws + (size_t)s * p.M * p.N + o);
            p.y[o] = acc;
          }
        }
        if (t == 0) p.counters[tile] = 0u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, (uint32_t)p.tmem_cols);
  }
}

// ---- host side ----------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

int raw_slot_bytes(int qtype) {
  // block bytes plus room for a 16-byte-aligned envelope, padded so that 8 consecutive
  // rows read 16-byte words from distinct bank groups (row stride = 4 words mod 32)
  return qtype == RRR_Q4_K ? 144 : qtype == RRR_Q5_K ? 176 : 240;
}

int next_pow2_cols(int tn) {
  int c = 32;
  while (c < tn) c <<= 1;
  return c;
}

template <int QT>
cudaError_t launch_t(const LaunchEnv& env, const TcPlan& pl, const void* w, const uint16_t* x,
                     float* y, int M, int K, int N, const TcWorkspace& wsp) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)pl.tn};
  const cuuint32_t estr[2] = {1, 1};
  CUresult cr = fn(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(x), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return cudaErrorInvalidValue;

  TcParams p{};
  p.w = static_cast<const uint8_t*>(w);
  p.bb = KQ<QT>::kBlockBytes;
  p.nb = K / 256;
  p.row_bytes = (long long)p.nb * p.bb;
  p.w_end = p.w + p.row_bytes * N;
  p.y = y;
  p.ws = wsp.ws;
  p.counters = wsp.counters;
  p.M = M;
  p.K = K;
  p.N = N;
  p.tn = pl.tn;
  p.splits = pl.splits;
  p.stages = pl.stages;
  p.slot = raw_slot_bytes(QT);
  p.tmem_cols = pl.tmem_cols;
  p.n_tiles = pl.n_tiles;
  p.off_b = (uint32_t)(pl.stages * kABytes);
  p.off_raw = p.off_b + (uint32_t)(pl.stages * pl.tn * 128);
  p.off_bar = p.off_raw + (uint32_t)(kRawStages * kBM * p.slot);
  // instruction descriptor: f32 accumulator (bits 4-5 = 1), A and B bf16 (bits 7-9 and
  // 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 (bits 17-22), M >> 4 (bits 24-28)
  p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(pl.tn >> 3) << 17) |
            ((uint32_t)(kBM >> 4) << 24);
  p.err = env.d_err;

  auto kern = gemm_kq_tc_kernel<QT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem);
  if (e != cudaSuccess) return e;
  const dim3 grid(pl.n_tiles, pl.m_tiles, pl.splits);
  kern<<<grid, kThreads, pl.smem, env.stream>>>(map, p);
  return cudaGetLastError();
}

}  // namespace

bool plan_gemm_kq_tc(int qtype, int M, int K, int N, int sm_count, TcPlan* pl) {
  if (M < 16 || K < 256 || K % 256 || N < 1 || kq_block_bytes(qtype) == 0) return false;
  TcPlan r{};
  r.m_tiles = (M + 255) / 256;
  r.tn = ((M + r.m_tiles - 1) / r.m_tiles + 15) / 16 * 16;
  r.n_tiles = (N + kBM - 1) / kBM;
  r.tmem_cols = next_pow2_cols(r.tn);
  const int raw = kRawStages * kBM * raw_slot_bytes(qtype);
  const int per_stage = kABytes + r.tn * 128;
  const int fixed = 1024 + raw + 256;
  r.stages = (kSmemBudget - fixed) / per_stage;
  if (r.stages > kMaxStages) r.stages = kMaxStages;
  if (r.stages < 2) return false;
  r.smem = fixed + r.stages * per_stage;
  // one CTA per SM (the launch bounds and the TMEM columns assume it)
  if (r.smem < kSmemBudget / 2 + 1024) r.smem = kSmemBudget / 2 + 1024;
  const int nb = K / 256;
  const int base = r.n_tiles * r.m_tiles;
  int splits = sm_count > 0 ? sm_count / base : 1;
  if (splits > nb / 2) splits = nb / 2;
  if (splits < 1) splits = 1;
  r.splits = splits;
  r.ws_floats = splits > 1 ? (size_t)splits * M * N : 0;
  r.n_counters = splits > 1 ? base : 0;
  *pl = r;
  return true;
}

cudaError_t launch_gemm_kq_tc(const LaunchEnv& env, int qtype, const void* w,
                              const uint16_t* x_bf16, float* y, int M, int K, int N,
                              const TcPlan& pl, const TcWorkspace& wsp) {
  if (pl.splits > 1 && (!wsp.ws || !wsp.counters)) return cudaErrorInvalidValue;
  switch (qtype) {
    case RRR_Q4_K: return launch_t<RRR_Q4_K>(env, pl, w, x_bf16, y, M, K, N, wsp);
    case RRR_Q5_K: return launch_t<RRR_Q5_K>(env, pl, w, x_bf16, y, M, K, N, wsp);
    case RRR_Q6_K: return launch_t<RRR_Q6_K>(env, pl, w, x_bf16, y, M, K, N, wsp);
    default: return cudaErrorNotSupported;
  }
}

}  // namespace rrr
