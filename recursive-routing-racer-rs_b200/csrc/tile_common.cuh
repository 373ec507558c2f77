// tile_common.cuh — pieces shared by the batched-token GEMM kernels (gemm_kq_tc.cu on the
// tcgen05 tensor cores, gemm_kq_mma.cu on register-level mma.sync): TMA tile loads, the
// 128-byte swizzle, cluster barriers and distributed shared memory, warp-uniform bounded
// waits, the packed exact-offset dequantisation of K-quant runs to bf16, and the host-side
// tensor-map encoding and raw-stage pitch. Only sm_100a is targeted.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "kquant.cuh"
#include "rrr_common.cuh"

namespace rrr {

// Device error code of a tile kernel's bounded wait (kDevErr* of rrr_common.cuh are 1..3).
constexpr int kDevErrTileWait = 4;

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

// Barrier over every thread of every CTA of the cluster (release / acquire).
__device__ __forceinline__ void cluster_sync() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}
// 16-byte load from the shared memory of cluster CTA `rank` at this CTA's shared address.
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t local_addr, uint32_t rank) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(local_addr), "r"(rank));
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(ra)
               : "memory");
  return v;
}

// Byte offset of 16-byte chunk c (0..7) of row r inside a 128-byte-swizzled tile.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// ---- tcgen05 primitives (one CTA group) ----------------------------------------------

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
// The same for tf32 inputs (32-bit containers; K = 8 per instruction).
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The same with the A operand in tensor memory (M = 128 lanes, one tf32 element per 32-bit
// column, K = 8 columns from a_tmem).
__device__ __forceinline__ void umma_tf32_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns from registers: thread i writes lane (base + i).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
      "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
      "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
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

// Bounded wait by every lane of a warp; the warp agrees on the outcome.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err,
                                          int code = kDevErrTileWait) {
  const bool ok = mbar_wait_bounded(bar, parity, err, code);
  return __all_sync(0xffffffffu, ok);
}

// The CTA's abort flag as one value for the whole warp (warp-collective code below must
// not diverge on it).
__device__ __forceinline__ bool warp_aborted(volatile int* flag) {
  return __any_sync(0xffffffffu, *flag != 0);
}

// Scale pair of one run of weights v*a - b (v a small integer) in the form the packed
// FMA uses: the integer is placed in bits 16-22 of an f32 with exponent 23, which is the
// exact value f = 2^23 + 65536 v; then f * (a / 65536) + c with c = -(128 a + b) equals
// v*a - b up to one rounding of the FMA and the rounding of c (about 2^-17 a).
struct RunScale {
  float2 a, c;
};
__device__ __forceinline__ RunScale run_scale(float a, float b) {
  const float ap = a * (1.0f / 65536.0f);
  const float c = -fmaf(128.f, a, b);
  return {make_float2(ap, ap), make_float2(c, c)};
}

// Four values (bytes of w, each < 128) -> two bf16x2 words (round to nearest).
__device__ __forceinline__ void emit4(uint32_t w, const RunScale& sc, uint32_t* o) {
  const float2 f01 = make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7044)),
                                 __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7144)));
  const float2 f23 = make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7244)),
                                 __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7344)));
  const __nv_bfloat162 b01 = __float22bfloat162_rn(__ffma2_rn(f01, sc.a, sc.c));
  const __nv_bfloat162 b23 = __float22bfloat162_rn(__ffma2_rn(f23, sc.a, sc.c));
  o[0] = *reinterpret_cast<const uint32_t*>(&b01);
  o[1] = *reinterpret_cast<const uint32_t*>(&b23);
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

// 16 bytes at a 2-byte-aligned shared address, via aligned 32-bit loads and funnel shifts.
__device__ __forceinline__ void ld16_a2(const uint8_t* p, uint32_t* o) {
  const uint32_t* q = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(p) & ~(uintptr_t)3);
  const uint32_t sh = (uint32_t)(reinterpret_cast<uintptr_t>(p) & 3) * 8;
  uint32_t w[5];
#pragma unroll
  for (int i = 0; i < 5; ++i) w[i] = q[i];
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = __funnelshift_r(w[i], w[i + 1], sh);
}

inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// Row pitch of a raw stage of `kbs` super-blocks: the blocks plus room for the 16-byte
// envelope of a block run that does not start 16-byte aligned (Q6_K), rounded to an odd
// number of 16-byte units so that 8 consecutive rows read 16-byte words from distinct
// bank groups.
inline int raw_slot_bytes(int qtype, int kbs) {
  const int bytes = kq_block_bytes(qtype) * kbs + (qtype == RRR_Q6_K ? 14 : 0);
  int units = (bytes + 15) / 16;
  if ((units & 1) == 0) ++units;
  return units * 16;
}

inline int next_pow2_cols(int tn) {
  int c = 32;
  while (c < tn) c <<= 1;
  return c;
}

// Tensor map of a 2-D row-major array: `inner` elements of `elem_bytes` per row (row
// pitch `pitch_bytes`, a multiple of 16), `rows` rows; box = box_inner x box_rows.
inline bool encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
               uint64_t rows, uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_rows,
               CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)pitch_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Clusters of `cluster` CTAs of `kern` (launch config `cfg`; its grid and attributes are
// replaced) that can be resident at once. A cluster must fit in one GPC, so at one CTA per
// SM clusters of 3 or more leave SMs unused (on a 148-SM B200: 45 x 3, 33 x 4, 26 x 5,
// 22 x 6, 15 x 8). Cached per (kernel, device, shared memory, cluster size).
inline int max_active_clusters(const void* kern, cudaLaunchConfig_t cfg, int cluster) {
  struct Entry {
    const void* k;
    int dev, smem, c, n;
  };
  static std::mutex mu;
  static Entry cache[128];
  static int n_cache = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    for (int i = 0; i < n_cache; ++i)
      if (cache[i].k == kern && cache[i].dev == dev && cache[i].smem == (int)cfg.dynamicSmemBytes &&
          cache[i].c == cluster)
        return cache[i].n;
  }
  cudaLaunchAttribute a[1];
  a[0].id = cudaLaunchAttributeClusterDimension;
  a[0].val.clusterDim.x = 1;
  a[0].val.clusterDim.y = 1;
  a[0].val.clusterDim.z = cluster;
  cfg.gridDim = dim3(1, 1, cluster);
  cfg.attrs = a;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (n_cache < 128) cache[n_cache++] = Entry{kern, dev, (int)cfg.dynamicSmemBytes, cluster, n};
  return n;
}

// Split-K factor for `base` output tiles of `nb` K-blocks each, at most `max_s`: the s
// whose waves (ceil(base / resident clusters of s)) times K-blocks per CTA (ceil(nb / s))
// is smallest; ties go to the smaller s (less reduction).
inline int pick_splits(const void* kern, const cudaLaunchConfig_t& cfg, int base, int nb,
                       int max_s) {
  int best = 1;
  long long best_cost = -1;
  for (int s = 1; s <= max_s; ++s) {
    const int fit = max_active_clusters(kern, cfg, s);
    if (fit < 1) continue;
    const long long cost = (long long)((base + fit - 1) / fit) * ((nb + s - 1) / s);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

// Candidate tile height of a row-tiled GEMM launch: weight rows per CTA, its block size and
// dynamic shared memory.
struct TileCand {
  int rows, threads, smem;
};
// Picks a candidate (given tallest first) and its split count. For each height the split
// count is pick_splits' (fewest waves x K-blocks per CTA); the tallest height whose
// first wave puts at least 3/4 of the SMs to work in one wave wins (tall tiles re-read X
// least and spread the fixed cost per CTA over the most rows); if no height fills the
// GPU, the least work on the busiest SM wins: waves x CTAs per SM x K-blocks per CTA x
// rows. Returns the index (-1: none fits) and the split count in *splits.
inline int choose_tile(const void* kern, cudaStream_t stream, const TileCand* c, int n, int N,
                       int m_tiles, int nb, int max_s, int sm_count, int* splits) {
  cudaLaunchConfig_t cfg = {};
  cfg.stream = stream;
  int best = -1, best_s = 1;
  long long best_work = -1;
  for (int i = 0; i < n; ++i) {
    cfg.blockDim = dim3(c[i].threads);
    cfg.dynamicSmemBytes = c[i].smem;
    const int base = m_tiles * ((N + c[i].rows - 1) / c[i].rows);
    int s_best = 0, fit_best = 0;
    long long cost_best = -1;
    for (int s = 1; s <= max_s; ++s) {
      const int fit = max_active_clusters(kern, cfg, s);
      if (fit < 1) continue;
      const long long cost = (long long)((base + fit - 1) / fit) * ((nb + s - 1) / s);
      if (cost_best < 0 || cost < cost_best) {
        cost_best = cost;
        s_best = s;
        fit_best = fit;
      }
    }
    if (s_best == 0) continue;
    const int waves = (base + fit_best - 1) / fit_best;
    const long long first = (long long)std::min(base, fit_best) * s_best;
    if (waves == 1 && 4 * first >= 3LL * sm_count) {
      *splits = s_best;
      return i;
    }
    const long long per_sm = (first + sm_count - 1) / sm_count;
    const long long work = (long long)waves * per_sm * ((nb + s_best - 1) / s_best) * c[i].rows;
    if (best_work < 0 || work < best_work) {
      best_work = work;
      best = i;
      best_s = s_best;
    }
  }
  *splits = best_s;
  return best;
}

}  // namespace rrr
