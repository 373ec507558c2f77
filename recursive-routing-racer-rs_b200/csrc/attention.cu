// attention.cu — decode glue at real positions: the embedding lookup, RoPE + f16 KV
// store, and GQA decode attention over the f16 caches.
//
//   embed_rows      out[t] = row tokens[t] of the embedding table, dequantised on the
//                   fly from its stored type (F32, F16, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K) with
//                   the reference's exact element formulas (dequant_tensor_f32 +
//                   Phi4Model::embed, src/model/phi4.rs:544-587, 2085-2089).
//   rope_kv_store   RoPE on the Q and K heads of each QKV row, in place (apply_rope_cfg,
//                   phi4.rs:238-256, same operation order, no FMA contraction), then K
//                   and V of the row rounded to f16 into cache row `pos` (the
//                   `rope_kv_store` / `kv_store` dispatches, phi4.rs:1115-1121, 1660-1677).
//   attention       softmax(q.K^T / sqrt(hd)) V per query head over cache rows 0..pos
//                   (the `attention` dispatch, push [seq_len, n_kv, heads_per_kv,
//                   head_dim], phi4.rs:1680-1688). One thread-block cluster per (KV head,
//                   token): its CTAs split the positions, each keeps an online-softmax
//                   partial (max, sum, weighted V) in shared memory, and the partials are
//                   merged over distributed shared memory in split order (deterministic,
//                   no workspace). The query heads that share a KV head read each K / V
//                   row once.
// The position can be a device integer (read after the grid dependency wait) so that a
// captured decode step replays at every position; pos_advance moves it on.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include <mutex>

#include "capi_internal.h"
#include "internal.h"
#include "kquant.cuh"
#include "rrr_common.cuh"

namespace rrr {
namespace {

constexpr int kAttnThreads = 256;
constexpr int kMaxHpk = 8;          // query heads per KV head
constexpr int kMaxSplits = 16;
constexpr int kMaxRopePairs = 64;

__device__ __forceinline__ void flag_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ------------------------------------------------------------------ embedding rows
// Element e of a row of `d` values stored as GGUF type T (row starts at `row`).
template <int T>
__device__ __forceinline__ float emb_elem(const uint8_t* row, int e);

template <>
__device__ __forceinline__ float emb_elem<0>(const uint8_t* row, int e) {
  return reinterpret_cast<const float*>(row)[e];
}
template <>
__device__ __forceinline__ float emb_elem<1>(const uint8_t* row, int e) {
  return f16_bits_to_f32(reinterpret_cast<const uint16_t*>(row)[e]);
}
// Q5_0 (22 B per 32): d, qh (u32), qs[16]; q = (nibble | qh bit j << 4) - 16,
// value d * q (phi4.rs:555-570).
template <>
__device__ __forceinline__ float emb_elem<6>(const uint8_t* row, int e) {
  const uint8_t* b = row + (e >> 5) * 22;
  const int j = e & 31;
  const float d = f16_bits_to_f32(rd16(b));
  const uint32_t qh = rd16(b + 2) | (rd16(b + 4) << 16);
  const uint32_t lo = j < 16 ? (b[6 + j] & 0xFu) : ((b[6 + j - 16] >> 4) & 0xFu);
  const int q = (int)(lo | (((qh >> j) & 1u) << 4)) - 16;
  return __fmul_rn(d, (float)q);
}
// Q8_0 (34 B per 32): d, qs[32] int8; value d * q (phi4.rs:544-553).
template <>
__device__ __forceinline__ float emb_elem<8>(const uint8_t* row, int e) {
  const uint8_t* b = row + (e >> 5) * 34;
  return __fmul_rn(f16_bits_to_f32(rd16(b)), (float)(int8_t)b[2 + (e & 31)]);
}
template <>
__device__ __forceinline__ float emb_elem<RRR_Q4_K>(const uint8_t* row, int e) {
  return kq_dequant_elem<RRR_Q4_K>(row + (e >> 8) * 144, e & 255);
}
template <>
__device__ __forceinline__ float emb_elem<RRR_Q5_K>(const uint8_t* row, int e) {
  return kq_dequant_elem<RRR_Q5_K>(row + (e >> 8) * 176, e & 255);
}
template <>
__device__ __forceinline__ float emb_elem<RRR_Q6_K>(const uint8_t* row, int e) {
  return kq_dequant_elem<RRR_Q6_K>(row + (e >> 8) * 210, e & 255);
}

template <int T>
__global__ void __launch_bounds__(256) embed_rows_kernel(const uint8_t* __restrict__ table,
                                                         long long n_rows, long long row_bytes,
                                                         int d, const int* __restrict__ tokens,
                                                         float* __restrict__ out, int* err) {
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.y;
  const int tok = tokens[t];
  const bool ok = tok >= 0 && (long long)tok < n_rows;
  if (!ok && blockIdx.x == 0 && threadIdx.x == 0) flag_error(err, kDevErrPosition);
  const uint8_t* row = table + (ok ? (long long)tok * row_bytes : 0);
  for (int e = blockIdx.x * 256 + threadIdx.x; e < d; e += gridDim.x * 256)
    out[(long long)t * d + e] = ok ? emb_elem<T>(row, e) : 0.f;
}

// ------------------------------------------------------------------ RoPE + KV store
struct RopeParams {
  float* qkv;
  long long row_stride;  // floats between QKV rows
  const int* d_pos;      // position of row 0 (device), or null: pos0
  int pos0, rows;
  int nh, nkv, hd, rope_pairs;
  float attn_factor;
  const float* factors;
  int n_factors;
  __half* kc;
  __half* vc;
  int max_seq;
  int* err;
  float base_freq[kMaxRopePairs];  // 1 / theta^((2i)/rope_dim), f32 powf on the host
};

// Pair (x0, x1) of a head rotated for position pos with the operations of apply_rope_cfg
// (phi4.rs:241-251): freq = base / factor, angle = pos * freq, (sin, cos) * attn_factor,
// (x0 c - x1 s, x0 s + x1 c); every product and sum rounded separately (no FMA).
__device__ __forceinline__ void rope_pair(float& x0, float& x1, int pos, float base_freq,
                                          float factor, float attn_factor) {
  const float freq = __fdiv_rn(base_freq, factor);
  const float angle = __fmul_rn((float)pos, freq);
  float s, c;
  sincosf(angle, &s, &c);
  const float cs = __fmul_rn(c, attn_factor), ss = __fmul_rn(s, attn_factor);
  const float y0 = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, ss));
  const float y1 = __fadd_rn(__fmul_rn(x0, ss), __fmul_rn(x1, cs));
  x0 = y0;
  x1 = y1;
}

// One CTA per (head of Q then K, row); thread i owns the pair (2i, 2i+1) of its head.
__global__ void rope_kv_store_kernel(const __grid_constant__ RopeParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int h = blockIdx.x, row = blockIdx.y;
  const int pos = (p.d_pos ? *p.d_pos : p.pos0) + row;
  if (pos < 0 || pos >= p.max_seq) {
    if (h == 0 && threadIdx.x == 0) flag_error(p.err, kDevErrPosition);
    return;
  }
  float* x = p.qkv + (long long)row * p.row_stride + (long long)h * p.hd;
  const bool is_k = h >= p.nh;
  const int kvs = p.nkv * p.hd;
  for (int i = threadIdx.x; 2 * i < p.hd; i += blockDim.x) {
    float x0 = x[2 * i], x1 = x[2 * i + 1];
    if (i < p.rope_pairs) {
      rope_pair(x0, x1, pos, p.base_freq[i], i < p.n_factors ? p.factors[i] : 1.0f, p.attn_factor);
      x[2 * i] = x0;
      x[2 * i + 1] = x1;
    }
    if (is_k) {
      const long long o = (long long)pos * kvs + (long long)(h - p.nh) * p.hd + 2 * i;
      const float* v = x + kvs;  // V of the same KV head
      *reinterpret_cast<__half2*>(p.kc + o) = __halves2half2(__float2half_rn(x0), __float2half_rn(x1));
      *reinterpret_cast<__half2*>(p.vc + o) =
          __halves2half2(__float2half_rn(v[2 * i]), __float2half_rn(v[2 * i + 1]));
    }
  }
}

// ------------------------------------------------------------------ decode attention
struct AttnParams {
  const float* q;
  long long q_stride;  // floats between query rows
  const int* d_pos;
  int pos0, rows;
  const __half* kc;
  const __half* vc;
  float* out;          // [rows, nh*hd]
  int nh, nkv, hpk;
  int max_seq, splits;
  float scale;               // 1 / sqrt(hd)
  int* err;
  // fused RoPE + KV store (one token: q is its QKV row, K and V follow the query heads)
  int fused, rope_pairs, n_factors;
  float attn_factor;
  const float* factors;
  __half* kc_w;
  __half* vc_w;
  float base_freq[kMaxRopePairs];
};

__device__ __forceinline__ float ld_dsmem_f32(const float* local, uint32_t rank) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_addr(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
  return v;
}

__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// The CTA's positions are processed in tiles of 8192 / head_dim rows (64 for 128): the K and V rows of a tile
// (head g) are copied into shared memory with 16-byte cp.async, double-buffered so that
// the next tile streams in while this one is computed; an online softmax (running max
// and sum per query head, the accumulator rescaled per tile) carries across tiles.
// Shared memory: K [2][kTile][HD] f16 | V [2][kTile][HD] f16 | new K, V row [2][HD] f16 |
// q [hpk][HD] f32 |
// probabilities [hpk][kTile] | rescale [hpk] | red [groups][hpk][HD] | partial acc
// [hpk][HD] | partial max [hpk] | partial sum [hpk].
template <int HD>
constexpr int attn_tile() { return 8192 / HD; }  // K + V double buffer = 64 KB

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(16) uint8_t smraw[];
  constexpr int LPK = HD / 8;             // lanes per key row (16 bytes each)
  constexpr int KPW = 32 / LPK;           // keys per warp step
  constexpr int NW = kAttnThreads / 32;
  constexpr int PAIRS = HD / 2;           // V dims per thread: 2
  constexpr int GROUPS = kAttnThreads / PAIRS;
  constexpr int CH = HD / 8;              // 16-byte chunks per row
  constexpr int kTile = attn_tile<HD>();
  const int hpk = p.hpk;
  __half* kt = reinterpret_cast<__half*>(smraw);
  __half* vt = kt + 2 * kTile * HD;
  __half* knew = vt + 2 * kTile * HD;
  __half* vnew = knew + HD;
  float* qs = reinterpret_cast<float*>(vnew + HD);
  float* pr = qs + hpk * HD;
  float* alpha = pr + hpk * kTile;
  float* red = alpha + kMaxHpk;
  float* pacc = red + GROUPS * hpk * HD;
  float* pmax = pacc + hpk * HD;
  float* psum = pmax + hpk;

  const int split = blockIdx.x, g = blockIdx.y, row = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvs = p.nkv * HD;
  pdl_launch_dependents();
  pdl_wait();
  const int pos = (p.d_pos ? *p.d_pos : p.pos0) + row;
  const bool pos_ok = pos >= 0 && pos < p.max_seq;
  if (!pos_ok && split == 0 && g == 0 && threadIdx.x == 0) flag_error(p.err, kDevErrPosition);
  const int seq = pos_ok ? pos + 1 : 0;
  const int per = (seq + p.splits - 1) / p.splits;
  const int t0 = min(seq, split * per), t1 = min(seq, t0 + per);
  const bool own_new = p.fused && pos_ok && t1 == seq && t0 < t1;

  const float* qrow = p.q + (long long)row * p.q_stride;
  for (int i = threadIdx.x; i < hpk * HD; i += kAttnThreads) qs[i] = qrow[(long long)(g * hpk) * HD + i];
  // the CTA whose positions end at `pos` stores the token's K (rotated) and V row of KV
  // head g into the caches, and keeps them in shared memory for its own last tile (the
  // bulk reads skip that row)
  if (own_new) {
    const float* kr = qrow + (long long)p.nh * HD + (long long)g * HD;
    const float* vr = kr + kvs;
    const long long o = (long long)pos * kvs + (long long)g * HD;
    for (int i = threadIdx.x; i < HD / 2; i += kAttnThreads) {
      float x0 = kr[2 * i], x1 = kr[2 * i + 1];
      if (i < p.rope_pairs)
        rope_pair(x0, x1, pos, p.base_freq[i], i < p.n_factors ? p.factors[i] : 1.0f, p.attn_factor);
      const __half2 k2 = __halves2half2(__float2half_rn(x0), __float2half_rn(x1));
      const __half2 v2 = __halves2half2(__float2half_rn(vr[2 * i]), __float2half_rn(vr[2 * i + 1]));
      *reinterpret_cast<__half2*>(p.kc_w + o + 2 * i) = k2;
      *reinterpret_cast<__half2*>(p.vc_w + o + 2 * i) = v2;
      *reinterpret_cast<__half2*>(knew + 2 * i) = k2;
      *reinterpret_cast<__half2*>(vnew + 2 * i) = v2;
    }
  }
  __syncthreads();
  if (p.fused && pos_ok) {
    // RoPE of this cluster's query heads (every CTA of the cluster, in shared memory)
    for (int i = threadIdx.x; i < hpk * p.rope_pairs; i += kAttnThreads) {
      const int j = i / p.rope_pairs, q2 = i % p.rope_pairs;
      float x0 = qs[j * HD + 2 * q2], x1 = qs[j * HD + 2 * q2 + 1];
      rope_pair(x0, x1, pos, p.base_freq[q2], q2 < p.n_factors ? p.factors[q2] : 1.0f, p.attn_factor);
      qs[j * HD + 2 * q2] = x0;
      qs[j * HD + 2 * q2 + 1] = x1;
    }
  }

  const int n_tiles = (t1 - t0 + kTile - 1) / kTile;
  auto issue = [&](int tile) {
    const int base = t0 + tile * kTile, nrows = min(kTile, t1 - base);
    __half* kd = kt + (tile & 1) * kTile * HD;
    __half* vd = vt + (tile & 1) * kTile * HD;
    for (int c = threadIdx.x; c < nrows * CH; c += kAttnThreads) {
      const int r = c / CH, cc = c % CH;
      if (own_new && base + r == pos) continue;
      const long long src = (long long)(base + r) * kvs + (long long)g * HD + cc * 8;
      cp_async16(kd + r * HD + cc * 8, p.kc + src);
      cp_async16(vd + r * HD + cc * 8, p.vc + src);
    }
    cp_async_commit();
  };
  if (n_tiles > 0) issue(0);

  // per-thread state: the query slice of the score lanes, and the running softmax /
  // accumulator of the PV threads (dims 2dp, 2dp+1 of every head, positions = grp mod GROUPS)
  const int sub = lane / LPK, kl = lane % LPK;
  const int grp = threadIdx.x / PAIRS, dp = threadIdx.x % PAIRS;
  float a0[kMaxHpk], a1[kMaxHpk];
#pragma unroll
  for (int j = 0; j < kMaxHpk; ++j) a0[j] = a1[j] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;  // warp j < hpk owns head j's running max / sum
  __syncthreads();
  float qr[kMaxHpk][8];
#pragma unroll
  for (int j = 0; j < kMaxHpk; ++j)
#pragma unroll
    for (int e = 0; e < 8; ++e) qr[j][e] = j < hpk ? qs[j * HD + kl * 8 + e] : 0.f;

  for (int tile = 0; tile < n_tiles; ++tile) {
    if (tile + 1 < n_tiles) {
      issue(tile + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int nrows = min(kTile, t1 - (t0 + tile * kTile));
    const __half* kb = kt + (tile & 1) * kTile * HD;
    const __half* vb = vt + (tile & 1) * kTile * HD;
    if (own_new && tile == n_tiles - 1) {  // the new row is the last one of the CTA
      const int r = pos - (t0 + tile * kTile);
      for (int c = threadIdx.x; c < 2 * CH; c += kAttnThreads) {
        const int cc = c % CH;
        __half* dst = (c < CH ? kt : vt) + (tile & 1) * kTile * HD + r * HD + cc * 8;
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>((c < CH ? knew : vnew) + cc * 8);
      }
      __syncthreads();
    }
    // ---- scores of the tile: LPK lanes per key, 8 dims per lane
    for (int kb0 = warp * KPW; kb0 < nrows; kb0 += NW * KPW) {
      const int k = kb0 + sub;
      float kf[8];
      if (k < nrows) {
        const uint4 raw = *reinterpret_cast<const uint4*>(kb + k * HD + kl * 8);
        const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(h2[e]);
          kf[2 * e] = f.x;
          kf[2 * e + 1] = f.y;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) kf[e] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < kMaxHpk; ++j) {
        if (j < hpk) {
          float dot = 0.f;
#pragma unroll
          for (int e = 0; e < 8; ++e) dot = fmaf(qr[j][e], kf[e], dot);
#pragma unroll
          for (int o = LPK / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
          if (kl == 0 && k < nrows) pr[j * kTile + k] = dot * p.scale;
        }
      }
    }
    __syncthreads();
    // ---- online softmax: warp j updates head j's running max / sum, writes the tile's
    // probabilities and the accumulator's rescale factor
    for (int j = warp; j < hpk; j += NW) {
      float m = -INFINITY;
      for (int i = lane; i < nrows; i += 32) m = fmaxf(m, pr[j * kTile + i]);
      m = fmaxf(warp_max(m), m_run);
      float l = 0.f;
      for (int i = lane; i < nrows; i += 32) {
        const float e = expf(pr[j * kTile + i] - m);
        pr[j * kTile + i] = e;
        l += e;
      }
      l = warp_sum(l);
      const float sc = m_run == -INFINITY ? 0.f : expf(m_run - m);
      l_run = l_run * sc + l;
      m_run = m;
      if (lane == 0) alpha[j] = sc;
    }
    __syncthreads();
    // ---- weighted V of the tile
    {
#pragma unroll
      for (int j = 0; j < kMaxHpk; ++j) {
        if (j < hpk) {
          const float sc = alpha[j];
          a0[j] *= sc;
          a1[j] *= sc;
        }
      }
      for (int k = grp; k < nrows; k += GROUPS) {
        const float2 v = __half22float2(*reinterpret_cast<const __half2*>(vb + k * HD + 2 * dp));
#pragma unroll
        for (int j = 0; j < kMaxHpk; ++j) {
          if (j < hpk) {
            const float w = pr[j * kTile + k];
            a0[j] = fmaf(w, v.x, a0[j]);
            a1[j] = fmaf(w, v.y, a1[j]);
          }
        }
      }
    }
    __syncthreads();  // the buffer and the probabilities are rewritten next tile
  }
  for (int j = warp; j < hpk; j += NW)
    if (lane == 0) {
      pmax[j] = m_run;
      psum[j] = l_run;
    }
#pragma unroll
  for (int j = 0; j < kMaxHpk; ++j) {
    if (j < hpk) {
      red[(grp * hpk + j) * HD + 2 * dp] = a0[j];
      red[(grp * hpk + j) * HD + 2 * dp + 1] = a1[j];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < hpk * HD; i += kAttnThreads) {
    float s = 0.f;
#pragma unroll
    for (int gi = 0; gi < GROUPS; ++gi) s += red[gi * hpk * HD + i];
    pacc[i] = s;
  }

  // ---- merge the splits' partials over distributed shared memory, in split order
  cluster_barrier();
  if (pos_ok) {
    const int tot = hpk * HD;
    const int share = (tot + p.splits - 1) / p.splits;
    const int i0 = split * share, i1 = min(tot, i0 + share);
    for (int i = i0 + threadIdx.x; i < i1; i += kAttnThreads) {
      const int j = i / HD;
      // all remote loads of the element first (independent), then the sums in split order
      float ms[kMaxSplits], ls[kMaxSplits], as[kMaxSplits];
#pragma unroll
      for (int s = 0; s < kMaxSplits; ++s) {
        if (s < p.splits) {
          ms[s] = ld_dsmem_f32(pmax + j, (uint32_t)s);
          ls[s] = ld_dsmem_f32(psum + j, (uint32_t)s);
          as[s] = ld_dsmem_f32(pacc + i, (uint32_t)s);
        }
      }
      float m = -INFINITY;
#pragma unroll
      for (int s = 0; s < kMaxSplits; ++s)
        if (s < p.splits) m = fmaxf(m, ms[s]);
      float l = 0.f, o = 0.f;
#pragma unroll
      for (int s = 0; s < kMaxSplits; ++s) {
        if (s < p.splits) {
          const float w = ms[s] == -INFINITY ? 0.f : expf(ms[s] - m);
          l = fmaf(w, ls[s], l);
          o = fmaf(w, as[s], o);
        }
      }
      p.out[(long long)row * p.nh * HD + (long long)g * hpk * HD + i] = o / l;
    }
  }
  cluster_barrier();
}

__global__ void pos_advance_kernel(int* d_pos, int delta) {
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x == 0) *d_pos += delta;
}

int attn_smem_bytes(int hd, int hpk) {
  const int groups = kAttnThreads / (hd / 2);
  const int tile = 8192 / hd;
  return 2 * 2 * 2 * tile * hd + 2 * 2 * hd +
         4 * (hpk * hd + hpk * tile + kMaxHpk + groups * hpk * hd + hpk * hd + 2 * hpk);
}

}  // namespace

// Splits of a decode-attention launch whose positions reach `seq_max`: about 64
// positions per CTA, at most 16 CTAs per cluster.
static int attn_splits(int seq_max) {
  int s = (seq_max + 63) / 64;
  return s < 1 ? 1 : s > kMaxSplits ? kMaxSplits : s;
}

cudaError_t launch_attention_f16kv(const LaunchEnv& env, const float* q, long long q_stride,
                                   int rows, int pos0, const int* d_pos, const uint16_t* kc,
                                   const uint16_t* vc, float* out, int nh, int nkv, int hd,
                                   int max_seq, int seq_max, const AttnRope* rope) {
  AttnParams p{};
  if (rope) {
    p.fused = 1;
    p.rope_pairs = rope->rope_dim / 2;
    p.attn_factor = rope->attn_factor;
    p.factors = rope->factors;
    p.n_factors = rope->factors ? rope->n_factors : 0;
    p.kc_w = reinterpret_cast<__half*>(const_cast<uint16_t*>(kc));
    p.vc_w = reinterpret_cast<__half*>(const_cast<uint16_t*>(vc));
    for (int i = 0; i < p.rope_pairs; ++i)
      p.base_freq[i] = 1.0f / powf(rope->theta, (2.0f * (float)i) / (float)rope->rope_dim);
  }
  p.q = q;
  p.q_stride = q_stride;
  p.d_pos = d_pos;
  p.pos0 = pos0;
  p.rows = rows;
  p.kc = reinterpret_cast<const __half*>(kc);
  p.vc = reinterpret_cast<const __half*>(vc);
  p.out = out;
  p.nh = nh;
  p.nkv = nkv;
  p.hpk = nh / nkv;
  p.max_seq = max_seq;
  p.splits = attn_splits(seq_max);
  p.scale = 1.0f / sqrtf((float)hd);
  p.err = env.d_err;
  const int smem = attn_smem_bytes(hd, p.hpk);
  void (*kern)(AttnParams) = nullptr;
  int hi;
  switch (hd) {
    case 64: kern = attention_kernel<64>; hi = 0; break;
    case 128: kern = attention_kernel<128>; hi = 1; break;
    case 256: kern = attention_kernel<256>; hi = 2; break;
    default: return cudaErrorInvalidValue;
  }
  // Kernel attributes and the cluster-size check are done once per kernel and split count
  // (the largest shared-memory size, 8 query heads per KV head, covers every launch).
  static std::mutex mu;
  static int dev_ready[8][3] = {};           // per device: attributes set
  static int8_t fits[8][3][kMaxSplits + 1];  // per device: 0 unknown, 1 fits, -1 does not
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 8) dev = 7;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = env.stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!dev_ready[dev][hi]) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               attn_smem_bytes(hd, kMaxHpk));
      if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess) return e;
      dev_ready[dev][hi] = 1;
    }
    for (;;) {
      int8_t& f = fits[dev][hi][p.splits];
      if (f == 0) {
        cfg.gridDim = dim3(p.splits, nkv, rows);
        attr[0].val.clusterDim.x = p.splits;
        cfg.numAttrs = 1;
        cfg.dynamicSmemBytes = attn_smem_bytes(hd, kMaxHpk);
        int n_clusters = 0;
        e = cudaOccupancyMaxActiveClusters(&n_clusters, kern, &cfg);
        cfg.dynamicSmemBytes = smem;
        f = (e == cudaSuccess && n_clusters > 0) ? 1 : -1;
      }
      if (f > 0) break;
      if (p.splits == 1) return cudaErrorInvalidConfiguration;
      // the cluster does not fit: half as many CTAs, each taking twice the positions
      p.splits = (p.splits + 1) / 2;
    }
  }
  cfg.gridDim = dim3(p.splits, nkv, rows);
  attr[0].val.clusterDim.x = p.splits;
  cfg.numAttrs = env.pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

int attention_smem_for(int hd, int hpk, int /*seq_max*/) { return attn_smem_bytes(hd, hpk); }

cudaError_t launch_rope_kv_store(const LaunchEnv& env, float* qkv, long long row_stride, int rows,
                                 int pos0, const int* d_pos, int nh, int nkv, int hd, int rope_dim,
                                 float theta, float attn_factor, const float* factors,
                                 int n_factors, uint16_t* kc, uint16_t* vc, int max_seq) {
  RopeParams p{};
  p.qkv = qkv;
  p.row_stride = row_stride;
  p.d_pos = d_pos;
  p.pos0 = pos0;
  p.rows = rows;
  p.nh = nh;
  p.nkv = nkv;
  p.hd = hd;
  p.rope_pairs = rope_dim / 2;
  p.attn_factor = attn_factor;
  p.factors = factors;
  p.n_factors = factors ? n_factors : 0;
  p.kc = reinterpret_cast<__half*>(kc);
  p.vc = reinterpret_cast<__half*>(vc);
  p.max_seq = max_seq;
  p.err = env.d_err;
  // the reference's f32 expression, 1.0 / theta.powf(2.0 * i as f32 / rope_dim as f32)
  for (int i = 0; i < p.rope_pairs; ++i)
    p.base_freq[i] = 1.0f / powf(theta, (2.0f * (float)i) / (float)rope_dim);
  int threads = hd / 2 < 32 ? 32 : hd / 2;
  if (threads > 256) threads = 256;
  return rrr_launch_pdl(rope_kv_store_kernel, dim3(nh + nkv, rows), dim3(threads), 0, env.stream,
                        env.pdl, p);
}

cudaError_t launch_embed_rows(const LaunchEnv& env, int type, const void* table, long long n_rows,
                              long long row_bytes, int d, const int* tokens, int n_tokens,
                              float* out) {
  const uint8_t* t = static_cast<const uint8_t*>(table);
  int gx = (d + 255) / 256;
  if (gx > 64) gx = 64;
  const dim3 grid(gx, n_tokens), block(256);
  switch (type) {
#define RRR_EMB_CASE(T)                                                                          \
  case T:                                                                                        \
    return rrr_launch_pdl(embed_rows_kernel<T>, grid, block, 0, env.stream, env.pdl, t, n_rows, \
                          row_bytes, d, tokens, out, env.d_err);
    RRR_EMB_CASE(0)
    RRR_EMB_CASE(1)
    RRR_EMB_CASE(6)
    RRR_EMB_CASE(8)
    RRR_EMB_CASE(RRR_Q4_K)
    RRR_EMB_CASE(RRR_Q5_K)
    RRR_EMB_CASE(RRR_Q6_K)
#undef RRR_EMB_CASE
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_pos_advance(const LaunchEnv& env, int* d_pos, int delta) {
  return rrr_launch_pdl(pos_advance_kernel, dim3(1), dim3(32), 0, env.stream, env.pdl, d_pos, delta);
}

}  // namespace rrr

using namespace rrr;

namespace {

int check_attn_desc(rrr_ctx* ctx, const rrr_attn_desc* a, const char* fn) {
  if (!a) return set_error(ctx, RRR_ERR_INVALID_ARG, "%s: null descriptor", fn);
  if (a->n_heads < 1 || a->n_kv_heads < 1 || a->n_heads % a->n_kv_heads ||
      a->n_heads / a->n_kv_heads > kMaxHpk ||
      (a->head_dim != 64 && a->head_dim != 128 && a->head_dim != 256) || a->rope_dim < 0 ||
      a->rope_dim % 2 || a->rope_dim > a->head_dim || a->rope_dim > 2 * kMaxRopePairs ||
      a->max_seq < 1 || a->n_rope_factors < 0)
    return set_error(ctx, RRR_ERR_BAD_SHAPE,
                     "%s: need n_heads %% n_kv_heads == 0 with at most 8 query heads per KV "
                     "head, head_dim 64/128/256, even rope_dim <= min(head_dim, 128), max_seq >= 1",
                     fn);
  return RRR_OK;
}

int check_rows(rrr_ctx* ctx, const rrr_attn_desc* a, int rows, int pos0, const int* d_pos,
               const char* fn) {
  if (rows < 0) return set_error(ctx, RRR_ERR_BAD_SHAPE, "%s: rows >= 0", fn);
  if (!d_pos && (pos0 < 0 || (int64_t)pos0 + rows > a->max_seq))
    return set_error(ctx, RRR_ERR_BAD_SHAPE, "%s: positions [%d, %d) outside the cache of %d rows",
                     fn, pos0, pos0 + rows, a->max_seq);
  return RRR_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" {

int rrr_rope_kv_store(rrr_ctx* ctx, const rrr_attn_desc* a, float* qkv, int64_t row_stride, int rows,
                      int pos0, const int* d_pos, uint16_t* k_cache, uint16_t* v_cache,
                      void* stream) {
  if (!ctx) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context");
  int rc = check_attn_desc(ctx, a, "rrr_rope_kv_store");
  if (rc) return rc;
  if ((rc = check_rows(ctx, a, rows, pos0, d_pos, "rrr_rope_kv_store"))) return rc;
  if (!qkv || !k_cache || !v_cache)
    return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_rope_kv_store: null pointer");
  const int64_t qkv_dim = (int64_t)(a->n_heads + 2 * a->n_kv_heads) * a->head_dim;
  if (row_stride < qkv_dim)
    return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_rope_kv_store: row_stride < (n_q + 2 n_kv) * head_dim");
  if (!aligned16(k_cache) || !aligned16(v_cache) || (reinterpret_cast<uintptr_t>(qkv) & 3))
    return set_error(ctx, RRR_ERR_MISALIGNED, "rrr_rope_kv_store: caches must be 16-byte aligned");
  if ((rc = bind_device(ctx))) return rc;
  if (rows == 0) return RRR_OK;
  cudaError_t e = launch_rope_kv_store(make_env(ctx, stream), qkv, row_stride, rows, pos0, d_pos,
                                       a->n_heads, a->n_kv_heads, a->head_dim, a->rope_dim,
                                       a->rope_theta, a->rope_attn_factor, a->rope_factors,
                                       a->n_rope_factors, k_cache, v_cache, a->max_seq);
  return e == cudaSuccess ? RRR_OK : cuda_error(ctx, e, "rrr_rope_kv_store launch");
}

int rrr_attention_f16kv(rrr_ctx* ctx, const rrr_attn_desc* a, const float* q, int64_t q_stride,
                        int rows, int pos0, const int* d_pos, const uint16_t* k_cache,
                        const uint16_t* v_cache, float* out, void* stream) {
  if (!ctx) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context");
  int rc = check_attn_desc(ctx, a, "rrr_attention_f16kv");
  if (rc) return rc;
  if ((rc = check_rows(ctx, a, rows, pos0, d_pos, "rrr_attention_f16kv"))) return rc;
  if (!q || !k_cache || !v_cache || !out)
    return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_attention_f16kv: null pointer");
  if (q_stride < (int64_t)a->n_heads * a->head_dim)
    return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_attention_f16kv: q_stride < n_heads * head_dim");
  if (!aligned16(k_cache) || !aligned16(v_cache))
    return set_error(ctx, RRR_ERR_MISALIGNED, "rrr_attention_f16kv: caches must be 16-byte aligned");
  const int seq_max = d_pos ? a->max_seq : pos0 + rows;
  if (attention_smem_for(a->head_dim, a->n_heads / a->n_kv_heads, seq_max > 0 ? seq_max : 1) >
      227 * 1024)
    return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_attention_f16kv: max_seq too large for one cluster");
  if ((rc = bind_device(ctx))) return rc;
  if (rows == 0) return RRR_OK;
  cudaError_t e = launch_attention_f16kv(make_env(ctx, stream), q, q_stride, rows, pos0, d_pos, k_cache,
                                         v_cache, out, a->n_heads, a->n_kv_heads, a->head_dim,
                                         a->max_seq, seq_max, nullptr);
  return e == cudaSuccess ? RRR_OK : cuda_error(ctx, e, "rrr_attention_f16kv launch");
}

int rrr_rope_attention_f16kv(rrr_ctx* ctx, const rrr_attn_desc* a, const float* qkv, int pos0,
                             const int* d_pos, uint16_t* k_cache, uint16_t* v_cache, float* out,
                             void* stream) {
  if (!ctx) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context");
  int rc = check_attn_desc(ctx, a, "rrr_rope_attention_f16kv");
  if (rc) return rc;
  if ((rc = check_rows(ctx, a, 1, pos0, d_pos, "rrr_rope_attention_f16kv"))) return rc;
  if (!qkv || !k_cache || !v_cache || !out)
    return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_rope_attention_f16kv: null pointer");
  if (!aligned16(k_cache) || !aligned16(v_cache))
    return set_error(ctx, RRR_ERR_MISALIGNED, "rrr_rope_attention_f16kv: caches must be 16-byte aligned");
  const int seq_max = d_pos ? a->max_seq : pos0 + 1;
  if (attention_smem_for(a->head_dim, a->n_heads / a->n_kv_heads, seq_max) > 227 * 1024)
    return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_rope_attention_f16kv: max_seq too large for one cluster");
  if ((rc = bind_device(ctx))) return rc;
  const AttnRope rope{a->rope_dim, a->rope_theta, a->rope_attn_factor, a->rope_factors,
                      a->n_rope_factors};
  const int64_t qkv_dim = (int64_t)(a->n_heads + 2 * a->n_kv_heads) * a->head_dim;
  cudaError_t e = launch_attention_f16kv(make_env(ctx, stream), qkv, qkv_dim, 1, pos0, d_pos, k_cache,
                                         v_cache, out, a->n_heads, a->n_kv_heads, a->head_dim,
                                         a->max_seq, seq_max, &rope);
  return e == cudaSuccess ? RRR_OK : cuda_error(ctx, e, "rrr_rope_attention_f16kv launch");
}

int rrr_position_advance(rrr_ctx* ctx, int* d_pos, int delta, void* stream) {
  if (!ctx) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context");
  if (!d_pos) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_position_advance: null position");
  int rc = bind_device(ctx);
  if (rc) return rc;
  cudaError_t e = launch_pos_advance(make_env(ctx, stream), d_pos, delta);
  return e == cudaSuccess ? RRR_OK : cuda_error(ctx, e, "rrr_position_advance launch");
}

int rrr_embed_rows(rrr_ctx* ctx, int ggml_type, const void* table, int64_t n_rows, int d,
                   const int32_t* tokens, int n_tokens, float* out, void* stream) {
  if (!ctx) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context");
  if (!table || !tokens || !out) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_embed_rows: null pointer");
  int64_t row_bytes;
  switch (ggml_type) {
    case 0: row_bytes = 4ll * d; break;
    case 1: row_bytes = 2ll * d; break;
    case 6: row_bytes = d % 32 ? -1 : (int64_t)(d / 32) * 22; break;
    case 8: row_bytes = d % 32 ? -1 : (int64_t)(d / 32) * 34; break;
    case RRR_Q4_K: case RRR_Q5_K: case RRR_Q6_K:
      row_bytes = d % 256 ? -1 : (int64_t)(d / 256) * kq_block_bytes(ggml_type);
      break;
    default:
      return set_error(ctx, RRR_ERR_BAD_QTYPE, "rrr_embed_rows: type %d is not one of 0, 1, 6, 8, 12, 13, 14",
                       ggml_type);
  }
  if (d < 1 || n_rows < 1 || n_tokens < 0 || row_bytes < 0)
    return set_error(ctx, RRR_ERR_BAD_SHAPE,
                     "rrr_embed_rows: d must be a multiple of the type's block (32 or 256 values)");
  if ((ggml_type == 0 && (reinterpret_cast<uintptr_t>(table) & 3)) ||
      (ggml_type == 1 && (reinterpret_cast<uintptr_t>(table) & 1)))
    return set_error(ctx, RRR_ERR_MISALIGNED, "rrr_embed_rows: table misaligned for its element type");
  int rc = bind_device(ctx);
  if (rc) return rc;
  if (n_tokens == 0) return RRR_OK;
  cudaError_t e = launch_embed_rows(make_env(ctx, stream), ggml_type, table, n_rows, row_bytes, d,
                                    tokens, n_tokens, out);
  return e == cudaSuccess ? RRR_OK : cuda_error(ctx, e, "rrr_embed_rows launch");
}

}  // extern "C"
