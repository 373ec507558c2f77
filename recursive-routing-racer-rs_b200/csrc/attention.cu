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
__device__ __forceinline__ void rope_cs(int pos, float base_freq, float factor, float attn_factor,
                                        float& cs, float& ss) {
  const float freq = __fdiv_rn(base_freq, factor);
  const float angle = __fmul_rn((float)pos, freq);
  float s, c;
  sincosf(angle, &s, &c);
  cs = __fmul_rn(c, attn_factor);
  ss = __fmul_rn(s, attn_factor);
}
__device__ __forceinline__ void rope_apply(float& x0, float& x1, float cs, float ss) {
  const float y0 = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, ss));
  const float y1 = __fadd_rn(__fmul_rn(x0, ss), __fmul_rn(x1, cs));
  x0 = y0;
  x1 = y1;
}
__device__ __forceinline__ void rope_pair(float& x0, float& x1, int pos, float base_freq,
                                          float factor, float attn_factor) {
  float cs, ss;
  rope_cs(pos, base_freq, factor, attn_factor, cs, ss);
  rope_apply(x0, x1, cs, ss);
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

__device__ __forceinline__ void st_dsmem_f32(float* local, uint32_t rank, float v) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_addr(local)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(v) : "memory");
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

// The CTA's positions are processed in tiles of 8192 / head_dim rows (64 for 128): the K and
// V rows of a tile (head g) are copied into shared memory with 16-byte cp.async,
// double-buffered so that the next tile streams in while this one is computed. The first
// tile is requested as soon as the position is known, before the query is read.
//
// Every warp runs its own online softmax over the tile's rows (R = 32 / HB rows per warp
// step, HB >= the query heads per KV head): lane l holds dims D*l .. D*l + D - 1 of the
// query heads (in registers, RoPE applied) and of its accumulators. A step's HB*R partial
// dot products are reduced with one 31-shuffle transpose, after which lane i holds the score
// of (head i / R, row i % R); each lane then takes one exponential, and the probabilities
// are broadcast for the weighted V rows. No CTA barrier is taken inside a tile. At the end
// the warps' partials are merged in warp order through shared memory, and the CTAs of the
// cluster over distributed shared memory in split order.
//
// Shared memory: K [2][kTile][HD] f16 | V [2][kTile][HD] f16 | warp max, sum, merge weight
// [NW][HB] each | warp accumulators [NW][hpk][HD] | CTA accumulator [hpk][HD] | CTA max,
// sum [HB] | new K, V row [2][HD] f16 | received split maxima, sums [kMaxSplits][HB] each |
// received accumulators [kMaxSplits][share].
template <int HD>
constexpr int attn_tile() { return 8192 / HD; }  // K + V double buffer = 64 KB

template <int HD, int HB>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(16) uint8_t smraw[];
  constexpr int NW = kAttnThreads / 32;
  constexpr int D = HD / 32;  // dims per lane
  constexpr int CH = HD / 8;  // 16-byte chunks per row
  constexpr int R = 32 / HB;  // rows per warp step
  constexpr int kTile = attn_tile<HD>();
  const int hpk = p.hpk;  // <= HB
  __half* kt = reinterpret_cast<__half*>(smraw);
  __half* vt = kt + 2 * kTile * HD;
  float* wm = reinterpret_cast<float*>(vt + 2 * kTile * HD);
  float* wl = wm + NW * HB;
  float* ww = wl + NW * HB;
  float* wacc = ww + NW * HB;
  float* pacc = wacc + NW * hpk * HD;
  float* pmax = pacc + hpk * HD;
  float* psum = pmax + HB;
  __half* knew = reinterpret_cast<__half*>(psum + HB);
  __half* vnew = knew + HD;
  float* rm = reinterpret_cast<float*>(vnew + HD);  // [kMaxSplits][HB]
  float* rl = rm + kMaxSplits * HB;                 // [kMaxSplits][HB]
  float* racc = rl + kMaxSplits * HB;               // [kMaxSplits][share]

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
  // the query heads of KV head g, this lane's dims (loads in flight while the first tile's
  // copies are issued), then rotated (RoPE of the fused one-token path)
  const float* qrow = p.q + (long long)row * p.q_stride;
  float q[HB][D];
#pragma unroll
  for (int j = 0; j < HB; ++j)
#pragma unroll
    for (int d = 0; d < D; ++d) q[j][d] = j < hpk ? qrow[(long long)(g * hpk + j) * HD + D * lane + d] : 0.f;
  if (n_tiles > 0) issue(0);
  if (p.fused && pos_ok) {
#pragma unroll
    for (int pp = 0; pp < D / 2; ++pp) {
      const int pair = (D * lane) / 2 + pp;
      if (pair < p.rope_pairs) {
        float cs, ss;
        rope_cs(pos, p.base_freq[pair], pair < p.n_factors ? p.factors[pair] : 1.0f, p.attn_factor, cs, ss);
#pragma unroll
        for (int j = 0; j < HB; ++j)
          if (j < hpk) rope_apply(q[j][2 * pp], q[j][2 * pp + 1], cs, ss);
      }
    }
  }
  // the CTA whose positions end at `pos` stores the token's K (rotated) and V row of KV
  // head g into the caches and keeps them for its last tile (the bulk reads skip that row)
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
    __syncthreads();  // (own_new is uniform over the CTA)
  }

  float m[HB], l[HB], acc[HB][D];
#pragma unroll
  for (int j = 0; j < HB; ++j) {
    m[j] = -INFINITY;
    l[j] = 0.f;
#pragma unroll
    for (int d = 0; d < D; ++d) acc[j][d] = 0.f;
  }
  const int my_j = lane / R, my_r = lane % R;  // the (head, row) this lane scores after the transpose

  for (int tile = 0; tile < n_tiles; ++tile) {
    if (tile + 1 < n_tiles) {
      __syncthreads();  // every warp is done with the buffer the next tile overwrites
      issue(tile + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    const int base = t0 + tile * kTile, nrows = min(kTile, t1 - base);
    __half* kb = kt + (tile & 1) * kTile * HD;
    __half* vb = vt + (tile & 1) * kTile * HD;
    if (own_new && tile == n_tiles - 1) {  // the new row is the last one of the CTA
      const int r = pos - base;
      for (int c = threadIdx.x; c < 2 * CH; c += kAttnThreads) {
        const int cc = c % CH;
        __half* dst = (c < CH ? kb : vb) + r * HD + cc * 8;
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>((c < CH ? knew : vnew) + cc * 8);
      }
    }
    __syncthreads();  // the tile (and the new row) is visible to every warp
    for (int r0 = warp * R; r0 < nrows; r0 += NW * R) {
      // partial dot products of this lane's dims: s[j*R + rr]
      float s[HB * R];
#pragma unroll
      for (int rr = 0; rr < R; ++rr) {
        const int r = r0 + rr;
        float kf[D];
        if (r < nrows) {
          const __half2* k2 = reinterpret_cast<const __half2*>(kb + r * HD + D * lane);
#pragma unroll
          for (int e = 0; e < D / 2; ++e) {
            const float2 f = __half22float2(k2[e]);
            kf[2 * e] = f.x;
            kf[2 * e + 1] = f.y;
          }
        } else {
#pragma unroll
          for (int e = 0; e < D; ++e) kf[e] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < HB; ++j) {
          float dot = 0.f;
          if (j < hpk) {
#pragma unroll
            for (int e = 0; e < D; ++e) dot = fmaf(q[j][e], kf[e], dot);
          }
          s[j * R + rr] = dot;
        }
      }
      // transpose reduction: afterwards s[0] of lane i is the full dot of (i / R, i % R)
#pragma unroll
      for (int o = 16, n = 32; o > 0; o >>= 1, n >>= 1) {
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
          const float send = up ? s[i] : s[i + n / 2];
          const float keep = up ? s[i + n / 2] : s[i];
          s[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      const bool valid = my_j < hpk && r0 + my_r < nrows;
      const float sc = valid ? s[0] * p.scale : -INFINITY;
      // the step's max per head over its R lanes, the new running max and the rescale
      float mx = sc;
#pragma unroll
      for (int o = R / 2; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float m_old = -INFINITY;
#pragma unroll
      for (int j = 0; j < HB; ++j)
        if (j == my_j) m_old = m[j];
      const float m_new = fmaxf(m_old, mx);
      const float pr = valid ? expf(sc - m_new) : 0.f;
      const float alpha = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
      float ps = pr;
#pragma unroll
      for (int o = R / 2; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      // every lane: the heads' rescale, running max and sum, then the weighted V rows
#pragma unroll
      for (int j = 0; j < HB; ++j) {
        if (j < hpk) {
          const float a = __shfl_sync(0xffffffffu, alpha, j * R);
          m[j] = __shfl_sync(0xffffffffu, m_new, j * R);
          l[j] = fmaf(l[j], a, __shfl_sync(0xffffffffu, ps, j * R));
#pragma unroll
          for (int d = 0; d < D; ++d) acc[j][d] *= a;
        }
      }
#pragma unroll
      for (int rr = 0; rr < R; ++rr) {
        const int r = r0 + rr;
        if (r < nrows) {
          float vf[D];
          const __half2* v2 = reinterpret_cast<const __half2*>(vb + r * HD + D * lane);
#pragma unroll
          for (int e = 0; e < D / 2; ++e) {
            const float2 f = __half22float2(v2[e]);
            vf[2 * e] = f.x;
            vf[2 * e + 1] = f.y;
          }
#pragma unroll
          for (int j = 0; j < HB; ++j) {
            if (j < hpk) {
              const float w = __shfl_sync(0xffffffffu, pr, j * R + rr);
#pragma unroll
              for (int d = 0; d < D; ++d) acc[j][d] = fmaf(w, vf[d], acc[j][d]);
            }
          }
        }
      }
    }
  }

  // ---- the warps' partials, merged in warp order into the CTA's (max, sum, accumulator)
#pragma unroll
  for (int j = 0; j < HB; ++j) {
    if (j < hpk) {
      if (lane == 0) {
        wm[warp * HB + j] = m[j];
        wl[warp * HB + j] = l[j];
      }
#pragma unroll
      for (int d = 0; d < D; ++d) wacc[(warp * hpk + j) * HD + D * lane + d] = acc[j][d];
    }
  }
  __syncthreads();
  // merge weights exp(m_w - M) of every (head, warp), one per thread
  if (threadIdx.x < hpk * NW) {
    const int j = threadIdx.x / NW, w = threadIdx.x % NW;
    float M = -INFINITY;
#pragma unroll
    for (int w2 = 0; w2 < NW; ++w2) M = fmaxf(M, wm[w2 * HB + j]);
    ww[w * HB + j] = wm[w * HB + j] == -INFINITY ? 0.f : expf(wm[w * HB + j] - M);
    if (w == 0) pmax[j] = M;
  }
  __syncthreads();
  if (threadIdx.x < hpk) {
    const int j = threadIdx.x;
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) L = fmaf(ww[w * HB + j], wl[w * HB + j], L);
    psum[j] = L;
  }
  for (int i = threadIdx.x; i < hpk * HD; i += kAttnThreads) {
    const int j = i / HD;
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) a = fmaf(ww[w * HB + j], wacc[w * hpk * HD + i], a);
    pacc[i] = a;
  }

  // ---- merge the splits' partials over distributed shared memory, in split order. Element
  // i of the hpk*HD outputs is merged by CTA i / share. Every CTA pushes its maxima and sums
  // to every CTA of the cluster and its accumulator elements to the CTA that merges them
  // (remote stores, no round trip); the cluster barrier publishes them, and the merge then
  // reads only its own shared memory. Nothing is read remotely after the barrier, so no
  // second barrier holds the CTAs.
  const int S = p.splits;
  const int tot = hpk * HD;
  const int share = (tot + S - 1) / S;
  __syncthreads();  // the CTA's partial is complete
  for (int t = threadIdx.x; t < S * hpk; t += kAttnThreads) {
    const int dst = t / hpk, j = t % hpk;
    st_dsmem_f32(rm + split * HB + j, (uint32_t)dst, pmax[j]);
    st_dsmem_f32(rl + split * HB + j, (uint32_t)dst, psum[j]);
  }
  for (int i = threadIdx.x; i < tot; i += kAttnThreads)
    st_dsmem_f32(racc + split * share + i % share, (uint32_t)(i / share), pacc[i]);
  cluster_barrier();
  if (pos_ok) {
    // weights exp(m_s - M) of every (head, split), the sums in split order, then this CTA's
    // elements (the warp accumulators are free again: they hold the weights)
    float* sw = wacc;               // [HB][kMaxSplits]
    float* sL = sw + HB * kMaxSplits;
    if (threadIdx.x < hpk * S) {
      const int j = threadIdx.x / S, s2 = threadIdx.x % S;
      float M = -INFINITY;
      for (int t = 0; t < S; ++t) M = fmaxf(M, rm[t * HB + j]);
      const float mv = rm[s2 * HB + j];
      sw[j * kMaxSplits + s2] = mv == -INFINITY ? 0.f : expf(mv - M);
    }
    __syncthreads();
    if (threadIdx.x < hpk) {
      const int j = threadIdx.x;
      float L = 0.f;
      for (int t = 0; t < S; ++t) L = fmaf(sw[j * kMaxSplits + t], rl[t * HB + j], L);
      sL[j] = L;
    }
    __syncthreads();
    const int i0 = split * share, i1 = min(tot, i0 + share);
    for (int i = i0 + threadIdx.x; i < i1; i += kAttnThreads) {
      const int j = i / HD;
      float o = 0.f;
      for (int t = 0; t < S; ++t) o = fmaf(sw[j * kMaxSplits + t], racc[t * share + (i - i0)], o);
      p.out[(long long)row * p.nh * HD + (long long)g * hpk * HD + i] = o / sL[j];
    }
  }
}

__global__ void pos_advance_kernel(int* d_pos, int delta) {
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x == 0) *d_pos += delta;
}

// Query heads per KV head the kernel variant is built for (registers per lane scale with it).
int attn_hb(int hpk) { return hpk <= 4 ? 4 : 8; }

int attn_smem_bytes(int hd, int hpk) {
  constexpr int NW = kAttnThreads / 32;
  const int hb = attn_hb(hpk);
  const int tile = 8192 / hd;
  return 2 * 2 * 2 * tile * hd + 4 * (3 * NW * hb + NW * hpk * hd + hpk * hd + 2 * hb) + 2 * 2 * hd +
         4 * (2 * kMaxSplits * hb + hpk * hd + kMaxSplits);
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
  if (p.hpk < 1 || p.hpk > kMaxHpk) return cudaErrorInvalidValue;
  const int smem = attn_smem_bytes(hd, p.hpk);
  const int hb = attn_hb(p.hpk);
  void (*kern)(AttnParams) = nullptr;
  int hi;
  switch (hd * 16 + hb) {
    case 64 * 16 + 4: kern = attention_kernel<64, 4>; hi = 0; break;
    case 64 * 16 + 8: kern = attention_kernel<64, 8>; hi = 1; break;
    case 128 * 16 + 4: kern = attention_kernel<128, 4>; hi = 2; break;
    case 128 * 16 + 8: kern = attention_kernel<128, 8>; hi = 3; break;
    case 256 * 16 + 4: kern = attention_kernel<256, 4>; hi = 4; break;
    case 256 * 16 + 8: kern = attention_kernel<256, 8>; hi = 5; break;
    default: return cudaErrorInvalidValue;
  }
  // Kernel attributes and the cluster-size check are done once per kernel and split count
  // (the largest shared-memory size, 8 query heads per KV head, covers every launch).
  static std::mutex mu;
  static int dev_ready[8][6] = {};           // per device: attributes set
  static int8_t fits[8][6][kMaxSplits + 1];  // per device: 0 unknown, 1 fits, -1 does not
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
