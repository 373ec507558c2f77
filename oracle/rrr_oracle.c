/*
 * rrr_oracle.c — CPU restatement of RRR's weight-path arithmetic (TEST INFRASTRUCTURE
 * ONLY; see rrr_oracle.h). Every function cites the reference line it restates
 * (Peterc3-dev/recursive-routing-racer-rs). Build with -O2 -ffp-contract=off, no
 * -ffast-math: each float operation below is one IEEE binary32 operation, in the
 * reference's evaluation order.
 */
#include "rrr_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

/* half 2.7.1 `f16::to_f32` (phi4.rs:442): exact widening; NaN keeps its payload with
 * the quiet bit set. */
float rrro_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0x1F) {
    bits = man ? (sign | 0x7FC00000u | (man << 13)) : (sign | 0x7F800000u);
  } else if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do { man <<= 1; e++; } while ((man & 0x400u) == 0);
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13);
    }
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

uint16_t rrro_f32_to_f16_rne(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t exp = (x >> 23) & 0xFFu;
  uint32_t man = x & 0x7FFFFFu;
  if (exp == 0xFF) return (uint16_t)(sign | 0x7C00u | (man ? (0x200u | (man >> 13)) : 0));
  int e = (int)exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7C00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    int shift = 14 - e;
    uint32_t m = man >> shift, rem = man & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (m & 1u))) m++;
    return (uint16_t)(sign | m);
  }
  uint32_t m = man >> 13, rem = man & 0x1FFFu;
  uint32_t h = sign | ((uint32_t)e << 10) | m;
  if (rem > 0x1000u || (rem == 0x1000u && (m & 1u))) h++;
  return (uint16_t)h;
}

/* gguf.rs:173-195 */
int rrro_block_bytes(int t) {
  switch (t) {
    case 0: return 4; case 1: return 2; case 2: return 18; case 3: return 20;
    case 6: return 22; case 7: return 24; case 8: return 34; case 9: return 36;
    case 12: return 144; case 13: return 176; case 14: return 210;
    default: return -1;
  }
}
int rrro_block_elems(int t) {
  switch (t) {
    case 0: case 1: return 1;
    case 2: case 3: case 6: case 7: case 8: case 9: return 32;
    case 12: case 13: case 14: return 256;
    default: return -1;
  }
}

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* dequant_q6_k, phi4.rs:444-479. out = (d * scale) * q, scale index is = g*8 + l/16
 * (phi4.rs:463, the README's bug #8 fix). */
void rrro_dequant_q6_k(const uint8_t* data, int64_t n_elements, float* out) {
  int64_t n_blocks = n_elements / 256;
  for (int64_t bi = 0; bi < n_blocks; ++bi) {
    const uint8_t* b = data + bi * 210;
    const uint8_t* ql = b;
    const uint8_t* qh = b + 128;
    const int8_t* scales = (const int8_t*)(b + 192);
    float d = rrro_f16_to_f32(rd16(b + 208));
    float* o = out + bi * 256;
    for (int g = 0; g < 2; ++g) {
      for (int l = 0; l < 32; ++l) {
        uint8_t ql_lo = ql[g * 64 + l], ql_hi = ql[g * 64 + l + 32], qh_b = qh[g * 32 + l];
        int is = g * 8 + l / 16;
        int q1 = (int)((ql_lo & 0x0F) | (((qh_b >> 0) & 3) << 4)) - 32;
        int q2 = (int)((ql_hi & 0x0F) | (((qh_b >> 2) & 3) << 4)) - 32;
        int q3 = (int)((ql_lo >> 4) | (((qh_b >> 4) & 3) << 4)) - 32;
        int q4 = (int)((ql_hi >> 4) | (((qh_b >> 6) & 3) << 4)) - 32;
        float* p = o + g * 128;
        p[l] = d * (float)scales[is] * (float)q1;
        p[l + 32] = d * (float)scales[is + 2] * (float)q2;
        p[l + 64] = d * (float)scales[is + 4] * (float)q3;
        p[l + 96] = d * (float)scales[is + 6] * (float)q4;
      }
    }
  }
}

/* 6-bit scale/min unpack shared by Q4_K and Q5_K, phi4.rs:492-498 / 522-528. */
static inline void scale_min_k4(const uint8_t* sc, int sub, uint32_t* sv, uint32_t* mv) {
  if (sub < 4) {
    *sv = sc[sub] & 0x3Fu;
    *mv = sc[sub + 4] & 0x3Fu;
  } else {
    int i = sub - 4;
    *sv = (sc[8 + i] & 0x0Fu) | ((uint32_t)(sc[i] >> 6) << 4);
    *mv = (uint32_t)(sc[8 + i] >> 4) | ((uint32_t)(sc[4 + i] >> 6) << 4);
  }
}

/* dequant_q4_k, phi4.rs:481-510: out = q * (d*sv) - (dmin*mv). */
void rrro_dequant_q4_k(const uint8_t* data, int64_t n_elements, float* out) {
  int64_t n_blocks = n_elements / 256;
  for (int64_t bi = 0; bi < n_blocks; ++bi) {
    const uint8_t* b = data + bi * 144;
    float d = rrro_f16_to_f32(rd16(b)), dmin = rrro_f16_to_f32(rd16(b + 2));
    const uint8_t* sc = b + 4;
    const uint8_t* qs = b + 16;
    float* o = out + bi * 256;
    for (int sub = 0; sub < 8; ++sub) {
      uint32_t sv, mv;
      scale_min_k4(sc, sub, &sv, &mv);
      float s = d * (float)sv, m = dmin * (float)mv;
      int pair = sub / 2;
      for (int j = 0; j < 32; ++j) {
        uint8_t qb = qs[pair * 32 + j];
        uint32_t qi = (sub % 2 == 0) ? (qb & 0xFu) : ((qb >> 4) & 0xFu);
        o[sub * 32 + j] = (float)qi * s - m;
      }
    }
  }
}

/* dequant_q5_k, phi4.rs:512-542: 5-bit q = nibble | ((qh[j] >> sub) & 1) << 4. */
void rrro_dequant_q5_k(const uint8_t* data, int64_t n_elements, float* out) {
  int64_t n_blocks = n_elements / 256;
  for (int64_t bi = 0; bi < n_blocks; ++bi) {
    const uint8_t* b = data + bi * 176;
    float d = rrro_f16_to_f32(rd16(b)), dmin = rrro_f16_to_f32(rd16(b + 2));
    const uint8_t* sc = b + 4;
    const uint8_t* qh = b + 16;
    const uint8_t* qs = b + 48;
    float* o = out + bi * 256;
    for (int sub = 0; sub < 8; ++sub) {
      uint32_t sv, mv;
      scale_min_k4(sc, sub, &sv, &mv);
      float s = d * (float)sv, m = dmin * (float)mv;
      int pair = sub / 2;
      for (int j = 0; j < 32; ++j) {
        uint8_t qb = qs[pair * 32 + j];
        uint32_t lo = (sub % 2 == 0) ? (qb & 0xFu) : ((qb >> 4) & 0xFu);
        uint32_t hb = (qh[j] >> sub) & 1u;
        uint32_t qi = lo | (hb << 4);
        o[sub * 32 + j] = (float)qi * s - m;
      }
    }
  }
}

/* dequant_q8_0, phi4.rs:544-553 */
void rrro_dequant_q8_0(const uint8_t* data, int64_t n_elements, float* out) {
  int64_t n_blocks = n_elements / 32;
  for (int64_t bi = 0; bi < n_blocks; ++bi) {
    const uint8_t* b = data + bi * 34;
    float d = rrro_f16_to_f32(rd16(b));
    for (int j = 0; j < 32; ++j) out[bi * 32 + j] = d * (float)(int8_t)b[2 + j];
  }
}

/* dequant_q5_0, phi4.rs:555-570 */
void rrro_dequant_q5_0(const uint8_t* data, int64_t n_elements, float* out) {
  int64_t n_blocks = n_elements / 32;
  for (int64_t bi = 0; bi < n_blocks; ++bi) {
    const uint8_t* b = data + bi * 22;
    float d = rrro_f16_to_f32(rd16(b));
    uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) |
                  ((uint32_t)b[5] << 24);
    for (int j = 0; j < 32; ++j) {
      uint32_t lo = j < 16 ? (b[6 + j] & 0xFu) : ((b[6 + j - 16] >> 4) & 0xFu);
      uint32_t hb = (qh >> j) & 1u;
      int qi = (int)(lo | (hb << 4)) - 16;
      out[bi * 32 + j] = d * (float)qi;
    }
  }
}

/* dequant_tensor_f32, phi4.rs:572-587 */
int rrro_dequant(int t, const uint8_t* data, int64_t n, float* out) {
  switch (t) {
    case 0: memcpy(out, data, (size_t)n * 4); return 0;
    case 1:
      for (int64_t i = 0; i < n; ++i) out[i] = rrro_f16_to_f32(rd16(data + 2 * i));
      return 0;
    case 6: rrro_dequant_q5_0(data, n, out); return 0;
    case 8: rrro_dequant_q8_0(data, n, out); return 0;
    case 12: rrro_dequant_q4_k(data, n, out); return 0;
    case 13: rrro_dequant_q5_k(data, n, out); return 0;
    case 14: rrro_dequant_q6_k(data, n, out); return 0;
    default: return -1;
  }
}

/* rms_norm, phi4.rs:593-599: sequential sum of squares; out = w * x * inv. */
void rrro_rms_norm(const float* x, const float* w, float* out, int n, float eps) {
  float sum_sq = 0.0f;
  for (int i = 0; i < n; ++i) sum_sq += x[i] * x[i];
  float inv_rms = 1.0f / sqrtf(sum_sq / (float)n + eps);
  for (int i = 0; i < n; ++i) out[i] = w[i] * x[i] * inv_rms;
}

/* cpu_silu, phi4.rs:601-606 */
void rrro_silu(float* x, int n) {
  for (int i = 0; i < n; ++i) x[i] = x[i] / (1.0f + expf(-x[i]));
}

/* SiLU(gate) * up, phi4.rs:1368-1373 */
void rrro_silu_gate(const float* gu, float* out, int F) {
  for (int i = 0; i < F; ++i) {
    float gate = gu[i];
    float silu = gate / (1.0f + expf(-gate));
    out[i] = silu * gu[F + i];
  }
}

/* elemwise_add, phi4.rs:608-610 */
void rrro_add(const float* a, const float* b, float* out, int n) {
  for (int i = 0; i < n; ++i) out[i] = a[i] + b[i];
}

/* ------------------------------------------------------------------ threading */
typedef struct job {
  int kind; /* 0 gemv_f32, 1 gemv_kq rows, 2 dequant rows, 3 dot rows */
  int qtype;
  const uint8_t* raw;
  const float* W;
  const float* x;
  float* y;
  float* scratch;
  int64_t K, r0, r1;
} job;

static void dequant_rows(int qtype, const uint8_t* raw, int64_t K, int64_t r0, int64_t r1,
                         float* out /* [(r1-r0)*K] */) {
  int64_t nb = K / 256, bb = rrro_block_bytes(qtype);
  const uint8_t* src = raw + r0 * nb * bb;
  rrro_dequant(qtype, src, (r1 - r0) * K, out);
}

static void* job_run(void* arg) {
  job* j = (job*)arg;
  if (j->kind == 0 || j->kind == 3) {
    const float* W = j->kind == 0 ? j->W : j->scratch;
    for (int64_t r = j->r0; r < j->r1; ++r) {
      const float* row = W + r * j->K;
      float acc = 0.0f;
      for (int64_t k = 0; k < j->K; ++k) acc += row[k] * j->x[k];
      j->y[r] = acc;
    }
  } else if (j->kind == 1) {
    float* buf = (float*)malloc((size_t)j->K * sizeof(float));
    for (int64_t r = j->r0; r < j->r1; ++r) {
      dequant_rows(j->qtype, j->raw, j->K, r, r + 1, buf);
      float acc = 0.0f;
      for (int64_t k = 0; k < j->K; ++k) acc += buf[k] * j->x[k];
      j->y[r] = acc;
    }
    free(buf);
  } else if (j->kind == 2) {
    dequant_rows(j->qtype, j->raw, j->K, j->r0, j->r1, j->scratch + j->r0 * j->K);
  }
  return NULL;
}

static void run_parallel(job proto, int64_t N, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  if ((int64_t)threads > N) threads = (int)(N > 0 ? N : 1);
  pthread_t tid[256];
  job jobs[256];
  int64_t per = (N + threads - 1) / threads;
  int started = 0;
  for (int t = 0; t < threads; ++t) {
    jobs[t] = proto;
    jobs[t].r0 = t * per;
    jobs[t].r1 = (t + 1) * per < N ? (t + 1) * per : N;
    if (jobs[t].r0 >= jobs[t].r1) break;
    if (threads == 1) {
      job_run(&jobs[t]);
    } else {
      pthread_create(&tid[t], NULL, job_run, &jobs[t]);
      started++;
    }
  }
  for (int t = 0; t < started; ++t) pthread_join(tid[t], NULL);
}

void rrro_gemv_f32(const float* W, const float* x, float* y, int64_t N, int64_t K,
                   int threads) {
  job p;
  memset(&p, 0, sizeof p);
  p.kind = 0; p.W = W; p.x = x; p.y = y; p.K = K;
  run_parallel(p, N, threads);
}

void rrro_matmul_f32(const float* A, const float* B, float* C, int M, int K, int N) {
  for (int m = 0; m < M; ++m)
    for (int n = 0; n < N; ++n) {
      float acc = 0.0f;
      for (int k = 0; k < K; ++k) acc += A[(int64_t)m * K + k] * B[(int64_t)k * N + n];
      C[(int64_t)m * N + n] = acc;
    }
}

static int kq_ok(int qtype, int64_t K) {
  return (qtype == 12 || qtype == 13 || qtype == 14) && K > 0 && K % 256 == 0;
}

int rrro_gemv_kq(int qtype, const uint8_t* raw, const float* x, float* y, int64_t K,
                 int64_t N, int threads) {
  if (!kq_ok(qtype, K) || N < 0) return -1;
  job p;
  memset(&p, 0, sizeof p);
  p.kind = 1; p.qtype = qtype; p.raw = raw; p.x = x; p.y = y; p.K = K;
  run_parallel(p, N, threads);
  return 0;
}

static double now_s(void) {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return ts.tv_sec + 1e-9 * ts.tv_nsec;
}

int rrro_gemv_kq_baseline(int qtype, const uint8_t* raw, const float* x, float* y,
                          int64_t K, int64_t N, int threads, float* scratch,
                          double* t_dequant, double* t_dot) {
  if (!kq_ok(qtype, K) || N < 0 || !scratch) return -1;
  job p;
  memset(&p, 0, sizeof p);
  p.qtype = qtype; p.raw = raw; p.x = x; p.y = y; p.K = K; p.scratch = scratch;
  double t0 = now_s();
  p.kind = 2;
  run_parallel(p, N, threads);
  double t1 = now_s();
  p.kind = 3;
  run_parallel(p, N, threads);
  double t2 = now_s();
  if (t_dequant) *t_dequant = t1 - t0;
  if (t_dot) *t_dot = t2 - t1;
  return 0;
}

/* ------------------------------------------------------------------ generator */
static inline uint64_t splitmix64(uint64_t* s) {
  uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

/* f16 bits of a value uniform in [1e-4, 1e-2]: lo + u*step with u a 24-bit integer. */
static inline uint16_t gen_scale_f16(uint64_t r) {
  const float lo = 0x1.a36e2ep-14f;   /* 1e-4f */
  const float step = 0x1.446738p-31f; /* (1e-2f - 1e-4f) / 2^24 */
  float u = (float)(uint32_t)(r >> 40);
  float v = lo + u * step;
  return rrro_f32_to_f16_rne(v);
}

void rrro_fill_kquant_random(int qtype, uint8_t* dst, int64_t block0, int64_t n_blocks,
                             uint64_t seed) {
  int bb = rrro_block_bytes(qtype);
  for (int64_t i = 0; i < n_blocks; ++i) {
    uint64_t blk = (uint64_t)(block0 + i);
    uint64_t s = seed ^ (blk * 0xD1B54A32D192ED03ull);
    uint8_t* b = dst + i * bb;
    for (int o = 0; o < bb; o += 8) {
      uint64_t r = splitmix64(&s);
      for (int k = 0; k < 8 && o + k < bb; ++k) b[o + k] = (uint8_t)(r >> (8 * k));
    }
    if (qtype == 14) {
      for (int k = 0; k < 16; ++k) b[192 + k] = (uint8_t)(int8_t)((int)(b[192 + k] & 63) - 32);
      uint16_t d = gen_scale_f16(splitmix64(&s));
      b[208] = (uint8_t)d; b[209] = (uint8_t)(d >> 8);
    } else {
      uint16_t d = gen_scale_f16(splitmix64(&s));
      uint16_t dm = gen_scale_f16(splitmix64(&s));
      b[0] = (uint8_t)d; b[1] = (uint8_t)(d >> 8);
      b[2] = (uint8_t)dm; b[3] = (uint8_t)(dm >> 8);
    }
  }
}

/* ------------------------------------------------------------------ decode step */
/* Position-0 decode step (phi4.rs:1006-1064 with seq_len 1): the attention output of
 * Q head h is V of KV head h / (n_heads / n_kv_heads) (push layout phi4.rs:1120). */
int rrro_decode_step(int d, int nh, int nkv, int hd, int ffn, int nl, int vocab, float eps,
                     const rrro_layer* L, const float* out_norm, const float* w_out,
                     float* h, float* logits, int threads) {
  if (d <= 0 || nh <= 0 || nkv <= 0 || nh % nkv || hd <= 0 || nh * hd != d) return -1;
  int qkv_dim = nh * hd + 2 * nkv * hd;
  float* normed = (float*)malloc(sizeof(float) * (size_t)d);
  float* qkv = (float*)malloc(sizeof(float) * (size_t)qkv_dim);
  float* attn = (float*)malloc(sizeof(float) * (size_t)d);
  float* tmp = (float*)malloc(sizeof(float) * (size_t)d);
  float* gu = (float*)malloc(sizeof(float) * (size_t)2 * ffn);
  float* mid = (float*)malloc(sizeof(float) * (size_t)ffn);
  int hpk = nh / nkv;
  for (int l = 0; l < nl; ++l) {
    rrro_rms_norm(h, L[l].attn_norm, normed, d, eps);
    rrro_gemv_kq(L[l].qkv_type, L[l].w_qkv, normed, qkv, d, qkv_dim, threads);
    const float* v = qkv + nh * hd + nkv * hd;
    for (int q = 0; q < nh; ++q)
      for (int e = 0; e < hd; ++e) attn[q * hd + e] = v[(q / hpk) * hd + e];
    rrro_gemv_kq(L[l].o_type, L[l].w_o, attn, tmp, d, d, threads);
    rrro_add(h, tmp, h, d);
    rrro_rms_norm(h, L[l].ffn_norm, normed, d, eps);
    rrro_gemv_kq(L[l].gate_up_type, L[l].w_gate_up, normed, gu, d, 2 * ffn, threads);
    rrro_silu_gate(gu, mid, ffn);
    rrro_gemv_kq(L[l].down_type, L[l].w_down, mid, tmp, ffn, d, threads);
    rrro_add(h, tmp, h, d);
  }
  rrro_rms_norm(h, out_norm, normed, d, eps);
  rrro_gemv_f32(w_out, normed, logits, vocab, d, threads);
  free(normed); free(qkv); free(attn); free(tmp); free(gu); free(mid);
  return 0;
}

/* ---------------------------------------------------------------- RoPE / KV / attention */
void rrro_rope(float* x, int pos, int n_heads, int head_dim, int rope_dim, float theta,
               float attn_factor, const float* factors, int n_factors) {
  for (int h = 0; h < n_heads; ++h) {
    const int base = h * head_dim;
    for (int i = 0; i < rope_dim / 2; ++i) {
      const float base_freq = 1.0f / powf(theta, (2.0f * (float)i) / (float)rope_dim);
      const float factor = i < n_factors ? factors[i] : 1.0f;
      const float freq = base_freq / factor;
      const float angle = (float)pos * freq;
      const float sin_t = sinf(angle), cos_t = cosf(angle);
      const float cs = cos_t * attn_factor, ss = sin_t * attn_factor;
      const float x0 = x[base + 2 * i], x1 = x[base + 2 * i + 1];
      x[base + 2 * i] = x0 * cs - x1 * ss;
      x[base + 2 * i + 1] = x0 * ss + x1 * cs;
    }
  }
}

void rrro_kv_store(const float* k, const float* v, uint16_t* k_cache, uint16_t* v_cache,
                   int pos, int kv_stride) {
  for (int i = 0; i < kv_stride; ++i) {
    k_cache[(size_t)pos * kv_stride + i] = rrro_f32_to_f16_rne(k[i]);
    v_cache[(size_t)pos * kv_stride + i] = rrro_f32_to_f16_rne(v[i]);
  }
}

void rrro_attention_f16kv(const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                          float* out, int seq_len, int n_heads, int n_kv_heads, int head_dim) {
  const int hpk = n_heads / n_kv_heads, kv_stride = n_kv_heads * head_dim;
  double* s = (double*)malloc(sizeof(double) * (size_t)(seq_len > 0 ? seq_len : 1));
  double* acc = (double*)malloc(sizeof(double) * (size_t)head_dim);
  const double scale = 1.0 / sqrt((double)head_dim);
  for (int h = 0; h < n_heads; ++h) {
    const int g = h / hpk;
    const float* qh = q + (size_t)h * head_dim;
    double m = -INFINITY;
    for (int t = 0; t < seq_len; ++t) {
      const uint16_t* kr = k_cache + (size_t)t * kv_stride + (size_t)g * head_dim;
      double dot = 0.0;
      for (int e = 0; e < head_dim; ++e) dot += (double)qh[e] * (double)rrro_f16_to_f32(kr[e]);
      s[t] = dot * scale;
      if (s[t] > m) m = s[t];
    }
    double l = 0.0;
    for (int e = 0; e < head_dim; ++e) acc[e] = 0.0;
    for (int t = 0; t < seq_len; ++t) {
      const double p = exp(s[t] - m);
      l += p;
      const uint16_t* vr = v_cache + (size_t)t * kv_stride + (size_t)g * head_dim;
      for (int e = 0; e < head_dim; ++e) acc[e] += p * (double)rrro_f16_to_f32(vr[e]);
    }
    for (int e = 0; e < head_dim; ++e) out[(size_t)h * head_dim + e] = (float)(acc[e] / l);
  }
  free(s);
  free(acc);
}

int rrro_decode_step_kv(int d, int nh, int nkv, int hd, int ffn, int nl, int vocab, float eps,
                        int rope_dim, float theta, float attn_factor, const float* factors,
                        int n_factors, int pos, int max_seq, uint16_t* k_caches,
                        uint16_t* v_caches, const rrro_layer* L, const float* out_norm,
                        const float* w_out, float* h, float* logits, int threads) {
  if (d <= 0 || nh <= 0 || nkv <= 0 || nh % nkv || hd <= 0 || nh * hd != d || pos < 0 ||
      pos >= max_seq || rope_dim < 0 || rope_dim > hd || rope_dim % 2)
    return -1;
  const int qkv_dim = nh * hd + 2 * nkv * hd, kv_stride = nkv * hd;
  float* normed = (float*)malloc(sizeof(float) * (size_t)d);
  float* qkv = (float*)malloc(sizeof(float) * (size_t)qkv_dim);
  float* attn = (float*)malloc(sizeof(float) * (size_t)d);
  float* tmp = (float*)malloc(sizeof(float) * (size_t)d);
  float* gu = (float*)malloc(sizeof(float) * (size_t)2 * ffn);
  float* mid = (float*)malloc(sizeof(float) * (size_t)ffn);
  for (int l = 0; l < nl; ++l) {
    uint16_t* kc = k_caches + (size_t)l * max_seq * kv_stride;
    uint16_t* vc = v_caches + (size_t)l * max_seq * kv_stride;
    rrro_rms_norm(h, L[l].attn_norm, normed, d, eps);
    rrro_gemv_kq(L[l].qkv_type, L[l].w_qkv, normed, qkv, d, qkv_dim, threads);
    float* q = qkv;
    float* k = qkv + nh * hd;
    float* v = k + kv_stride;
    rrro_rope(q, pos, nh, hd, rope_dim, theta, attn_factor, factors, n_factors);
    rrro_rope(k, pos, nkv, hd, rope_dim, theta, attn_factor, factors, n_factors);
    rrro_kv_store(k, v, kc, vc, pos, kv_stride);
    rrro_attention_f16kv(q, kc, vc, attn, pos + 1, nh, nkv, hd);
    rrro_gemv_kq(L[l].o_type, L[l].w_o, attn, tmp, d, d, threads);
    rrro_add(h, tmp, h, d);
    rrro_rms_norm(h, L[l].ffn_norm, normed, d, eps);
    rrro_gemv_kq(L[l].gate_up_type, L[l].w_gate_up, normed, gu, d, 2 * ffn, threads);
    rrro_silu_gate(gu, mid, ffn);
    rrro_gemv_kq(L[l].down_type, L[l].w_down, mid, tmp, ffn, d, threads);
    rrro_add(h, tmp, h, d);
  }
  rrro_rms_norm(h, out_norm, normed, d, eps);
  rrro_gemv_f32(w_out, normed, logits, vocab, d, threads);
  free(normed); free(qkv); free(attn); free(tmp); free(gu); free(mid);
  return 0;
}
