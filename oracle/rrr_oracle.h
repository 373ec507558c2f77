/*
 * rrr_oracle.h — CPU restatement of RRR's weight-path arithmetic. TEST INFRASTRUCTURE
 * ONLY: it is the checker for the CUDA kernels (tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py use it) and is never linked into the product library.
 *
 * Reference: Peterc3-dev/recursive-routing-racer-rs, src/model/phi4.rs. Compiled with
 * -ffp-contract=off (Rust never contracts a*b+c into an FMA), so every dequantised value
 * is bit-identical to the reference's CPU dequant. Parity pin: the reference is Rust and
 * cannot be built in this image (no rustc/cargo), so these functions are pinned against
 * gguf-py 0.19.0's independent dequantisers (tests/golden/make_golden.py writes the
 * fixtures) and hand-derived known-answer blocks (tests/test_oracle.py).
 */
#ifndef RRR_ORACLE_H
#define RRR_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

float rrro_f16_to_f32(uint16_t bits);          /* half 2.7.1 f16::to_f32, phi4.rs:442 */
uint16_t rrro_f32_to_f16_rne(float f);         /* IEEE round-to-nearest-even */
int rrro_block_bytes(int ggml_type);           /* gguf.rs:173-195 (per block) */
int rrro_block_elems(int ggml_type);

/* phi4.rs:444-479 / 481-510 / 512-542 / 544-553 / 555-570 */
void rrro_dequant_q6_k(const uint8_t* data, int64_t n_elements, float* out);
void rrro_dequant_q4_k(const uint8_t* data, int64_t n_elements, float* out);
void rrro_dequant_q5_k(const uint8_t* data, int64_t n_elements, float* out);
void rrro_dequant_q8_0(const uint8_t* data, int64_t n_elements, float* out);
void rrro_dequant_q5_0(const uint8_t* data, int64_t n_elements, float* out);
/* dequant_tensor_f32 dispatcher, phi4.rs:572-587 (types 0,1,6,8,12,13,14); 0 on
 * success, -1 on an unsupported type. */
int rrro_dequant(int ggml_type, const uint8_t* data, int64_t n_elements, float* out);

/* phi4.rs:593-599 (eps passed in; the reference's CPU path uses 1e-5, phi4.rs:111) */
void rrro_rms_norm(const float* x, const float* w, float* out, int n, float eps);
/* phi4.rs:601-606 and the SiLU*up loop of phi4.rs:1368-1373 */
void rrro_silu(float* x, int n);
void rrro_silu_gate(const float* gate_up, float* out, int F);
void rrro_add(const float* a, const float* b, float* out, int n); /* phi4.rs:608-610 */

/* Plain f32 GEMV, y[n] = sum_k W[n*K+k]*x[k], sequential accumulation per row. */
void rrro_gemv_f32(const float* W, const float* x, float* y, int64_t N, int64_t K,
                   int threads);
/* f32 C[M,N] = A[M,K] B[K,N] (matmul_tiled semantics). */
void rrro_matmul_f32(const float* A, const float* B, float* C, int M, int K, int N);

/* K-quant GEMV checker: each row is dequantised exactly as the reference, then dotted
 * in f32 (sequential). Works row by row (no whole-matrix buffer). threads >= 1. */
int rrro_gemv_kq(int qtype, const uint8_t* raw, const float* x, float* y, int64_t K,
                 int64_t N, int threads);
/* CPU baseline of the reference path: dequantise the whole matrix to f32 (phi4.rs
 * dequant_*), then a row-parallel f32 dot, both over `threads` threads. Returns the
 * seconds spent in each phase. scratch: f32[N*K] (caller-provided). */
int rrro_gemv_kq_baseline(int qtype, const uint8_t* raw, const float* x, float* y,
                          int64_t K, int64_t N, int threads, float* scratch,
                          double* t_dequant, double* t_dot);

/* Seeded synthetic blocks, identical to the product's device generator
 * (rrr_fill_kquant_random): blocks [block0, block0+n_blocks) of the stream `seed`. */
void rrro_fill_kquant_random(int qtype, uint8_t* dst, int64_t block0, int64_t n_blocks,
                             uint64_t seed);

/* Decode step at position 0 (see rrr_phi4_forward). Host pointers. hidden updated in
 * place; logits f32[vocab]. Returns 0, or -1 on a bad argument. */
typedef struct rrro_layer {
  const uint8_t* w_qkv; int qkv_type;
  const uint8_t* w_o; int o_type;
  const uint8_t* w_gate_up; int gate_up_type;
  const uint8_t* w_down; int down_type;
  const float* attn_norm; const float* ffn_norm;
} rrro_layer;
int rrro_decode_step(int d_model, int n_heads, int n_kv_heads, int head_dim, int ffn_dim,
                     int n_layers, int vocab, float eps, const rrro_layer* layers,
                     const float* output_norm, const float* w_out, float* hidden,
                     float* logits, int threads);

/* RoPE exactly as apply_rope_cfg (phi4.rs:238-256): for each of n_heads heads of
 * head_dim values and i < rope_dim/2: base = 1 / theta^((2i)/rope_dim) (f32 powf),
 * freq = base / factor_i (factor 1 past the table), angle = pos * freq, (sin, cos) of the
 * angle times attn_factor, then (x0, x1) = (x0 c - x1 s, x0 s + x1 c) on the pair
 * (2i, 2i+1). In place. */
void rrro_rope(float* x, int pos, int n_heads, int head_dim, int rope_dim, float theta,
               float attn_factor, const float* factors, int n_factors);
/* The f16 KV store of the `kv_store` dispatch (phi4.rs:1660-1677): row `pos` of the
 * caches (kv_stride f16 per row) = k, v rounded to nearest even. */
void rrro_kv_store(const float* k, const float* v, uint16_t* k_cache, uint16_t* v_cache,
                   int pos, int kv_stride);
/* Decode attention of the `attention` dispatch (push [seq_len, n_kv, heads_per_kv,
 * head_dim], phi4.rs:1680-1688). The shader is not part of the reference (un-vendored
 * torch-vulkan), so this is the standard definition it implements: query head h uses KV
 * head h / (n_heads / n_kv_heads); scores q.k / sqrt(head_dim) over positions
 * 0..seq_len-1 of the f16 caches, softmax (max subtracted), weighted sum of V. Dot
 * products and sums in double. out f32[n_heads*head_dim]. */
void rrro_attention_f16kv(const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                          float* out, int seq_len, int n_heads, int n_kv_heads, int head_dim);
/* Decode step at position `pos` with RoPE and the f16 KV caches (forward_dynamic,
 * phi4.rs:1593-1760): per layer rms -> QKV -> RoPE(Q), RoPE(K) -> store K, V at row pos
 * -> attention over pos+1 rows -> O -> residual -> FFN as rrro_decode_step.
 * k_caches / v_caches: n_layers x max_seq x (n_kv_heads*head_dim) f16, updated. */
int rrro_decode_step_kv(int d_model, int n_heads, int n_kv_heads, int head_dim, int ffn_dim,
                        int n_layers, int vocab, float eps, int rope_dim, float theta,
                        float attn_factor, const float* factors, int n_factors, int pos,
                        int max_seq, uint16_t* k_caches, uint16_t* v_caches,
                        const rrro_layer* layers, const float* output_norm,
                        const float* w_out, float* hidden, float* logits, int threads);

#ifdef __cplusplus
}
#endif
#endif
