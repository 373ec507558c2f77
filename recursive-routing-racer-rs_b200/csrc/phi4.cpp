// phi4.cpp — Phi-4-mini-shape decode step on the weight-path kernels (replaces
// Phi4Model::forward_gpu, src/model/phi4.rs:1099-1196, and its 378-dispatch table,
// phi4.rs:969-1064).
//
// Per layer the reference issues 11 dispatches (rmsnorm, qkv, rope_kv_store, attention,
// o-proj, residual_add, rmsnorm, ffn_up, silu_gate, ffn_down, residual_add). Here the
// norms, the attention output at position 0 and both residual adds are fused into the
// GEMV prologues / epilogues (rrr_gemv_kq_ex) and SiLU(gate)*up into the gate_up GEMV's
// epilogue (rrr_gemv_kq_swiglu), so a layer is 4 launches and the step is
// 4*L + logits chunks (+ argmax). The whole step can be captured once into a CUDA graph.
//
// With a KV cache (max_seq > 0, forward_dynamic, phi4.rs:1593-1760) a layer is 5 launches:
// QKV (RMSNorm prologue), RoPE + f16 KV store + attention over rows 0..pos (one fused
// kernel), O-proj (residual epilogue), gate_up (SwiGLU), down (residual); the position
// lives on the device and a one-thread kernel advances it at the end of the step, so one
// captured graph serves every position.
#include <cuda_runtime.h>

#include <vector>

#include "capi_internal.h"
#include "internal.h"

using namespace rrr;

struct rrr_phi4 {
  rrr_ctx* ctx = nullptr;
  rrr_phi4_desc d{};
  std::vector<rrr_phi4_layer> layers;
  float* qkv = nullptr;      // f32[n_q*hd + 2*n_kv*hd]
  float* mid = nullptr;      // f32[ffn]: silu(gate) * up
  void* argmax_scratch = nullptr;  // 16 B, kept zeroed by the argmax kernel
  // KV-cache decode
  uint16_t* kv = nullptr;    // f16 [n_layers][2][max_seq][n_kv*hd]
  float* attn = nullptr;     // f32[n_q*hd]: attention output, the O-projection's input
  int* d_pos = nullptr;      // device position of the next token
  int pos = 0;               // host copy
  rrr_attn_desc attn_desc{};
  // graph cache
  cudaGraphExec_t exec = nullptr;
  cudaGraph_t graph = nullptr;
  cudaStream_t cap_stream = nullptr;
  float* g_hidden = nullptr;
  float* g_logits = nullptr;
  int* g_argmax = nullptr;
  // batched forward (M tokens): scratch for b_cap rows in one allocation, and its graph
  int b_cap = 0;
  void* b_arena = nullptr;
  uint16_t* b_xn = nullptr;   // bf16 [M][d]: RMSNorm output, the GEMM input
  float* b_qkv = nullptr;     // f32 [M][qkv_dim]
  uint16_t* b_a = nullptr;    // bf16 [M][n_q*hd]: attention output (O-proj input)
  float* b_attn = nullptr;    // f32 [M][n_q*hd] (KV-cache mode)
  float* b_gu = nullptr;      // f32 [M][2 ffn]
  uint16_t* b_mid = nullptr;  // bf16 [M][ffn]: silu(gate) * up
  float* b_xnorm = nullptr;   // f32 [M][d]: output RMSNorm of the logits
  cudaGraphExec_t b_exec = nullptr;
  cudaGraph_t b_graph = nullptr;
  float* bg_hidden = nullptr;
  float* bg_logits = nullptr;
  int* bg_argmax = nullptr;
  int bg_M = 0;
};

static int phi4_issue(rrr_phi4* m, float* hidden, float* logits, int* argmax, void* stream) {
  const rrr_phi4_desc& d = m->d;
  rrr_ctx* ctx = m->ctx;
  const int qkv_dim = (d.n_heads + 2 * d.n_kv_heads) * d.head_dim;
  int rc;
  const size_t cache = (size_t)d.max_seq * d.n_kv_heads * d.head_dim;
  for (int l = 0; l < d.n_layers; ++l) {
    const rrr_phi4_layer& L = m->layers[l];
    rrr_gemv_prologue pn{RRR_X_RMSNORM, L.attn_norm, d.rms_eps, 0, 0, 0};
    if ((rc = rrr_gemv_kq_ex(ctx, L.qkv_type, L.w_qkv, hidden, m->qkv, d.d_model, qkv_dim, nullptr,
                             &pn, stream)))
      return rc;
    if (d.max_seq > 0) {
      uint16_t* kc = m->kv + 2 * cache * l;
      uint16_t* vc = kc + cache;
      if ((rc = rrr_rope_attention_f16kv(ctx, &m->attn_desc, m->qkv, 0, m->d_pos, kc, vc, m->attn,
                                         stream)) ||
          (rc = rrr_gemv_kq_ex(ctx, L.o_type, L.w_o, m->attn, hidden, d.n_heads * d.head_dim,
                               d.d_model, hidden, nullptr, stream)))
        return rc;
    } else {
      rrr_gemv_prologue pv{RRR_X_GQA_V, nullptr, 0.f, d.n_heads, d.n_kv_heads, d.head_dim};
      if ((rc = rrr_gemv_kq_ex(ctx, L.o_type, L.w_o, m->qkv, hidden, d.n_heads * d.head_dim,
                               d.d_model, hidden, &pv, stream)))
        return rc;
    }
    rrr_gemv_prologue pf{RRR_X_RMSNORM, L.ffn_norm, d.rms_eps, 0, 0, 0};
    if ((rc = rrr_gemv_kq_swiglu(ctx, L.gate_up_type, L.w_gate_up, hidden, m->mid, d.d_model,
                                 d.ffn_dim, &pf, stream)))
      return rc;
    if ((rc = rrr_gemv_kq_ex(ctx, L.down_type, L.w_down, m->mid, hidden, d.ffn_dim, d.d_model,
                             hidden, nullptr, stream)))
      return rc;
  }
  if ((rc = rrr_logits_f32(ctx, d.w_out, hidden, logits, d.vocab, d.d_model, d.logits_chunk_rows,
                           d.output_norm, d.rms_eps, stream)))
    return rc;
  if (argmax) {
    cudaError_t e = launch_argmax(make_env(ctx, stream), logits, d.vocab, argmax, m->argmax_scratch);
    if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_phi4_forward: argmax launch");
  }
  if (d.max_seq > 0) {
    cudaError_t e = launch_pos_advance(make_env(ctx, stream), m->d_pos, 1);
    if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_phi4_forward: position launch");
  }
  return RRR_OK;
}

// Scratch rows for a batched forward of M tokens (grown, never shrunk).
static int phi4_batch_scratch(rrr_phi4* m, int M) {
  if (M <= m->b_cap) return RRR_OK;
  const rrr_phi4_desc& d = m->d;
  const size_t qkv_dim = (size_t)(d.n_heads + 2 * d.n_kv_heads) * d.head_dim;
  const size_t qd = (size_t)d.n_heads * d.head_dim;
  auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
  const size_t sz[7] = {al((size_t)M * d.d_model * 2), al((size_t)M * qkv_dim * 4), al((size_t)M * qd * 2),
                        al((size_t)M * qd * 4), al((size_t)M * 2 * d.ffn_dim * 4),
                        al((size_t)M * d.ffn_dim * 2), al((size_t)M * d.d_model * 4)};
  size_t tot = 0;
  for (size_t b : sz) tot += b;
  // the old arena may still be read by work in flight
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_error(m->ctx, e, "rrr_phi4_forward_batched: synchronise");
  if (m->b_arena) cudaFree(m->b_arena);
  m->b_arena = nullptr;
  m->b_cap = 0;
  e = cudaMalloc(&m->b_arena, tot);
  if (e != cudaSuccess) {
    m->b_arena = nullptr;
    return cuda_error(m->ctx, e, "rrr_phi4_forward_batched: scratch allocation");
  }
  char* p = static_cast<char*>(m->b_arena);
  m->b_xn = reinterpret_cast<uint16_t*>(p);     p += sz[0];
  m->b_qkv = reinterpret_cast<float*>(p);       p += sz[1];
  m->b_a = reinterpret_cast<uint16_t*>(p);      p += sz[2];
  m->b_attn = reinterpret_cast<float*>(p);      p += sz[3];
  m->b_gu = reinterpret_cast<float*>(p);        p += sz[4];
  m->b_mid = reinterpret_cast<uint16_t*>(p);    p += sz[5];
  m->b_xnorm = reinterpret_cast<float*>(p);
  m->b_cap = M;
  return RRR_OK;
}

// M tokens through the layer stack (forward_prefill_batched, phi4.rs:1200-1445): per
// layer RMSNorm -> bf16, QKV GEMM; at position 0 the attention output is V of each head's
// KV group (GQA-V), with a KV cache RoPE + f16 KV store of rows p..p+M-1 and causal
// attention over rows 0..p+t; O GEMM with the residual in its epilogue; RMSNorm -> bf16,
// gate_up GEMM, SiLU(gate)*up -> bf16, down GEMM with the residual; then the output
// RMSNorm + logits of all M rows, the argmax of each row, and the position advance.
static int phi4_issue_batched(rrr_phi4* m, float* hidden, float* logits, int* argmax, int M,
                              void* stream) {
  const rrr_phi4_desc& d = m->d;
  rrr_ctx* ctx = m->ctx;
  const int qkv_dim = (d.n_heads + 2 * d.n_kv_heads) * d.head_dim;
  const int qd = d.n_heads * d.head_dim;
  const size_t cache = (size_t)d.max_seq * d.n_kv_heads * d.head_dim;
  int rc;
  for (int l = 0; l < d.n_layers; ++l) {
    const rrr_phi4_layer& L = m->layers[l];
    if ((rc = rrr_rmsnorm_bf16(ctx, hidden, L.attn_norm, m->b_xn, M, d.d_model, d.rms_eps, stream)) ||
        (rc = rrr_gemm_kq_batched(ctx, L.qkv_type, L.w_qkv, m->b_xn, m->b_qkv, M, d.d_model, qkv_dim,
                                  stream)))
      return rc;
    if (d.max_seq > 0) {
      uint16_t* kc = m->kv + 2 * cache * l;
      uint16_t* vc = kc + cache;
      if ((rc = rrr_rope_kv_store(ctx, &m->attn_desc, m->b_qkv, qkv_dim, M, 0, m->d_pos, kc, vc, stream)) ||
          (rc = rrr_attention_f16kv(ctx, &m->attn_desc, m->b_qkv, qkv_dim, M, 0, m->d_pos, kc, vc,
                                    m->b_attn, stream)) ||
          (rc = rrr_window_bf16(ctx, m->b_attn, m->b_a, M, qd, qd, 0, stream)))
        return rc;
    } else if ((rc = rrr_gqa_v_bf16(ctx, m->b_qkv, m->b_a, M, d.n_heads, d.n_kv_heads, d.head_dim, qd, 0,
                                    stream))) {
      return rc;
    }
    if ((rc = rrr_gemm_kq_batched_ex(ctx, L.o_type, L.w_o, m->b_a, hidden, M, qd, d.d_model, hidden,
                                     stream)) ||
        (rc = rrr_rmsnorm_bf16(ctx, hidden, L.ffn_norm, m->b_xn, M, d.d_model, d.rms_eps, stream)) ||
        (rc = rrr_gemm_kq_batched(ctx, L.gate_up_type, L.w_gate_up, m->b_xn, m->b_gu, M, d.d_model,
                                  2 * d.ffn_dim, stream)) ||
        (rc = rrr_silu_gate_bf16(ctx, m->b_gu, m->b_mid, M, d.ffn_dim, stream)) ||
        (rc = rrr_gemm_kq_batched_ex(ctx, L.down_type, L.w_down, m->b_mid, hidden, M, d.ffn_dim,
                                     d.d_model, hidden, stream)))
      return rc;
  }
  if ((rc = rrr_logits_f32_batched(ctx, d.w_out, hidden, m->b_xnorm, logits, M, d.vocab, d.d_model,
                                   d.output_norm, d.rms_eps, stream)))
    return rc;
  if (argmax) {
    cudaError_t e = launch_argmax_rows(make_env(ctx, stream), logits, d.vocab, d.vocab, argmax, M);
    if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_phi4_forward_batched: argmax launch");
  }
  if (d.max_seq > 0) {
    cudaError_t e = launch_pos_advance(make_env(ctx, stream), m->d_pos, M);
    if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_phi4_forward_batched: position launch");
  }
  return RRR_OK;
}

static void phi4_drop_batched_graph(rrr_phi4* m) {
  if (m->b_exec) cudaGraphExecDestroy(m->b_exec);
  if (m->b_graph) cudaGraphDestroy(m->b_graph);
  m->b_exec = nullptr;
  m->b_graph = nullptr;
}

static void phi4_drop_graph(rrr_phi4* m) {
  if (m->exec) cudaGraphExecDestroy(m->exec);
  if (m->graph) cudaGraphDestroy(m->graph);
  m->exec = nullptr;
  m->graph = nullptr;
}

extern "C" {

int rrr_phi4_create(rrr_ctx* ctx, const rrr_phi4_desc* desc, rrr_phi4** out) {
  if (!ctx) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context");
  if (!desc || !out) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_phi4_create: null argument");
  *out = nullptr;
  const rrr_phi4_desc& d = *desc;
  if (d.d_model <= 0 || d.n_heads <= 0 || d.n_kv_heads <= 0 || d.head_dim <= 0 || d.ffn_dim <= 0 ||
      d.n_layers < 0 || d.vocab <= 0 || d.n_heads % d.n_kv_heads != 0 ||
      d.n_heads * d.head_dim != d.d_model || d.d_model % 256 != 0 || d.ffn_dim % 256 != 0 ||
      d.head_dim % 8 != 0)
    return set_error(ctx, RRR_ERR_BAD_SHAPE,
                     "rrr_phi4_create: need n_heads*head_dim == d_model, d_model and ffn_dim "
                     "multiples of 256, head_dim %% 8 == 0, n_heads %% n_kv_heads == 0");
  if ((d.n_layers > 0 && !d.layers) || !d.output_norm || !d.w_out)
    return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_phi4_create: missing weights");
  for (int l = 0; l < d.n_layers; ++l) {
    const rrr_phi4_layer& L = d.layers[l];
    if (!L.w_qkv || !L.w_o || !L.w_gate_up || !L.w_down || !L.attn_norm || !L.ffn_norm)
      return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_phi4_create: layer %d has a null weight", l);
  }
  rrr_attn_desc ad{};
  if (d.max_seq > 0) {
    ad.n_heads = d.n_heads;
    ad.n_kv_heads = d.n_kv_heads;
    ad.head_dim = d.head_dim;
    ad.rope_dim = d.rope_dim;
    ad.rope_theta = d.rope_theta;
    ad.rope_attn_factor = d.rope_attn_factor;
    ad.rope_factors = d.rope_factors;
    ad.n_rope_factors = d.rope_factors ? d.n_rope_factors : 0;
    ad.max_seq = d.max_seq;
    const int hpk = d.n_heads / d.n_kv_heads;
    if ((d.head_dim != 64 && d.head_dim != 128 && d.head_dim != 256) || hpk > 8 || d.rope_dim < 0 ||
        d.rope_dim % 2 || d.rope_dim > d.head_dim || d.rope_dim > 128 || d.n_rope_factors < 0 ||
        attention_smem_for(d.head_dim, hpk, d.max_seq) > 227 * 1024)
      return set_error(ctx, RRR_ERR_BAD_SHAPE,
                       "rrr_phi4_create: KV-cache decode needs head_dim 64/128/256, at most 8 query "
                       "heads per KV head, even rope_dim <= min(head_dim, 128), a max_seq that fits");
  } else if (d.max_seq < 0) {
    return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_phi4_create: max_seq >= 0");
  }
  int rc = bind_device(ctx);
  if (rc) return rc;
  rrr_phi4* m = new rrr_phi4();
  m->attn_desc = ad;
  m->ctx = ctx;
  m->d = d;
  m->layers.assign(d.layers, d.layers + d.n_layers);
  m->d.layers = nullptr;
  const size_t qkv_dim = (size_t)(d.n_heads + 2 * d.n_kv_heads) * d.head_dim;
  cudaError_t e = cudaMalloc(&m->qkv, qkv_dim * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&m->mid, (size_t)d.ffn_dim * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&m->argmax_scratch, 64);
  if (e == cudaSuccess) e = cudaMemset(m->argmax_scratch, 0, 64);
  if (e == cudaSuccess && d.max_seq > 0) {
    const size_t cache = (size_t)d.max_seq * d.n_kv_heads * d.head_dim;
    e = cudaMalloc(&m->kv, 2 * cache * d.n_layers * sizeof(uint16_t) + 16);
    if (e == cudaSuccess) e = cudaMalloc(&m->attn, (size_t)d.d_model * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&m->d_pos, 16);
    if (e == cudaSuccess) e = cudaMemset(m->d_pos, 0, 16);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
  }
  if (e != cudaSuccess) {
    rrr_phi4_destroy(m);
    return cuda_error(ctx, e, "rrr_phi4_create: scratch allocation");
  }
  *out = m;
  return RRR_OK;
}

int rrr_phi4_forward(rrr_phi4* m, float* hidden, float* logits, int* argmax_out, int use_graph,
                     void* stream) {
  if (!m) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null model");
  rrr_ctx* ctx = m->ctx;
  if (!hidden || !logits) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_phi4_forward: null buffer");
  int rc = bind_device(ctx);
  if (rc) return rc;
  if (m->d.max_seq > 0 && m->pos >= m->d.max_seq)
    return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_phi4_forward: position %d is past the cache (%d rows)",
                     m->pos, m->d.max_seq);
  if (!use_graph) {
    rc = phi4_issue(m, hidden, logits, argmax_out, stream);
    if (rc == RRR_OK && m->d.max_seq > 0) ++m->pos;
    return rc;
  }
  if (!m->exec || m->g_hidden != hidden || m->g_logits != logits || m->g_argmax != argmax_out) {
    phi4_drop_graph(m);
    if (!m->cap_stream) {
      cudaError_t e = cudaStreamCreateWithFlags(&m->cap_stream, cudaStreamNonBlocking);
      if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_phi4_forward: stream");
    }
    cudaError_t e;
    e = cudaStreamBeginCapture(m->cap_stream, cudaStreamCaptureModeRelaxed);
    if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_phi4_forward: begin capture");
    rc = phi4_issue(m, hidden, logits, argmax_out, m->cap_stream);
    cudaGraph_t g = nullptr;
    e = cudaStreamEndCapture(m->cap_stream, &g);
    if (rc) {
      if (g) cudaGraphDestroy(g);
      return rc;
    }
    if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_phi4_forward: end capture");
    e = cudaGraphInstantiate(&m->exec, g, 0);
    if (e != cudaSuccess) {
      cudaGraphDestroy(g);
      return cuda_error(ctx, e, "rrr_phi4_forward: instantiate");
    }
    m->graph = g;
    m->g_hidden = hidden;
    m->g_logits = logits;
    m->g_argmax = argmax_out;
  }
  cudaError_t e = cudaGraphLaunch(m->exec, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_phi4_forward: graph launch");
  if (m->d.max_seq > 0) ++m->pos;
  return RRR_OK;
}

int rrr_phi4_forward_batched(rrr_phi4* m, float* hidden, float* logits, int* argmax_out, int M,
                             int use_graph, void* stream) {
  if (!m) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null model");
  rrr_ctx* ctx = m->ctx;
  if (!hidden || !logits) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_phi4_forward_batched: null buffer");
  if (M < 1) return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_phi4_forward_batched: M >= 1");
  if (m->d.max_seq > 0 && m->pos + M > m->d.max_seq)
    return set_error(ctx, RRR_ERR_BAD_SHAPE,
                     "rrr_phi4_forward_batched: positions %d..%d are past the cache (%d rows)", m->pos,
                     m->pos + M - 1, m->d.max_seq);
  int rc = bind_device(ctx);
  if (rc) return rc;
  if (M > m->b_cap) {
    phi4_drop_batched_graph(m);
    if ((rc = phi4_batch_scratch(m, M))) return rc;
  }
  if (use_graph && m->b_exec && m->bg_hidden == hidden && m->bg_logits == logits &&
      m->bg_argmax == argmax_out && m->bg_M == M) {
    cudaError_t e = cudaGraphLaunch(m->b_exec, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_phi4_forward_batched: graph launch");
    if (m->d.max_seq > 0) m->pos += M;
    return RRR_OK;
  }
  // the step itself, eagerly (this also creates the cuBLAS state the logits GEMM needs
  // before any capture)
  rc = phi4_issue_batched(m, hidden, logits, argmax_out, M, stream);
  if (rc) return rc;
  if (m->d.max_seq > 0) m->pos += M;
  if (!use_graph) return RRR_OK;
  // then the graph for the next calls with these buffers and M (capture executes nothing;
  // the position is read on the device when the graph runs)
  phi4_drop_batched_graph(m);
  if (!m->cap_stream) {
    cudaError_t e = cudaStreamCreateWithFlags(&m->cap_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_phi4_forward_batched: stream");
  }
  cudaError_t e = cudaStreamBeginCapture(m->cap_stream, cudaStreamCaptureModeRelaxed);
  if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_phi4_forward_batched: begin capture");
  rc = phi4_issue_batched(m, hidden, logits, argmax_out, M, m->cap_stream);
  cudaGraph_t g = nullptr;
  e = cudaStreamEndCapture(m->cap_stream, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_phi4_forward_batched: end capture");
  e = cudaGraphInstantiate(&m->b_exec, g, 0);
  if (e != cudaSuccess) {
    cudaGraphDestroy(g);
    m->b_exec = nullptr;
    return cuda_error(ctx, e, "rrr_phi4_forward_batched: instantiate");
  }
  m->b_graph = g;
  m->bg_hidden = hidden;
  m->bg_logits = logits;
  m->bg_argmax = argmax_out;
  m->bg_M = M;
  return RRR_OK;
}

int rrr_phi4_launches_per_step(rrr_phi4* m, int* n) {
  if (!m || !n) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null argument");
  const int chunk = m->d.logits_chunk_rows > 0 ? m->d.logits_chunk_rows : m->d.vocab;
  *n = (m->d.max_seq > 0 ? 5 : 4) * m->d.n_layers + (m->d.vocab + chunk - 1) / chunk +
       (m->d.max_seq > 0 ? 1 : 0);
  return RRR_OK;
}

int rrr_phi4_set_position(rrr_phi4* m, int pos, void* stream) {
  if (!m) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null model");
  if (m->d.max_seq <= 0)
    return set_error(m->ctx, RRR_ERR_UNSUPPORTED, "rrr_phi4_set_position: model has no KV cache");
  if (pos < 0 || pos >= m->d.max_seq)
    return set_error(m->ctx, RRR_ERR_BAD_SHAPE, "rrr_phi4_set_position: need 0 <= pos < %d", m->d.max_seq);
  int rc = bind_device(m->ctx);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(m->d_pos, &pos, sizeof(int), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_error(m->ctx, e, "rrr_phi4_set_position");
  m->pos = pos;
  return RRR_OK;
}

int rrr_phi4_position(rrr_phi4* m, int* pos) {
  if (!m || !pos) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null argument");
  *pos = m->pos;
  return RRR_OK;
}

int rrr_phi4_kv_cache(rrr_phi4* m, int layer, uint16_t** k_cache, uint16_t** v_cache) {
  if (!m || !k_cache || !v_cache) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null argument");
  if (m->d.max_seq <= 0)
    return set_error(m->ctx, RRR_ERR_UNSUPPORTED, "rrr_phi4_kv_cache: model has no KV cache");
  if (layer < 0 || layer >= m->d.n_layers)
    return set_error(m->ctx, RRR_ERR_BAD_SHAPE, "rrr_phi4_kv_cache: layer out of range");
  const size_t cache = (size_t)m->d.max_seq * m->d.n_kv_heads * m->d.head_dim;
  *k_cache = m->kv + 2 * cache * layer;
  *v_cache = *k_cache + cache;
  return RRR_OK;
}

int rrr_phi4_destroy(rrr_phi4* m) {
  if (!m) return RRR_OK;
  bind_device(m->ctx);
  phi4_drop_graph(m);
  phi4_drop_batched_graph(m);
  if (m->b_arena) cudaFree(m->b_arena);
  if (m->cap_stream) cudaStreamDestroy(m->cap_stream);
  if (m->qkv) cudaFree(m->qkv);
  if (m->mid) cudaFree(m->mid);
  if (m->argmax_scratch) cudaFree(m->argmax_scratch);
  if (m->kv) cudaFree(m->kv);
  if (m->attn) cudaFree(m->attn);
  if (m->d_pos) cudaFree(m->d_pos);
  delete m;
  return RRR_OK;
}

}  // extern "C"
