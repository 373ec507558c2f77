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
