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
//
// A tensor-parallel rank (rrr_phi4_tp_create) all-reduces the hidden state after each
// O-projection and down and all-gathers the logits. On a peer-memory channel with a fused
// region (rrr_comm_create_ex, ranks on distinct GPUs) the one-token step fuses the
// all-reduces into the GEMVs instead (GemvFuse): O-projection / down push their partial rows,
// tagged with the step's epoch, to every rank, and the next RMSNorm GEMV (gate_up, the next
// layer's QKV) sums the ranks' rows in rank order in its prologue. Exchange site s = 2l
// (O-projection of layer l) or 2l+1 (down); each rank's region holds [site][rank][d_model]
// words. The last site is summed by one small kernel, which is followed by the epoch advance.
#include <cuda_runtime.h>

#include <cstring>
#include <vector>

#include "capi_internal.h"
#include "internal.h"

using namespace rrr;

struct rrr_phi4 {
  rrr_ctx* ctx = nullptr;
  rrr_phi4_desc d{};
  std::vector<rrr_phi4_layer> layers;
  // Tensor parallelism: this rank's shard (G = 1: the whole model on this GPU) and the
  // channel of its exchanges; the rank-local extents below follow from the shard.
  rrr_tp_shard sh{};
  rrr_tp_comm* comm = nullptr;
  int q_loc = 0, kv_loc = 0, f_loc = 0, v_loc = 0;
  bool fused = false;                            // all-reduces fused into the GEMVs
  unsigned long long* fz_base[kMaxTpRanks] = {};  // each rank's fused region, mapped here
  unsigned* fz_epoch = nullptr;                   // the step epoch (the channel's, on this GPU)
  float* qkv = nullptr;      // f32[qkv_dim of the shard]
  float* mid = nullptr;      // f32[ffn of the shard]: silu(gate) * up
  float* logits_loc = nullptr;  // f32[vocab rows of the shard] (G > 1)
  void* argmax_scratch = nullptr;  // 16 B, kept zeroed by the argmax kernel
  // KV-cache decode
  uint16_t* kv = nullptr;    // f16 [n_layers][2][max_seq][kv heads of the shard * hd]
  float* attn = nullptr;     // f32[o_k]: attention output in the O-projection's window
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
  uint16_t* b_a = nullptr;    // bf16 [M][o_k]: attention output (O-proj input window)
  float* b_attn = nullptr;    // f32 [M][heads * hd] (KV-cache mode)
  float* b_gu = nullptr;      // f32 [M][2 ffn]
  uint16_t* b_mid = nullptr;  // bf16 [M][ffn]: silu(gate) * up
  float* b_xnorm = nullptr;   // f32 [M][d]: output RMSNorm of the logits
  float* b_logits_loc = nullptr;  // f32 [M][vocab rows] (G > 1)
  cudaGraphExec_t b_exec = nullptr;
  cudaGraph_t b_graph = nullptr;
  float* bg_hidden = nullptr;
  float* bg_logits = nullptr;
  int* bg_argmax = nullptr;
  int bg_M = 0;
};

// A step is 2 segments per layer (the attention half ending with the O-projection, the FFN
// half ending with down) plus the logits and a tail (argmax, position). With G > 1 the
// hidden state is all-reduced after each layer segment and the logits are all-gathered
// after the logits segment; the one-GPU emulation of a split runs the segments of all ranks
// in lockstep with local exchanges in between.
static int phi4_segments(const rrr_phi4* m) { return 2 * m->d.n_layers + 2; }

// The fused exchange that a GEMV of the one-token step takes part in: the sum of site
// `site`'s rows in its prologue (the sum also stored to h_out), or the push of its rows to
// site `site`.
static GemvFuse phi4_fuse_sum(const rrr_phi4* m, int site, float* h_out) {
  GemvFuse f;
  f.G = m->sh.G;
  f.epoch = m->fz_epoch;
  f.sum_in = m->fz_base[m->sh.g] + (size_t)site * m->sh.G * m->d.d_model;
  f.h_out = h_out;
  return f;
}
static GemvFuse phi4_fuse_push(const rrr_phi4* m, int site) {
  GemvFuse f;
  f.G = m->sh.G;
  f.epoch = m->fz_epoch;
  for (int r = 0; r < m->sh.G; ++r)
    f.push[r] = m->fz_base[r] + ((size_t)site * m->sh.G + m->sh.g) * m->d.d_model;
  return f;
}

// One GEMV of the one-token step (SwiGLU epilogue when `swiglu`, N = F), checked like the
// C ABI's rrr_gemv_kq_ex / rrr_gemv_kq_swiglu, with the fused exchange `fz` when it is not
// null.
static int phi4_gemv(rrr_phi4* m, int qtype, const void* w, const float* x, float* y, int K, int N,
                     const float* residual, const rrr_gemv_prologue* pro, bool swiglu,
                     const GemvFuse* fz, void* stream) {
  rrr_ctx* ctx = m->ctx;
  int rc = check_gemv(ctx, qtype, w, x, y, K, N, residual, pro, swiglu);
  if (rc) return rc;
  const LaunchEnv env = make_env(ctx, stream);
  cudaError_t e = swiglu ? launch_gemv_kq_swiglu(env, qtype, w, x, y, K, N, pro, fz)
                         : launch_gemv_kq(env, qtype, w, x, y, K, N, residual, pro, fz);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? RRR_OK : cuda_error(ctx, e, "rrr_phi4_forward: GEMV launch");
}

// Segment `seg` of the one-token step (forward_gpu, phi4.rs:1099-1196).
static int phi4_issue_seg(rrr_phi4* m, int seg, float* hidden, float* logits, int* argmax,
                          void* stream) {
  const rrr_phi4_desc& d = m->d;
  const rrr_tp_shard& sh = m->sh;
  rrr_ctx* ctx = m->ctx;
  const int L = d.n_layers;
  float* res = sh.g == 0 ? hidden : nullptr;  // the residual enters the sum once
  const bool fz = m->fused;
  int rc;
  if (seg < 2 * L) {
    const rrr_phi4_layer& Ly = m->layers[seg / 2];
    const int l = seg / 2;
    // fused exchanges: this segment's GEMVs sum site seg - 1 and push site seg
    GemvFuse fin, fout;
    if (fz) {
      if (seg > 0) fin = phi4_fuse_sum(m, seg - 1, hidden);
      fout = phi4_fuse_push(m, seg);
    }
    const GemvFuse* pin = fz && seg > 0 ? &fin : nullptr;
    const GemvFuse* pout = fz ? &fout : nullptr;
    if ((seg & 1) == 0) {
      rrr_gemv_prologue pn{RRR_X_RMSNORM, Ly.attn_norm, d.rms_eps, 0, 0, 0, 0};
      if ((rc = phi4_gemv(m, Ly.qkv_type, Ly.w_qkv, hidden, m->qkv, d.d_model, sh.qkv_dim,
                          nullptr, &pn, false, pin, stream)))
        return rc;
      if (d.max_seq > 0) {
        const size_t cache = (size_t)d.max_seq * m->kv_loc * d.head_dim;
        uint16_t* kc = m->kv + 2 * cache * l;
        uint16_t* vc = kc + cache;
        if ((rc = rrr_rope_attention_f16kv(ctx, &m->attn_desc, m->qkv, 0, m->d_pos, kc, vc,
                                           m->attn + sh.o_k_offset, stream)) ||
            (rc = phi4_gemv(m, Ly.o_type, Ly.w_o, m->attn, hidden, sh.o_k, d.d_model, res,
                            nullptr, false, pout, stream)))
          return rc;
      } else {
        rrr_gemv_prologue pv{RRR_X_GQA_V, nullptr, 0.f, m->q_loc, m->kv_loc, d.head_dim, sh.o_k_offset};
        if ((rc = phi4_gemv(m, Ly.o_type, Ly.w_o, m->qkv, hidden, sh.o_k, d.d_model, res, &pv,
                            false, pout, stream)))
          return rc;
      }
      return RRR_OK;
    }
    rrr_gemv_prologue pf{RRR_X_RMSNORM, Ly.ffn_norm, d.rms_eps, 0, 0, 0, 0};
    if ((rc = phi4_gemv(m, Ly.gate_up_type, Ly.w_gate_up, hidden, m->mid, d.d_model, m->f_loc,
                        nullptr, &pf, true, pin, stream)) ||
        (rc = phi4_gemv(m, Ly.down_type, Ly.w_down, m->mid, hidden, m->f_loc, d.d_model, res,
                        nullptr, false, pout, stream)))
      return rc;
    if (fz && l == L - 1) {
      // the last site's sum is the final hidden state; then the next step's epoch
      const LaunchEnv env = make_env(ctx, stream);
      cudaError_t e = launch_fused_sum(env, phi4_fuse_sum(m, seg, nullptr).sum_in, hidden, d.d_model,
                                       sh.G, m->fz_epoch);
      if (e == cudaSuccess) e = launch_epoch_advance(env, m->fz_epoch);
      if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_phi4_forward: fused exchange launch");
    }
    return RRR_OK;
  }
  if (seg == 2 * L)
    return rrr_logits_f32(ctx, d.w_out, hidden, sh.G > 1 ? m->logits_loc : logits, m->v_loc,
                          d.d_model, d.logits_chunk_rows, d.output_norm, d.rms_eps, stream);
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

// Segment `seg` of the M-token step (forward_prefill_batched, phi4.rs:1200-1445): per
// layer RMSNorm -> bf16, QKV GEMM; at position 0 the attention output is V of each head's
// KV group (GQA-V), with a KV cache RoPE + f16 KV store of rows p..p+M-1 and causal
// attention over rows 0..p+t; O GEMM with the residual in its epilogue; RMSNorm -> bf16,
// gate_up GEMM, SiLU(gate)*up -> bf16, down GEMM with the residual; then the output
// RMSNorm + logits of all M rows, the argmax of each row, and the position advance.
static int phi4_issue_batched_seg(rrr_phi4* m, int seg, float* hidden, float* logits,
                                  int* argmax, int M, void* stream) {
  const rrr_phi4_desc& d = m->d;
  const rrr_tp_shard& sh = m->sh;
  rrr_ctx* ctx = m->ctx;
  const int L = d.n_layers;
  const int qd = m->q_loc * d.head_dim;
  float* res = sh.g == 0 ? hidden : nullptr;
  int rc;
  if (seg < 2 * L) {
    const int l = seg / 2;
    const rrr_phi4_layer& Ly = m->layers[l];
    if ((seg & 1) == 0) {
      if ((rc = rrr_rmsnorm_bf16(ctx, hidden, Ly.attn_norm, m->b_xn, M, d.d_model, d.rms_eps, stream)) ||
          (rc = rrr_gemm_kq_batched(ctx, Ly.qkv_type, Ly.w_qkv, m->b_xn, m->b_qkv, M, d.d_model,
                                    sh.qkv_dim, stream)))
        return rc;
      if (d.max_seq > 0) {
        const size_t cache = (size_t)d.max_seq * m->kv_loc * d.head_dim;
        uint16_t* kc = m->kv + 2 * cache * l;
        uint16_t* vc = kc + cache;
        if ((rc = rrr_rope_kv_store(ctx, &m->attn_desc, m->b_qkv, sh.qkv_dim, M, 0, m->d_pos, kc, vc,
                                    stream)) ||
            (rc = rrr_attention_f16kv(ctx, &m->attn_desc, m->b_qkv, sh.qkv_dim, M, 0, m->d_pos, kc, vc,
                                      m->b_attn, stream)) ||
            (rc = rrr_window_bf16(ctx, m->b_attn, m->b_a, M, qd, sh.o_k, sh.o_k_offset, stream)))
          return rc;
      } else if ((rc = rrr_gqa_v_bf16(ctx, m->b_qkv, m->b_a, M, m->q_loc, m->kv_loc, d.head_dim,
                                      sh.o_k, sh.o_k_offset, stream))) {
        return rc;
      }
      return rrr_gemm_kq_batched_ex(ctx, Ly.o_type, Ly.w_o, m->b_a, hidden, M, sh.o_k, d.d_model,
                                    res, stream);
    }
    if ((rc = rrr_rmsnorm_bf16(ctx, hidden, Ly.ffn_norm, m->b_xn, M, d.d_model, d.rms_eps, stream)) ||
        (rc = rrr_gemm_kq_batched(ctx, Ly.gate_up_type, Ly.w_gate_up, m->b_xn, m->b_gu, M, d.d_model,
                                  2 * m->f_loc, stream)) ||
        (rc = rrr_silu_gate_bf16(ctx, m->b_gu, m->b_mid, M, m->f_loc, stream)))
      return rc;
    return rrr_gemm_kq_batched_ex(ctx, Ly.down_type, Ly.w_down, m->b_mid, hidden, M, m->f_loc,
                                  d.d_model, res, stream);
  }
  if (seg == 2 * L)
    return rrr_logits_f32_batched(ctx, d.w_out, hidden, m->b_xnorm,
                                  sh.G > 1 ? m->b_logits_loc : logits, M, m->v_loc, d.d_model,
                                  d.output_norm, d.rms_eps, stream);
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

// The exchange that follows segment `seg` on one rank (rows = tokens of the step).
static int phi4_exchange(rrr_phi4* m, int seg, float* hidden, float* logits, int rows,
                         void* stream) {
  if (m->sh.G == 1) return RRR_OK;
  const int L = m->d.n_layers;
  if (seg < 2 * L) return tp_allreduce(m->comm, hidden, (int64_t)rows * m->d.d_model, stream);
  if (seg == 2 * L)
    return tp_allgather_rows(m->comm, logits, rows == 1 ? m->logits_loc : m->b_logits_loc, rows,
                             m->v_loc, stream);
  return RRR_OK;
}

static int phi4_issue(rrr_phi4* m, float* hidden, float* logits, int* argmax, void* stream) {
  int rc;
  for (int seg = 0; seg < phi4_segments(m); ++seg) {
    if ((rc = phi4_issue_seg(m, seg, hidden, logits, argmax, stream))) return rc;
    // (the layers' all-reduces are inside the GEMVs when fused)
    if ((!m->fused || seg >= 2 * m->d.n_layers) &&
        (rc = phi4_exchange(m, seg, hidden, logits, 1, stream)))
      return rc;
  }
  return RRR_OK;
}

static int phi4_issue_batched(rrr_phi4* m, float* hidden, float* logits, int* argmax, int M,
                              void* stream) {
  int rc;
  for (int seg = 0; seg < phi4_segments(m); ++seg)
    if ((rc = phi4_issue_batched_seg(m, seg, hidden, logits, argmax, M, stream)) ||
        (rc = phi4_exchange(m, seg, hidden, logits, M, stream)))
      return rc;
  return RRR_OK;
}

// Scratch rows for a batched forward of M tokens (grown, never shrunk).
static int phi4_batch_scratch(rrr_phi4* m, int M) {
  if (M <= m->b_cap) return RRR_OK;
  const rrr_phi4_desc& d = m->d;
  const size_t qkv_dim = (size_t)m->sh.qkv_dim;
  const size_t qd = (size_t)m->q_loc * d.head_dim;
  auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
  const size_t sz[8] = {al((size_t)M * d.d_model * 2), al((size_t)M * qkv_dim * 4),
                        al((size_t)M * m->sh.o_k * 2), al((size_t)M * qd * 4),
                        al((size_t)M * 2 * m->f_loc * 4), al((size_t)M * m->f_loc * 2),
                        al((size_t)M * d.d_model * 4),
                        m->sh.G > 1 ? al((size_t)M * m->v_loc * 4) : 0};
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
  m->b_xnorm = reinterpret_cast<float*>(p);     p += sz[6];
  m->b_logits_loc = m->sh.G > 1 ? reinterpret_cast<float*>(p) : nullptr;
  m->b_cap = M;
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

// Captures `issue` on the model's capture stream into a new graph (nothing executes).
template <class F>
static int phi4_capture(rrr_phi4* m, F issue, cudaGraph_t* graph, cudaGraphExec_t* exec,
                        const char* what) {
  rrr_ctx* ctx = m->ctx;
  if (!m->cap_stream) {
    cudaError_t e = cudaStreamCreateWithFlags(&m->cap_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return cuda_error(ctx, e, what);
  }
  cudaError_t e = cudaStreamBeginCapture(m->cap_stream, cudaStreamCaptureModeRelaxed);
  if (e != cudaSuccess) return cuda_error(ctx, e, what);
  const int rc = issue(m->cap_stream);
  cudaGraph_t g = nullptr;
  e = cudaStreamEndCapture(m->cap_stream, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) return cuda_error(ctx, e, what);
  e = cudaGraphInstantiate(exec, g, 0);
  if (e != cudaSuccess) {
    cudaGraphDestroy(g);
    *exec = nullptr;
    return cuda_error(ctx, e, what);
  }
  *graph = g;
  return RRR_OK;
}

// Model object for the rank `sh` of a split of `desc` (G = 1: the whole model).
static int phi4_make(rrr_ctx* ctx, const rrr_phi4_desc* desc, const rrr_tp_shard& sh,
                     rrr_tp_comm* comm, rrr_phi4** out) {
  const rrr_phi4_desc& d = *desc;
  if ((d.n_layers > 0 && !d.layers) || !d.output_norm || !d.w_out)
    return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_phi4_create: missing weights");
  for (int l = 0; l < d.n_layers; ++l) {
    const rrr_phi4_layer& L = d.layers[l];
    if (!L.w_qkv || !L.w_o || !L.w_gate_up || !L.w_down || !L.attn_norm || !L.ffn_norm)
      return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_phi4_create: layer %d has a null weight", l);
  }
  const int q_loc = sh.q_head1 - sh.q_head0, kv_loc = sh.kv_head1 - sh.kv_head0;
  rrr_attn_desc ad{};
  if (d.max_seq > 0) {
    ad.n_heads = q_loc;
    ad.n_kv_heads = kv_loc;
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
  m->sh = sh;
  m->comm = comm;
  m->q_loc = q_loc;
  m->kv_loc = kv_loc;
  m->f_loc = sh.ffn1 - sh.ffn0;
  m->v_loc = sh.vocab1 - sh.vocab0;
  if (comm && sh.G > 1 && d.n_layers > 0) {
    rrr_comm* pc = tp_comm_p2p_of(comm);
    unsigned long long* bases[kMaxTpRanks] = {};
    unsigned* epoch = nullptr;
    const int64_t words = pc ? comm_fused(pc, bases, &epoch) : 0;
    const int64_t need = 2ll * d.n_layers * sh.G * d.d_model;
    if (words > 0 && words < need) {
      delete m;
      return set_error(ctx, RRR_ERR_BAD_SHAPE,
                       "rrr_phi4_tp_create: the channel's fused region holds %lld words, the step "
                       "needs 2 * n_layers * world * d_model = %lld",
                       (long long)words, (long long)need);
    }
    if (words > 0) {
      m->fused = true;
      for (int r = 0; r < sh.G; ++r) m->fz_base[r] = bases[r];
      m->fz_epoch = epoch;
    }
  }
  cudaError_t e = cudaMalloc(&m->qkv, (size_t)sh.qkv_dim * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&m->mid, (size_t)m->f_loc * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&m->argmax_scratch, 64);
  if (e == cudaSuccess) e = cudaMemset(m->argmax_scratch, 0, 64);
  if (e == cudaSuccess && sh.G > 1) e = cudaMalloc(&m->logits_loc, (size_t)m->v_loc * sizeof(float));
  if (e == cudaSuccess && d.max_seq > 0) {
    const size_t cache = (size_t)d.max_seq * kv_loc * d.head_dim;
    e = cudaMalloc(&m->kv, 2 * cache * d.n_layers * sizeof(uint16_t) + 16);
    // the O-projection input: the heads' attention output inside the window, zero around it
    if (e == cudaSuccess) e = cudaMalloc(&m->attn, (size_t)sh.o_k * sizeof(float));
    if (e == cudaSuccess) e = cudaMemset(m->attn, 0, (size_t)sh.o_k * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&m->d_pos, 16);
    if (e == cudaSuccess) e = cudaMemset(m->d_pos, 0, 16);
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    rrr_phi4_destroy(m);
    return cuda_error(ctx, e, "rrr_phi4_create: scratch allocation");
  }
  *out = m;
  return RRR_OK;
}

static int phi4_check_dims(rrr_ctx* ctx, const rrr_phi4_desc* desc) {
  const rrr_phi4_desc& d = *desc;
  if (d.d_model <= 0 || d.n_heads <= 0 || d.n_kv_heads <= 0 || d.head_dim <= 0 || d.ffn_dim <= 0 ||
      d.n_layers < 0 || d.vocab <= 0 || d.n_heads % d.n_kv_heads != 0 ||
      d.n_heads * d.head_dim != d.d_model || d.d_model % 256 != 0 || d.ffn_dim % 256 != 0 ||
      d.head_dim % 8 != 0)
    return set_error(ctx, RRR_ERR_BAD_SHAPE,
                     "rrr_phi4_create: need n_heads*head_dim == d_model, d_model and ffn_dim "
                     "multiples of 256, head_dim %% 8 == 0, n_heads %% n_kv_heads == 0");
  return RRR_OK;
}

extern "C" {

int rrr_phi4_create(rrr_ctx* ctx, const rrr_phi4_desc* desc, rrr_phi4** out) {
  if (!ctx) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context");
  if (!desc || !out) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_phi4_create: null argument");
  *out = nullptr;
  int rc = phi4_check_dims(ctx, desc);
  if (rc) return rc;
  const rrr_phi4_desc& d = *desc;
  rrr_tp_shard whole{};
  if ((rc = rrr_tp_plan(d.d_model, d.n_heads, d.n_kv_heads, d.head_dim, d.ffn_dim, d.vocab, 1, 0,
                        &whole)))
    return set_error(ctx, rc, "rrr_phi4_create: %s", rrr_last_error(nullptr));
  return phi4_make(ctx, desc, whole, nullptr, out);
}

int rrr_phi4_tp_create(rrr_ctx* ctx, const rrr_phi4_desc* desc, const rrr_tp_shard* shard,
                       rrr_tp_comm* comm, rrr_phi4** out) {
  if (!ctx) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null context");
  if (!desc || !shard || !out) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_phi4_tp_create: null argument");
  *out = nullptr;
  int rc = phi4_check_dims(ctx, desc);
  if (rc) return rc;
  const rrr_phi4_desc& d = *desc;
  rrr_tp_shard want{};
  if ((rc = rrr_tp_plan(d.d_model, d.n_heads, d.n_kv_heads, d.head_dim, d.ffn_dim, d.vocab, shard->G,
                        shard->g, &want)))
    return set_error(ctx, rc, "rrr_phi4_tp_create: %s", rrr_last_error(nullptr));
  if (memcmp(&want, shard, sizeof want) != 0)
    return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_phi4_tp_create: the shard is not rrr_tp_plan's for rank %d of %d",
                     shard->g, shard->G);
  if (shard->G > kMaxTpRanks)
    return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_phi4_tp_create: at most %d ranks", kMaxTpRanks);
  if (comm && (tp_comm_world(comm) != shard->G || tp_comm_rank(comm) != shard->g))
    return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_phi4_tp_create: the communicator is not rank %d of %d",
                     shard->g, shard->G);
  return phi4_make(ctx, desc, *shard, comm, out);
}

int rrr_phi4_forward(rrr_phi4* m, float* hidden, float* logits, int* argmax_out, int use_graph,
                     void* stream) {
  if (!m) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null model");
  rrr_ctx* ctx = m->ctx;
  if (!hidden || !logits) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_phi4_forward: null buffer");
  if (m->sh.G > 1 && !m->comm)
    return set_error(ctx, RRR_ERR_INVALID_ARG,
                     "rrr_phi4_forward: a tensor-parallel rank needs a communicator (or run it "
                     "through rrr_phi4_tp_forward_emulated)");
  int rc = bind_device(ctx);
  if (rc) return rc;
  if (m->d.max_seq > 0 && m->pos >= m->d.max_seq)
    return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_phi4_forward: position %d is past the cache (%d rows)",
                     m->pos, m->d.max_seq);
  if (use_graph && m->exec && m->g_hidden == hidden && m->g_logits == logits &&
      m->g_argmax == argmax_out) {
    cudaError_t e = cudaGraphLaunch(m->exec, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_phi4_forward: graph launch");
    if (m->d.max_seq > 0) ++m->pos;
    return RRR_OK;
  }
  // the step itself, eagerly (a communicator's first collectives also set it up here,
  // outside any capture)
  rc = phi4_issue(m, hidden, logits, argmax_out, stream);
  if (rc) return rc;
  if (m->d.max_seq > 0) ++m->pos;
  if (!use_graph) return RRR_OK;
  // then the graph for the next calls with these buffers (capture executes nothing; the
  // position is read on the device when the graph runs)
  phi4_drop_graph(m);
  rc = phi4_capture(
      m, [&](cudaStream_t s) { return phi4_issue(m, hidden, logits, argmax_out, s); }, &m->graph,
      &m->exec, "rrr_phi4_forward: capture");
  if (rc) return rc;
  m->g_hidden = hidden;
  m->g_logits = logits;
  m->g_argmax = argmax_out;
  return RRR_OK;
}

int rrr_phi4_forward_batched(rrr_phi4* m, float* hidden, float* logits, int* argmax_out, int M,
                             int use_graph, void* stream) {
  if (!m) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null model");
  rrr_ctx* ctx = m->ctx;
  if (!hidden || !logits) return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_phi4_forward_batched: null buffer");
  if (M < 1) return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_phi4_forward_batched: M >= 1");
  if (m->sh.G > 1 && !m->comm)
    return set_error(ctx, RRR_ERR_INVALID_ARG, "rrr_phi4_forward_batched: a tensor-parallel rank needs a communicator");
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
  // the step itself, eagerly (it also sizes the staging of the exchanges before a capture)
  rc = phi4_issue_batched(m, hidden, logits, argmax_out, M, stream);
  if (rc) return rc;
  if (m->d.max_seq > 0) m->pos += M;
  if (!use_graph) return RRR_OK;
  phi4_drop_batched_graph(m);
  rc = phi4_capture(
      m, [&](cudaStream_t s) { return phi4_issue_batched(m, hidden, logits, argmax_out, M, s); },
      &m->b_graph, &m->b_exec, "rrr_phi4_forward_batched: capture");
  if (rc) return rc;
  m->bg_hidden = hidden;
  m->bg_logits = logits;
  m->bg_argmax = argmax_out;
  m->bg_M = M;
  return RRR_OK;
}

int rrr_phi4_tp_forward_emulated(rrr_phi4* const* ranks, int G, float* const* hidden,
                                 float* const* logits, int* const* argmax, int M, void* stream) {
  if (!ranks || !hidden || !logits || G < 1 || G > kMaxTpRanks)
    return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_phi4_tp_forward_emulated: bad arguments");
  for (int r = 0; r < G; ++r) {
    if (!ranks[r] || !hidden[r] || !logits[r])
      return set_error(nullptr, RRR_ERR_INVALID_ARG, "rrr_phi4_tp_forward_emulated: null entry %d", r);
    const rrr_phi4* m = ranks[r];
    if (m->sh.G != G || m->sh.g != r || m->ctx != ranks[0]->ctx || m->pos != ranks[0]->pos)
      return set_error(nullptr, RRR_ERR_INVALID_ARG,
                       "rrr_phi4_tp_forward_emulated: entry %d is not rank %d of %d of one context at "
                       "one position", r, r, G);
  }
  rrr_phi4* m0 = ranks[0];
  rrr_ctx* ctx = m0->ctx;
  if (M < 0) return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_phi4_tp_forward_emulated: M >= 0");
  const int rows = M > 0 ? M : 1;
  if (m0->d.max_seq > 0 && m0->pos + rows > m0->d.max_seq)
    return set_error(ctx, RRR_ERR_BAD_SHAPE, "rrr_phi4_tp_forward_emulated: positions past the cache");
  int rc = bind_device(ctx);
  if (rc) return rc;
  if (M > 0)
    for (int r = 0; r < G; ++r)
      if (M > ranks[r]->b_cap) {
        phi4_drop_batched_graph(ranks[r]);
        if ((rc = phi4_batch_scratch(ranks[r], M))) return rc;
      }
  const LaunchEnv env = make_env(ctx, stream);
  const int L = m0->d.n_layers;
  float* hs[kMaxTpRanks];
  float* outs[kMaxTpRanks];
  const float* parts[kMaxTpRanks];
  for (int r = 0; r < G; ++r) {
    hs[r] = hidden[r];
    outs[r] = logits[r];
    parts[r] = M > 0 ? ranks[r]->b_logits_loc : ranks[r]->logits_loc;
  }
  for (int seg = 0; seg < phi4_segments(m0); ++seg) {
    for (int r = 0; r < G; ++r) {
      int* am = argmax ? argmax[r] : nullptr;
      rc = M > 0 ? phi4_issue_batched_seg(ranks[r], seg, hidden[r], logits[r], am, M, stream)
                 : phi4_issue_seg(ranks[r], seg, hidden[r], logits[r], am, stream);
      if (rc) return rc;
    }
    if (G == 1) continue;
    cudaError_t e = cudaSuccess;
    if (seg < 2 * L)
      e = launch_local_allreduce(env, hs, G, (int64_t)rows * m0->d.d_model);
    else if (seg == 2 * L)
      e = launch_local_allgather_rows(env, parts, outs, G, rows, m0->v_loc);
    if (e != cudaSuccess) return cuda_error(ctx, e, "rrr_phi4_tp_forward_emulated: exchange");
  }
  if (m0->d.max_seq > 0)
    for (int r = 0; r < G; ++r) ranks[r]->pos += rows;
  return RRR_OK;
}

int rrr_phi4_launches_per_step(rrr_phi4* m, int* n) {
  if (!m || !n) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null argument");
  const int chunk = m->d.logits_chunk_rows > 0 ? m->d.logits_chunk_rows : m->v_loc;
  const int L = m->d.n_layers;
  *n = (m->d.max_seq > 0 ? 5 : 4) * L + (m->v_loc + chunk - 1) / chunk + (m->d.max_seq > 0 ? 1 : 0);
  // the peer-memory exchanges are kernels of this library (NCCL's are not counted); fused:
  // the last site's sum, the epoch advance and the logits all-gather
  if (m->sh.G > 1 && m->comm && tp_comm_is_p2p(m->comm))
    *n += m->fused ? 3 : 2 * L + 1;
  return RRR_OK;
}

int rrr_phi4_tp_fused(rrr_phi4* m, int* fused) {
  if (!m || !fused) return set_error(nullptr, RRR_ERR_INVALID_ARG, "null argument");
  *fused = m->fused ? 1 : 0;
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
  const size_t cache = (size_t)m->d.max_seq * m->kv_loc * m->d.head_dim;
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
  if (m->logits_loc) cudaFree(m->logits_loc);
  if (m->argmax_scratch) cudaFree(m->argmax_scratch);
  if (m->kv) cudaFree(m->kv);
  if (m->attn) cudaFree(m->attn);
  if (m->d_pos) cudaFree(m->d_pos);
  delete m;
  return RRR_OK;
}

}  // extern "C"
