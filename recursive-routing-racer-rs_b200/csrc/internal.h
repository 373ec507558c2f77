// internal.h — host-side launch functions shared between the kernel translation units
// and the C ABI (capi.cpp). Not part of the public interface.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/rrr_cuda.h"

namespace rrr {

// The context's device error block (256 bytes): int [0] is the error flag kernels set, the
// 64-bit word at int index kWaitLimitSlot holds the bounded waits' limit in ns (0 = the
// 1 s default), bytes 64-79 the argmax key and counter.
constexpr int kWaitLimitSlot = 8;

struct LaunchEnv {
  cudaStream_t stream;
  int sm_count;
  int* d_err;  // device error flag of the context
  bool pdl;    // launch with programmatic stream serialisation
  // GEMV timeline of the context (rrr_set_trace; null: off): records, their number, the
  // next free record and the launch counter (host memory of the context)
  unsigned long long* trace = nullptr;
  int64_t trace_cap = 0;
  int64_t* trace_next = nullptr;
  int64_t* trace_seq = nullptr;
};

// Shape limits of the K-quant GEMV (checked by the C ABI before launching).
constexpr int kGemvMaxK = 16384;
constexpr int kMaxTpRanks = 8;

// The tensor-parallel exchange of a decode step fused into its GEMVs (peer-memory channel
// with a fused region, ranks on distinct GPUs). Every exchange site has, in every rank's
// region, one slot of K tagged words (value low, step epoch high) per source rank.
//  * sum_in (prologue, RMSNORM mode): the GEMV input is the sum, in rank order, of the G
//    slots sum_in[r*K ...] once they carry the step's epoch; CTA 0 also stores it to h_out.
//  * push (epilogue, plain output): each finished row, tagged, goes to push[r][row] for
//    r < G (this rank's slot of the site in every rank's region) instead of y; a rank whose
//    device error flag is set pushes nothing, so its peers' waits run out too.
// The step's epoch is *epoch + 1 (read after the preceding kernels have completed).
struct GemvFuse {
  const unsigned long long* sum_in = nullptr;
  float* h_out = nullptr;
  unsigned long long* push[kMaxTpRanks] = {};
  int G = 0;
  const unsigned* epoch = nullptr;
};

// x_early: the input is not written by any kernel this launch can overlap under
// programmatic dependent launch (e.g. a prebuilt table in which no earlier dispatch writes
// it), so the CTAs prepare it before the grid dependency wait; the rows are still stored
// after it.
cudaError_t launch_gemv_kq(const LaunchEnv& env, int qtype, const void* w, const float* x,
                           float* y, int K, int N, const float* residual,
                           const rrr_gemv_prologue* pro, const GemvFuse* fuse = nullptr,
                           bool x_early = false);

// One GEMV: the arguments of launch_gemv_kq (swiglu: of launch_gemv_kq_swiglu, N = F output
// rows of a 2F-row weight).
struct GemvDesc {
  int qtype = 0;
  const void* w = nullptr;
  const float* x = nullptr;
  float* y = nullptr;
  int K = 0, N = 0;
  const float* residual = nullptr;
  rrr_gemv_prologue pro{};  // mode RRR_X_PLAIN
  bool swiglu = false;
  GemvFuse fuse;            // G = 0: no fused exchange
  bool x_early = false;     // see launch_gemv_kq
};
// GEMV with a bf16 input vector (one token of the batched path when M < 16).
cudaError_t launch_gemv_kq_bf16(const LaunchEnv& env, int qtype, const void* w,
                                const uint16_t* x, float* y, int K, int N,
                                const float* residual);
cudaError_t launch_dequant_kq(const LaunchEnv& env, int qtype, const void* w, float* out,
                              int64_t n_blocks);
cudaError_t launch_rmsnorm(const LaunchEnv& env, const float* x, const float* gamma, float* y,
                           int rows, int d, float eps);
cudaError_t launch_logits_f32(const LaunchEnv& env, const float* W, const float* x, float* y,
                              int V, int K, const float* gamma, float eps);
cudaError_t launch_silu_gate(const LaunchEnv& env, const float* gu, float* out, int F);
cudaError_t launch_residual_add(const LaunchEnv& env, const float* a, const float* b,
                                float* out, int n);
// scratch: 16 bytes of zero-initialised device memory (a 64-bit key and a 32-bit counter),
// left zeroed by every completed launch; one launch at a time per scratch slot.
cudaError_t launch_argmax(const LaunchEnv& env, const float* x, int n, int* out_index,
                          void* scratch);
// Greedy argmax of each row of x ([rows] rows of n values, row pitch ld elements).
cudaError_t launch_argmax_rows(const LaunchEnv& env, const float* x, int n, long long ld,
                               int* out_index, int rows);
// gate_up GEMV with the SwiGLU epilogue: W has 2F rows [gate; up], y[i] = silu(gate_i) * up_i.
cudaError_t launch_gemv_kq_swiglu(const LaunchEnv& env, int qtype, const void* w,
                                  const float* x, float* y, int K, int F,
                                  const rrr_gemv_prologue* pro, const GemvFuse* fuse = nullptr);
cudaError_t launch_matmul_f32(const LaunchEnv& env, const float* A, const float* B, float* C,
                              int M, int K, int N);
cudaError_t launch_fill_kquant(const LaunchEnv& env, int qtype, void* dst, int64_t rows,
                               int64_t bpr, int64_t src_row, int64_t block0, uint64_t seed);
cudaError_t launch_fill_f32(const LaunchEnv& env, float* dst, int64_t n, int64_t offset,
                            int normal, float a, float b, uint64_t seed);
cudaError_t launch_bf16_to_f32_rows(const LaunchEnv& env, const uint16_t* x, float* out,
                                    int64_t n);
// Batched-token GEMM on the tensor cores (gemm_kq_tc.cu). plan_gemm_kq_tc picks the tile
// shape, the ring depth and the split-K factor for this GPU; it returns false for shapes
// the kernel does not handle (M < 16).
struct TcPlan {
  int tn;          // tokens per tile (MMA N), multiple of 16, <= 256
  int m_tiles, n_tiles;
  int splits;      // K splits = CTAs per cluster (1..8)
  int stages, smem, tmem_cols;
  int raw_stages;  // raw-block ring depth
  int kbs;         // super-blocks per raw stage
  int raw_tma;     // raw blocks staged by one 2-D TMA box per stage
};
bool plan_gemm_kq_tc(int qtype, int M, int K, int N, int sm_count, TcPlan* plan);
cudaError_t launch_gemm_kq_tc(const LaunchEnv& env, int qtype, const void* w,
                              const uint16_t* x_bf16, float* y, int M, int K, int N,
                              const TcPlan& plan, const float* residual);
// Batched F32 logits Y[M, V] = X[M, K] W[V, K]^T on the tcgen05 tensor cores with three
// tf32 products per K step (logits_tc.cu); K % 4 == 0, W and x 16-byte aligned.
constexpr int kMaxTokTile = 128;  // tokens per tile of that kernel
cudaError_t launch_logits_tc(const LaunchEnv& env, const float* W, const float* x, float* y,
                             int M, int V, int K);
// Self-test of the integer tensor-core fragment layout used by the GEMV (writes 1 to
// *d_ok when the device result matches the expected product).
cudaError_t launch_mma_selftest(const LaunchEnv& env, int* d_ok);

// Batched-token GEMM for 1 <= M <= 64 on mma.sync (gemm_kq_mma.cu): 256-row tiles, the
// weights dequantised into A fragments in registers. plan_gemm_kq_mma returns false for
// shapes it does not handle (M outside [1, 64], rows not 16-byte aligned). The automatic
// choice takes it from kMmaMinTokens tokens (fewer run one GEMV per token).
constexpr int kMmaMinTokens = 3;
struct MmaPlan {
  int tn;          // tokens per tile: M rounded up to 16
  int m_tiles, n_tiles;
  int splits;      // K splits = CTAs per cluster (1..8)
  int stages, smem;
  int kbs;         // super-blocks per stage
};
bool plan_gemm_kq_mma(int qtype, int M, int K, int N, int sm_count, MmaPlan* plan);
cudaError_t launch_gemm_kq_mma(const LaunchEnv& env, int qtype, const void* w,
                               const uint16_t* x_bf16, float* y, int M, int K, int N,
                               const MmaPlan& plan, const float* residual);

// Batched-token GEMM for 1 <= M <= 64 on integer mma.sync (gemm_kq_i8.cu): raw quants as
// the A operand against int8 digits of X, which a preparation kernel writes into `scratch`
// (i8_scratch_bytes(K) bytes; one GEMM at a time per scratch buffer, in stream order).
struct I8Plan {
  int tn;          // tokens per tile: M rounded up to 16
  int m_tiles, n_tiles;
  int splits;      // K splits = CTAs per cluster (1..8)
  int stages, smem;
  int kbs;         // super-blocks per stage
};
size_t i8_digit_bytes(int K);
size_t i8_scratch_bytes(int K);
bool plan_gemm_kq_i8(int qtype, int M, int K, int N, int sm_count, I8Plan* plan);
cudaError_t launch_gemm_kq_i8(const LaunchEnv& env, int qtype, const void* w,
                              const uint16_t* x_bf16, float* y, int M, int K, int N,
                              const I8Plan& plan, const float* residual, void* scratch);

// Decode attention at real positions (attention.cu).
cudaError_t launch_rope_kv_store(const LaunchEnv& env, float* qkv, long long row_stride, int rows,
                                 int pos0, const int* d_pos, int nh, int nkv, int hd, int rope_dim,
                                 float theta, float attn_factor, const float* factors,
                                 int n_factors, uint16_t* kc, uint16_t* vc, int max_seq);
// RoPE parameters of the fused one-token path (rope != null in launch_attention_f16kv):
// q is the token's QKV row; its query heads are rotated in shared memory and its K
// (rotated) and V rows are stored into the caches at the token's position first.
struct AttnRope {
  int rope_dim;
  float theta, attn_factor;
  const float* factors;
  int n_factors;
};
cudaError_t launch_attention_f16kv(const LaunchEnv& env, const float* q, long long q_stride,
                                   int rows, int pos0, const int* d_pos, const uint16_t* kc,
                                   const uint16_t* vc, float* out, int nh, int nkv, int hd,
                                   int max_seq, int seq_max, const AttnRope* rope);
int attention_smem_for(int hd, int hpk, int seq_max);
cudaError_t launch_embed_rows(const LaunchEnv& env, int type, const void* table, long long n_rows,
                              long long row_bytes, int d, const int* tokens, int n_tokens,
                              float* out);
// Exchanges of the one-GPU emulation of a tensor-parallel split (tp_exchange.cu): bufs[r]
// (G <= 8) summed in rank order into every bufs[r]; parts[r] [rows][npr] gathered into
// every outs[r] [rows][G * npr]; and the NCCL row all-gather's reorder, tmp [G][rows][npr]
// -> out [rows][G * npr].
cudaError_t launch_local_allreduce(const LaunchEnv& env, float* const* bufs, int G, int64_t n);
cudaError_t launch_local_allgather_rows(const LaunchEnv& env, const float* const* parts,
                                        float* const* outs, int G, int rows, int64_t npr);
cudaError_t launch_rows_from_ranks(const LaunchEnv& env, const float* tmp, float* out, int G,
                                   int rows, int64_t npr);
// *d_pos += delta after the preceding kernels of the stream have completed.
cudaError_t launch_pos_advance(const LaunchEnv& env, int* d_pos, int delta);
// The end of a step's fused exchanges (tp_exchange.cu): out[i] = sum over ranks, in rank
// order, of slots[r*n + i] once they carry the epoch *epoch + 1 (bounded waits), then
// *epoch += 1 by a second launch once every reader of this step's epoch has completed.
cudaError_t launch_fused_sum(const LaunchEnv& env, const unsigned long long* slots, float* out,
                             int n, int G, const unsigned* epoch);
cudaError_t launch_epoch_advance(const LaunchEnv& env, unsigned* epoch);

}  // namespace rrr
