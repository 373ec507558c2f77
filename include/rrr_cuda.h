/*
 * rrr_cuda.h — C ABI of the B200 (sm_100a) weight-path kernels for Recursive Routing
 * Racer (RRR, Peterc3-dev/recursive-routing-racer-rs).
 *
 * This header replaces RRR's Vulkan `ComputeEngine` (src/gpu/engine.rs:15-29) and the
 * weight-path dispatch helpers built on it (src/model/phi4.rs:631-697, 1081-1096,
 * src/gpu/ops.rs:65-84). A Rust host binds it with a thin `extern "C"` block; Python
 * binds it with ctypes. Every citation below is a file:line in the reference project.
 *
 * Conventions (all entry points):
 *   - Return 0 (RRR_OK) on success and a negative rrr_status on failure. Nothing panics
 *     or throws across the ABI. rrr_last_error(ctx) returns a message for the last
 *     failure on that context (thread-local per context use; one host thread at a time).
 *   - Weight, activation and output pointers are DEVICE pointers unless a name says
 *     "host". K-quant weights are raw GGUF super-blocks (Q4_K 144 B, Q5_K 176 B,
 *     Q6_K 210 B per 256 elements), row-major: row n's K/256 blocks are contiguous at
 *     byte offset n*(K/256)*block_bytes. No repacking (the reference's repack_q*k,
 *     src/model/phi4.rs:278-436, is not needed).
 *   - Kernels are asynchronous on the given `stream` (a cudaStream_t passed as void*;
 *     NULL = the legacy default stream). The caller synchronises (rrr_sync).
 *   - qtype uses GGUF type ids: 12 = Q4_K, 13 = Q5_K, 14 = Q6_K (phi4.rs:154-156).
 */
#ifndef RRR_CUDA_H
#define RRR_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RRR_ABI_VERSION 1

typedef enum rrr_status {
  RRR_OK = 0,
  RRR_ERR_INVALID_ARG = -1,  /* null pointer, bad count, unknown name */
  RRR_ERR_BAD_QTYPE = -2,    /* qtype not 12/13/14 */
  RRR_ERR_BAD_SHAPE = -3,    /* K % 256 != 0, K or N out of the supported range */
  RRR_ERR_MISALIGNED = -4,   /* pointer alignment rule violated */
  RRR_ERR_CUDA = -5,         /* a CUDA runtime call failed */
  RRR_ERR_NCCL = -6,         /* an NCCL call failed or NCCL is unavailable */
  RRR_ERR_TIMEOUT = -7,      /* a bounded device-side wait gave up (kernel error flag) */
  RRR_ERR_OOM = -8,          /* device allocation failed */
  RRR_ERR_UNSUPPORTED = -9,  /* known operation that this build does not implement */
  RRR_ERR_IO = -10,          /* file open / mmap / parse failure (GGUF) */
  RRR_ERR_BUFFER_TOO_SMALL = -11 /* a buffer size given to a dispatch is too small */
} rrr_status;

enum { RRR_Q4_K = 12, RRR_Q5_K = 13, RRR_Q6_K = 14 };

typedef struct rrr_ctx rrr_ctx;

/* ---- context, memory, streams (replaces ComputeEngine::new / alloc_buffer /
 *      upload / download: engine.rs:49-128, 200-229; phi4.rs:616-626) ---------------- */

/* Create a context on CUDA device `device`. Fails with RRR_ERR_CUDA if no device. */
int rrr_init(int device, rrr_ctx** out);
/* Destroy a context (frees its internal buffers; user allocations must be freed first). */
int rrr_destroy(rrr_ctx* ctx);
/* Message of the last failure on this context ("" if none). ctx may be NULL: then the
 * message of the last failure of a call that had no context (e.g. rrr_init). */
const char* rrr_last_error(rrr_ctx* ctx);
/* Name of a status code. */
const char* rrr_status_string(int status);
int rrr_abi_version(void);

int rrr_alloc(rrr_ctx* ctx, size_t bytes, void** dptr);  /* 256-B aligned device memory */
int rrr_free(rrr_ctx* ctx, void* dptr);
int rrr_alloc_host(rrr_ctx* ctx, size_t bytes, void** hptr);  /* pinned host memory */
int rrr_free_host(rrr_ctx* ctx, void* hptr);
int rrr_h2d(rrr_ctx* ctx, void* dst_dev, const void* src_host, size_t bytes, void* stream);
int rrr_d2h(rrr_ctx* ctx, void* dst_host, const void* src_dev, size_t bytes, void* stream);
int rrr_d2d(rrr_ctx* ctx, void* dst_dev, const void* src_dev, size_t bytes, void* stream);
int rrr_memset(rrr_ctx* ctx, void* dst_dev, int value, size_t bytes, void* stream);
int rrr_sync(rrr_ctx* ctx, void* stream);
/* Reads and clears the context's device error flag, which kernels set when a bounded
 * wait gives up (codes 1-5: RRR_ERR_TIMEOUT) or meet a position outside the KV cache /
 * a token id outside the embedding table (code 6: RRR_ERR_BAD_SHAPE). Synchronises the
 * device. *code = 0 if no kernel reported an error. */
int rrr_check_device_error(rrr_ctx* ctx, int* code);
/* Limit of every bounded device-side wait of this context's kernels (bulk-copy and ring
 * barriers, peer flags of the exchanges), in ns; 0 restores the default of 1 s. A wait
 * that runs out records its code in the device error flag and the kernel returns, so
 * rrr_check_device_error reports RRR_ERR_TIMEOUT and the context stays usable. Range
 * [1e5, 6e10] ns. No reference counterpart (the reference's fence waits are unbounded,
 * engine.rs:312,369). */
int rrr_set_wait_limit(rrr_ctx* ctx, uint64_t ns);
/* Device-side timeline of the single-token K-quant GEMVs (tracing; the reference has none).
 * With `bytes` of device memory set, every GEMV launch of this context (rrr_gemv_kq*,
 * named dispatches, prebuilt tables, the decode steps) is given one 64-byte record per CTA,
 * assigned on the host at launch or capture time, round-robin over the buffer (a launch
 * that does not fit in the rest of the buffer starts again at record 0; a graph replays
 * into the records of its capture). u64 fields, %globaltimer ns: [0] CTA start, [1] first
 * weight copy issued, [2] grid dependency resolved, [3] GEMV input prepared, [4] rows
 * stored, [5] last weight copy issued, [6] qtype << 56 | K << 28 | N, [7] launch sequence
 * number << 16 | CTA index. buffer = NULL turns it off (the default). */
int rrr_set_trace(rrr_ctx* ctx, void* buffer, int64_t bytes);
/* The next record the tracer will assign and the GEMV launches traced since rrr_set_trace. */
int rrr_trace_position(rrr_ctx* ctx, int64_t* next_record, int64_t* launches);
/* Programmatic dependent launch (default on): each kernel of the library may start while
 * the previous kernel on its stream finishes (weights stream early; inputs are read after
 * the grid dependency wait). enable = 0 serialises every launch (a debugging aid). */
int rrr_set_pdl(rrr_ctx* ctx, int enable);
/* Number of streaming multiprocessors of the context's device. */
int rrr_device_sm_count(rrr_ctx* ctx, int* sms);
/* Diagnostic: runs the integer tensor-core fragment-layout check the GEMV relies on
 * (one warp, known operands); *ok = 1 when the device result is exact. No reference
 * counterpart (the reference has no GPU self-tests). */
int rrr_selftest_mma(rrr_ctx* ctx, int* ok);

/* ---- kernel (1): fused raw-block K-quant GEMV, y = W x (+ residual) ------------------
 * Replaces gpu_matmul_kquant / kquant_dispatch (phi4.rs:631-658, 1081-1096) and the
 * `matmul_q{4,5,6}k` / `matmul_gpuq{4,5,6}` shaders they dispatch (push [K, N],
 * workgroups [N,1,1]). W: N rows x K (raw blocks, 16-B aligned base), x: f32[K]
 * (16-B aligned), y: f32[N]. residual: NULL or f32[N]; when given, y = residual + W x
 * (the residual_add shader, phi4.rs:1028,1033, fused). y may alias residual.
 * Supported: K % 256 == 0, 256 <= K <= 16384, N >= 1.
 * With programmatic dependent launch on (the default), the GEMV starts streaming weight
 * blocks before the previous kernel on its stream has finished, so W must not be written
 * by the kernel launched just before it on the same stream. The library's own fills
 * (rrr_fill_*) end with a marker kernel that keeps this rule; a caller that writes
 * weights with its own kernel must synchronise, or launch something between. */
int rrr_gemv_kq(rrr_ctx* ctx, int qtype, const void* w_raw, const float* x, float* y,
                int K, int N, const float* residual, void* stream);

/* Same GEMV with the input produced in the prologue (fusions of the decode step,
 * phi4.rs:1006-1033):
 *   RRR_X_RMSNORM : x_in f32[K], gamma f32[K]; the GEMV input is rms_norm(x_in)*gamma
 *                   (phi4.rs:593-599, `rmsnorm` shader slot before QKV / FFN-up).
 *   RRR_X_SILU_GATE: x_in f32[2K] = [gate; up]; input = silu(gate) * up
 *                   (phi4.rs:601-606, 1359-1378, `silu_gate` shader).
 *   RRR_X_GQA_V   : x_in = qkv f32[n_q*hd + 2*n_kv*hd]; input[h*hd + d] =
 *                   V[(h / (n_q/n_kv))*hd + d] — attention output at position 0
 *                   (seq_len 1: softmax = 1, output = V of the head's KV group;
 *                   `attention` push [seq_len, n_kv, heads_per_kv, head_dim],
 *                   phi4.rs:1120). K = n_q*hd for the whole model. A tensor-parallel
 *                   shard whose heads do not cover whole super-blocks passes the
 *                   super-block window around them: input[k] is the head output at
 *                   k - k_offset for k_offset <= k < k_offset + n_q*hd and 0 elsewhere
 *                   (k_offset % 8 == 0, k_offset + n_q*hd <= K). The window has no
 *                   reference counterpart (the reference runs on one GPU). */
enum { RRR_X_PLAIN = 0, RRR_X_RMSNORM = 1, RRR_X_SILU_GATE = 2, RRR_X_GQA_V = 3 };
typedef struct rrr_gemv_prologue {
  int mode;            /* RRR_X_* */
  const float* gamma;  /* RRR_X_RMSNORM */
  float eps;           /* RRR_X_RMSNORM */
  int n_q_heads, n_kv_heads, head_dim; /* RRR_X_GQA_V */
  int k_offset;        /* RRR_X_GQA_V: first input element of the heads (0: no window) */
} rrr_gemv_prologue;
int rrr_gemv_kq_ex(rrr_ctx* ctx, int qtype, const void* w_raw, const float* x_in,
                   float* y, int K, int N, const float* residual,
                   const rrr_gemv_prologue* pro, void* stream);

/* gate_up GEMV with the SwiGLU epilogue (the `silu_gate` shader fused, phi4.rs:1023,
 * 1368-1373): W has 2F rows [gate; up] (the Phi-3 ffn_up layout), y f32[F] =
 * silu(W_gate . x_in) * (W_up . x_in), silu(g) = g / (1 + e^-g). pro: NULL, RRR_X_PLAIN or
 * RRR_X_RMSNORM. No residual. */
int rrr_gemv_kq_swiglu(rrr_ctx* ctx, int qtype, const void* w_raw, const float* x_in,
                       float* y, int K, int F, const rrr_gemv_prologue* pro, void* stream);

/* Bit-exact dequantisation of n_blocks raw blocks to f32 (n_blocks*256 values), the
 * reference's CPU dequant_q4_k / dequant_q5_k / dequant_q6_k (phi4.rs:481-542, 444-479)
 * on the GPU, with no FMA contraction. */
int rrr_dequant_kq(rrr_ctx* ctx, int qtype, const void* w_raw, float* out,
                   int64_t n_blocks, void* stream);

/* ---- kernel (2): batched-token K-quant GEMM, Y[M,N] = X[M,K] W^T (f32 out) ----------
 * Replaces the `matmul_gpuq{4,5,6}_batch` dispatches (push [K, N, M], workgroups
 * [N, M, 1], phi4.rs:1257-1268, 1346-1357, 1380-1391). X is bf16 [M,K] row-major
 * (uint16 bit patterns). Tensor cores: register-level mma.sync for 3 <= M <= 64 when
 * every weight row is a multiple of 16 bytes, tcgen05 otherwise from M = 16; M <= 2 (and
 * M < 16 with unaligned rows) runs the GEMV kernel once per token. */
int rrr_gemm_kq_batched(rrr_ctx* ctx, int qtype, const void* w_raw, const uint16_t* x_bf16,
                        float* y, int M, int K, int N, void* stream);

/* Same with an optional f32 residual [M, N] added in the epilogue (may equal y), for the
 * residual adds of the batched decode step (phi4.rs:1393-1403, done on the CPU there). */
int rrr_gemm_kq_batched_ex(rrr_ctx* ctx, int qtype, const void* w_raw, const uint16_t* x_bf16,
                           float* y, int M, int K, int N, const float* residual, void* stream);
/* The same GEMM with the kernel chosen explicitly (tests, benchmarks): RRR_GEMM_AUTO is
 * rrr_gemm_kq_batched_ex's choice (mma.sync for 3 <= M <= 64 when every weight row is a
 * multiple of 16 bytes, the integer mma.sync kernel there when K <= 1024, tcgen05 for
 * larger M or unaligned rows from M = 16, one GEMV per token otherwise); the others force
 * one kernel (mma.sync takes 1 <= M <= 64, tcgen05
 * M >= 16) and fail with RRR_ERR_BAD_SHAPE where it does not apply. RRR_GEMM_MMA_I8 is
 * the integer mma.sync kernel (raw quants against int8 digits of X, 1 <= M <= 64, rows of
 * a multiple of 16 bytes); it prepares the digits in the context's scratch buffer, so two
 * of its calls on one context must not run concurrently on different streams. */
enum {
  RRR_GEMM_AUTO = 0,
  RRR_GEMM_TCGEN05 = 1,
  RRR_GEMM_MMA = 2,
  RRR_GEMM_PER_TOKEN = 3,
  RRR_GEMM_MMA_I8 = 4
};
int rrr_gemm_kq_batched_path(rrr_ctx* ctx, int qtype, const void* w_raw, const uint16_t* x_bf16,
                             float* y, int M, int K, int N, const float* residual, int path,
                             void* stream);

/* ---- batched decode-step glue (M tokens, each at position 0) -----------------------
 * Producers of the bf16 GEMM inputs (phi4.rs:1198-1445 computes these per token on the
 * CPU): rmsnorm rows -> bf16; the position-0 attention output V of each head's KV group
 * from qkv rows [n_q*hd | n_kv*hd | n_kv*hd] into a k_window-wide bf16 row, zero outside
 * [k_offset, k_offset + n_q*hd) (the tensor-parallel window, see RRR_X_GQA_V); SiLU(gate)*up
 * rows ([gate | up] f32 [rows, 2F]) -> bf16 [rows, F]. The batched logits normalise the M
 * rows (gamma != NULL, into x_norm f32 [M, K]) and multiply by the row-major [V, K] f32
 * matrix with one cuBLAS SGEMM (a plain library GEMM): y f32 [M, V]. */
int rrr_rmsnorm_bf16(rrr_ctx* ctx, const float* x, const float* gamma, uint16_t* y, int rows,
                     int d, float eps, void* stream);
int rrr_gqa_v_bf16(rrr_ctx* ctx, const float* qkv, uint16_t* y, int rows, int n_q, int n_kv,
                   int head_dim, int k_window, int k_offset, void* stream);
int rrr_silu_gate_bf16(rrr_ctx* ctx, const float* gu, uint16_t* y, int rows, int F, void* stream);
/* y[m][k] = bf16(x[m][k - k_offset]) for k - k_offset in [0, n), 0 elsewhere in
 * [0, k_window): a rank's attention output [rows, n] placed in its O-projection window. */
int rrr_window_bf16(rrr_ctx* ctx, const float* x, uint16_t* y, int rows, int n, int k_window,
                    int k_offset, void* stream);
/* Logits of M rows (the batched prefill's logits, phi4.rs:1408-1434): x_norm[m] =
 * rms_norm(x[m]) * gamma (gamma NULL: x used as is), then y[m][v] = W[v] . x_norm[m] for a
 * row-major f32 [V, K] W, on the tcgen05 tensor cores with three tf32 products per element
 * pair (3xTF32: W and x split into a tf32 part and an f32 remainder; the dropped
 * remainder-by-remainder product is 2^-22 of the product), so the result carries f32-level
 * accuracy; W is streamed once per 128 rows of x. K % 4 == 0; W and the GEMM input
 * (x_norm with gamma, else x) 16-byte aligned (RRR_ERR_MISALIGNED otherwise). */
int rrr_logits_f32_batched(rrr_ctx* ctx, const float* W, const float* x, float* x_norm, float* y,
                           int M, int V, int K, const float* gamma, float eps, void* stream);

/* ---- kernel (3): RMSNorm, y = gamma * x / sqrt(mean(x^2) + eps), `rows` rows of d ---
 * Replaces gpu_rmsnorm / the `rmsnorm` shader (phi4.rs:680-697, push [num_rows, d]). */
int rrr_rmsnorm(rrr_ctx* ctx, const float* x, const float* gamma, float* y, int rows,
                int d, float eps, void* stream);

/* ---- kernel (4): F32 logits GEMV over the vocab, y[v] = sum_k W[v,k] x[k] ----------
 * Replaces the logits `matmul_tiled` chunks (phi4.rs:866-893, 1049-1064). W is
 * row-major [V, K] f32 (16-B aligned); the vocab is processed in chunks of chunk_rows
 * (0 = one launch). gamma != NULL fuses the output RMSNorm (phi4.rs:1043-1047):
 * the GEMV input is rms_norm(x)*gamma with eps. K % 4 == 0, K <= 16384. */
int rrr_logits_f32(rrr_ctx* ctx, const float* W, const float* x, float* y, int V, int K,
                   int chunk_rows, const float* gamma, float eps, void* stream);

/* Decode glue (phi4.rs:601-610, shaders silu_gate / residual_add, phi4.rs:736-737). */
int rrr_silu_gate(rrr_ctx* ctx, const float* gate_up, float* out, int F, void* stream);
int rrr_residual_add(rrr_ctx* ctx, const float* a, const float* b, float* out, int n,
                     void* stream);
/* Greedy argmax over f32[n] (replaces the CPU scan, phi4.rs:1172-1183). First index
 * wins on ties, NaN is never selected. out_index: device int32[1]. */
int rrr_argmax_f32(rrr_ctx* ctx, const float* x, int n, int* out_index, void* stream);

/* Allocation-free argmax (no counterpart in the reference). For callers that cannot
 * allocate device memory — a host whose memory is fully reserved by its own caching
 * allocator, code running inside a stream capture it does not own (cudaMalloc is not
 * allowed there), latency-critical paths that cannot afford cudaMalloc's implicit
 * synchronisation — and so cannot create a context: takes no context, calls no
 * cudaMalloc / cudaFree, and uses a fixed file-scope device scratch array (16 KB on every
 * GPU that loads this library, until the process exits). Same result as rrr_argmax_f32.
 * Limit: 1 <= n <= 8,388,608 (larger n is rejected with RRR_ERR_BAD_SHAPE). The first
 * call in a CUDA context looks up the scratch array's device address (cached per
 * context, so a context created again after cudaDeviceReset gets a fresh lookup); make
 * that first call before any stream capture. Every call shares the scratch array, so calls that overlap
 * on the GPU (concurrent streams) race; serialise them. Errors: rrr_last_error(NULL). */
int rrr_argmax_f32_noalloc(const float* x, int n, int* out_index, void* stream);

/* f32 GEMM C[M,N] = A[M,K] B[K,N] with B in the reference's transposed chunk layout
 * ([K, N] row-major, phi4.rs:874-893); the `matmul_tiled` / `matmul_reg_tiled`
 * shaders (push [M, K, N], ops.rs:65-84). */
int rrr_matmul_f32(rrr_ctx* ctx, const float* A, const float* B, float* C, int M, int K,
                   int N, void* stream);

/* ---- named dispatch (replaces ComputeEngine::dispatch_by_name, engine.rs:476-554) ---
 * `name` is a reference shader name; buffers/sizes follow its bindings and push
 * constants its push layout:
 *   matmul_q4k | matmul_q5k | matmul_q6k   bufs [x, W, y]            push u32[K, N]
 *   matmul_q4k_batch | _q5k_ | _q6k_batch  bufs [X(bf16), W, Y]      push u32[K, N, M]
 *   rmsnorm                                 bufs [x, gamma, y]        push u32[rows, d]
 *   matmul_tiled | matmul_reg_tiled         bufs [A, B, C]            push u32[M, K, N]
 *   silu_gate                               bufs [gate_up, out]       push u32[F]
 *   residual_add                            bufs [a, b, out]          push u32[n]
 * Sizes are byte sizes of each binding (checked: RRR_ERR_BUFFER_TOO_SMALL). Names of
 * the reference's repacked-layout shaders (matmul_gpuq*) return RRR_ERR_UNSUPPORTED,
 * as do attention / rope / rope_kv_store / kv_store (outside the weight path).
 * The rmsnorm eps is 1e-5 (phi4.rs:111). */
int rrr_dispatch_by_name(rrr_ctx* ctx, const char* name, void* const* buffers,
                         const uint64_t* sizes, int n_buffers, const void* push,
                         int push_bytes, void* stream);

/* ---- prebuilt dispatch table as a CUDA graph (replaces pre_allocate_desc_set +
 *      dispatch_batch_persistent_v2, engine.rs:244-268, 317-370; phi4.rs:969-1064) ---- */
typedef struct rrr_batch rrr_batch;
int rrr_batch_create(rrr_ctx* ctx, rrr_batch** out);
/* Append one named dispatch (same arguments as rrr_dispatch_by_name, validated now). */
int rrr_batch_add(rrr_batch* b, const char* name, void* const* buffers,
                  const uint64_t* sizes, int n_buffers, const void* push, int push_bytes);
/* Launch all dispatches in order on `stream` (captured into a CUDA graph on first use). */
int rrr_batch_launch(rrr_batch* b, void* stream);
int rrr_batch_size(rrr_batch* b, int* n);
int rrr_batch_destroy(rrr_batch* b);

/* ---- GGUF loader (replaces GGUFModel, src/model/gguf.rs:125-195) -------------------- */
typedef struct rrr_gguf rrr_gguf;
typedef struct rrr_gguf_tensor {
  const char* name;
  int n_dims;
  uint64_t shape[4];   /* ne0 (contiguous) first */
  uint32_t type;       /* GGML type id */
  uint64_t offset;     /* relative to the data section */
  uint64_t n_bytes;    /* byte size by type (gguf.rs:173-195) */
  const void* data;    /* zero-copy pointer into the mapping */
} rrr_gguf_tensor;
int rrr_gguf_open(const char* path, rrr_gguf** out);
int rrr_gguf_close(rrr_gguf* g);
int rrr_gguf_n_tensors(rrr_gguf* g, int64_t* n);
int rrr_gguf_tensor_at(rrr_gguf* g, int64_t index, rrr_gguf_tensor* out);
int rrr_gguf_find_tensor(rrr_gguf* g, const char* name, rrr_gguf_tensor* out);
/* Metadata readers (MetaValue::as_u64 / as_f32 / as_str, gguf.rs:41-62). */
int rrr_gguf_meta_u64(rrr_gguf* g, const char* key, uint64_t* out);
int rrr_gguf_meta_f32(rrr_gguf* g, const char* key, float* out);
int rrr_gguf_meta_str(rrr_gguf* g, const char* key, const char** out);
int rrr_gguf_version(rrr_gguf* g, uint32_t* version);
int rrr_gguf_data_offset(rrr_gguf* g, uint64_t* off);
/* Copy one tensor's raw bytes from the mapping to a new device buffer (raw, no repack;
 * the weight upload of load_weight_gpu, phi4.rs:744-771, without repack_q*k): one
 * rrr_gguf_load of one tensor. Free *dptr with rrr_free. */
int rrr_gguf_upload(rrr_ctx* ctx, rrr_gguf* g, const char* name, void** dptr,
                    uint64_t* n_bytes);
/* Upload n tensors into ONE new device allocation (each 256-byte aligned, in the order
 * given): dptrs[i] receives tensor i's device address (dptrs[0] is the allocation: free it
 * with rrr_free to release all), n_bytes[i] (may be NULL) its size, *seconds (may be NULL)
 * the wall time. The bytes go from the mapping into two reusable pinned buffers (32 MB,
 * filled by 8 host threads) and from there to the device with cudaMemcpyAsync on the
 * file's copy stream, each DMA overlapping the host copy of the next chunk; the call
 * returns when the data is on the device. Replaces load_weight_gpu's per-tensor upload
 * into mapped memory (phi4.rs:744-771). The staging stays with the file (rrr_gguf_close
 * frees it) and serves one device. */
int rrr_gguf_load(rrr_ctx* ctx, rrr_gguf* g, const char* const* names, int n, void** dptrs,
                  uint64_t* n_bytes, double* seconds);

/* ---- decode attention at real positions (per-layer glue between the QKV and the
 *      O-projection GEMVs of forward_gpu / forward_dynamic: phi4.rs:1115-1121,
 *      1284-1309, 1656-1690) ------------------------------------------------------
 * RoPE as apply_rope_cfg (phi4.rs:238-256), the f16 KV cache of max_seq rows per layer
 * (MAX_SEQ = 2048, phi4.rs:181, 897-904) and GQA decode attention. */
typedef struct rrr_attn_desc {
  int n_heads, n_kv_heads, head_dim;  /* head_dim 64/128/256; n_heads / n_kv_heads <= 8 */
  int rope_dim;                       /* rotated values per head: even, <= head_dim, <= 128 */
  float rope_theta;                   /* rope.freq_base (10000 for Phi-4-mini) */
  float rope_attn_factor;             /* rope.scaling.attn_factor (1.190238; 1 = standard) */
  const float* rope_factors;          /* device f32[n_rope_factors] (rope_factors_short) or NULL */
  int n_rope_factors;                 /* pair i uses factor i, 1 past the table */
  int max_seq;                        /* rows of each cache */
} rrr_attn_desc;
/* Row t of qkv (f32 [rows][row_stride]: Q | K | V of n_q + 2 n_kv heads) is the token at
 * position p + t, p = *d_pos (a device int read when the kernel runs, so that a captured
 * step replays at any position) or pos0 when d_pos is NULL. RoPE on its Q and K heads in
 * place (pair (2i, 2i+1), i < rope_dim/2, same operations as apply_rope_cfg); K and V
 * rounded to f16 (nearest even) into row p + t of k_cache / v_cache (f16
 * [max_seq][n_kv*head_dim], 16-byte aligned). Positions outside [0, max_seq): rejected
 * (pos0) or recorded in the device error flag with nothing written (d_pos). */
int rrr_rope_kv_store(rrr_ctx* ctx, const rrr_attn_desc* a, float* qkv, int64_t row_stride,
                      int rows, int pos0, const int* d_pos, uint16_t* k_cache,
                      uint16_t* v_cache, void* stream);
/* out[t][h*hd + e] = sum over s in [0, p + t] of softmax_s(q[t]_h . k[s]_g / sqrt(hd)) *
 * v[s]_g[e], g = h / (n_q / n_kv) (causal: row t sees the rows stored up to its own
 * position). q: rows of q_stride floats whose first n_q*hd values are the query heads
 * (the Q part of QKV rows: q = qkv, q_stride = the QKV row stride). out f32 [rows][n_q*hd]. */
int rrr_attention_f16kv(rrr_ctx* ctx, const rrr_attn_desc* a, const float* q, int64_t q_stride,
                        int rows, int pos0, const int* d_pos, const uint16_t* k_cache,
                        const uint16_t* v_cache, float* out, void* stream);
/* One token, fused: RoPE of its query heads (in shared memory; qkv is not modified), its
 * K (rotated) and V rows stored into the caches at position p, then attention over rows
 * 0..p. Same results as rrr_rope_kv_store followed by rrr_attention_f16kv for rows = 1,
 * in one launch (the decode step's path). qkv: one f32 QKV row. */
int rrr_rope_attention_f16kv(rrr_ctx* ctx, const rrr_attn_desc* a, const float* qkv, int pos0,
                             const int* d_pos, uint16_t* k_cache, uint16_t* v_cache, float* out,
                             void* stream);
/* *d_pos += delta on the stream, after the kernels before it (the KVCache.len += 1 of the
 * reference's decode loop for a device-resident position; capturable in a CUDA graph). */
int rrr_position_advance(rrr_ctx* ctx, int* d_pos, int delta, void* stream);
/* Embedding rows (Phi4Model::embed on the table dequantised by dequant_tensor_f32,
 * phi4.rs:709, 572-587, 2085-2089): out[t] = row tokens[t] of an [n_rows, d] table stored
 * as GGUF type ggml_type (0 F32, 1 F16, 6 Q5_0, 8 Q8_0, 12 Q4_K, 13 Q5_K, 14 Q6_K; d a
 * multiple of the type's block), dequantised bit-exactly on the fly. tokens: device
 * int32[n_tokens]; an id outside [0, n_rows) gives a zero row and sets the device error
 * flag (the reference panics on the slice). */
int rrr_embed_rows(rrr_ctx* ctx, int ggml_type, const void* table, int64_t n_rows, int d,
                   const int32_t* tokens, int n_tokens, float* out, void* stream);

/* ---- Phi-4-mini-shape decode step (replaces forward_gpu, phi4.rs:1099-1196) --------
 * max_seq == 0: one token at position 0 (attention output = V, see RRR_X_GQA_V): per layer
 *   h += Wo . expand(V(Wqkv . rms(h)*g_attn)); h += Wdown . (silu(g) * u),
 *   [g; u] = Wgate_up . rms(h)*g_ffn; then logits = Wout . rms(h)*g_out.
 * max_seq > 0: one token at the model's current position p (forward_dynamic,
 * phi4.rs:1593-1760): after the QKV GEMV, RoPE + the f16 KV store at row p and
 * attention over rows 0..p (rrr_rope_attention_f16kv, one launch) give the
 * O-projection's input; the model owns the caches (2 x n_layers x max_seq x n_kv*hd f16)
 * and a device position that starts at 0 and advances by one per forward.
 * All pointers are device pointers that the caller owns and keeps alive. */
typedef struct rrr_phi4_layer {
  const void* w_qkv;      int qkv_type;      /* [n_q*hd + 2*n_kv*hd, d] */
  const void* w_o;        int o_type;        /* [d, n_q*hd] */
  const void* w_gate_up;  int gate_up_type;  /* [2*ffn, d] */
  const void* w_down;     int down_type;     /* [d, ffn] */
  const float* attn_norm; /* f32[d] */
  const float* ffn_norm;  /* f32[d] */
} rrr_phi4_layer;
typedef struct rrr_phi4_desc {
  int d_model, n_heads, n_kv_heads, head_dim, ffn_dim, n_layers, vocab;
  float rms_eps;
  int logits_chunk_rows;        /* 0 = whole vocab per launch */
  const rrr_phi4_layer* layers; /* n_layers entries (copied) */
  const float* output_norm;     /* f32[d] */
  const float* w_out;           /* f32 [vocab, d] row-major */
  int max_seq;                  /* 0: position-0 step; > 0: KV-cache decode */
  int rope_dim;                 /* KV-cache decode: RoPE of rrr_attn_desc */
  float rope_theta, rope_attn_factor;
  const float* rope_factors;    /* device f32[n_rope_factors] or NULL */
  int n_rope_factors;
} rrr_phi4_desc;
typedef struct rrr_phi4 rrr_phi4;
int rrr_phi4_create(rrr_ctx* ctx, const rrr_phi4_desc* desc, rrr_phi4** out);
/* hidden: device f32[d], updated in place (the residual stream); logits: device
 * f32[vocab]; argmax_out: NULL or device int32[1]. use_graph != 0 replays a CUDA graph
 * of the step (captured on the first call for this stream and these pointers). */
int rrr_phi4_forward(rrr_phi4* m, float* hidden, float* logits, int* argmax_out,
                     int use_graph, void* stream);
/* M tokens in one step (Phi4Model::forward_prefill_batched, phi4.rs:1200-1445): hidden
 * device f32 [M][d] (in/out), logits device f32 [M][vocab], argmax_out NULL or device
 * int32[M] (greedy argmax of each row). Every layer GEMM runs on the tensor cores
 * (rrr_gemm_kq_batched; one GEMV per token below 16 rows) on bf16-rounded inputs, so the
 * result is within the batched path's tolerance of the one-token step, not bit-equal.
 * Without a KV cache the M tokens are independent (each at position 0); with one they are
 * consecutive positions p..p+M-1 from the model's position p (a prefill chunk: RoPE, KV
 * store of the M rows, causal attention), and the position advances by M. use_graph != 0:
 * the first call for these pointers and M runs the step and captures it; later calls
 * replay the graph. */
int rrr_phi4_forward_batched(rrr_phi4* m, float* hidden, float* logits, int* argmax_out, int M,
                             int use_graph, void* stream);
/* Number of kernel launches one forward issues. */
int rrr_phi4_launches_per_step(rrr_phi4* m, int* n);
/* KV-cache decode: the position of the next forward (the KVCache.len of the reference;
 * 0 after create). set_position moves it (0 <= pos < max_seq; cache rows >= pos are
 * overwritten as decoding proceeds); position reads the host-side copy. */
int rrr_phi4_set_position(rrr_phi4* m, int pos, void* stream);
int rrr_phi4_position(rrr_phi4* m, int* pos);
/* KV-cache decode: the device caches of one layer (f16 [max_seq][n_kv*hd]). */
int rrr_phi4_kv_cache(rrr_phi4* m, int layer, uint16_t** k_cache, uint16_t** v_cache);
int rrr_phi4_destroy(rrr_phi4* m);

/* ---- exchanges between the GPUs of one box (tensor-parallel decode step) ------------
 * No reference counterpart (the reference runs on one GPU). One process per GPU; every
 * rank creates its exchange buffer, passes its 64-byte CUDA IPC handle to the other
 * ranks (any host channel: torch.distributed, a file, MPI) and connects with all
 * world handles in rank order. The exchanges then run as one kernel over NVLink peer
 * memory (peer stores of values tagged with the call's epoch in one 8-byte word, the
 * receiver waiting on the words themselves; no NCCL), capturable in CUDA graphs:
 *   all-reduce: x[i] = sum over ranks in rank order (identical bits on every rank; from
 *     4 ranks, exchanges of n * (world - 2) * 8 >= 2 MB bytes take two trips: each slice
 *     summed by its owner rank, the sums sent back; the environment variable
 *     RRR_COMM_TWO_TRIP=1 / 0 forces two trips for every all-reduce / for none),
 *   all-gather: out[r*n + i] = rank r's part[i] (part may be out + rank*n).
 * Every rank must issue the same sequence of calls with the same n <= max_elems. A wait
 * that exceeds about a second records an error in the context's device flag. */
typedef struct rrr_comm rrr_comm;
int rrr_comm_create(rrr_ctx* ctx, int rank, int world, int64_t max_elems, rrr_comm** out,
                    void* ipc_handle_out /* 64 bytes */);
/* The same with a fused-exchange region of `fused_words` 8-byte words after the exchange
 * slots, in the same IPC-shared allocation. A tensor-parallel rank made on this channel
 * (rrr_phi4_tp_create) fuses the all-reduces of its one-token step into the GEMVs when the
 * region holds 2 * n_layers * world * d_model words and every peer is on another GPU: the
 * O-projection and down GEMVs push their partial rows, tagged with the step's epoch, into
 * the peers' regions and the next RMSNorm GEMV sums them in rank order in its prologue (the
 * bits of the exchange kernel's all-reduce; no exchange kernels between the GEMVs). The
 * step epoch lives in the channel, so rank models made one after another on it stay in
 * step; one rank model at a time per channel. */
int rrr_comm_create_ex(rrr_ctx* ctx, int rank, int world, int64_t max_elems, int64_t fused_words,
                       rrr_comm** out, void* ipc_handle_out /* 64 bytes */);
int rrr_comm_connect(rrr_comm* comm, const void* ipc_handles /* world x 64 bytes */);
int rrr_comm_allreduce_f32(rrr_comm* comm, float* x, int64_t n, void* stream);
int rrr_comm_allgather_f32(rrr_comm* comm, float* out, const float* part, int64_t n_per_rank,
                           void* stream);
/* All-gather of row-split rows: part f32 [rows, n_per_row] of every rank into
 * out f32 [rows, world * n_per_row] (rank r's row m at out[m][r*n_per_row ...]); out must
 * not overlap part. (rows * n_per_row <= max_elems.) */
int rrr_comm_allgather_rows_f32(rrr_comm* comm, float* out, const float* part, int rows,
                                int64_t n_per_row, void* stream);
/* Unmaps the other ranks' buffers (after this rank's last exchange has completed). Call
 * it on every rank and synchronise the ranks before any rank calls rrr_comm_destroy,
 * which frees this rank's buffer (and disconnects first if needed). */
int rrr_comm_disconnect(rrr_comm* comm);
int rrr_comm_destroy(rrr_comm* comm);

/* ---- tensor-parallel decode step over G GPUs of one box ------
 * No reference counterpart: the reference runs the model on one GPU (forward_gpu,
 * phi4.rs:1099-1196, its dispatch table replayed by dispatch_batch_persistent_v2,
 * engine.rs:317-370). A Rust host that keeps forward_gpu's call pattern replaces the
 * one-GPU rrr_phi4 with one rank of this split per process:
 *   QKV      rows of the rank's query heads [q_head0, q_head1) and of their KV heads
 *            [kv_head0, kv_head1), in Q, K, V order (position-0 attention stays local);
 *   O-proj   the super-block window [o_block0, o_block1) of its K around the heads' columns
 *            (the GEMV input is zero outside the heads, from o_k_offset); partial sums
 *            all-reduced, the residual added by rank 0 only;
 *   gate_up  gate rows [ffn0, ffn1) and the same up rows (SwiGLU local); down the matching
 *            K columns, all-reduced;
 *   logits   vocabulary rows [vocab0, vocab1), all-gathered; argmax replicated.
 * Two all-reduces per layer and one all-gather per step. */
typedef struct rrr_tp_shard {
  int G, g;                 /* ranks, this rank */
  int q_head0, q_head1;     /* query heads */
  int kv_head0, kv_head1;   /* KV heads */
  int qkv_rows[3][2];       /* Q, K, V row ranges of the full QKV matrix */
  int qkv_dim;              /* rows of the rank's QKV shard */
  int o_block0, o_block1;   /* super-block window of the O-projection's K */
  int o_k, o_k_offset;      /* window width (256 per block); first head column in it */
  int ffn0, ffn1;           /* gate / up rows; down's K columns */
  int vocab0, vocab1;       /* logits rows */
} rrr_tp_shard;
/* The shard ranges of rank g of G for a model of these dimensions (host only, no GPU
 * needed). RRR_ERR_BAD_SHAPE when the model does not split G ways: n_heads, n_kv_heads
 * and vocab multiples of G, ffn_dim a multiple of 256*G, n_heads a multiple of n_kv_heads. */
int rrr_tp_plan(int d_model, int n_heads, int n_kv_heads, int head_dim, int ffn_dim, int vocab,
                int G, int g, rrr_tp_shard* out);

/* The exchange channel of one rank. NCCL (loaded at run time: libnccl.so.2, the copy
 * already in the process if there is one): rank 0 creates a 128-byte unique id, the host
 * sends it to every rank (any channel), every rank creates its communicator with it.
 * Peer memory: a connected rrr_comm (not owned; destroy it after this). */
typedef struct rrr_tp_comm rrr_tp_comm;
int rrr_tp_nccl_unique_id(void* id_out /* 128 bytes */);
int rrr_tp_comm_nccl(rrr_ctx* ctx, const void* unique_id, int rank, int world, rrr_tp_comm** out);
int rrr_tp_comm_p2p(rrr_comm* comm, rrr_tp_comm** out);
/* Host-side failure detection: waits for the work issued on `stream` with a deadline,
 * polling the communicator's asynchronous error (NCCL) and the device error flag. On a
 * communicator error the communicator is aborted and RRR_ERR_NCCL is returned; past the
 * deadline it is aborted and RRR_ERR_TIMEOUT is returned (an aborted NCCL communicator
 * refuses further use; recreate it). The reference waits on its fences without a limit
 * (engine.rs:312,369). */
int rrr_tp_wait(rrr_tp_comm* comm, void* stream, int timeout_ms);
int rrr_tp_comm_destroy(rrr_tp_comm* comm);

/* One rank's decode step. desc carries the FULL model's dimensions (d_model, n_heads,
 * n_kv_heads, head_dim, ffn_dim, vocab) and this rank's shard tensors: w_qkv [qkv_dim, d],
 * w_o [d, o_k] (the block window), w_gate_up [2*(ffn1-ffn0), d] (gate rows then up rows),
 * w_down [d, ffn1-ffn0], the norms whole, w_out [vocab1-vocab0, d]. shard must be
 * rrr_tp_plan's for (desc, G, g). comm may be NULL when G == 1 or when the rank is only run
 * through rrr_phi4_tp_forward_emulated. The returned model is driven by rrr_phi4_forward /
 * rrr_phi4_forward_batched / rrr_phi4_set_position / rrr_phi4_destroy like the 1-GPU one
 * (hidden and logits full-size on every rank; the exchanges run inside the step and are
 * captured in its CUDA graph). Every rank must run the same calls in the same order. */
int rrr_phi4_tp_create(rrr_ctx* ctx, const rrr_phi4_desc* desc, const rrr_tp_shard* shard,
                       rrr_tp_comm* comm, rrr_phi4** out);
/* 1 when the one-token step's all-reduces are fused into its GEMVs (rrr_comm_create_ex),
 * else 0. */
int rrr_phi4_tp_fused(rrr_phi4* m, int* fused);
/* All G ranks of one split on the calling process's GPU, run in lockstep with the
 * exchanges done by local kernels (sums in rank order): for checking the split on one GPU.
 * ranks[r] are rrr_phi4_tp_create models of ranks r = 0..G-1 of one context; hidden[r],
 * logits[r], argmax[r] (NULL entries or a NULL array: no argmax) their buffers. M = 0: the
 * one-token step (rrr_phi4_forward); M >= 1: the batched step of M tokens. */
int rrr_phi4_tp_forward_emulated(rrr_phi4* const* ranks, int G, float* const* hidden,
                                 float* const* logits, int* const* argmax, int M, void* stream);

/* ---- seeded synthetic data on the device (bench / tests) --------------------------
 * Blocks follow the distributions of the benchmark configs: d, dmin f16 ~ U[1e-4,1e-2];
 * Q6_K scales int8 ~ U[-32,31]; all other bytes uniform. Block i depends only on
 * (seed, i) through splitmix64, so any row range can be regenerated on the host. */
int rrr_fill_kquant_random(rrr_ctx* ctx, int qtype, void* dst, int64_t n_blocks,
                           uint64_t seed, void* stream);
int rrr_fill_f32_normal(rrr_ctx* ctx, float* dst, int64_t n, float mean, float std,
                        uint64_t seed, void* stream);
int rrr_fill_f32_uniform(rrr_ctx* ctx, float* dst, int64_t n, float lo, float hi,
                         uint64_t seed, void* stream);
/* Sub-ranges of the same streams, for tensor-parallel shards that must equal slices of
 * the full tensors: dst block (r, c), r < rows, c < blocks_per_row, row-major, is generator
 * block block0 + r*src_row_blocks + c of rrr_fill_kquant_random's stream; dst[i] of
 * rrr_fill_f32_range is element offset + i of rrr_fill_f32_normal (normal != 0: a = mean,
 * b = std) or rrr_fill_f32_uniform (a = lo, b = hi). No reference counterpart. */
int rrr_fill_kquant_random_2d(rrr_ctx* ctx, int qtype, void* dst, int64_t rows,
                              int64_t blocks_per_row, int64_t src_row_blocks, int64_t block0,
                              uint64_t seed, void* stream);
int rrr_fill_f32_range(rrr_ctx* ctx, float* dst, int64_t n, int64_t offset, int normal, float a,
                       float b, uint64_t seed, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* RRR_CUDA_H */
