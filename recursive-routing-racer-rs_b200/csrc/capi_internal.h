// capi_internal.h — the context object and error helpers shared by the C-ABI sources.
#pragma once
#include <cuda_runtime.h>

#include <string>

#include "../../include/rrr_cuda.h"
#include "internal.h"

struct rrr_ctx {
  int device = 0;
  int sm_count = 0;
  int* d_err = nullptr;  // 256 B: [0] device error flag written by kernels whose bounded
                         // waits give up; [64..79] argmax key + counter (kept zeroed)
  bool pdl = true;       // launch kernels with programmatic dependent launch
  // GEMV timeline (rrr_set_trace): device records of 8 u64, the next record and the launch
  // sequence number, assigned on the host at launch (or capture) time
  unsigned long long* trace = nullptr;
  int64_t trace_cap = 0, trace_next = 0, trace_seq = 0;
  // int8 digits of the batched GEMM input (gemm_kq_i8.cu), i8_scratch_bytes(kGemvMaxK) bytes
  void* xdig = nullptr;
  std::string last_error;
  void* argmax_scratch() { return reinterpret_cast<char*>(d_err) + 64; }
};

namespace rrr {
// Records a message for rrr_last_error and returns `code`.
int set_error(rrr_ctx* ctx, int code, const char* fmt, ...);
int cuda_error(rrr_ctx* ctx, cudaError_t e, const char* what);
int bind_device(rrr_ctx* ctx);
LaunchEnv make_env(rrr_ctx* ctx, void* stream);
// Tensor parallelism (tp.cpp): the exchanges of a rank, in-place sum of n floats over the
// ranks and all-gather of `rows` rows of npr floats (part [rows][npr] -> out
// [rows][world * npr]); the peer-memory communicator's parameters.
int tp_comm_world(const rrr_tp_comm* c);
int tp_comm_rank(const rrr_tp_comm* c);
bool tp_comm_is_p2p(const rrr_tp_comm* c);
int tp_allreduce(rrr_tp_comm* c, float* x, int64_t n, void* stream);
int tp_allgather_rows(rrr_tp_comm* c, float* out, const float* part, int rows, int64_t npr,
                      void* stream);
void comm_info(const rrr_comm* c, rrr_ctx** ctx, int* rank, int* world, int64_t* max_elems);
// The fused-exchange regions of every rank of a connected communicator (bases[r]: rank r's,
// mapped into this process) and the step epoch of the fused exchanges (device counter,
// zero at creation); returns the regions' size in 8-byte words, 0 when there is none or a
// peer shares this rank's GPU.
int64_t comm_fused(const rrr_comm* c, unsigned long long** bases, unsigned** epoch);
// The rrr_comm of a peer-memory channel (NULL for NCCL).
rrr_comm* tp_comm_p2p_of(rrr_tp_comm* c);
// Argument rules of one single-token GEMV (rrr_gemv_kq_ex; swiglu: rrr_gemv_kq_swiglu
// with N = F).
int check_gemv(rrr_ctx* ctx, int qtype, const void* w, const float* x, float* y, int K, int N,
               const float* residual, const rrr_gemv_prologue* pro, bool swiglu);
}  // namespace rrr
