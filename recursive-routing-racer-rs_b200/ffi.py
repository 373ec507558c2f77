"""ctypes binding of include/rrr_cuda.h (librrr_cuda.so, built in-tree for sm_100a).

This is the Python side of the C ABI; a Rust host binds the same header with an
`extern "C"` block. Loading fails loudly if the library is missing: there is no fallback
implementation.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_int64, c_size_t, c_uint16, c_uint32, \
    c_uint64, c_void_p

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librrr_cuda.so")

RRR_OK = 0
STATUS = {
    0: "RRR_OK", -1: "RRR_ERR_INVALID_ARG", -2: "RRR_ERR_BAD_QTYPE", -3: "RRR_ERR_BAD_SHAPE",
    -4: "RRR_ERR_MISALIGNED", -5: "RRR_ERR_CUDA", -6: "RRR_ERR_NCCL", -7: "RRR_ERR_TIMEOUT",
    -8: "RRR_ERR_OOM", -9: "RRR_ERR_UNSUPPORTED", -10: "RRR_ERR_IO", -11: "RRR_ERR_BUFFER_TOO_SMALL",
}
Q4_K, Q5_K, Q6_K = 12, 13, 14
X_PLAIN, X_RMSNORM, X_SILU_GATE, X_GQA_V = 0, 1, 2, 3


class RRRError(RuntimeError):
    """A non-zero status from the C ABI (the Rust reference would have panicked)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{STATUS.get(code, code)}: {message}")
        self.code = code


class GemvPrologue(ctypes.Structure):
    _fields_ = [("mode", c_int), ("gamma", c_void_p), ("eps", c_float), ("n_q_heads", c_int),
                ("n_kv_heads", c_int), ("head_dim", c_int), ("k_offset", c_int)]


class GGUFTensor(ctypes.Structure):
    _fields_ = [("name", c_char_p), ("n_dims", c_int), ("shape", c_uint64 * 4), ("type", c_uint32),
                ("offset", c_uint64), ("n_bytes", c_uint64), ("data", c_void_p)]


class Phi4Layer(ctypes.Structure):
    _fields_ = [("w_qkv", c_void_p), ("qkv_type", c_int), ("w_o", c_void_p), ("o_type", c_int),
                ("w_gate_up", c_void_p), ("gate_up_type", c_int), ("w_down", c_void_p),
                ("down_type", c_int), ("attn_norm", c_void_p), ("ffn_norm", c_void_p)]


class Phi4Desc(ctypes.Structure):
    _fields_ = [("d_model", c_int), ("n_heads", c_int), ("n_kv_heads", c_int), ("head_dim", c_int),
                ("ffn_dim", c_int), ("n_layers", c_int), ("vocab", c_int), ("rms_eps", c_float),
                ("logits_chunk_rows", c_int), ("layers", POINTER(Phi4Layer)),
                ("output_norm", c_void_p), ("w_out", c_void_p), ("max_seq", c_int),
                ("rope_dim", c_int), ("rope_theta", c_float), ("rope_attn_factor", c_float),
                ("rope_factors", c_void_p), ("n_rope_factors", c_int)]


class TPShard(ctypes.Structure):
    """rrr_tp_shard (include/rrr_cuda.h): rank g of G's ranges, [start, stop)."""
    _fields_ = [("G", c_int), ("g", c_int), ("q_head0", c_int), ("q_head1", c_int),
                ("kv_head0", c_int), ("kv_head1", c_int), ("qkv_rows", (c_int * 2) * 3),
                ("qkv_dim", c_int), ("o_block0", c_int), ("o_block1", c_int), ("o_k", c_int),
                ("o_k_offset", c_int), ("ffn0", c_int), ("ffn1", c_int), ("vocab0", c_int),
                ("vocab1", c_int)]


class AttnDesc(ctypes.Structure):
    _fields_ = [("n_heads", c_int), ("n_kv_heads", c_int), ("head_dim", c_int), ("rope_dim", c_int),
                ("rope_theta", c_float), ("rope_attn_factor", c_float), ("rope_factors", c_void_p),
                ("n_rope_factors", c_int), ("max_seq", c_int)]


vp = c_void_p
PROTOS = {
    "rrr_abi_version": (c_int, []),
    "rrr_status_string": (c_char_p, [c_int]),
    "rrr_last_error": (c_char_p, [vp]),
    "rrr_init": (c_int, [c_int, POINTER(vp)]),
    "rrr_destroy": (c_int, [vp]),
    "rrr_alloc": (c_int, [vp, c_size_t, POINTER(vp)]),
    "rrr_free": (c_int, [vp, vp]),
    "rrr_alloc_host": (c_int, [vp, c_size_t, POINTER(vp)]),
    "rrr_free_host": (c_int, [vp, vp]),
    "rrr_h2d": (c_int, [vp, vp, vp, c_size_t, vp]),
    "rrr_d2h": (c_int, [vp, vp, vp, c_size_t, vp]),
    "rrr_d2d": (c_int, [vp, vp, vp, c_size_t, vp]),
    "rrr_memset": (c_int, [vp, vp, c_int, c_size_t, vp]),
    "rrr_sync": (c_int, [vp, vp]),
    "rrr_check_device_error": (c_int, [vp, POINTER(c_int)]),
    "rrr_device_sm_count": (c_int, [vp, POINTER(c_int)]),
    "rrr_selftest_mma": (c_int, [vp, POINTER(c_int)]),
    "rrr_gemv_kq": (c_int, [vp, c_int, vp, vp, vp, c_int, c_int, vp, vp]),
    "rrr_gemv_kq_ex": (c_int, [vp, c_int, vp, vp, vp, c_int, c_int, vp, POINTER(GemvPrologue), vp]),
    "rrr_gemv_kq_swiglu": (c_int, [vp, c_int, vp, vp, vp, c_int, c_int, POINTER(GemvPrologue), vp]),
    "rrr_dequant_kq": (c_int, [vp, c_int, vp, vp, c_int64, vp]),
    "rrr_gemm_kq_batched": (c_int, [vp, c_int, vp, vp, vp, c_int, c_int, c_int, vp]),
    "rrr_rmsnorm": (c_int, [vp, vp, vp, vp, c_int, c_int, c_float, vp]),
    "rrr_gemm_kq_batched_ex": (c_int, [vp, c_int, vp, vp, vp, c_int, c_int, c_int, vp, vp]),
    "rrr_rmsnorm_bf16": (c_int, [vp, vp, vp, vp, c_int, c_int, c_float, vp]),
    "rrr_gqa_v_bf16": (c_int, [vp, vp, vp, c_int, c_int, c_int, c_int, c_int, c_int, vp]),
    "rrr_silu_gate_bf16": (c_int, [vp, vp, vp, c_int, c_int, vp]),
    "rrr_logits_f32_batched": (c_int, [vp, vp, vp, vp, vp, c_int, c_int, c_int, vp, c_float, vp]),
    "rrr_logits_f32": (c_int, [vp, vp, vp, vp, c_int, c_int, c_int, vp, c_float, vp]),
    "rrr_silu_gate": (c_int, [vp, vp, vp, c_int, vp]),
    "rrr_residual_add": (c_int, [vp, vp, vp, vp, c_int, vp]),
    "rrr_argmax_f32": (c_int, [vp, vp, c_int, vp, vp]),
    "rrr_argmax_f32_noalloc": (c_int, [vp, c_int, vp, vp]),
    "rrr_matmul_f32": (c_int, [vp, vp, vp, vp, c_int, c_int, c_int, vp]),
    "rrr_dispatch_by_name": (c_int, [vp, c_char_p, POINTER(vp), POINTER(c_uint64), c_int, vp, c_int, vp]),
    "rrr_batch_create": (c_int, [vp, POINTER(vp)]),
    "rrr_batch_add": (c_int, [vp, c_char_p, POINTER(vp), POINTER(c_uint64), c_int, vp, c_int]),
    "rrr_batch_launch": (c_int, [vp, vp]),
    "rrr_batch_size": (c_int, [vp, POINTER(c_int)]),
    "rrr_batch_destroy": (c_int, [vp]),
    "rrr_gguf_open": (c_int, [c_char_p, POINTER(vp)]),
    "rrr_gguf_close": (c_int, [vp]),
    "rrr_gguf_n_tensors": (c_int, [vp, POINTER(c_int64)]),
    "rrr_gguf_tensor_at": (c_int, [vp, c_int64, POINTER(GGUFTensor)]),
    "rrr_gguf_find_tensor": (c_int, [vp, c_char_p, POINTER(GGUFTensor)]),
    "rrr_gguf_meta_u64": (c_int, [vp, c_char_p, POINTER(c_uint64)]),
    "rrr_gguf_meta_f32": (c_int, [vp, c_char_p, POINTER(c_float)]),
    "rrr_gguf_meta_str": (c_int, [vp, c_char_p, POINTER(c_char_p)]),
    "rrr_gguf_version": (c_int, [vp, POINTER(c_uint32)]),
    "rrr_gguf_data_offset": (c_int, [vp, POINTER(c_uint64)]),
    "rrr_gguf_upload": (c_int, [vp, vp, c_char_p, POINTER(vp), POINTER(c_uint64)]),
    "rrr_gguf_load": (c_int, [vp, vp, POINTER(c_char_p), c_int, POINTER(vp), POINTER(c_uint64),
                              POINTER(ctypes.c_double)]),
    "rrr_phi4_create": (c_int, [vp, POINTER(Phi4Desc), POINTER(vp)]),
    "rrr_phi4_forward": (c_int, [vp, vp, vp, vp, c_int, vp]),
    "rrr_phi4_forward_batched": (c_int, [vp, vp, vp, vp, c_int, c_int, vp]),
    "rrr_phi4_launches_per_step": (c_int, [vp, POINTER(c_int)]),
    "rrr_phi4_destroy": (c_int, [vp]),
    "rrr_set_pdl": (c_int, [vp, c_int]),
    "rrr_set_wait_limit": (c_int, [vp, c_uint64]),
    "rrr_tp_plan": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, POINTER(TPShard)]),
    "rrr_tp_nccl_unique_id": (c_int, [vp]),
    "rrr_tp_comm_nccl": (c_int, [vp, vp, c_int, c_int, POINTER(vp)]),
    "rrr_tp_comm_p2p": (c_int, [vp, POINTER(vp)]),
    "rrr_tp_wait": (c_int, [vp, vp, c_int]),
    "rrr_tp_comm_destroy": (c_int, [vp]),
    "rrr_phi4_tp_create": (c_int, [vp, POINTER(Phi4Desc), POINTER(TPShard), vp, POINTER(vp)]),
    "rrr_phi4_tp_fused": (c_int, [vp, POINTER(c_int)]),
    "rrr_set_trace": (c_int, [vp, vp, c_int64]),
    "rrr_trace_position": (c_int, [vp, POINTER(c_int64), POINTER(c_int64)]),
    "rrr_phi4_tp_forward_emulated": (c_int, [POINTER(vp), c_int, POINTER(vp), POINTER(vp), POINTER(vp),
                                             c_int, vp]),
    "rrr_position_advance": (c_int, [vp, vp, c_int, vp]),
    "rrr_window_bf16": (c_int, [vp, vp, vp, c_int, c_int, c_int, c_int, vp]),
    "rrr_gemm_kq_batched_path": (c_int, [vp, c_int, vp, vp, vp, c_int, c_int, c_int, vp, c_int, vp]),
    "rrr_phi4_set_position": (c_int, [vp, c_int, vp]),
    "rrr_phi4_position": (c_int, [vp, POINTER(c_int)]),
    "rrr_phi4_kv_cache": (c_int, [vp, c_int, POINTER(vp), POINTER(vp)]),
    "rrr_rope_kv_store": (c_int, [vp, POINTER(AttnDesc), vp, c_int64, c_int, c_int, vp, vp, vp, vp]),
    "rrr_attention_f16kv": (c_int, [vp, POINTER(AttnDesc), vp, c_int64, c_int, c_int, vp, vp, vp, vp, vp]),
    "rrr_rope_attention_f16kv": (c_int, [vp, POINTER(AttnDesc), vp, c_int, vp, vp, vp, vp, vp]),
    "rrr_embed_rows": (c_int, [vp, c_int, vp, c_int64, c_int, vp, c_int, vp, vp]),
    "rrr_fill_kquant_random": (c_int, [vp, c_int, vp, c_int64, c_uint64, vp]),
    "rrr_fill_f32_normal": (c_int, [vp, vp, c_int64, c_float, c_float, c_uint64, vp]),
    "rrr_fill_f32_uniform": (c_int, [vp, vp, c_int64, c_float, c_float, c_uint64, vp]),
    "rrr_comm_create": (c_int, [vp, c_int, c_int, c_int64, POINTER(vp), vp]),
    "rrr_comm_create_ex": (c_int, [vp, c_int, c_int, c_int64, c_int64, POINTER(vp), vp]),
    "rrr_comm_connect": (c_int, [vp, vp]),
    "rrr_comm_allreduce_f32": (c_int, [vp, vp, c_int64, vp]),
    "rrr_comm_allgather_f32": (c_int, [vp, vp, vp, c_int64, vp]),
    "rrr_comm_allgather_rows_f32": (c_int, [vp, vp, vp, c_int, c_int64, vp]),
    "rrr_comm_disconnect": (c_int, [vp]),
    "rrr_comm_destroy": (c_int, [vp]),
    "rrr_fill_kquant_random_2d": (c_int, [vp, c_int, vp, c_int64, c_int64, c_int64, c_int64, c_uint64, vp]),
    "rrr_fill_f32_range": (c_int, [vp, vp, c_int64, c_int64, c_int, c_float, c_float, c_uint64, vp]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load librrr_cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run __graft_entry__.build() (no fallback "
                               "implementation exists)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in PROTOS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error(ctx=None) -> str:
    m = lib().rrr_last_error(ctx)
    return m.decode() if m else ""


def check(rc: int, ctx=None) -> None:
    if rc != RRR_OK:
        raise RRRError(rc, last_error(ctx))


class Context:
    """One rrr_ctx on one CUDA device (one host thread at a time)."""

    def __init__(self, device: int = 0):
        h = c_void_p()
        check(lib().rrr_init(device, ctypes.byref(h)))
        self.h = h
        self.device = device

    def close(self) -> None:
        if self.h:
            lib().rrr_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def check(self, rc: int) -> None:
        check(rc, self.h)

    def sm_count(self) -> int:
        n = c_int()
        self.check(lib().rrr_device_sm_count(self.h, ctypes.byref(n)))
        return n.value

    def device_error(self) -> int:
        code = c_int()
        rc = lib().rrr_check_device_error(self.h, ctypes.byref(code))
        if rc not in (RRR_OK, -7, -3):
            self.check(rc)
        return code.value
