"""ctypes wrapper and numpy helpers for the CPU oracle (TEST INFRASTRUCTURE ONLY).

The oracle restates RRR's CPU arithmetic (Peterc3-dev/recursive-routing-racer-rs,
src/model/phi4.rs) in C compiled with -ffp-contract=off; see rrr_oracle.h. Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline / reference legs use this module, as
the checker. Parity pin: gguf-py 0.19.0 dequantisers + hand-derived known answers
(the Rust reference cannot be built here).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD_DIR = os.path.join(HERE, "build")
LIB_PATH = os.path.join(BUILD_DIR, "liboracle.so")

BLOCK_BYTES = {12: 144, 13: 176, 14: 210}
QNAMES = {12: "Q4_K", 13: "Q5_K", 14: "Q6_K"}


def build(force: bool = False) -> str:
    """Compile rrr_oracle.c into build/liboracle.so (gcc, -O2 -ffp-contract=off)."""
    src = os.path.join(HERE, "rrr_oracle.c")
    hdr = os.path.join(HERE, "rrr_oracle.h")
    if (not force and os.path.exists(LIB_PATH)
            and os.path.getmtime(LIB_PATH) >= max(os.path.getmtime(src), os.path.getmtime(hdr))):
        return LIB_PATH
    os.makedirs(BUILD_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = ["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
           "-std=c11", "-D_POSIX_C_SOURCE=200809L", "-Wall", "-o", tmp, src, "-lm", "-pthread"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        u8p = ctypes.POINTER(ctypes.c_uint8)
        f32p = ctypes.POINTER(ctypes.c_float)
        i64 = ctypes.c_int64
        L.rrro_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.rrro_f16_to_f32.restype = ctypes.c_float
        L.rrro_f32_to_f16_rne.argtypes = [ctypes.c_float]
        L.rrro_f32_to_f16_rne.restype = ctypes.c_uint16
        L.rrro_dequant.argtypes = [ctypes.c_int, u8p, i64, f32p]
        L.rrro_dequant.restype = ctypes.c_int
        L.rrro_rms_norm.argtypes = [f32p, f32p, f32p, ctypes.c_int, ctypes.c_float]
        L.rrro_silu_gate.argtypes = [f32p, f32p, ctypes.c_int]
        L.rrro_silu.argtypes = [f32p, ctypes.c_int]
        L.rrro_gemv_f32.argtypes = [f32p, f32p, f32p, i64, i64, ctypes.c_int]
        L.rrro_matmul_f32.argtypes = [f32p, f32p, f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.rrro_gemv_kq.argtypes = [ctypes.c_int, u8p, f32p, f32p, i64, i64, ctypes.c_int]
        L.rrro_gemv_kq.restype = ctypes.c_int
        L.rrro_gemv_kq_baseline.argtypes = [ctypes.c_int, u8p, f32p, f32p, i64, i64, ctypes.c_int,
                                            f32p, ctypes.POINTER(ctypes.c_double),
                                            ctypes.POINTER(ctypes.c_double)]
        L.rrro_gemv_kq_baseline.restype = ctypes.c_int
        L.rrro_fill_kquant_random.argtypes = [ctypes.c_int, u8p, i64, i64, ctypes.c_uint64]
        L.rrro_decode_step.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.POINTER(t))


def f16_to_f32(bits: int) -> float:
    return lib().rrro_f16_to_f32(bits)


def dequant(qtype: int, raw: np.ndarray, n_elements: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.empty(n_elements, dtype=np.float32)
    rc = lib().rrro_dequant(qtype, _p(raw, ctypes.c_uint8), n_elements, _p(out, ctypes.c_float))
    if rc != 0:
        raise ValueError(f"unsupported type {qtype}")
    return out


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    lib().rrro_rms_norm(_p(x, ctypes.c_float), _p(w, ctypes.c_float), _p(out, ctypes.c_float),
                        x.size, eps)
    return out


def silu_gate(gu: np.ndarray) -> np.ndarray:
    gu = np.ascontiguousarray(gu, np.float32)
    F = gu.size // 2
    out = np.empty(F, np.float32)
    lib().rrro_silu_gate(_p(gu, ctypes.c_float), _p(out, ctypes.c_float), F)
    return out


def gemv_f32(W: np.ndarray, x: np.ndarray, threads: int = 1) -> np.ndarray:
    W = np.ascontiguousarray(W, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    N, K = W.shape
    y = np.empty(N, np.float32)
    lib().rrro_gemv_f32(_p(W, ctypes.c_float), _p(x, ctypes.c_float), _p(y, ctypes.c_float), N, K,
                        threads)
    return y


def matmul_f32(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    M, K = A.shape
    N = B.shape[1]
    C = np.empty((M, N), np.float32)
    lib().rrro_matmul_f32(_p(A, ctypes.c_float), _p(B, ctypes.c_float), _p(C, ctypes.c_float),
                          M, K, N)
    return C


def gemv_kq(qtype: int, raw: np.ndarray, x: np.ndarray, K: int, N: int,
            threads: int = 1) -> np.ndarray:
    raw = np.ascontiguousarray(raw, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    assert raw.size >= N * (K // 256) * BLOCK_BYTES[qtype] and x.size >= K
    y = np.empty(N, np.float32)
    rc = lib().rrro_gemv_kq(qtype, _p(raw, ctypes.c_uint8), _p(x, ctypes.c_float),
                            _p(y, ctypes.c_float), K, N, threads)
    if rc != 0:
        raise ValueError("bad gemv_kq arguments")
    return y


def gemv_kq_baseline(qtype: int, raw: np.ndarray, x: np.ndarray, K: int, N: int,
                     threads: int, scratch: np.ndarray | None = None):
    """CPU baseline: whole-matrix dequant + row-parallel dot. Returns (y, t_deq, t_dot)."""
    raw = np.ascontiguousarray(raw, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    if scratch is None or scratch.size < N * K:
        scratch = np.empty(N * K, np.float32)
    y = np.empty(N, np.float32)
    td = ctypes.c_double()
    tt = ctypes.c_double()
    rc = lib().rrro_gemv_kq_baseline(qtype, _p(raw, ctypes.c_uint8), _p(x, ctypes.c_float),
                                     _p(y, ctypes.c_float), K, N, threads,
                                     _p(scratch, ctypes.c_float), ctypes.byref(td),
                                     ctypes.byref(tt))
    if rc != 0:
        raise ValueError("bad baseline arguments")
    return y, td.value, tt.value


def fill_kquant_random(qtype: int, n_blocks: int, seed: int, block0: int = 0) -> np.ndarray:
    """Same bytes as the device generator rrr_fill_kquant_random for blocks
    [block0, block0+n_blocks)."""
    out = np.empty(n_blocks * BLOCK_BYTES[qtype], np.uint8)
    lib().rrro_fill_kquant_random(qtype, _p(out, ctypes.c_uint8), block0, n_blocks,
                                  ctypes.c_uint64(seed))
    return out


class _Layer(ctypes.Structure):
    _fields_ = [("w_qkv", ctypes.c_void_p), ("qkv_type", ctypes.c_int),
                ("w_o", ctypes.c_void_p), ("o_type", ctypes.c_int),
                ("w_gate_up", ctypes.c_void_p), ("gate_up_type", ctypes.c_int),
                ("w_down", ctypes.c_void_p), ("down_type", ctypes.c_int),
                ("attn_norm", ctypes.c_void_p), ("ffn_norm", ctypes.c_void_p)]


def decode_step(cfg: dict, layers: list, output_norm: np.ndarray, w_out: np.ndarray,
                hidden: np.ndarray, threads: int = 1):
    """Position-0 decode step on the CPU. layers: list of dicts with keys w_qkv, qkv_type,
    w_o, o_type, w_gate_up, gate_up_type, w_down, down_type, attn_norm, ffn_norm (numpy).
    Returns (hidden_out, logits)."""
    arr = (_Layer * len(layers))()
    keep = []
    for i, L in enumerate(layers):
        for k in ("w_qkv", "w_o", "w_gate_up", "w_down"):
            a = np.ascontiguousarray(L[k], np.uint8)
            keep.append(a)
            setattr(arr[i], k, a.ctypes.data)
        for k in ("attn_norm", "ffn_norm"):
            a = np.ascontiguousarray(L[k], np.float32)
            keep.append(a)
            setattr(arr[i], k, a.ctypes.data)
        for k in ("qkv_type", "o_type", "gate_up_type", "down_type"):
            setattr(arr[i], k, int(L[k]))
    on = np.ascontiguousarray(output_norm, np.float32)
    wo = np.ascontiguousarray(w_out, np.float32)
    h = np.array(hidden, dtype=np.float32, copy=True)
    logits = np.empty(cfg["vocab"], np.float32)
    L_ = lib()
    L_.rrro_decode_step.argtypes = [ctypes.c_int] * 7 + [ctypes.c_float, ctypes.POINTER(_Layer),
                                                         ctypes.c_void_p, ctypes.c_void_p,
                                                         ctypes.c_void_p, ctypes.c_void_p,
                                                         ctypes.c_int]
    rc = L_.rrro_decode_step(cfg["d_model"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"],
                             cfg["ffn_dim"], cfg["n_layers"], cfg["vocab"], cfg.get("eps", 1e-5),
                             arr, on.ctypes.data, wo.ctypes.data, h.ctypes.data,
                             logits.ctypes.data, threads)
    if rc != 0:
        raise ValueError("bad decode_step config")
    return h, logits


def rope(x: np.ndarray, pos: int, n_heads: int, head_dim: int, rope_dim: int, theta: float,
         attn_factor: float, factors=None) -> np.ndarray:
    """apply_rope_cfg (phi4.rs:238-256) on a copy of x (f32[n_heads*head_dim])."""
    y = np.array(x, dtype=np.float32, copy=True)
    f = np.ascontiguousarray(factors if factors is not None else np.zeros(0), np.float32)
    L = lib()
    L.rrro_rope.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                            ctypes.c_float, ctypes.c_float, ctypes.c_void_p, ctypes.c_int]
    L.rrro_rope(y.ctypes.data, pos, n_heads, head_dim, rope_dim, theta, attn_factor,
                f.ctypes.data, len(f))
    return y


def f32_to_f16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f16 bit patterns (the KV-cache store)."""
    return np.asarray(a, np.float32).astype(np.float16).view(np.uint16)


def attention_f16kv(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, seq_len: int,
                    n_heads: int, n_kv_heads: int, head_dim: int) -> np.ndarray:
    """Decode attention over rows 0..seq_len-1 of the f16 caches (uint16 bit patterns,
    [rows, n_kv_heads*head_dim])."""
    qq = np.ascontiguousarray(q, np.float32)
    kc = np.ascontiguousarray(k_cache, np.uint16)
    vc = np.ascontiguousarray(v_cache, np.uint16)
    out = np.empty(n_heads * head_dim, np.float32)
    L = lib()
    L.rrro_attention_f16kv.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 4
    L.rrro_attention_f16kv(qq.ctypes.data, kc.ctypes.data, vc.ctypes.data, out.ctypes.data,
                           seq_len, n_heads, n_kv_heads, head_dim)
    return out


def decode_step_kv(cfg: dict, layers: list, output_norm: np.ndarray, w_out: np.ndarray,
                   hidden: np.ndarray, pos: int, k_caches: np.ndarray, v_caches: np.ndarray,
                   rope_dim: int, theta: float, attn_factor: float, factors=None,
                   threads: int = 1):
    """Decode step at position `pos` with RoPE and f16 KV caches (forward_dynamic,
    phi4.rs:1593-1760). k_caches / v_caches: uint16 [n_layers, max_seq, n_kv*hd], updated
    in place. Returns (hidden_out, logits)."""
    arr = (_Layer * len(layers))()
    keep = []
    for i, Ly in enumerate(layers):
        for k in ("w_qkv", "w_o", "w_gate_up", "w_down"):
            a = np.ascontiguousarray(Ly[k], np.uint8)
            keep.append(a)
            setattr(arr[i], k, a.ctypes.data)
        for k in ("attn_norm", "ffn_norm"):
            a = np.ascontiguousarray(Ly[k], np.float32)
            keep.append(a)
            setattr(arr[i], k, a.ctypes.data)
        for k in ("qkv_type", "o_type", "gate_up_type", "down_type"):
            setattr(arr[i], k, int(Ly[k]))
    assert k_caches.dtype == np.uint16 and k_caches.flags.c_contiguous
    assert v_caches.dtype == np.uint16 and v_caches.flags.c_contiguous
    on = np.ascontiguousarray(output_norm, np.float32)
    wo = np.ascontiguousarray(w_out, np.float32)
    f = np.ascontiguousarray(factors if factors is not None else np.zeros(0), np.float32)
    h = np.array(hidden, dtype=np.float32, copy=True)
    logits = np.empty(cfg["vocab"], np.float32)
    L = lib()
    L.rrro_decode_step_kv.argtypes = ([ctypes.c_int] * 7 + [ctypes.c_float, ctypes.c_int,
                                      ctypes.c_float, ctypes.c_float, ctypes.c_void_p,
                                      ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                      ctypes.c_void_p, ctypes.POINTER(_Layer)]
                                      + [ctypes.c_void_p] * 4 + [ctypes.c_int])
    L.rrro_decode_step_kv.restype = ctypes.c_int
    rc = L.rrro_decode_step_kv(cfg["d_model"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"],
                               cfg["ffn_dim"], cfg["n_layers"], cfg["vocab"], cfg.get("eps", 1e-5),
                               rope_dim, theta, attn_factor, f.ctypes.data, len(f), pos,
                               k_caches.shape[1], k_caches.ctypes.data, v_caches.ctypes.data, arr,
                               on.ctypes.data, wo.ctypes.data, h.ctypes.data, logits.ctypes.data,
                               threads)
    if rc != 0:
        raise ValueError("bad decode_step_kv config")
    return h, logits


# ---------------------------------------------------------------- synthetic data (numpy)
def _f16_bits_uniform(rng: np.random.Generator, n: int, lo=1e-4, hi=1e-2) -> np.ndarray:
    return rng.uniform(lo, hi, n).astype(np.float32).astype(np.float16).view(np.uint16)


def random_blocks(qtype: int, n_blocks: int, rng: np.random.Generator) -> np.ndarray:
    """Seeded synthetic raw blocks with the benchmark distributions (numpy PCG64):
    d, dmin f16 ~ U[1e-4,1e-2]; Q6_K scales int8 ~ U[-32,31]; other bytes uniform."""
    bb = BLOCK_BYTES[qtype]
    b = rng.integers(0, 256, size=(n_blocks, bb), dtype=np.uint8)
    if qtype == 14:
        b[:, 192:208] = rng.integers(-32, 32, size=(n_blocks, 16)).astype(np.int8).view(np.uint8)
        b[:, 208:210] = _f16_bits_uniform(rng, n_blocks).view(np.uint8).reshape(n_blocks, 2)
    else:
        b[:, 0:2] = _f16_bits_uniform(rng, n_blocks).view(np.uint8).reshape(n_blocks, 2)
        b[:, 2:4] = _f16_bits_uniform(rng, n_blocks).view(np.uint8).reshape(n_blocks, 2)
    return np.ascontiguousarray(b.reshape(-1))
