"""Phi-4-mini-shape weight path on the C ABI: model configuration (phi4.rs:8-116), the
per-layer GEMV set, seeded synthetic weights resident in HBM, and the decode step
(rrr_phi4_forward; reference Phi4Model::forward_gpu, phi4.rs:1099-1196).
"""
from __future__ import annotations

import ctypes
from ctypes import c_int, c_void_p
from dataclasses import dataclass

from . import ffi

BLOCK_BYTES = {12: 144, 13: 176, 14: 210}


@dataclass
class ModelConfig:
    """phi4.rs:10-27 (the fields the weight path uses). Defaults are the legacy constants
    of phi4.rs:104-116 (Phi-4-mini, arch phi3)."""
    d_model: int = 3072
    n_heads: int = 24
    n_kv_heads: int = 8
    head_dim: int = 128
    ffn_dim: int = 8192
    n_layers: int = 32
    vocab_size: int = 200064
    rms_eps: float = 1e-5
    rope_dim: int = 96            # ROPE_DIM, phi4.rs:114
    rope_theta: float = 10000.0   # ROPE_THETA, phi4.rs:115
    rope_attn_factor: float = 1.190238  # ROPE_ATTN_FACTOR, phi4.rs:116
    qkv_type: int = 13      # Q5_K (Q4_K_M assignment in the benchmark configs)
    o_type: int = 12        # Q4_K
    gate_up_type: int = 12  # Q4_K
    down_type: int = 14     # Q6_K
    # Rows of the F32 logits per launch; 0 = all rows in one launch. The reference dispatches
    # 32768-row chunks (phi4.rs:866-893, a dispatch-size limit of its backend); the rows and
    # bytes are the same either way, and one launch saves a ramp and a tail per chunk.
    logits_chunk_rows: int = 0

    def qkv_dim(self) -> int:
        return self.n_heads * self.head_dim + 2 * self.n_kv_heads * self.head_dim

    def gate_up_dim(self) -> int:
        return 2 * self.ffn_dim

    @classmethod
    def from_gguf(cls, gguf) -> "ModelConfig":
        """ModelConfig::from_gguf, phi4.rs:31-97 (fields used by the weight path)."""
        arch = gguf.meta_str("general.architecture") or "llama"
        g = lambda k: gguf.meta_u64(f"{arch}.{k}")
        d = g("embedding_length")
        nh = g("attention.head_count")
        eps = gguf.meta_f32(f"{arch}.attention.layer_norm_rms_epsilon")
        vocab = next((t.shape[1] for t in gguf.tensor_infos if t.name == "token_embd.weight"), 0)
        hd = d // nh if nh else 128
        rd = g("rope.dimension_count")
        theta = gguf.meta_f32(f"{arch}.rope.freq_base")
        af = gguf.meta_f32(f"{arch}.rope.scaling.attn_factor")
        return cls(d_model=d, n_heads=nh, n_kv_heads=g("attention.head_count_kv"),
                   head_dim=hd, ffn_dim=g("feed_forward_length"),
                   n_layers=g("block_count"), vocab_size=vocab, rms_eps=eps if eps > 0 else 1e-5,
                   rope_dim=rd if rd > 0 else hd, rope_theta=theta if theta > 0 else 10000.0,
                   rope_attn_factor=af if af > 0 else 1.0)

    def layer_gemvs(self):
        """(name, qtype, K, N) of the four per-layer GEMVs (benchmark config 1)."""
        return [("qkv", self.qkv_type, self.d_model, self.qkv_dim()),
                ("o_proj", self.o_type, self.n_heads * self.head_dim, self.d_model),
                ("gate_up", self.gate_up_type, self.d_model, self.gate_up_dim()),
                ("down", self.down_type, self.ffn_dim, self.d_model)]

    def weight_bytes(self, qtype: int, K: int, N: int) -> int:
        return N * (K // 256) * BLOCK_BYTES[qtype]

    def step_bytes(self) -> int:
        """Algorithmic bytes of one decode step (weights + norms + logits matrix)."""
        layer = sum(self.weight_bytes(q, K, N) for _, q, K, N in self.layer_gemvs())
        norms = (2 * self.n_layers + 1) * self.d_model * 4
        return layer * self.n_layers + norms + self.vocab_size * self.d_model * 4


class DeviceArena:
    """Owns device allocations made through the C ABI."""

    def __init__(self, ctx: ffi.Context):
        self.ctx = ctx
        self.ptrs = []

    def alloc(self, nbytes: int) -> int:
        p = c_void_p()
        self.ctx.check(ffi.lib().rrr_alloc(self.ctx.h, nbytes, ctypes.byref(p)))
        self.ptrs.append(p.value)
        return p.value

    def free_all(self) -> None:
        for p in self.ptrs:
            ffi.lib().rrr_free(self.ctx.h, c_void_p(p))
        self.ptrs = []


def tensor_seed(seed: int, layer: int, name: str) -> int:
    """One generator stream per (seed, layer, tensor) (stable across runs)."""
    h = 1469598103934665603
    for ch in f"{seed}/{layer}/{name}".encode():
        h = ((h ^ ch) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


class SyntheticPhi4:
    """Seeded synthetic Phi-4-mini-shape weights generated in HBM (benchmark config 2):
    K-quant blocks with the config distributions, norms gamma ~ U[0.5, 1.5], logits
    matrix W ~ N(0, 0.02) row-major [vocab, d]."""

    def __init__(self, ctx: ffi.Context, cfg: ModelConfig, seed: int = 0, stream=None):
        self.ctx, self.cfg, self.seed = ctx, cfg, seed
        self.arena = DeviceArena(ctx)
        L = ffi.lib()
        s = stream
        self.layers = []
        for l in range(cfg.n_layers):
            ent = {}
            for name, qt, K, N in cfg.layer_gemvs():
                nb = N * (K // 256)
                p = self.arena.alloc(nb * BLOCK_BYTES[qt])
                ctx.check(L.rrr_fill_kquant_random(ctx.h, qt, p, nb, tensor_seed(seed, l, name), s))
                ent[name] = (p, qt, K, N)
            for nn in ("attn_norm", "ffn_norm"):
                p = self.arena.alloc(cfg.d_model * 4)
                ctx.check(L.rrr_fill_f32_uniform(ctx.h, p, cfg.d_model, 0.5, 1.5,
                                                 tensor_seed(seed, l, nn), s))
                ent[nn] = p
            self.layers.append(ent)
        self.output_norm = self.arena.alloc(cfg.d_model * 4)
        ctx.check(L.rrr_fill_f32_uniform(ctx.h, self.output_norm, cfg.d_model, 0.5, 1.5,
                                         tensor_seed(seed, -1, "output_norm"), s))
        self.w_out = self.arena.alloc(cfg.vocab_size * cfg.d_model * 4)
        ctx.check(L.rrr_fill_f32_normal(ctx.h, self.w_out, cfg.vocab_size * cfg.d_model, 0.0, 0.02,
                                        tensor_seed(seed, -1, "output"), s))
        # LongRoPE short factors (rope_factors_short.weight, one per rotated pair) ~ U[1, 1.5]
        self.n_rope_factors = cfg.rope_dim // 2
        self.rope_factors = self.arena.alloc(max(1, self.n_rope_factors) * 4)
        if self.n_rope_factors:
            ctx.check(L.rrr_fill_f32_uniform(ctx.h, self.rope_factors, self.n_rope_factors, 1.0, 1.5,
                                             tensor_seed(seed, -1, "rope_factors"), s))
        ctx.check(L.rrr_sync(ctx.h, s))

    def desc(self, max_seq: int = 0):
        """rrr_phi4_desc; max_seq > 0 selects KV-cache decode with RoPE."""
        cfg = self.cfg
        arr = (ffi.Phi4Layer * cfg.n_layers)()
        for i, e in enumerate(self.layers):
            arr[i].w_qkv, arr[i].qkv_type = e["qkv"][0], e["qkv"][1]
            arr[i].w_o, arr[i].o_type = e["o_proj"][0], e["o_proj"][1]
            arr[i].w_gate_up, arr[i].gate_up_type = e["gate_up"][0], e["gate_up"][1]
            arr[i].w_down, arr[i].down_type = e["down"][0], e["down"][1]
            arr[i].attn_norm, arr[i].ffn_norm = e["attn_norm"], e["ffn_norm"]
        d = ffi.Phi4Desc(cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim,
                         cfg.n_layers, cfg.vocab_size, cfg.rms_eps, cfg.logits_chunk_rows,
                         ctypes.cast(arr, ctypes.POINTER(ffi.Phi4Layer)), self.output_norm, self.w_out,
                         max_seq, cfg.rope_dim, cfg.rope_theta, cfg.rope_attn_factor,
                         self.rope_factors, self.n_rope_factors)
        return d, arr

    def close(self) -> None:
        self.arena.free_all()


class Phi4Decoder:
    """The decode step (rrr_phi4_*), a drop-in for Phi4Model::forward_gpu's GPU chain."""

    def __init__(self, ctx: ffi.Context, weights: SyntheticPhi4, max_seq: int = 0):
        self.ctx = ctx
        self.max_seq = max_seq
        d, self._keep = weights.desc(max_seq)
        h = c_void_p()
        ctx.check(ffi.lib().rrr_phi4_create(ctx.h, ctypes.byref(d), ctypes.byref(h)))
        self.h = h

    def forward(self, hidden_ptr: int, logits_ptr: int, argmax_ptr: int | None = None,
                use_graph: bool = True, stream=None) -> None:
        s = None if stream is None else c_void_p(stream if isinstance(stream, int) else stream.cuda_stream)
        self.ctx.check(ffi.lib().rrr_phi4_forward(self.h, c_void_p(hidden_ptr), c_void_p(logits_ptr),
                                                  c_void_p(argmax_ptr) if argmax_ptr else None,
                                                  1 if use_graph else 0, s))

    def forward_batched(self, hidden_ptr: int, logits_ptr: int, M: int, argmax_ptr: int | None = None,
                        use_graph: bool = True, stream=None) -> None:
        """M tokens in one step (forward_prefill_batched): hidden f32 [M, d] in/out, logits
        f32 [M, vocab], argmax int32 [M] or None; consecutive positions with a KV cache."""
        s = None if stream is None else c_void_p(stream if isinstance(stream, int) else stream.cuda_stream)
        self.ctx.check(ffi.lib().rrr_phi4_forward_batched(
            self.h, c_void_p(hidden_ptr), c_void_p(logits_ptr), c_void_p(argmax_ptr) if argmax_ptr else None,
            M, 1 if use_graph else 0, s))

    def launches_per_step(self) -> int:
        n = c_int()
        self.ctx.check(ffi.lib().rrr_phi4_launches_per_step(self.h, ctypes.byref(n)))
        return n.value

    def set_position(self, pos: int, stream=None) -> None:
        """KV-cache decode: position of the next forward (KVCache.len)."""
        s = None if stream is None else c_void_p(stream if isinstance(stream, int) else stream.cuda_stream)
        self.ctx.check(ffi.lib().rrr_phi4_set_position(self.h, pos, s))

    @property
    def position(self) -> int:
        n = c_int()
        self.ctx.check(ffi.lib().rrr_phi4_position(self.h, ctypes.byref(n)))
        return n.value

    def kv_cache(self, layer: int):
        """Device pointers (k, v) of one layer's f16 [max_seq, n_kv*hd] caches."""
        k, v = c_void_p(), c_void_p()
        self.ctx.check(ffi.lib().rrr_phi4_kv_cache(self.h, layer, ctypes.byref(k), ctypes.byref(v)))
        return k.value, v.value

    def close(self) -> None:
        if self.h:
            ffi.lib().rrr_phi4_destroy(self.h)
            self.h = None
