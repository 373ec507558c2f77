"""Tensor-parallel decode step of the weight path over G GPUs of one box (one process per
GPU, torch.distributed over NCCL for the exchanges).

The reference runs the whole model on one GPU (src/model/phi4.rs:1099-1196); this module
splits the same per-layer weight GEMVs so that every rank streams 1/G of the bytes:

    QKV       rows of the rank's query heads [h0, h1) and their KV heads [v0, v1): the
              position-0 attention (output = V of the head's KV group) is then local
    O-proj    the K columns of those heads (Megatron split). When the heads do not cover
              whole 256-wide super-blocks (8 GPUs: 384 columns), the rank keeps the
              super-block window around them and the GEMV input is zero outside the
              heads (RRR_X_GQA_V with k_offset), so no block is split; the partial
              outputs are summed with an all-reduce
    gate_up   rows [f0, f1) of gate and the same rows of up: SiLU(gate)*up stays local
    down      the matching K columns [f0, f1) of every row; all-reduce of the partials
    logits    vocab rows [V*g/G, V*(g+1)/G), output RMSNorm fused; all-gather of the rows

The residual is added by rank 0 only (in its O-proj / down epilogue), so the all-reduced
sum carries it once. Everything else (RMSNorm, the argmax) is replicated. Per token: 2
all-reduces per layer and one all-gather.
"""
from __future__ import annotations

import ctypes
from ctypes import c_void_p
from dataclasses import dataclass

from . import ffi
from .phi4 import BLOCK_BYTES, DeviceArena, ModelConfig, tensor_seed


@dataclass(frozen=True)
class TPShard:
    """Rows and K windows of rank g's shards (all ranges are [start, stop))."""
    G: int
    g: int
    q_heads: tuple
    kv_heads: tuple
    qkv_rows: tuple          # row ranges of the full QKV matrix, in shard order (Q, K, V)
    o_blocks: tuple          # super-block window of O-proj's K (n_heads*head_dim)
    o_k_offset: int          # first column of the rank's heads inside the window
    ffn: tuple               # rows [f0, f1) of gate and of up; K columns of down
    vocab: tuple             # rows of the logits matrix

    @property
    def qkv_dim(self) -> int:
        return sum(b - a for a, b in self.qkv_rows)

    @property
    def o_k(self) -> int:
        return 256 * (self.o_blocks[1] - self.o_blocks[0])

    @property
    def ffn_dim(self) -> int:
        return self.ffn[1] - self.ffn[0]

    @property
    def vocab_rows(self) -> int:
        return self.vocab[1] - self.vocab[0]


def plan(cfg: ModelConfig, G: int, g: int) -> TPShard:
    """Shard ranges of rank g of G (the split of the tensor-parallel section above)."""
    if G < 1 or not 0 <= g < G:
        raise ValueError(f"bad rank {g} of {G}")
    nq, nkv, hd, F, V = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim, cfg.vocab_size
    if nq % G or nkv % G or nq % nkv:
        raise ValueError(f"{nq} query / {nkv} KV heads do not split over {G} GPUs")
    if F % (256 * G):
        raise ValueError(f"ffn_dim {F} is not a multiple of 256*{G}")
    if V % G:
        raise ValueError(f"vocab {V} is not a multiple of {G}")
    h0, h1 = nq * g // G, nq * (g + 1) // G
    v0, v1 = nkv * g // G, nkv * (g + 1) // G
    qkv_rows = ((h0 * hd, h1 * hd),
                (nq * hd + v0 * hd, nq * hd + v1 * hd),
                ((nq + nkv) * hd + v0 * hd, (nq + nkv) * hd + v1 * hd))
    c0, c1 = h0 * hd, h1 * hd
    b0, b1 = c0 // 256, (c1 + 255) // 256
    f0, f1 = F * g // G, F * (g + 1) // G
    return TPShard(G, g, (h0, h1), (v0, v1), qkv_rows, (b0, b1), c0 - 256 * b0, (f0, f1),
                   (V * g // G, V * (g + 1) // G))


class SyntheticPhi4TP:
    """Rank g's shards of SyntheticPhi4(cfg, seed): every shard holds exactly the bytes of
    the corresponding slice of the 1-GPU model (same generator streams), so a G-GPU step
    can be checked against the 1-GPU step."""

    def __init__(self, ctx: ffi.Context, cfg: ModelConfig, shard: TPShard, seed: int = 0,
                 stream=None):
        self.ctx, self.cfg, self.shard, self.seed = ctx, cfg, shard, seed
        self.arena = DeviceArena(ctx)
        L = ffi.lib()
        s = stream
        sh = shard
        d, F = cfg.d_model, cfg.ffn_dim

        def kq(qt, name, l, rows_ranges, nb_row, blocks=None):
            """Rows `rows_ranges` of tensor `name` of layer l (nb_row blocks per row),
            restricted to the super-block column window `blocks`."""
            c0, c1 = blocks if blocks else (0, nb_row)
            n_rows = sum(b - a for a, b in rows_ranges)
            p = self.arena.alloc(n_rows * (c1 - c0) * BLOCK_BYTES[qt])
            off, sd = 0, tensor_seed(seed, l, name)
            for a, b in rows_ranges:
                ctx.check(L.rrr_fill_kquant_random_2d(ctx.h, qt, c_void_p(p + off), b - a, c1 - c0,
                                                      nb_row, a * nb_row + c0, sd, s))
                off += (b - a) * (c1 - c0) * BLOCK_BYTES[qt]
            return p

        self.layers = []
        for l in range(cfg.n_layers):
            ent = {
                "qkv": kq(cfg.qkv_type, "qkv", l, sh.qkv_rows, d // 256),
                "o_proj": kq(cfg.o_type, "o_proj", l, ((0, d),), cfg.n_heads * cfg.head_dim // 256,
                             sh.o_blocks),
                "gate_up": kq(cfg.gate_up_type, "gate_up", l,
                              (sh.ffn, (F + sh.ffn[0], F + sh.ffn[1])), d // 256),
                "down": kq(cfg.down_type, "down", l, ((0, d),), F // 256,
                           (sh.ffn[0] // 256, sh.ffn[1] // 256)),
            }
            for nn in ("attn_norm", "ffn_norm"):
                p = self.arena.alloc(d * 4)
                ctx.check(L.rrr_fill_f32_uniform(ctx.h, p, d, 0.5, 1.5, tensor_seed(seed, l, nn), s))
                ent[nn] = p
            self.layers.append(ent)
        self.output_norm = self.arena.alloc(d * 4)
        ctx.check(L.rrr_fill_f32_uniform(ctx.h, self.output_norm, d, 0.5, 1.5,
                                         tensor_seed(seed, -1, "output_norm"), s))
        v0, v1 = sh.vocab
        self.w_out = self.arena.alloc((v1 - v0) * d * 4)
        ctx.check(L.rrr_fill_f32_range(ctx.h, self.w_out, (v1 - v0) * d, v0 * d, 1, 0.0, 0.02,
                                       tensor_seed(seed, -1, "output"), s))
        # LongRoPE factors, replicated (the same stream as SyntheticPhi4's)
        self.n_rope_factors = cfg.rope_dim // 2
        self.rope_factors = self.arena.alloc(max(1, self.n_rope_factors) * 4)
        if self.n_rope_factors:
            ctx.check(L.rrr_fill_f32_uniform(ctx.h, self.rope_factors, self.n_rope_factors, 1.0, 1.5,
                                             tensor_seed(seed, -1, "rope_factors"), s))
        ctx.check(L.rrr_sync(ctx.h, s))

    def shard_bytes(self) -> int:
        """Weight bytes one decode step streams on this rank."""
        c, sh = self.cfg, self.shard
        d = c.d_model
        b = (sh.qkv_dim * (d // 256) * BLOCK_BYTES[c.qkv_type]
             + d * (sh.o_blocks[1] - sh.o_blocks[0]) * BLOCK_BYTES[c.o_type]
             + 2 * sh.ffn_dim * (d // 256) * BLOCK_BYTES[c.gate_up_type]
             + d * (sh.ffn_dim // 256) * BLOCK_BYTES[c.down_type])
        return b * c.n_layers + (2 * c.n_layers + 1) * d * 4 + sh.vocab_rows * d * 4

    def close(self) -> None:
        self.arena.free_all()


class TPTimeout(RuntimeError):
    """A collective did not complete before its host deadline (or its group failed); the
    process group has been torn down, so no later collective can wait on it."""


def all_reduce_with_deadline(t, timeout_s: float, group=None) -> None:
    """dist.all_reduce(t) (sum, in place) that gives up after `timeout_s` seconds of host
    time: a rank that skipped the collective, stalled or died makes the call raise
    TPTimeout instead of blocking, and the group is destroyed (its pending work is
    abandoned). The reference waits on its fences without a limit (engine.rs:312,369)."""
    import datetime
    import torch.distributed as dist
    work = dist.all_reduce(t, group=group, async_op=True)
    try:
        done = work.wait(timeout=datetime.timedelta(seconds=timeout_s))
        err = None if done is not False else "the wait returned False"
    except RuntimeError as e:
        err = str(e)
    if err is not None:
        try:
            dist.destroy_process_group(group)
        except Exception:
            pass
        raise TPTimeout(f"all_reduce missed its {timeout_s:g} s host deadline or its group "
                        f"failed: {err}")


class P2PComm:
    """The C ABI's NVLink peer-memory exchanges (rrr_comm_*) for one rank; the 64-byte IPC
    handles are swapped with torch.distributed.all_gather_object."""

    def __init__(self, ctx: ffi.Context, rank: int, world: int, max_elems: int, group=None):
        import torch.distributed as dist
        L = ffi.lib()
        self.ctx, self.group = ctx, group
        h = c_void_p()
        buf = ctypes.create_string_buffer(64)
        ctx.check(L.rrr_comm_create(ctx.h, rank, world, max_elems, ctypes.byref(h), buf))
        self.h = h
        handles = [None] * world
        dist.all_gather_object(handles, bytes(buf.raw), group=group)
        allh = ctypes.create_string_buffer(b"".join(handles), 64 * world)
        ctx.check(L.rrr_comm_connect(self.h, allh))
        dist.barrier(group=group)

    def all_reduce(self, t, stream) -> None:
        self.ctx.check(ffi.lib().rrr_comm_allreduce_f32(self.h, c_void_p(t.data_ptr()), t.numel(), stream))

    def all_gather(self, out, part, stream) -> None:
        self.ctx.check(ffi.lib().rrr_comm_allgather_f32(self.h, c_void_p(out.data_ptr()),
                                                        c_void_p(part.data_ptr()), part.numel(), stream))

    def close(self) -> None:
        """Collective: every rank unmaps the others' buffers, then frees its own."""
        import torch.distributed as dist
        if self.h:
            ffi.lib().rrr_comm_disconnect(self.h)
            dist.barrier(group=self.group)
            ffi.lib().rrr_comm_destroy(self.h)
            self.h = None


class TPDecoder:
    """One rank's decode step: the kernels of the 1-GPU step on the rank's shards, with
    torch.distributed all-reduce / all-gather (NCCL) or the peer-memory kernels between
    them. The step can be captured into a CUDA graph (kernels and collectives) and
    replayed.

    max_seq = 0: every token at position 0 (attention output = V; forward_batched runs M
    independent sequences). max_seq > 0: a KV cache of the rank's KV heads (f16, max_seq
    rows per layer) and a device position: forward decodes one token at the position and
    advances it (RoPE, KV store and attention fused in one launch per layer);
    forward_batched is a prefill of M consecutive tokens of one sequence (RoPE + KV store
    of the M rows, causal attention, phi4.rs:1270-1309) and advances the position by M."""

    def __init__(self, ctx: ffi.Context, weights: SyntheticPhi4TP, group=None, comm: str = "nccl",
                 max_batch: int = 1, max_seq: int = 0):
        """comm: "nccl" (torch.distributed collectives) or "p2p" (rrr_comm_* kernels over
        NVLink peer memory); max_batch: the largest M of forward_batched; max_seq: KV-cache
        rows (0: position-0 steps)."""
        import torch
        import torch.distributed as dist
        self.torch, self.dist = torch, dist
        self.ctx, self.w, self.group = ctx, weights, group
        self.p2p = None
        if comm == "p2p" and weights.shard.G > 1:
            self.p2p = P2PComm(ctx, weights.shard.g, weights.shard.G,
                               max_batch * max(weights.cfg.d_model, weights.shard.vocab_rows), group)
        elif comm not in ("nccl", "p2p"):
            raise ValueError(f"unknown comm {comm!r}")
        cfg, sh = weights.cfg, weights.shard
        dev = torch.device("cuda", ctx.device)
        self.qkv = torch.empty(sh.qkv_dim, device=dev)
        self.mid = torch.empty(sh.ffn_dim, device=dev)
        self.logits_loc = torch.empty(sh.vocab_rows, device=dev)
        self.graph = None
        self._graph_key = None
        self._bm = 0  # batch size of the batched buffers
        self.max_seq = max_seq
        self.pos = 0  # host copy of the device position
        if max_seq:
            nq_loc = sh.q_heads[1] - sh.q_heads[0]
            nkv_loc = sh.kv_heads[1] - sh.kv_heads[0]
            self.kc = torch.zeros(cfg.n_layers, max_seq, nkv_loc * cfg.head_dim, dtype=torch.int16, device=dev)
            self.vc = torch.zeros_like(self.kc)
            self.d_pos = torch.zeros(1, dtype=torch.int32, device=dev)
            self.attn_desc = ffi.AttnDesc(nq_loc, nkv_loc, cfg.head_dim, cfg.rope_dim, cfg.rope_theta,
                                          cfg.rope_attn_factor, c_void_p(weights.rope_factors),
                                          weights.n_rope_factors, max_seq)
            # O-projection input: the heads' attention output inside the window, zeros around
            self.attn_in = torch.zeros(sh.o_k, device=dev)

    def set_position(self, pos: int) -> None:
        """KV-cache decode: position of the next token (KVCache.len)."""
        if not 0 <= pos < self.max_seq:
            raise ValueError(f"position {pos} outside the cache of {self.max_seq} rows")
        self.d_pos.fill_(pos)
        self.pos = pos

    def _cache(self, l):
        kv = self.kc[l].data_ptr(), self.vc[l].data_ptr()
        return c_void_p(kv[0]), c_void_p(kv[1])

    def steps(self, hidden, logits, argmax, stream=None):
        """The step as a generator: launches the kernels on `stream` (default: the current
        torch stream) and yields at each exchange ("all_reduce", t) -- sum t over the
        ranks in place -- and ("all_gather", out, part) -- out = concatenation of every
        rank's part. hidden: f32[d] (in/out); logits: f32[vocab]; argmax: int32[1] or None."""
        L, ctx, cfg, sh, w = ffi.lib(), self.ctx, self.w.cfg, self.w.shard, self.w
        torch = self.torch
        st = c_void_p(stream if stream is not None else torch.cuda.current_stream().cuda_stream)
        d, hd = cfg.d_model, cfg.head_dim
        hp = c_void_p(hidden.data_ptr())
        res = hp if sh.g == 0 else None
        nq_loc = sh.q_heads[1] - sh.q_heads[0]
        nkv_loc = sh.kv_heads[1] - sh.kv_heads[0]
        qkv_p, mid_p = c_void_p(self.qkv.data_ptr()), c_void_p(self.mid.data_ptr())
        if self.max_seq:
            if self.pos >= self.max_seq:
                raise ValueError(f"position {self.pos} is past the cache of {self.max_seq} rows")
            ad, dpos = ctypes.byref(self.attn_desc), c_void_p(self.d_pos.data_ptr())
            attn_out = c_void_p(self.attn_in.data_ptr() + 4 * sh.o_k_offset)
        for l, e in enumerate(w.layers):
            pn = ffi.GemvPrologue(1, e["attn_norm"], cfg.rms_eps, 0, 0, 0, 0)
            ctx.check(L.rrr_gemv_kq_ex(ctx.h, cfg.qkv_type, c_void_p(e["qkv"]), hp, qkv_p, d,
                                       sh.qkv_dim, None, ctypes.byref(pn), st))
            if self.max_seq:
                kc, vc = self._cache(l)
                ctx.check(L.rrr_rope_attention_f16kv(ctx.h, ad, qkv_p, 0, dpos, kc, vc, attn_out, st))
                ctx.check(L.rrr_gemv_kq_ex(ctx.h, cfg.o_type, c_void_p(e["o_proj"]),
                                           c_void_p(self.attn_in.data_ptr()), hp, sh.o_k, d, res, None, st))
            else:
                pv = ffi.GemvPrologue(3, None, 0.0, nq_loc, nkv_loc, hd, sh.o_k_offset)
                ctx.check(L.rrr_gemv_kq_ex(ctx.h, cfg.o_type, c_void_p(e["o_proj"]), qkv_p, hp, sh.o_k,
                                           d, res, ctypes.byref(pv), st))
            if sh.G > 1:
                yield ("all_reduce", hidden)
            pf = ffi.GemvPrologue(1, e["ffn_norm"], cfg.rms_eps, 0, 0, 0, 0)
            ctx.check(L.rrr_gemv_kq_swiglu(ctx.h, cfg.gate_up_type, c_void_p(e["gate_up"]), hp, mid_p,
                                           d, sh.ffn_dim, ctypes.byref(pf), st))
            ctx.check(L.rrr_gemv_kq_ex(ctx.h, cfg.down_type, c_void_p(e["down"]), mid_p, hp, sh.ffn_dim,
                                       d, res, None, st))
            if sh.G > 1:
                yield ("all_reduce", hidden)
        lp = c_void_p(self.logits_loc.data_ptr() if sh.G > 1 else logits.data_ptr())
        ctx.check(L.rrr_logits_f32(ctx.h, c_void_p(w.w_out), hp, lp, sh.vocab_rows, d,
                                   cfg.logits_chunk_rows, c_void_p(w.output_norm), cfg.rms_eps, st))
        if sh.G > 1:
            yield ("all_gather", logits, self.logits_loc)
        if argmax is not None:
            ctx.check(L.rrr_argmax_f32(ctx.h, c_void_p(logits.data_ptr()), cfg.vocab_size,
                                       c_void_p(argmax.data_ptr()), st))
        if self.max_seq:
            ctx.check(L.rrr_position_advance(ctx.h, c_void_p(self.d_pos.data_ptr()), 1, st))
            self.pos += 1

    def _issue(self, hidden, logits, argmax):
        """The step with its exchanges as torch.distributed collectives (NCCL) or as the
        peer-memory kernels."""
        st = c_void_p(self.torch.cuda.current_stream().cuda_stream)
        for op in self.steps(hidden, logits, argmax):
            self._exchange(op, st)

    def close(self) -> None:
        self.release_graph()
        if self.p2p is not None:
            self.p2p.close()
            self.p2p = None

    def _ensure_batch(self, M: int) -> None:
        if self._bm >= M:
            return
        torch = self.torch
        cfg, sh = self.w.cfg, self.w.shard
        dev = torch.device("cuda", self.ctx.device)
        self.b_xn = torch.empty(M, cfg.d_model, dtype=torch.int16, device=dev)       # bf16 bits
        self.b_qkv = torch.empty(M, sh.qkv_dim, device=dev)
        self.b_a = torch.empty(M, sh.o_k, dtype=torch.int16, device=dev)             # bf16 bits
        self.b_gu = torch.empty(M, 2 * sh.ffn_dim, device=dev)
        self.b_mid = torch.empty(M, sh.ffn_dim, dtype=torch.int16, device=dev)       # bf16 bits
        self.b_xnorm = torch.empty(M, cfg.d_model, device=dev)
        self.b_logits_loc = torch.empty(M, sh.vocab_rows, device=dev)
        if self.max_seq:
            self.b_attn = torch.empty(M, (sh.q_heads[1] - sh.q_heads[0]) * cfg.head_dim, device=dev)
        self._bm = M

    def steps_batched(self, hidden, logits, M: int, stream=None):
        """M tokens (the batched-prefill call sites, phi4.rs:1198-1445, with every GEMM on
        the tensor cores): at position 0 each (max_seq = 0), or a prefill of M consecutive
        positions from the current one (max_seq > 0). hidden f32 [M, d] (in/out), logits
        f32 [M, vocab]. Yields at each exchange like steps(); the logits exchange is
        ("all_gather_rows", out [M, vocab], part [M, vocab/G], M)."""
        L, ctx, cfg, sh, w = ffi.lib(), self.ctx, self.w.cfg, self.w.shard, self.w
        torch = self.torch
        self._ensure_batch(M)
        st = c_void_p(stream if stream is not None else torch.cuda.current_stream().cuda_stream)
        d, hd = cfg.d_model, cfg.head_dim
        hp = c_void_p(hidden.data_ptr())
        res = hp if sh.g == 0 else None
        nq_loc = sh.q_heads[1] - sh.q_heads[0]
        nkv_loc = sh.kv_heads[1] - sh.kv_heads[0]
        xn, qkv, a = c_void_p(self.b_xn.data_ptr()), c_void_p(self.b_qkv.data_ptr()), c_void_p(self.b_a.data_ptr())
        gu, mid = c_void_p(self.b_gu.data_ptr()), c_void_p(self.b_mid.data_ptr())
        if self.max_seq:
            if self.pos + M > self.max_seq:
                raise ValueError(f"positions {self.pos}..{self.pos + M - 1} exceed the cache of "
                                 f"{self.max_seq} rows")
            ad, dpos = ctypes.byref(self.attn_desc), c_void_p(self.d_pos.data_ptr())
            att = c_void_p(self.b_attn.data_ptr())
        for l, e in enumerate(w.layers):
            ctx.check(L.rrr_rmsnorm_bf16(ctx.h, hp, c_void_p(e["attn_norm"]), xn, M, d, cfg.rms_eps, st))
            ctx.check(L.rrr_gemm_kq_batched(ctx.h, cfg.qkv_type, c_void_p(e["qkv"]), xn, qkv, M, d,
                                            sh.qkv_dim, st))
            if self.max_seq:
                kc, vc = self._cache(l)
                ctx.check(L.rrr_rope_kv_store(ctx.h, ad, qkv, sh.qkv_dim, M, 0, dpos, kc, vc, st))
                ctx.check(L.rrr_attention_f16kv(ctx.h, ad, qkv, sh.qkv_dim, M, 0, dpos, kc, vc, att, st))
                ctx.check(L.rrr_window_bf16(ctx.h, att, a, M, nq_loc * hd, sh.o_k, sh.o_k_offset, st))
            else:
                ctx.check(L.rrr_gqa_v_bf16(ctx.h, qkv, a, M, nq_loc, nkv_loc, hd, sh.o_k, sh.o_k_offset, st))
            ctx.check(L.rrr_gemm_kq_batched_ex(ctx.h, cfg.o_type, c_void_p(e["o_proj"]), a, hp, M, sh.o_k,
                                               d, res, st))
            if sh.G > 1:
                yield ("all_reduce", hidden)
            ctx.check(L.rrr_rmsnorm_bf16(ctx.h, hp, c_void_p(e["ffn_norm"]), xn, M, d, cfg.rms_eps, st))
            ctx.check(L.rrr_gemm_kq_batched(ctx.h, cfg.gate_up_type, c_void_p(e["gate_up"]), xn, gu, M, d,
                                            2 * sh.ffn_dim, st))
            ctx.check(L.rrr_silu_gate_bf16(ctx.h, gu, mid, M, sh.ffn_dim, st))
            ctx.check(L.rrr_gemm_kq_batched_ex(ctx.h, cfg.down_type, c_void_p(e["down"]), mid, hp, M,
                                               sh.ffn_dim, d, res, st))
            if sh.G > 1:
                yield ("all_reduce", hidden)
        lp = self.b_logits_loc if sh.G > 1 else logits
        ctx.check(L.rrr_logits_f32_batched(ctx.h, c_void_p(w.w_out), hp, c_void_p(self.b_xnorm.data_ptr()),
                                           c_void_p(lp.data_ptr()), M, sh.vocab_rows, d,
                                           c_void_p(w.output_norm), cfg.rms_eps, st))
        if sh.G > 1:
            yield ("all_gather_rows", logits, self.b_logits_loc[:M], M)
        if self.max_seq:
            ctx.check(L.rrr_position_advance(ctx.h, dpos, M, st))
            self.pos += M

    def _exchange(self, op, st) -> None:
        dist = self.dist
        if self.p2p is not None:
            if op[0] == "all_reduce":
                self.p2p.all_reduce(op[1], st)
            elif op[0] == "all_gather":
                self.p2p.all_gather(op[1], op[2], st)
            else:
                self.ctx.check(ffi.lib().rrr_comm_allgather_rows_f32(
                    self.p2p.h, c_void_p(op[1].data_ptr()), c_void_p(op[2].data_ptr()), op[3],
                    op[2].numel() // op[3], st))
        elif op[0] == "all_reduce":
            dist.all_reduce(op[1], group=self.group)
        elif op[0] == "all_gather":
            dist.all_gather_into_tensor(op[1], op[2], group=self.group)
        else:
            G, M = self.w.shard.G, op[3]
            tmp = self.torch.empty(G * op[2].numel(), device=op[2].device)
            dist.all_gather_into_tensor(tmp, op[2].reshape(-1), group=self.group)
            op[1].view(M, G, -1).copy_(tmp.view(G, M, -1).permute(1, 0, 2))

    def forward_batched(self, hidden, logits, M: int, use_graph: bool = False) -> None:
        """One batched step of M tokens on the current stream (see steps_batched); with
        use_graph the step is captured on the first call for these tensors and M."""
        torch = self.torch
        if not use_graph:
            st = c_void_p(torch.cuda.current_stream().cuda_stream)
            for op in self.steps_batched(hidden, logits, M):
                self._exchange(op, st)
            return
        key = ("b", hidden.data_ptr(), logits.data_ptr(), M)
        if self.max_seq and self.pos + M > self.max_seq:
            raise ValueError(f"positions {self.pos}..{self.pos + M - 1} exceed the cache of "
                             f"{self.max_seq} rows")
        if self.graph is None or self._graph_key != key:
            self.release_graph()
            saved = hidden.clone()
            p0 = self.pos
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                for op in self.steps_batched(hidden, logits, M):
                    self._exchange(op, c_void_p(s.cuda_stream))
            torch.cuda.current_stream().wait_stream(s)
            hidden.copy_(saved)
            if self.max_seq:  # the warm-up wrote these positions' cache rows: run them again
                self.set_position(p0)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, capture_error_mode="relaxed"):
                st = c_void_p(torch.cuda.current_stream().cuda_stream)
                for op in self.steps_batched(hidden, logits, M):
                    self._exchange(op, st)
            self.pos = p0
            self.graph, self._graph_key = g, key
        self.graph.replay()
        if self.max_seq:
            self.pos += M

    def launches_per_step(self) -> int:
        """Kernels of this library per step (NCCL collectives not counted; the peer-memory
        exchanges are)."""
        cfg = self.w.cfg
        n = 4 * cfg.n_layers + -(-self.w.shard.vocab_rows // cfg.logits_chunk_rows) + 1
        if self.max_seq:
            n += cfg.n_layers + 1  # fused RoPE + KV + attention per layer, position advance
        if self.p2p is not None:
            n += 2 * cfg.n_layers + 1
        return n

    def forward(self, hidden, logits, argmax=None, use_graph: bool = False) -> None:
        """One step on the current stream. hidden / logits / argmax are torch tensors on
        this rank's device; with use_graph the step is captured on the first call for these
        tensors and replayed afterwards."""
        if not use_graph:
            self._issue(hidden, logits, argmax)
            return
        torch = self.torch
        key = (hidden.data_ptr(), logits.data_ptr(), None if argmax is None else argmax.data_ptr())
        if self.max_seq and self.pos >= self.max_seq:
            raise ValueError(f"position {self.pos} is past the cache of {self.max_seq} rows")
        if self.graph is None or self._graph_key != key:
            self.release_graph()
            saved = hidden.clone()
            p0 = self.pos
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                # warm-up outside the capture (first collectives set up the communicator)
                self._issue(hidden, logits, argmax)
            torch.cuda.current_stream().wait_stream(s)
            hidden.copy_(saved)
            if self.max_seq:  # the warm-up wrote this position's cache row: decode it again
                self.set_position(p0)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, capture_error_mode="relaxed"):
                self._issue(hidden, logits, argmax)
            self.pos = p0
            self.graph, self._graph_key = g, key
        self.graph.replay()
        if self.max_seq:
            self.pos += 1

    def release_graph(self) -> None:
        """Drop the captured graph (it holds NCCL calls: release it before the process
        group is destroyed)."""
        if self.graph is not None:
            self.graph.reset()
            self.graph = None
            self._graph_key = None


def emulate_step(decoders, hiddens, logits_list, argmaxes=None, batch: int = 0) -> None:
    """Runs the ranks' steps of one process (all shards on the current device) in lockstep,
    doing each exchange with torch ops: the sum of the ranks' tensors for an all-reduce,
    the concatenation for an all-gather. batch > 0: the batched step of that many tokens.
    For checking the split on one GPU."""
    import torch
    if batch:
        gens = [dec.steps_batched(h, lg, batch) for dec, h, lg in zip(decoders, hiddens, logits_list)]
    else:
        gens = [dec.steps(h, lg, None if argmaxes is None else argmaxes[i])
                for i, (dec, h, lg) in enumerate(zip(decoders, hiddens, logits_list))]
    while True:
        ops = []
        for gi in gens:
            try:
                ops.append(next(gi))
            except StopIteration:
                ops.append(None)
        if all(o is None for o in ops):
            return
        if any(o is None for o in ops):
            raise RuntimeError("ranks disagree on the exchange sequence")
        if ops[0][0] == "all_reduce":
            total = torch.stack([o[1] for o in ops]).sum(0)
            for o in ops:
                o[1].copy_(total)
        elif ops[0][0] == "all_gather":
            full = torch.cat([o[2] for o in ops])
            for o in ops:
                o[1].copy_(full)
        else:
            M = ops[0][3]
            full = torch.cat([o[2].reshape(M, -1) for o in ops], dim=1)
            for o in ops:
                o[1].view(M, -1).copy_(full)
