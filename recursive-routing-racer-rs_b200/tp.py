"""Tensor-parallel decode step of the weight path over G GPUs of one box (one process per
GPU): the Python host of the C ABI's rrr_tp_* / rrr_phi4_tp_* entry points.

The reference runs the whole model on one GPU (src/model/phi4.rs:1099-1196); the split
(rrr_tp_plan) makes every rank stream 1/G of the bytes:

    QKV       rows of the rank's query heads [h0, h1) and their KV heads [v0, v1): the
              position-0 attention (output = V of the head's KV group) is then local
    O-proj    the K columns of those heads (Megatron split). When the heads do not cover
              whole 256-wide super-blocks (8 GPUs: 384 columns), the rank keeps the
              super-block window around them and the GEMV input is zero outside the
              heads, so no block is split; the partial outputs are summed (all-reduce)
    gate_up   rows [f0, f1) of gate and the same rows of up: SiLU(gate)*up stays local
    down      the matching K columns [f0, f1) of every row; all-reduce of the partials
    logits    vocab rows [V*g/G, V*(g+1)/G), output RMSNorm fused; all-gather of the rows

The residual is added by rank 0 only, so the all-reduced sum carries it once. RMSNorm and
the argmax are replicated. The step itself (kernels and exchanges, one CUDA graph) runs in
C++ (rrr_phi4_forward on a rank made by rrr_phi4_tp_create); this module generates the
synthetic shards, sets up the exchange channel (NCCL through a unique id broadcast over
torch.distributed, or the peer-memory rrr_comm with IPC handles all-gathered the same
way) and runs the one-GPU emulation of a split (rrr_phi4_tp_forward_emulated).
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
    """Shard ranges of rank g of G (rrr_tp_plan of the C ABI; no GPU needed)."""
    sh = ffi.TPShard()
    rc = ffi.lib().rrr_tp_plan(cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim,
                               cfg.vocab_size, G, g, ctypes.byref(sh))
    if rc != 0:
        raise ValueError(ffi.last_error(None))
    return TPShard(sh.G, sh.g, (sh.q_head0, sh.q_head1), (sh.kv_head0, sh.kv_head1),
                   tuple((sh.qkv_rows[i][0], sh.qkv_rows[i][1]) for i in range(3)),
                   (sh.o_block0, sh.o_block1), sh.o_k_offset, (sh.ffn0, sh.ffn1),
                   (sh.vocab0, sh.vocab1))


def c_shard(shard: TPShard) -> "ffi.TPShard":
    """The rrr_tp_shard of a plan (what rrr_phi4_tp_create checks against its own plan)."""
    sh = ffi.TPShard()
    sh.G, sh.g = shard.G, shard.g
    sh.q_head0, sh.q_head1 = shard.q_heads
    sh.kv_head0, sh.kv_head1 = shard.kv_heads
    for i, (a, b) in enumerate(shard.qkv_rows):
        sh.qkv_rows[i][0], sh.qkv_rows[i][1] = a, b
    sh.qkv_dim = shard.qkv_dim
    sh.o_block0, sh.o_block1 = shard.o_blocks
    sh.o_k, sh.o_k_offset = shard.o_k, shard.o_k_offset
    sh.ffn0, sh.ffn1 = shard.ffn
    sh.vocab0, sh.vocab1 = shard.vocab
    return sh


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

    def desc(self, max_seq: int = 0):
        """rrr_phi4_desc of the shard tensors (full model dimensions); returns (desc, keep)."""
        cfg = self.cfg
        arr = (ffi.Phi4Layer * cfg.n_layers)()
        for i, e in enumerate(self.layers):
            arr[i].w_qkv, arr[i].qkv_type = e["qkv"], cfg.qkv_type
            arr[i].w_o, arr[i].o_type = e["o_proj"], cfg.o_type
            arr[i].w_gate_up, arr[i].gate_up_type = e["gate_up"], cfg.gate_up_type
            arr[i].w_down, arr[i].down_type = e["down"], cfg.down_type
            arr[i].attn_norm, arr[i].ffn_norm = e["attn_norm"], e["ffn_norm"]
        d = ffi.Phi4Desc(cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim,
                         cfg.n_layers, cfg.vocab_size, cfg.rms_eps, cfg.logits_chunk_rows,
                         ctypes.cast(arr, ctypes.POINTER(ffi.Phi4Layer)), self.output_norm, self.w_out,
                         max_seq, cfg.rope_dim, cfg.rope_theta, cfg.rope_attn_factor,
                         self.rope_factors, self.n_rope_factors)
        return d, arr

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
    handles are swapped with torch.distributed.all_gather_object. `tp` is its
    rrr_tp_comm for rrr_phi4_tp_create. fused_words > 0 adds the fused-exchange region
    (rrr_comm_create_ex) that lets a rank's step push its partial rows from the GEMVs."""

    def __init__(self, ctx: ffi.Context, rank: int, world: int, max_elems: int, group=None,
                 fused_words: int = 0):
        import torch.distributed as dist
        L = ffi.lib()
        self.ctx, self.group = ctx, group
        h = c_void_p()
        buf = ctypes.create_string_buffer(64)
        ctx.check(L.rrr_comm_create_ex(ctx.h, rank, world, max_elems, fused_words, ctypes.byref(h), buf))
        self.h = h
        handles = [None] * world
        dist.all_gather_object(handles, bytes(buf.raw), group=group)
        allh = ctypes.create_string_buffer(b"".join(handles), 64 * world)
        ctx.check(L.rrr_comm_connect(self.h, allh))
        dist.barrier(group=group)
        self.tp = c_void_p()
        ctx.check(L.rrr_tp_comm_p2p(self.h, ctypes.byref(self.tp)))

    def close(self) -> None:
        """Collective: every rank unmaps the others' buffers, then frees its own."""
        import torch.distributed as dist
        L = ffi.lib()
        if self.tp:
            L.rrr_tp_comm_destroy(self.tp)
            self.tp = None
        if self.h:
            L.rrr_comm_disconnect(self.h)
            dist.barrier(group=self.group)
            L.rrr_comm_destroy(self.h)
            self.h = None


class NcclComm:
    """An NCCL communicator made by the C ABI (rrr_tp_comm_nccl); rank 0's unique id is
    broadcast with torch.distributed."""

    def __init__(self, ctx: ffi.Context, rank: int, world: int, group=None):
        import torch.distributed as dist
        L = ffi.lib()
        uid = ctypes.create_string_buffer(128)
        if rank == 0:
            ffi.check(L.rrr_tp_nccl_unique_id(uid))
        obj = [bytes(uid.raw)]
        dist.broadcast_object_list(obj, src=0, group=group)
        uid = ctypes.create_string_buffer(obj[0], 128)
        self.tp = c_void_p()
        ctx.check(L.rrr_tp_comm_nccl(ctx.h, uid, rank, world, ctypes.byref(self.tp)))

    def close(self) -> None:
        if self.tp:
            ffi.lib().rrr_tp_comm_destroy(self.tp)
            self.tp = None


class TPDecoder:
    """One rank's decode step on the C ABI (rrr_phi4_tp_create + rrr_phi4_forward[_batched]):
    the kernels of the 1-GPU step on the rank's shards with the exchanges between them
    (NCCL, or the peer-memory kernels), capturable into one CUDA graph.

    max_seq = 0: every token at position 0 (attention output = V; forward_batched runs M
    independent sequences). max_seq > 0: a KV cache of the rank's KV heads (f16, max_seq
    rows per layer) and a device position: forward decodes one token at the position and
    advances it (RoPE, KV store and attention fused in one launch per layer);
    forward_batched is a prefill of M consecutive tokens of one sequence (RoPE + KV store
    of the M rows, causal attention, phi4.rs:1270-1309) and advances the position by M.
    comm = None with G > 1: the rank is only run through emulate_step."""

    def __init__(self, ctx: ffi.Context, weights: SyntheticPhi4TP, group=None, comm: str | None = None,
                 max_batch: int = 1, max_seq: int = 0, fused: bool = True):
        """comm: "nccl" (rrr_tp_comm_nccl), "p2p" (rrr_comm_* kernels over NVLink peer
        memory) or None; max_batch: the largest M of forward_batched (sizes the peer-memory
        buffers); max_seq: KV-cache rows (0: position-0 steps); fused: on "p2p", fuse the
        one-token step's all-reduces into its GEMVs (taken when every rank has its own GPU)."""
        self.ctx, self.w, self.group = ctx, weights, group
        self.max_seq = max_seq
        sh = weights.shard
        self.channel = None
        if comm not in (None, "nccl", "p2p"):
            raise ValueError(f"unknown comm {comm!r}")
        if comm == "p2p" and sh.G > 1:
            fw = 2 * weights.cfg.n_layers * sh.G * weights.cfg.d_model if fused else 0
            self.channel = P2PComm(ctx, sh.g, sh.G,
                                   max_batch * max(weights.cfg.d_model, sh.vocab_rows), group, fw)
        elif comm == "nccl" and sh.G > 1:
            self.channel = NcclComm(ctx, sh.g, sh.G, group)
        d, self._keep = weights.desc(max_seq)
        self._shard = c_shard(sh)
        h = c_void_p()
        ctx.check(ffi.lib().rrr_phi4_tp_create(ctx.h, ctypes.byref(d), ctypes.byref(self._shard),
                                               self.channel.tp if self.channel else None, ctypes.byref(h)))
        self.h = h

    @staticmethod
    def _stream(stream):
        import torch
        if stream is None:
            return c_void_p(torch.cuda.current_stream().cuda_stream)
        return c_void_p(stream if isinstance(stream, int) else stream.cuda_stream)

    @staticmethod
    def _ptr(t):
        return None if t is None else c_void_p(t if isinstance(t, int) else t.data_ptr())

    def forward(self, hidden, logits, argmax=None, use_graph: bool = False, stream=None) -> None:
        """One step on `stream` (default: the current torch stream). hidden f32[d] in/out,
        logits f32[vocab] (full on every rank), argmax int32[1] or None. use_graph: the first
        call runs the step and captures it; later calls with these buffers replay it."""
        self.ctx.check(ffi.lib().rrr_phi4_forward(self.h, self._ptr(hidden), self._ptr(logits),
                                                  self._ptr(argmax), 1 if use_graph else 0,
                                                  self._stream(stream)))

    def forward_batched(self, hidden, logits, M: int, argmax=None, use_graph: bool = False,
                        stream=None) -> None:
        """M tokens in one step: hidden f32 [M, d] in/out, logits f32 [M, vocab], argmax int32[M]
        or None."""
        self.ctx.check(ffi.lib().rrr_phi4_forward_batched(self.h, self._ptr(hidden), self._ptr(logits),
                                                          self._ptr(argmax), M, 1 if use_graph else 0,
                                                          self._stream(stream)))

    def wait(self, timeout_ms: int, stream=None) -> None:
        """Host deadline on the step's stream (rrr_tp_wait): raises RRRError with
        RRR_ERR_TIMEOUT / RRR_ERR_NCCL (the communicator aborted) on failure."""
        if self.channel is None:
            raise ValueError("no communicator")
        self.ctx.check(ffi.lib().rrr_tp_wait(self.channel.tp, self._stream(stream), timeout_ms))

    def set_position(self, pos: int) -> None:
        """KV-cache decode: position of the next token (KVCache.len)."""
        self.ctx.check(ffi.lib().rrr_phi4_set_position(self.h, pos, None))

    @property
    def pos(self) -> int:
        n = ctypes.c_int()
        self.ctx.check(ffi.lib().rrr_phi4_position(self.h, ctypes.byref(n)))
        return n.value

    @property
    def fused(self) -> bool:
        """Whether the one-token step's all-reduces run inside its GEMVs."""
        n = ctypes.c_int()
        self.ctx.check(ffi.lib().rrr_phi4_tp_fused(self.h, ctypes.byref(n)))
        return bool(n.value)

    def launches_per_step(self) -> int:
        """Kernels of this library per step (NCCL collectives not counted; the peer-memory
        exchanges are)."""
        n = ctypes.c_int()
        self.ctx.check(ffi.lib().rrr_phi4_launches_per_step(self.h, ctypes.byref(n)))
        return n.value

    def close(self) -> None:
        """Destroys the rank's step (its graphs hold the collectives: before the process
        group goes) and its channel (collective for the peer-memory one)."""
        if self.h:
            ffi.lib().rrr_phi4_destroy(self.h)
            self.h = None
        if self.channel is not None:
            self.channel.close()
            self.channel = None


def emulate_step(decoders, hiddens, logits_list, argmaxes=None, batch: int = 0, stream=None) -> None:
    """Runs the G ranks of one split (decoders made with comm=None, all on the current GPU)
    in lockstep with local exchanges (rrr_phi4_tp_forward_emulated): sums in rank order,
    concatenation for the logits. batch > 0: the batched step of that many tokens. For
    checking the split on one GPU."""
    G = len(decoders)
    ranks = (c_void_p * G)(*[dec.h.value for dec in decoders])
    hs = (c_void_p * G)(*[h.data_ptr() for h in hiddens])
    lgs = (c_void_p * G)(*[lg.data_ptr() for lg in logits_list])
    ams = None
    if argmaxes is not None:
        ams = (c_void_p * G)(*[a.data_ptr() if a is not None else None for a in argmaxes])
    ctx = decoders[0].ctx
    ctx.check(ffi.lib().rrr_phi4_tp_forward_emulated(ranks, G, hs, lgs, ams, batch,
                                                     TPDecoder._stream(stream)))
