"""Tensor-parallel split of the decode step (recursive-routing-racer-rs_b200/tp.py).

CPU: the shard plan covers every head, row, column and vocab entry exactly once; and a
2-rank gloo run of the sharded step, each rank computing its shards with the oracle and
exchanging partial sums with all-reduce / all-gather, reproduces the oracle's 1-GPU
decode step (the shards are slices of the full seeded tensors).
GPU (2+ devices): the NCCL step on the C ABI equals the 1-GPU rrr_phi4_forward step.
"""
import importlib
import os
import socket

import numpy as np
import pytest

tp = importlib.import_module("recursive-routing-racer-rs_b200.tp")
phi4 = importlib.import_module("recursive-routing-racer-rs_b200.phi4")

BB = {12: 144, 13: 176, 14: 210}


def _phi4_cfg():
    return phi4.ModelConfig()


@pytest.mark.parametrize("G", [1, 2, 4, 8])
def test_plan_partitions_phi4(G):
    cfg = _phi4_cfg()
    hd, nq, nkv, F, V = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads, cfg.ffn_dim, cfg.vocab_size
    heads, kvs, qkv_rows, ffn, vocab = [], [], [], [], []
    for g in range(G):
        s = tp.plan(cfg, G, g)
        heads += list(range(*s.q_heads))
        kvs += list(range(*s.kv_heads))
        for a, b in s.qkv_rows:
            qkv_rows += list(range(a, b))
        ffn += list(range(*s.ffn))
        vocab.append(s.vocab)
        # every local query head maps to a local KV head
        hpk = nq // nkv
        assert s.q_heads[0] // hpk == s.kv_heads[0] and (s.q_heads[1] - 1) // hpk == s.kv_heads[1] - 1
        # the O-proj window holds the heads' columns, whole super-blocks
        c0 = s.q_heads[0] * hd
        assert 256 * s.o_blocks[0] + s.o_k_offset == c0
        assert s.o_k_offset + (s.q_heads[1] - s.q_heads[0]) * hd <= s.o_k
        assert s.o_k_offset % 8 == 0 and 0 <= s.o_k_offset < 256
        assert s.ffn[0] % 256 == 0 and s.ffn[1] % 256 == 0
    assert sorted(heads) == list(range(nq)) and sorted(kvs) == list(range(nkv))
    assert sorted(qkv_rows) == list(range(cfg.qkv_dim()))
    assert sorted(ffn) == list(range(F))
    assert vocab[0][0] == 0 and vocab[-1][1] == V and all(vocab[i][1] == vocab[i + 1][0] for i in range(G - 1))


def test_plan_rejects_bad_splits():
    cfg = _phi4_cfg()
    with pytest.raises(ValueError):
        tp.plan(cfg, 3, 0)          # 8 KV heads do not split 3 ways
    with pytest.raises(ValueError):
        tp.plan(cfg, 2, 2)


# ------------------------------------------------------------------ 2-rank gloo run
SMALL = dict(d_model=768, n_heads=6, n_kv_heads=2, head_dim=128, ffn_dim=1024, n_layers=2,
             vocab=1000, eps=1e-5)
TYPES = dict(qkv_type=13, o_type=12, gate_up_type=12, down_type=14)


def _small_model(oracle, seed=3):
    """Full small model from the device generator's streams (oracle restatement)."""
    c = SMALL
    d, F = c["d_model"], c["ffn_dim"]
    qkv_dim = (c["n_heads"] + 2 * c["n_kv_heads"]) * c["head_dim"]
    shapes = {"qkv": (TYPES["qkv_type"], d, qkv_dim), "o_proj": (TYPES["o_type"], c["n_heads"] * c["head_dim"], d),
              "gate_up": (TYPES["gate_up_type"], d, 2 * F), "down": (TYPES["down_type"], F, d)}
    rng = np.random.default_rng(seed)
    layers = []
    for l in range(c["n_layers"]):
        e = {}
        for name, (qt, K, N) in shapes.items():
            e[name] = oracle.fill_kquant_random(qt, N * (K // 256), phi4.tensor_seed(seed, l, name))
        e["attn_norm"] = rng.uniform(0.5, 1.5, d).astype(np.float32)
        e["ffn_norm"] = rng.uniform(0.5, 1.5, d).astype(np.float32)
        layers.append(e)
    out_norm = rng.uniform(0.5, 1.5, d).astype(np.float32)
    w_out = (rng.standard_normal((c["vocab"], d)) * 0.02).astype(np.float32)
    hidden = rng.standard_normal(d).astype(np.float32)
    return shapes, layers, out_norm, w_out, hidden


def _rows(raw, qt, K, rows, blocks=None):
    """Rows (list of (a, b)) and a super-block column window of a raw [N, K] matrix."""
    nb = K // 256
    m = raw.reshape(-1, nb, BB[qt])
    c0, c1 = blocks if blocks else (0, nb)
    return np.concatenate([m[a:b, c0:c1].reshape(-1) for a, b in rows])


def _rank_main(rank, world, port, q):
    import torch.distributed as dist
    import torch
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "oracle"))
    import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = SMALL
        cfg = phi4.ModelConfig(d_model=c["d_model"], n_heads=c["n_heads"], n_kv_heads=c["n_kv_heads"],
                               head_dim=c["head_dim"], ffn_dim=c["ffn_dim"], n_layers=c["n_layers"],
                               vocab_size=c["vocab"], rms_eps=c["eps"], **TYPES)
        shapes, layers, out_norm, w_out, hidden = _small_model(oracle)
        s = tp.plan(cfg, world, rank)
        d, F, hd = cfg.d_model, cfg.ffn_dim, cfg.head_dim
        nq_l, nkv_l = s.q_heads[1] - s.q_heads[0], s.kv_heads[1] - s.kv_heads[0]
        hpk = cfg.n_heads // cfg.n_kv_heads
        h = hidden.copy()
        for l, e in enumerate(layers):
            qt, K, N = shapes["qkv"]
            qkv = oracle.gemv_kq(qt, _rows(e["qkv"], qt, K, s.qkv_rows), oracle.rms_norm(h, e["attn_norm"]),
                                 K, s.qkv_dim)
            xo = np.zeros(s.o_k, np.float32)   # GQA-V input with the super-block window
            v = qkv[(nq_l + nkv_l) * hd:]
            for i in range(nq_l):
                xo[s.o_k_offset + i * hd: s.o_k_offset + (i + 1) * hd] = v[(i // hpk) * hd:(i // hpk + 1) * hd]
            qt, K, N = shapes["o_proj"]
            y = oracle.gemv_kq(qt, _rows(e["o_proj"], qt, K, [(0, d)], s.o_blocks), xo, s.o_k, d)
            if rank == 0:
                y = y + h
            t = torch.from_numpy(y)
            dist.all_reduce(t)
            h = t.numpy().copy()
            qt, K, N = shapes["gate_up"]
            gu = oracle.gemv_kq(qt, _rows(e["gate_up"], qt, K, [s.ffn, (F + s.ffn[0], F + s.ffn[1])]),
                                oracle.rms_norm(h, e["ffn_norm"]), K, 2 * s.ffn_dim)
            mid = oracle.silu_gate(gu)
            qt, K, N = shapes["down"]
            y = oracle.gemv_kq(qt, _rows(e["down"], qt, K, [(0, d)], (s.ffn[0] // 256, s.ffn[1] // 256)),
                               mid, s.ffn_dim, d)
            if rank == 0:
                y = y + h
            t = torch.from_numpy(y)
            dist.all_reduce(t)
            h = t.numpy().copy()
        loc = oracle.gemv_f32(w_out[s.vocab[0]:s.vocab[1]], oracle.rms_norm(h, out_norm))
        parts = [torch.empty(s.vocab_rows) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(loc))
        logits = torch.cat(parts).numpy()
        if rank == 0:
            ref_layers = [dict(w_qkv=e["qkv"], w_o=e["o_proj"], w_gate_up=e["gate_up"], w_down=e["down"],
                               attn_norm=e["attn_norm"], ffn_norm=e["ffn_norm"], **TYPES) for e in layers]
            h_ref, lg_ref = oracle.decode_step(c, ref_layers, out_norm, w_out, hidden)
            q.put((float(np.linalg.norm(h - h_ref) / np.linalg.norm(h_ref)),
                   float(np.linalg.norm(logits - lg_ref) / np.linalg.norm(lg_ref)),
                   int(np.argmax(logits)), int(np.argmax(lg_ref))))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_tp_step_gloo_matches_oracle(oracle):
    """2 ranks (gloo): the sharded step with all-reduce / all-gather equals the full step."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    rh, rl, am, am_ref = q.get(timeout=10)
    assert rh < 1e-5 and rl < 1e-5
    assert am == am_ref
