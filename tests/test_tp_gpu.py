"""Tensor-parallel decode step on the GPU (recursive-routing-racer-rs_b200/tp.py).

* the range fills give exactly the slices of the full synthetic tensors;
* the G-rank split run in one process (exchanges done with torch ops, all shards on one
  GPU) equals the 1-GPU rrr_phi4_forward step at G = 2, 4 and 8 (8: O-proj windows that
  cut super-blocks) within 1e-4 relative L2 (only the summation order differs);
* with 2+ GPUs: the run with one process per GPU, eager and as a CUDA graph, with the
  exchanges as NCCL collectives, as the peer-memory kernels, or fused into the GEMVs
  (peer-memory pushes from the O-projection / down epilogues, sums in the next prologue),
  equals the 1-GPU step; the fused step has the bits of the unfused one.
"""
import importlib
import os
import socket
from ctypes import c_void_p

import numpy as np
import pytest

tp = importlib.import_module("recursive-routing-racer-rs_b200.tp")
phi4 = importlib.import_module("recursive-routing-racer-rs_b200.phi4")

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def test_range_fills_are_slices(rrr, ctx):
    import torch
    L = rrr.ffi.lib()
    qt, rows, nb = 14, 40, 12
    full = torch.empty(rows * nb * 210, dtype=torch.uint8, device="cuda")
    ctx.check(L.rrr_fill_kquant_random(ctx.h, qt, c_void_p(full.data_ptr()), rows * nb, 77, None))
    part = torch.empty(9 * 5 * 210, dtype=torch.uint8, device="cuda")
    # rows 30..38, block columns 4..8
    ctx.check(L.rrr_fill_kquant_random_2d(ctx.h, qt, c_void_p(part.data_ptr()), 9, 5, nb, 30 * nb + 4, 77, None))
    ref = full.view(rows, nb, 210)[30:39, 4:9].reshape(-1)
    assert torch.equal(part, ref)
    f = torch.empty(10000, device="cuda")
    g = torch.empty(3000, device="cuda")
    ctx.check(L.rrr_fill_f32_normal(ctx.h, c_void_p(f.data_ptr()), 10000, 0.0, 0.02, 5, None))
    ctx.check(L.rrr_fill_f32_range(ctx.h, c_void_p(g.data_ptr()), 3000, 6000, 1, 0.0, 0.02, 5, None))
    assert torch.equal(g, f[6000:9000])
    ctx.check(L.rrr_fill_f32_uniform(ctx.h, c_void_p(f.data_ptr()), 10000, 0.5, 1.5, 6, None))
    ctx.check(L.rrr_fill_f32_range(ctx.h, c_void_p(g.data_ptr()), 3000, 100, 0, 0.5, 1.5, 6, None))
    assert torch.equal(g, f[100:3100])


def _single_gpu(ctx, cfg, seed, hidden0):
    import torch
    m = phi4.SyntheticPhi4(ctx, cfg, seed=seed)
    dec = phi4.Phi4Decoder(ctx, m)
    h = hidden0.clone()
    lg = torch.empty(cfg.vocab_size, device="cuda")
    am = torch.zeros(1, dtype=torch.int32, device="cuda")
    dec.forward(h.data_ptr(), lg.data_ptr(), am.data_ptr(), False)
    torch.cuda.synchronize()
    out = (h.cpu().numpy(), lg.cpu().numpy(), int(am.item()))
    dec.close()
    m.close()
    return out


@pytest.mark.parametrize("G", [2, 4, 8])
def test_tp_split_emulated_matches_single_gpu(rrr, ctx, G):
    """Phi-4-mini shapes (2 layers, full vocab), all G ranks' shards on this GPU."""
    import torch
    cfg = phi4.ModelConfig(n_layers=2)
    seed = 11
    hidden0 = torch.randn(cfg.d_model, device="cuda")
    h1, lg1, am1 = _single_gpu(ctx, cfg, seed, hidden0)
    ws = [tp.SyntheticPhi4TP(ctx, cfg, tp.plan(cfg, G, g), seed=seed) for g in range(G)]
    decs = [tp.TPDecoder(ctx, w) for w in ws]
    hs = [hidden0.clone() for _ in range(G)]
    lgs = [torch.empty(cfg.vocab_size, device="cuda") for _ in range(G)]
    ams = [torch.zeros(1, dtype=torch.int32, device="cuda") for _ in range(G)]
    tp.emulate_step(decs, hs, lgs, ams)
    torch.cuda.synchronize()
    assert ctx.device_error() == 0
    for g in range(G):
        assert _rel(hs[g].cpu().numpy(), h1) < 1e-4
        assert _rel(lgs[g].cpu().numpy(), lg1) < 1e-4
        assert int(ams[g].item()) == am1
    for w in ws:
        w.close()


@pytest.mark.parametrize("G", [2, 4, 8])
def test_tp_kv_decode_emulated_matches_single_gpu(rrr, ctx, G):
    """KV-cache decode at positions 0..3 (RoPE, f16 caches of the rank's KV heads, fused
    attention; the O-projection input is the heads' attention output in the rank's column
    window): the emulated G-rank split equals the 1-GPU rrr_phi4_forward KV step."""
    import torch
    cfg = phi4.ModelConfig(n_layers=2)
    seed, max_seq = 13, 32
    m = phi4.SyntheticPhi4(ctx, cfg, seed=seed)
    dec1 = phi4.Phi4Decoder(ctx, m, max_seq=max_seq)
    ws = [tp.SyntheticPhi4TP(ctx, cfg, tp.plan(cfg, G, g), seed=seed) for g in range(G)]
    decs = [tp.TPDecoder(ctx, w, max_seq=max_seq) for w in ws]
    gen = torch.Generator(device="cuda").manual_seed(3)
    lg1 = torch.empty(cfg.vocab_size, device="cuda")
    am1 = torch.zeros(1, dtype=torch.int32, device="cuda")
    for pos in range(4):
        hidden0 = torch.randn(cfg.d_model, device="cuda", generator=gen)
        h1 = hidden0.clone()
        dec1.forward(h1.data_ptr(), lg1.data_ptr(), am1.data_ptr(), False)
        hs = [hidden0.clone() for _ in range(G)]
        lgs = [torch.empty(cfg.vocab_size, device="cuda") for _ in range(G)]
        ams = [torch.zeros(1, dtype=torch.int32, device="cuda") for _ in range(G)]
        tp.emulate_step(decs, hs, lgs, ams)
        torch.cuda.synchronize()
        assert ctx.device_error() == 0
        for g in range(G):
            assert _rel(hs[g].cpu().numpy(), h1.cpu().numpy()) < 1e-4, (pos, g)
            assert _rel(lgs[g].cpu().numpy(), lg1.cpu().numpy()) < 1e-4
            assert int(ams[g].item()) == int(am1.item())
            assert decs[g].pos == pos + 1
    dec1.close()
    m.close()
    for w in ws:
        w.close()


# ------------------------------------------------------------------ NCCL, 2 GPUs
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, q, comm, max_seq=0):
    import datetime
    import torch
    import torch.distributed as dist
    rrr = importlib.import_module("recursive-routing-racer-rs_b200")
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))
    dec = None
    try:
        ctx = rrr.Context(rank)
        cfg = phi4.ModelConfig(n_layers=2)
        seed = 12
        gen = torch.Generator(device="cuda").manual_seed(5)
        hidden0 = torch.randn(cfg.d_model, device="cuda", generator=gen)
        w = tp.SyntheticPhi4TP(ctx, cfg, tp.plan(cfg, world, rank), seed=seed)
        fused = comm == "p2p"
        dec = tp.TPDecoder(ctx, w, comm="p2p" if comm.startswith("p2p") else comm, max_seq=max_seq,
                           fused=fused)
        assert dec.fused == fused
        lg = torch.empty(cfg.vocab_size, device="cuda")
        am = torch.zeros(1, dtype=torch.int32, device="cuda")
        results = []
        for use_graph in (False, True, True):
            h = hidden0.clone()
            dec.forward(h, lg, am, use_graph=use_graph)
            torch.cuda.synchronize()
            results.append((h.cpu().numpy(), lg.cpu().numpy(), int(am.item())))
        dec.close()
        if rank == 0:
            if max_seq:
                # the same three tokens (positions 0, 1, 2) through the 1-GPU KV step
                m = phi4.SyntheticPhi4(ctx, cfg, seed=seed)
                d1 = phi4.Phi4Decoder(ctx, m, max_seq=max_seq)
                refs = []
                for _ in range(3):
                    h = hidden0.clone()
                    lg1 = torch.empty(cfg.vocab_size, device="cuda")
                    am1 = torch.zeros(1, dtype=torch.int32, device="cuda")
                    d1.forward(h.data_ptr(), lg1.data_ptr(), am1.data_ptr(), False)
                    torch.cuda.synchronize()
                    refs.append((h.cpu().numpy(), lg1.cpu().numpy(), int(am1.item())))
                d1.close()
                m.close()
            else:
                refs = [_single_gpu(ctx, cfg, seed, hidden0)] * 3
            q.put([(_rel(h, r[0]), _rel(lgr, r[1]), a == r[2]) for (h, lgr, a), r in zip(results, refs)]
                  + [ctx.device_error()])
        w.close()
    finally:
        if dec is not None:
            dec.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("comm,max_seq", [("nccl", 0), ("p2p", 0), ("p2p-unfused", 0), ("nccl", 16),
                                          ("p2p", 16), ("p2p-unfused", 16)])
def test_tp_nccl_two_gpus(comm, max_seq):
    """comm = nccl: torch.distributed collectives; p2p: the all-reduces fused into the
    GEMVs over peer memory; p2p-unfused: the rrr_comm_* peer-memory exchange kernels.
    max_seq > 0: three decode steps at positions 0, 1, 2 with the KV caches (eager, then
    captured and replayed), against the 1-GPU KV step."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = _free_port()
    procs = [mpc.Process(target=_nccl_rank, args=(r, 2, port, q, comm, max_seq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    res = q.get(timeout=10)
    assert res[-1] == 0
    for rh, rl, same in res[:-1]:
        assert rh < 1e-4 and rl < 1e-4 and same


# ------------------------------------------------------------------ fused vs unfused
def _fused_rank(rank, world, port, q, max_seq):
    import datetime
    import torch
    import torch.distributed as dist
    rrr = importlib.import_module("recursive-routing-racer-rs_b200")
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))
    try:
        ctx = rrr.Context(rank)
        cfg = phi4.ModelConfig(n_layers=3, vocab_size=8192)
        gen = torch.Generator(device="cuda").manual_seed(9)
        tokens = [torch.randn(cfg.d_model, device="cuda", generator=gen) for _ in range(4)]
        w = tp.SyntheticPhi4TP(ctx, cfg, tp.plan(cfg, world, rank), seed=21)
        runs, flags, launches = [], [], []
        for fused in (False, True):
            dec = tp.TPDecoder(ctx, w, comm="p2p", max_seq=max_seq, fused=fused)
            flags.append(dec.fused)
            launches.append(dec.launches_per_step())
            lg = torch.empty(cfg.vocab_size, device="cuda")
            am = torch.zeros(1, dtype=torch.int32, device="cuda")
            h = torch.empty(cfg.d_model, device="cuda")  # one buffer: the graph keeps it
            out = []
            # eager, captured, replayed, replayed: four tokens (positions 0..3 with a cache)
            for i, use_graph in enumerate((False, True, True, True)):
                h.copy_(tokens[i])
                dec.forward(h, lg, am, use_graph=use_graph)
                torch.cuda.synchronize()
                out.append((h.cpu().numpy().copy(), lg.cpu().numpy().copy(), int(am.item())))
            runs.append(out)
            dec.close()
        same = all(np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1]) and a[2] == b[2]
                   for a, b in zip(runs[0], runs[1]))
        q.put((rank, flags, launches, same, ctx.device_error()))
        w.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("max_seq", [0, 8])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_fused_exchange_bits_equal_unfused(world, max_seq):
    """One process per GPU: the one-token step with the all-reduces fused into the GEMVs
    (rank-order sums of tagged peer rows in the RMSNorm prologue) gives the same bits as the
    step with the exchange kernels, eager and replayed from its CUDA graph, at world 2, 4, 8
    (as many as the box has), with and without a KV cache, in fewer launches."""
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = _free_port()
    procs = [mpc.Process(target=_fused_rank, args=(r, world, port, q, max_seq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    for _ in range(world):
        rank, flags, launches, same, err = q.get(timeout=10)
        assert flags == [False, True], (rank, flags)
        assert launches[1] < launches[0], launches
        assert same, rank
        assert err == 0


# ------------------------------------------------------------------ exchange kernels
def _exchange_rank(rank, world, port, q, two_trip):
    import datetime
    import torch
    import torch.distributed as dist
    if two_trip is not None:
        os.environ["RRR_COMM_TWO_TRIP"] = two_trip
    rrr = importlib.import_module("recursive-routing-racer-rs_b200")
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))
    comm = None
    try:
        ctx = rrr.Context(rank)
        L = rrr.ffi.lib()
        big = 64 * 3072
        comm = tp.P2PComm(ctx, rank, world, max_elems=big)
        # large (two-trip) and small (one-trip) all-reduces, with an all-gather between them
        # that maps elements to CTAs differently; every call's inputs are known to every rank
        calls = ["ar", "ar_small", "ar", "ag", "ar", "ar", "ar_small", "ar"]
        results = []
        for k, kind in enumerate(calls):
            n = {"ar": big, "ar_small": 3072, "ag": 25000}[kind]
            inputs = [np.random.default_rng(1000 * k + r).standard_normal(n).astype(np.float32)
                      for r in range(world)]
            x = torch.from_numpy(inputs[rank]).cuda()
            if kind == "ag":
                out = torch.empty(world * n, device="cuda")
                ctx.check(L.rrr_comm_allgather_f32(comm.h, c_void_p(out.data_ptr()), c_void_p(x.data_ptr()),
                                                   n, None))
                want = np.concatenate(inputs)
            else:
                ctx.check(L.rrr_comm_allreduce_f32(comm.h, c_void_p(x.data_ptr()), n, None))
                out = x
                want = inputs[0].copy()
                for r in range(1, world):
                    want = want + inputs[r]  # rank order, f32
            torch.cuda.synchronize()
            results.append(bool(np.array_equal(out.cpu().numpy(), want)))
        q.put((rank, results, ctx.device_error()))
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("world,two_trip", [(2, None), (2, "1"), (4, None), (8, None)])
def test_comm_allreduce_two_trips_bits(world, two_trip):
    """The peer-memory all-reduce at 64 tokens x 3072 (two trips from 4 ranks: each rank's
    slice summed by its owner in rank order, the sums sent back) gives every rank the bits
    of the rank-order f32 sum, as the one-trip form does for small exchanges, across calls
    of different sizes and an all-gather in between. At 2 ranks once as built (one trip
    throughout) and once with RRR_COMM_TWO_TRIP=1 (two trips for every all-reduce)."""
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = _free_port()
    procs = [mpc.Process(target=_exchange_rank, args=(r, world, port, q, two_trip)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    for _ in range(world):
        rank, results, err = q.get(timeout=10)
        assert all(results), (rank, results)
        assert err == 0
