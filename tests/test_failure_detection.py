"""Failure detection, exercised without faulting, trapping or hanging a GPU.

* On the GPU: rank 0 of a 2-rank peer-memory exchange (rrr_comm, NVLink/IPC mappings)
  whose rank 1 process maps its buffer but never calls the exchange. Rank 0's bounded wait
  runs out after the context's wait limit (set to 50 ms), the kernel records its code and
  returns, rrr_check_device_error reports RRR_ERR_TIMEOUT, and the context and the GPU
  keep working (a GEMV afterwards matches the oracle). The reference waits on its fences
  with no limit (src/gpu/engine.rs:312,369: u64::MAX).
* On the host (gloo ranks on CPU): a collective that one rank skips ends on the other
  rank with a clean timeout error from the host deadline, and the group is torn down.
"""
import ctypes
import importlib
import multiprocessing as mp
import os
import socket
import time
from ctypes import c_void_p

import numpy as np
import pytest

from conftest import rel_l2

tp = importlib.import_module("recursive-routing-racer-rs_b200.tp")


def _idle_peer(q, done):
    """Rank 1: creates its exchange buffer, publishes the IPC handle, never exchanges."""
    rrr = importlib.import_module("recursive-routing-racer-rs_b200")
    L = rrr.ffi.lib()
    ctx = rrr.Context(0)
    comm = c_void_p()
    h = ctypes.create_string_buffer(64)
    ctx.check(L.rrr_comm_create(ctx.h, 1, 2, 4096, ctypes.byref(comm), h))
    q.put(bytes(h.raw))
    done.wait(120)
    L.rrr_comm_destroy(comm)
    ctx.close()


@pytest.mark.gpu
def test_exchange_wait_expires_when_a_rank_never_arrives(rrr, ctx, oracle):
    import torch
    L = rrr.ffi.lib()
    spawn = mp.get_context("spawn")
    q, done = spawn.Queue(), spawn.Event()
    peer = spawn.Process(target=_idle_peer, args=(q, done))
    peer.start()
    comm = c_void_p()
    try:
        peer_handle = q.get(timeout=120)
        mine = ctypes.create_string_buffer(64)
        ctx.check(L.rrr_comm_create(ctx.h, 0, 2, 4096, ctypes.byref(comm), mine))
        handles = (ctypes.c_char * 128).from_buffer_copy(bytes(mine.raw) + peer_handle)
        ctx.check(L.rrr_comm_connect(comm, handles))
        ctx.check(L.rrr_set_wait_limit(ctx.h, 50_000_000))          # 50 ms
        x = torch.ones(4096, device="cuda")
        torch.cuda.synchronize()
        t0 = time.time()
        ctx.check(L.rrr_comm_allreduce_f32(comm, c_void_p(x.data_ptr()), 4096, None))
        code = ctypes.c_int(0)
        rc = L.rrr_check_device_error(ctx.h, ctypes.byref(code))
        elapsed = time.time() - t0
        assert rc == -7, rrr.ffi.last_error(ctx.h)                   # RRR_ERR_TIMEOUT
        assert code.value == 5                                       # exchange wait gave up
        assert 0.04 < elapsed < 5.0, elapsed
        # the host deadline of the tensor-parallel channel (rrr_tp_wait) ends before the
        # device's own 400 ms limit; the kernel then gives up by itself
        tpc = c_void_p()
        ctx.check(L.rrr_tp_comm_p2p(comm, ctypes.byref(tpc)))
        ctx.check(L.rrr_set_wait_limit(ctx.h, 400_000_000))
        torch.cuda.synchronize()
        t0 = time.time()
        ctx.check(L.rrr_comm_allreduce_f32(comm, c_void_p(x.data_ptr()), 4096, None))
        rc = L.rrr_tp_wait(tpc, None, 30)
        waited = time.time() - t0
        assert rc == -7 and "30 ms" in rrr.ffi.last_error(ctx.h), rrr.ffi.last_error(ctx.h)
        assert waited < 0.3, waited
        rc = L.rrr_check_device_error(ctx.h, ctypes.byref(code))
        assert rc == -7 and code.value == 5
        assert time.time() - t0 > 0.35
        L.rrr_tp_comm_destroy(tpc)
        # the context and the GPU still answer: a GEMV checked against the oracle
        ctx.check(L.rrr_set_wait_limit(ctx.h, 0))
        rng = np.random.default_rng(5)
        K, N = 3072, 256
        raw = oracle.random_blocks(12, N * K // 256, rng)
        xv = rng.standard_normal(K).astype(np.float32)
        wd, xd = torch.from_numpy(raw).cuda(), torch.from_numpy(xv).cuda()
        y = torch.empty(N, device="cuda")
        ctx.check(L.rrr_gemv_kq(ctx.h, 12, c_void_p(wd.data_ptr()), c_void_p(xd.data_ptr()),
                                c_void_p(y.data_ptr()), K, N, None, None))
        assert rel_l2(y.cpu().numpy(), oracle.gemv_kq(12, raw, xv, K, N)) < 1e-4
        assert ctx.device_error() == 0
    finally:
        L.rrr_set_wait_limit(ctx.h, 0)
        if comm.value:
            L.rrr_comm_disconnect(comm)
            L.rrr_comm_destroy(comm)
        done.set()
        peer.join(60)
        if peer.is_alive():
            peer.kill()
    assert peer.exitcode == 0


@pytest.mark.gpu
def test_tp_wait_with_a_one_rank_nccl_communicator(rrr, ctx):
    """NCCL loaded at run time by the library: a 1-rank communicator, a tensor-parallel
    rank of G = 1 on it, one step, and rrr_tp_wait returning on the completed stream."""
    import torch
    phi4 = importlib.import_module("recursive-routing-racer-rs_b200.phi4")
    L = rrr.ffi.lib()
    uid = ctypes.create_string_buffer(128)
    ctx.check(L.rrr_tp_nccl_unique_id(uid))
    tpc = c_void_p()
    ctx.check(L.rrr_tp_comm_nccl(ctx.h, uid, 0, 1, ctypes.byref(tpc)))
    cfg = phi4.ModelConfig(n_layers=1, vocab_size=4096)
    w = tp.SyntheticPhi4TP(ctx, cfg, tp.plan(cfg, 1, 0), seed=2)
    d, keep = w.desc()
    sh = tp.c_shard(w.shard)
    m = c_void_p()
    ctx.check(L.rrr_phi4_tp_create(ctx.h, ctypes.byref(d), ctypes.byref(sh), tpc, ctypes.byref(m)))
    h = torch.randn(cfg.d_model, device="cuda")
    lg = torch.empty(cfg.vocab_size, device="cuda")
    ctx.check(L.rrr_phi4_forward(m, c_void_p(h.data_ptr()), c_void_p(lg.data_ptr()), None, 1, None))
    ctx.check(L.rrr_tp_wait(tpc, None, 10000))
    assert torch.isfinite(lg).all()
    # a shard that is not the plan's is refused
    bad = tp.c_shard(w.shard)
    bad.ffn1 -= 256
    m2 = c_void_p()
    assert L.rrr_phi4_tp_create(ctx.h, ctypes.byref(d), ctypes.byref(bad), tpc, ctypes.byref(m2)) == -3
    L.rrr_phi4_destroy(m)
    L.rrr_tp_comm_destroy(tpc)
    w.close()


def _fused_stall_rank(rank, port, q):
    """Two ranks on two GPUs with the all-reduces fused into the GEMVs; rank 1 makes its
    model but never steps, so rank 0's prologues wait for rows that never come."""
    import datetime
    import torch
    import torch.distributed as dist
    rrr = importlib.import_module("recursive-routing-racer-rs_b200")
    phi4 = importlib.import_module("recursive-routing-racer-rs_b200.phi4")
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
    L = rrr.ffi.lib()
    ctx = rrr.Context(rank)
    cfg = phi4.ModelConfig(n_layers=2, vocab_size=4096)
    w = tp.SyntheticPhi4TP(ctx, cfg, tp.plan(cfg, 2, rank), seed=3)
    dec = tp.TPDecoder(ctx, w, comm="p2p")
    res = None
    if rank == 0:
        ctx.check(L.rrr_set_wait_limit(ctx.h, 50_000_000))          # 50 ms
        h = torch.randn(cfg.d_model, device="cuda")
        lg = torch.empty(cfg.vocab_size, device="cuda")
        torch.cuda.synchronize()
        t0 = time.time()
        dec.forward(h, lg)
        code = ctypes.c_int(0)
        rc = L.rrr_check_device_error(ctx.h, ctypes.byref(code))
        elapsed = time.time() - t0
        ctx.check(L.rrr_set_wait_limit(ctx.h, 0))
        # the context still works afterwards
        x = torch.ones(1 << 20, device="cuda")
        ok_after = float(x.sum().item()) == float(1 << 20) and ctx.device_error() == 0
        res = (dec.fused, rc, code.value, elapsed, ok_after)
    dist.barrier()
    dec.close()
    w.close()
    q.put((rank, res))
    dist.destroy_process_group()


@pytest.mark.gpu
def test_fused_exchange_wait_expires_when_a_rank_never_steps():
    """The fused exchange's waits (tagged rows in the GEMV prologue, the last site's sum) are
    bounded like the exchange kernel's: with a 50 ms limit the step ends in well under a
    second, the device flag holds the exchange code (5, not the weight stream's) and the
    GPU keeps working. Needs two GPUs (fused exchanges run only between distinct GPUs)."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    spawn = mp.get_context("spawn")
    q = spawn.Queue()
    port = _free_port()
    procs = [spawn.Process(target=_fused_stall_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        r, res = q.get(timeout=240)
        out[r] = res
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    fused, rc, code, elapsed, ok_after = out[0]
    assert fused
    assert rc == -7 and code == 5, (rc, code)
    assert 0.04 < elapsed < 5.0, elapsed
    assert ok_after


def test_wait_limit_range_is_checked(rrr):
    """Out-of-range limits are rejected; no GPU is needed to reach the check."""
    L = rrr.ffi.lib()
    assert L.rrr_set_wait_limit(None, 0) == -1


# ------------------------------------------------------------------ host side, gloo
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, port, q):
    import datetime
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
    t = torch.ones(1000)
    # step 1: both ranks take part
    tp.all_reduce_with_deadline(t, timeout_s=30.0)
    ok1 = float(t[0]) == 2.0
    if rank == 1:
        # rank 1 stays alive but never joins the next collective (a stalled rank)
        q.put((rank, ok1, None, 0.0))
        time.sleep(6.0)
        return
    t0 = time.time()
    err = None
    try:
        tp.all_reduce_with_deadline(t, timeout_s=2.0)
    except tp.TPTimeout as e:
        err = str(e)
    q.put((rank, ok1, err, time.time() - t0))


def test_host_deadline_on_a_skipped_collective():
    spawn = mp.get_context("spawn")
    q = spawn.Queue()
    port = _free_port()
    procs = [spawn.Process(target=_gloo_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, ok1, err, el = q.get(timeout=120)
        res[r] = (ok1, err, el)
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    assert res[0][0] and res[1][0]
    assert res[0][1] is not None and "deadline" in res[0][1]
    assert 1.5 < res[0][2] < 20.0


def test_tp_watchdog_loop_with_fakes(tmp_path):
    """The host watchdog of the tensor-parallel step (csrc/tp_watchdog.h, behind
    rrr_tp_wait) compiled with g++ and run against fake stream / communicator operations:
    completion, a stream error, an asynchronous communicator error and a missed deadline,
    each with the communicator aborted exactly when it must be."""
    import subprocess
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    exe = str(tmp_path / "test_tp_watchdog")
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Werror",
                    "-I", os.path.join(root, "recursive-routing-racer-rs_b200", "csrc"),
                    os.path.join(root, "tests", "cpp", "test_tp_watchdog.cpp"), "-o", exe], check=True)
    out = subprocess.run([exe], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout + out.stderr
    assert out.stdout.strip() == "ok"
