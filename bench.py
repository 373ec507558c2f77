#!/usr/bin/env python
"""Benchmark of the B200 weight path of RRR (K-quant GEMV HBM GB/s; Phi-4-mini-shape
decode tok/s). Prints ONE JSON line on rank 0.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the metric's config): the four per-layer GEMVs of
Phi-4-mini at batch 1 (QKV Q5_K 5120x3072, O Q4_K 3072x3072, gate_up Q4_K 16384x3072,
down Q6_K 3072x8192). One step = that GEMV set over all 32 layers' weights (seeded
synthetic blocks resident in HBM, 2.08 GB per pass, larger than the 126 MB L2, so no
flush is needed between steps). `value` = algorithmic bytes (weights + x + y) of all
ranks / device time (max over ranks). Under torchrun each rank runs its own copy of the
layer stack (independent weights, no data-path collective): scaling "weak".
Also reported: per-GEMV GB/s, the batched GEMM, the batched logits, the
end-to-end number through the C ABI with host buffers, a CPU baseline (the oracle's
restatement of the reference's dequant + f32 dot on the host cores) and, last on the line,
the full decode step tok/s with its CUDA graph, the tensor-parallel decode
step over all ranks (configs[4]; at one GPU the 1-GPU steps) and the roofline of the
dominant kernel (the layer GEMV with the largest time per layer).
"""
from __future__ import annotations

import argparse
import ctypes
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from ctypes import c_void_p

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

# DRAM bytes (read + write) of one launch of each layer GEMV, from the ncu capture
# summarised in profiles/gemv_kq_phi4_layer_shapes.md (nothing is written back to DRAM:
# the outputs stay in L2).
DRAM_BYTES = {"o_proj": 5367552, "gate_up": 28370688, "down": 20738304}
METRIC = "K-quant GEMV HBM GB/s (% of peak) per B200; Phi-4-mini-shape decode tok/s"
KERNEL_NAMES = {"qkv": "gemv_kq_kernel<Q5_K> (QKV 5120x3072)", "o_proj": "gemv_kq_kernel<Q4_K> (O 3072x3072)",
                "gate_up": "gemv_kq_kernel<Q4_K> (gate_up 16384x3072)",
                "down": "gemv_kq_kernel<Q6_K> (down 3072x8192)"}


def bench_config(world: int) -> dict:
    """The workload of the headline metric (the same dict on both arms)."""
    return {"workload": "configs[1]: per-layer GEMV set at batch 1 (QKV Q5_K 5120x3072, O Q4_K 3072x3072, "
                        "gate_up Q4_K 16384x3072, down Q6_K 3072x8192) over 32 layers' weights per step",
            "l2": "inputs larger than L2 (2.08 GB rotation per step), no flush",
            "parallelism": f"independent layer stacks per GPU (x{world})"}


def peaks(tensor: bool = False):
    """(peak, source): HBM copy GB/s, or with tensor=True the dense bf16 TFLOP/s burst
    figure, from MEASURED_PEAKS.json; the pool's earlier measurement when it is absent."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return (float(d["bf16_tflops"]) if tensor else float(d["hbm_gbs"])), "measured"
    except Exception:
        return (1590.0 if tensor else 6650.0), "fallback"


class Clocks:
    """Samples SM clocks and throttle reasons with nvidia-smi during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-f", self.path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        try:
            with open(self.path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) >= 9:
                        rows.append(parts)
            os.unlink(self.path)
        except Exception:
            return None
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_baseline(oracle, cfg, seconds: float = 10.0, layer_seed: int = 0):
    """The reference path on the host cores: dequantise each weight matrix to f32 (the
    reference's dequant_*) then a row-parallel f32 dot, over all host threads. Sample:
    the four GEMVs of one layer, repeated for about `seconds`."""
    import numpy as np
    from importlib import import_module
    phi4 = import_module("recursive-routing-racer-rs_b200.phi4")
    threads = os.cpu_count() or 1
    mats = []
    for name, qt, K, N in cfg.layer_gemvs():
        raw = oracle.fill_kquant_random(qt, N * (K // 256), phi4.tensor_seed(layer_seed, 0, name))
        x = np.random.default_rng(1).standard_normal(K).astype(np.float32)
        mats.append((qt, raw, x, K, N, np.empty(N * K, np.float32)))
    nbytes = sum(raw.nbytes + 4 * K + 4 * N for _, raw, _, K, N, _ in mats)
    t_deq = t_dot = 0.0
    reps = 0
    t0 = time.time()
    while reps < 1 or (time.time() - t0 < seconds and reps < 50):
        for qt, raw, x, K, N, scratch in mats:
            _, td, tt = oracle.gemv_kq_baseline(qt, raw, x, K, N, threads, scratch)
            t_deq += td
            t_dot += tt
        reps += 1
    total = t_deq + t_dot
    return {"value": round(nbytes * reps / total / 1e9, 3), "unit": "GB/s", "cores": threads,
            "kind": "port",
            "sample": f"one layer's 4 GEMVs (QKV Q5_K, O Q4_K, gate_up Q4_K, down Q6_K; "
                      f"{nbytes / 1e6:.1f} MB algorithmic) x {reps} reps; dequant {t_deq:.2f}s + dot {t_dot:.2f}s",
            "dequant_s": round(t_deq, 3), "dot_s": round(t_dot, 3)}


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU path (oracle port; the Rust reference cannot be
    built in this image) on the host cores, same metric/config."""
    if rank != 0:
        return
    import oracle
    oracle.build()
    from importlib import import_module
    phi4 = import_module("recursive-routing-racer-rs_b200.phi4")
    cfg = phi4.ModelConfig()
    per_step = max(1.0, 60.0 / max(1, args.steps + args.warmup))
    for _ in range(args.warmup):
        cpu_baseline(oracle, cfg, seconds=0.0)
    t0 = time.time()
    vals = []
    for _ in range(args.steps):
        vals.append(cpu_baseline(oracle, cfg, seconds=min(per_step, 10.0)))
    el = time.time() - t0
    v = round(statistics.mean(x["value"] for x in vals), 3)
    cb = dict(vals[-1])
    cb["value"] = v
    line = {"metric": METRIC, "value": v, "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * el / max(1, args.steps), 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": bench_config(args.gpus),
            "cpu_baseline": cb, "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def bench_gguf_load(rrr, ctx):
    """Load GB/s of rrr_gguf_load for a synthetic 2 GB GGUF written with gguf-py."""
    import numpy as np
    try:
        import gguf
        from gguf import GGMLQuantizationType as T
    except Exception as e:  # gguf-py missing: the measurement is skipped, not faked
        return {"skipped": str(e)}
    path = os.path.join(tempfile.gettempdir(), f"rrr_bench_{os.getpid()}.gguf")
    try:
        w = gguf.GGUFWriter(path, "phi3")
        raw = np.random.default_rng(0).integers(0, 256, size=(16384, 8192), dtype=np.uint8)  # 128 MiB
        raw = np.ascontiguousarray(raw[:, : (8192 // 144) * 144])
        names = [f"blk.{i}.ffn_up.weight" for i in range(16)]
        for nm in names:
            w.add_tensor(nm, raw, raw_dtype=T.Q4_K)
        w.write_header_to_file()
        w.write_kv_data_to_file()
        w.write_tensors_to_file()
        w.close()
        g = rrr.GGUFModel.load(path)
        ptrs, sizes, secs = g.load_tensors(ctx, names)
        ffi = rrr.ffi
        ctx.check(ffi.lib().rrr_free(ctx.h, c_void_p(ptrs[0])))
        ptrs, sizes, secs = g.load_tensors(ctx, names)  # second load: staging set up
        ctx.check(ffi.lib().rrr_free(ctx.h, c_void_p(ptrs[0])))
        g.close()
        tot = sum(sizes)
        return {"bytes": tot, "s": round(secs, 4), "GBps": round(tot / secs / 1e9, 2), "tensors": len(names),
                "path": "mmap -> 2 x 32 MB pinned (8 host threads) -> cudaMemcpyAsync, overlapped; page cache warm"}
    finally:
        try:
            os.unlink(path)
        except OSError:
            pass


def run_ours(args, rank, world, local_rank):
    import numpy as np
    import torch
    rrr = importlib.import_module("recursive-routing-racer-rs_b200")
    importlib.import_module("recursive-routing-racer-rs_b200.build").build()
    phi4 = importlib.import_module("recursive-routing-racer-rs_b200.phi4")
    ffi = rrr.ffi
    L = ffi.lib()
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank),
                                timeout=datetime.timedelta(seconds=120))
    ctx = ffi.Context(local_rank)
    stream = torch.cuda.current_stream()
    sp = c_void_p(stream.cuda_stream)
    cfg = phi4.ModelConfig()
    model = phi4.SyntheticPhi4(ctx, cfg, seed=1000 + rank, stream=sp)
    gemvs = cfg.layer_gemvs()
    # x / y of every GEMV of the 32-layer pass, packed in one device buffer each (the
    # end-to-end leg copies them from / to pinned host memory in one transfer each)
    x_off, y_off, xo, yo = {}, {}, 0, 0
    for l in range(cfg.n_layers):
        for name, _, K, N in gemvs:
            x_off[l, name], y_off[l, name] = xo, yo
            xo += K
            yo += N
    X = torch.randn(xo, device="cuda")
    Y = torch.empty(yo, device="cuda")
    bytes_layer = sum(cfg.weight_bytes(q, K, N) + 4 * K + 4 * N for _, q, K, N in gemvs)
    bytes_step = bytes_layer * cfg.n_layers
    launches_step = 4 * cfg.n_layers
    qname = {12: "matmul_q4k", 13: "matmul_q5k", 14: "matmul_q6k"}

    def add_gemv(batch, l, name):
        p, qt, K, N = model.layers[l][name]
        bufs = (c_void_p * 3)(X.data_ptr() + 4 * x_off[l, name], p, Y.data_ptr() + 4 * y_off[l, name])
        sizes = (ctypes.c_uint64 * 3)(4 * K, cfg.weight_bytes(qt, K, N), 4 * N)
        push = ctypes.create_string_buffer(rrr.push_u32(K, N), 8)
        ctx.check(L.rrr_batch_add(batch, qname[qt].encode(), bufs, sizes, 3, push, 8))

    def make_batch(names):
        b = c_void_p()
        ctx.check(L.rrr_batch_create(ctx.h, ctypes.byref(b)))
        for l in range(cfg.n_layers):
            for name in names:
                add_gemv(b, l, name)
        return b

    # The step as a prebuilt dispatch table (the reference's pre_allocate_desc_set +
    # dispatch_batch_persistent_v2), replayed as one CUDA graph per step.
    step_batch = make_batch([g[0] for g in gemvs])

    def step():
        ctx.check(L.rrr_batch_launch(step_batch, sp))

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if not dist:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---------------- headline: per-layer GEMV set over 32 layers
    for _ in range(max(3, args.warmup)):
        step()
    clocks = Clocks(local_rank)
    barrier()
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    # ---------------- per-GEMV: one shape over the 32 layers' weights per replay
    per = {}
    for name, qt, K, N in gemvs:
        b = make_batch([name])
        ctx.check(L.rrr_batch_launch(b, sp))
        a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(5, args.steps)
        a.record(stream)
        for _ in range(reps):
            ctx.check(L.rrr_batch_launch(b, sp))
        z.record(stream)
        torch.cuda.synchronize()
        L.rrr_batch_destroy(b)
        us = 1e3 * a.elapsed_time(z) / (reps * cfg.n_layers)
        nb = cfg.weight_bytes(qt, K, N) + 4 * K + 4 * N
        per[name] = {"qtype": {12: "Q4_K", 13: "Q5_K", 14: "Q6_K"}[qt], "K": K, "N": N, "bytes": nb,
                     "us_per_launch": round(us, 3), "GBps": round(nb / us / 1e3, 1),
                     "frac": round(nb / us / 1e3 / peaks()[0], 4)}
    # ---------------- batched-token GEMM: tcgen05 tiles, one launch per layer's
    # weights (32 distinct matrices per pass, larger than L2), M tokens of bf16 input
    batched = {}
    # configs[3]'s M = 16 / 64 / 256, and 4 / 8 tokens (the mma.sync kernel's 16-token tile)
    for name, M in [(n, m) for n in ("gate_up", "down") for m in (4, 8, 16, 64, 256)]:
        _, qt, K, N = model.layers[0][name]
        Xb = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        Yb = torch.empty(M, N, device="cuda")

        def gemm(l):
            ctx.check(L.rrr_gemm_kq_batched(ctx.h, qt, c_void_p(model.layers[l][name][0]),
                                            c_void_p(Xb.data_ptr()), c_void_p(Yb.data_ptr()), M, K, N, sp))
        for l in range(3):
            gemm(l)
        a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        passes = 2
        a.record(stream)
        for _ in range(passes):
            for l in range(cfg.n_layers):
                gemm(l)
        z.record(stream)
        torch.cuda.synchronize()
        us = 1e3 * a.elapsed_time(z) / (passes * cfg.n_layers)
        flops = 2.0 * M * N * K
        wb = cfg.weight_bytes(qt, K, N) + 2 * M * K + 4 * M * N
        batched[f"{name}_M{M}"] = {
            "qtype": {12: "Q4_K", 13: "Q5_K", 14: "Q6_K"}[qt], "M": M, "K": K, "N": N,
            "path": "mma.sync" if 3 <= M <= 64 else "tcgen05" if M > 64 else "per-token GEMV",
            "us_per_launch": round(us, 3), "TFLOPs": round(flops / us / 1e6, 1),
            "tensor_frac": round(flops / us / 1e6 / peaks(tensor=True)[0], 4),
            "GBps": round(wb / us / 1e3, 1), "hbm_frac": round(wb / us / 1e3 / peaks()[0], 4)}
        del Xb, Yb
    clk = clocks.stop()
    peak, peak_src = peaks()
    # ---------------- decode step through the CUDA graph
    dec = phi4.Phi4Decoder(ctx, model)
    hidden = torch.randn(cfg.d_model, device="cuda")
    logits = torch.empty(cfg.vocab_size, device="cuda")
    am = torch.zeros(1, dtype=torch.int32, device="cuda")
    for _ in range(max(3, args.warmup)):
        dec.forward(hidden.data_ptr(), logits.data_ptr(), am.data_ptr(), True, stream)
    barrier()
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dsteps = max(args.steps, 10)
    d0.record(stream)
    for _ in range(dsteps):
        dec.forward(hidden.data_ptr(), logits.data_ptr(), am.data_ptr(), True, stream)
    d1.record(stream)
    barrier()
    dms = max_over_ranks(d0.elapsed_time(d1) / dsteps)
    dec_bytes = cfg.step_bytes()
    decode = {"tok_s": round(1e3 / dms, 2), "ms_per_token": round(dms, 4),
              "GBps": round(dec_bytes / dms / 1e6, 1), "bytes_per_token": dec_bytes,
              "frac_of_peak": round(dec_bytes / dms / 1e6 / peak, 4),
              "launches_per_token": dec.launches_per_step() + 1, "graph": True}
    dec.close()
    # the same step with the logits dispatched as the reference does, in 32768-row chunks
    # (7 launches instead of 1; identical rows and bytes)
    import dataclasses
    cfg_c = dataclasses.replace(cfg, logits_chunk_rows=32768)
    model.cfg, cfg0 = cfg_c, model.cfg
    cdec = phi4.Phi4Decoder(ctx, model)
    model.cfg = cfg0
    for _ in range(max(3, args.warmup)):
        cdec.forward(hidden.data_ptr(), logits.data_ptr(), am.data_ptr(), True, stream)
    barrier()
    d0.record(stream)
    for _ in range(dsteps):
        cdec.forward(hidden.data_ptr(), logits.data_ptr(), am.data_ptr(), True, stream)
    d1.record(stream)
    barrier()
    decode["tok_s_logits_32768_row_chunks"] = round(1e3 / max_over_ranks(d0.elapsed_time(d1) / dsteps), 2)
    cdec.close()
    # ---------------- decode at real positions (KV cache of 2048 rows, RoPE, attention):
    # graph replays at positions 1024 .. 1024 + steps (the position advances on the device)
    kdec = phi4.Phi4Decoder(ctx, model, max_seq=2048)
    P0 = 1024
    kdec.set_position(P0 - max(3, args.warmup), stream)
    for _ in range(max(3, args.warmup)):
        kdec.forward(hidden.data_ptr(), logits.data_ptr(), am.data_ptr(), True, stream)
    barrier()
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ksteps = max(args.steps, 10)
    k0.record(stream)
    for _ in range(ksteps):
        kdec.forward(hidden.data_ptr(), logits.data_ptr(), am.data_ptr(), True, stream)
    k1.record(stream)
    barrier()
    kms = max_over_ranks(k0.elapsed_time(k1) / ksteps)
    kv_bytes = 2 * 2 * cfg.n_kv_heads * cfg.head_dim * cfg.n_layers * (P0 + ksteps / 2)
    decode_kv = {"positions": [P0, P0 + ksteps], "tok_s": round(1e3 / kms, 2),
                 "ms_per_token": round(kms, 4),
                 "GBps": round((dec_bytes + kv_bytes) / kms / 1e6, 1),
                 "launches_per_token": kdec.launches_per_step() + 1, "graph": True}
    kdec.close()
    # ---------------- batched decode step, 64 tokens at position 0 (configs[4] batch 64 on
    # one GPU / one rank's replica) through the C++ driver (rrr_phi4_forward_batched):
    # tensor-core GEMMs for every layer GEMM, batched logits, argmax of every row
    BM = 64
    bdec = phi4.Phi4Decoder(ctx, model)
    bh = torch.randn(BM, cfg.d_model, device="cuda")
    blg = torch.empty(BM, cfg.vocab_size, device="cuda")
    bam = torch.zeros(BM, dtype=torch.int32, device="cuda")
    for _ in range(max(3, args.warmup)):
        bdec.forward_batched(bh.data_ptr(), blg.data_ptr(), BM, bam.data_ptr(), True, stream)
    barrier()
    b0e, b1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    bsteps = max(5, args.steps // 2)
    b0e.record(stream)
    for _ in range(bsteps):
        bdec.forward_batched(bh.data_ptr(), blg.data_ptr(), BM, bam.data_ptr(), True, stream)
    b1e.record(stream)
    barrier()
    bms = max_over_ranks(b0e.elapsed_time(b1e) / bsteps)
    decode_batch = {"batch": BM, "tok_s": round(BM * 1e3 / bms, 1), "ms_per_step": round(bms, 4),
                    "graph": True, "api": "rrr_phi4_forward_batched",
                    "path": "per layer: rmsnorm->bf16, 4 batched K-quant GEMMs (mma.sync at M <= 64, tcgen05 above; "
                            "residual in the epilogue), GQA-V / SiLU glue; logits on the 3xTF32 tcgen05 kernel, "
                            "row-wise argmax"}
    bdec.close()
    # ---------------- batched logits alone (rrr_logits_f32_batched: 3xTF32 tcgen05 kernel,
    # output RMSNorm fused) for the 64 tokens over the 200064 x 3072 f32 matrix (2.46 GB per
    # launch, larger than L2)
    lx = torch.randn(BM, cfg.d_model, device="cuda")
    lxn = torch.empty(BM, cfg.d_model, device="cuda")
    ly = torch.empty(BM, cfg.vocab_size, device="cuda")

    def logits_b():
        ctx.check(L.rrr_logits_f32_batched(ctx.h, c_void_p(model.w_out), c_void_p(lx.data_ptr()),
                                           c_void_p(lxn.data_ptr()), c_void_p(ly.data_ptr()), BM,
                                           cfg.vocab_size, cfg.d_model, c_void_p(model.output_norm),
                                           cfg.rms_eps, sp))
    for _ in range(3):
        logits_b()
    l0e, l1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0e.record(stream)
    for _ in range(5):
        logits_b()
    l1e.record(stream)
    torch.cuda.synchronize()
    lus = 1e3 * l0e.elapsed_time(l1e) / 5
    lbytes = 4 * cfg.vocab_size * cfg.d_model + 8 * BM * cfg.d_model + 4 * BM * cfg.vocab_size
    logits_batched = {"M": BM, "V": cfg.vocab_size, "K": cfg.d_model, "us": round(lus, 1),
                      "GBps": round(lbytes / lus / 1e3, 1), "hbm_frac": round(lbytes / lus / 1e3 / peaks()[0], 4),
                      "kernel": "logits_tc_kernel (3xTF32 tcgen05) + rmsnorm"}
    del lx, lxn, ly
    # ---------------- tensor-parallel decode step (configs[4], batch 1) over all ranks
    tp_decode = None
    if world > 1:
        tpm = importlib.import_module("recursive-routing-racer-rs_b200.tp")
        shard = tpm.plan(cfg, world, rank)
        tw = tpm.SyntheticPhi4TP(ctx, cfg, shard, seed=7, stream=sp)
        th = torch.randn(cfg.d_model, device="cuda")
        tl = torch.empty(cfg.vocab_size, device="cuda")
        ta = torch.zeros(1, dtype=torch.int32, device="cuda")

        def time_tp(comm, fused=True):
            tdec = tpm.TPDecoder(ctx, tw, comm=comm, fused=fused)
            is_fused = comm == "p2p" and tdec.fused
            for _ in range(max(3, args.warmup)):
                tdec.forward(th, tl, ta, use_graph=True)
            barrier()
            t0e, t1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0e.record(stream)
            for _ in range(dsteps):
                tdec.forward(th, tl, ta, use_graph=True)
            t1e.record(stream)
            barrier()
            t = max_over_ranks(t0e.elapsed_time(t1e) / dsteps)
            n_l = tdec.launches_per_step()
            tdec.close()
            return t, n_l, is_fused

        # the all-reduces fused into the GEMVs (peer-memory pushes), the exchange kernels
        # between the GEMVs, and NCCL collectives
        tms, tl_p2p, tp_fused = time_tp("p2p")
        tms_unf, tl_unf, _ = time_tp("p2p", fused=False)
        tms_nccl, _, _ = time_tp("nccl")
        # at real positions: KV caches of the rank's heads, positions 1024 .. 1024 + steps
        kdec = tpm.TPDecoder(ctx, tw, comm="p2p", max_seq=2048)
        kdec.set_position(1024 - max(3, args.warmup))
        for _ in range(max(3, args.warmup)):
            kdec.forward(th, tl, ta, use_graph=True)
        barrier()
        t0e, t1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0e.record(stream)
        for _ in range(dsteps):
            kdec.forward(th, tl, ta, use_graph=True)
        t1e.record(stream)
        barrier()
        tkms = max_over_ranks(t0e.elapsed_time(t1e) / dsteps)
        kdec.close()
        # batch 64 over the ranks (peer-memory exchanges of [64, 3072] and [64, V/G])
        tb = tpm.TPDecoder(ctx, tw, comm="p2p", max_batch=BM)
        tbh = torch.randn(BM, cfg.d_model, device="cuda")
        tblg = torch.empty(BM, cfg.vocab_size, device="cuda")
        for _ in range(max(3, args.warmup)):
            tb.forward_batched(tbh, tblg, BM, use_graph=True)
        barrier()
        t0e, t1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0e.record(stream)
        for _ in range(bsteps):
            tb.forward_batched(tbh, tblg, BM, use_graph=True)
        t1e.record(stream)
        barrier()
        tbms = max_over_ranks(t0e.elapsed_time(t1e) / bsteps)
        tb.close()
        # the tensor-parallel decode step over all ranks (peer-memory exchanges;
        # NCCL beside it), batch 1 at position 0 and at positions 1024+, and batch 64
        tp_decode = {"n_gpus": world, "tok_s": round(1e3 / tms, 2), "ms_per_token": round(tms, 4),
                     "fused_exchanges": tp_fused,
                     "tok_s_exchange_kernels": round(1e3 / tms_unf, 2),
                     "tok_s_nccl": round(1e3 / tms_nccl, 2),
                     "kv_tok_s": round(1e3 / tkms, 2), "batch64_tok_s": round(BM * 1e3 / tbms, 1),
                     "GBps_per_rank": round(tw.shard_bytes() / tms / 1e6, 1),
                     "exchange_kernels_per_token": (3 if tp_fused else 2 * cfg.n_layers + 1),
                     "launches_per_token": tl_p2p, "launches_per_token_exchange_kernels": tl_unf}
        tw.close()
    # ---------------- end to end through the C ABI with host buffers (pinned): copy every
    # x of the step in, replay the prebuilt table, copy every y out, synchronise
    hX = torch.randn(xo).pin_memory()
    hY = torch.empty(yo).pin_memory()
    h2d, d2h = hX.numel() * 4, hY.numel() * 4

    # In chunks of 8 layers: the chunk's x in on a copy stream, its prebuilt table (32 GEMVs)
    # on the compute stream once the copy has landed, its y out on a second copy stream, so
    # the copies of one chunk overlap the GEMVs of its neighbours.
    CH = 8
    n_ch = (cfg.n_layers + CH - 1) // CH
    chunk_batches = []
    for c in range(n_ch):
        b = c_void_p()
        ctx.check(L.rrr_batch_create(ctx.h, ctypes.byref(b)))
        for l in range(c * CH, min(cfg.n_layers, (c + 1) * CH)):
            for name in [g[0] for g in gemvs]:
                add_gemv(b, l, name)
        chunk_batches.append(b)
    first = gemvs[0][0]

    def span(off, total, c):
        lo = off[c * CH, first]
        hi = off[(c + 1) * CH, first] if (c + 1) * CH < cfg.n_layers else total
        return 4 * lo, 4 * (hi - lo)
    xr = [span(x_off, xo, c) for c in range(n_ch)]
    yr = [span(y_off, yo, c) for c in range(n_ch)]
    c_in, c_out = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(n_ch)]
    ev_out = [torch.cuda.Event() for _ in range(n_ch)]

    def e2e_step():
        main = torch.cuda.current_stream()
        c_in.wait_stream(main)
        c_out.wait_stream(main)
        for c in range(n_ch):
            (xo_, xb), (yo_, yb) = xr[c], yr[c]
            ctx.check(L.rrr_h2d(ctx.h, c_void_p(X.data_ptr() + xo_), c_void_p(hX.data_ptr() + xo_), xb,
                                c_void_p(c_in.cuda_stream)))
            ev_in[c].record(c_in)
            main.wait_event(ev_in[c])
            ctx.check(L.rrr_batch_launch(chunk_batches[c], c_void_p(main.cuda_stream)))
            ev_out[c].record(main)
            c_out.wait_event(ev_out[c])
            ctx.check(L.rrr_d2h(ctx.h, c_void_p(hY.data_ptr() + yo_), c_void_p(Y.data_ptr() + yo_), yb,
                                c_void_p(c_out.cuda_stream)))
        main.wait_stream(c_in)
        main.wait_stream(c_out)
        torch.cuda.synchronize()

    for _ in range(3):
        e2e_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e2e_ms = max_over_ranks(1e3 * (time.perf_counter() - t0) / args.steps)
    L.rrr_batch_destroy(step_batch)
    for b in chunk_batches:
        L.rrr_batch_destroy(b)
    code = ctx.device_error()
    if code:
        raise SystemExit(f"device error flag {code}")
    # ---------------- GGUF load (rank 0, N = 1 only): a synthetic 2 GB file of 16 Q4_K
    # tensors (page cache warm: the file was just written) into one device allocation
    # through rrr_gguf_load's pinned staging
    gguf_load = None
    if rank == 0 and world == 1:
        gguf_load = bench_gguf_load(rrr, ctx)
    # ---------------- CPU baseline (rank 0, N = 1 only)
    cb = None
    if rank == 0 and world == 1:
        import oracle
        oracle.build()
        cb = cpu_baseline(oracle, cfg, seconds=10.0)
    if rank == 0:
        gbs = bytes_step * world / ms / 1e6
        # the dominant kernel: the layer GEMV with the largest time per layer
        dom_name = max(per, key=lambda k: per[k]["us_per_launch"])
        dom = per[dom_name]
        cases = {k: [v["us_per_launch"], v["path"], v["TFLOPs"], v["tensor_frac"], v["hbm_frac"]]
                 for k, v in batched.items()}
        if tp_decode is None:
            # one GPU: the decode steps themselves are the 1-rank point of the TP curve
            tp_decode = {"n_gpus": 1, "tok_s": decode["tok_s"], "kv_tok_s": decode_kv["tok_s"],
                         "batch64_tok_s": decode_batch["tok_s"]}
        # Order: the bulky detail first, the figures a reader looks for last (the driver keeps
        # the tail of the line).
        line = {
            "metric": METRIC, "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8 (K-quant) x f32",
            "data": "synthetic",
            "config": bench_config(world),
            "batched_gemm": {"cols": ["us", "path", "TFLOPs", "tensor_frac", "hbm_frac"], "cases": cases},
            "decode_batch64": {"tok_s": decode_batch["tok_s"], "ms_per_step": decode_batch["ms_per_step"],
                               "api": decode_batch["api"]},
            "logits_batched": logits_batched,
            "gguf_load": gguf_load,
            "per_gemv": {k: {"us": v["us_per_launch"], "GBps": v["GBps"], "frac": v["frac"]} for k, v in per.items()},
            "frac_of_peak": round(gbs / world / peak, 4),
            "e2e": {"value": round(bytes_step / e2e_ms / 1e6, 1), "unit": "GB/s", "ms_per_step": round(e2e_ms, 3),
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "rrr_h2d (copy stream) -> rrr_batch_launch of a prebuilt table of 32 GEMVs -> rrr_d2h "
                            "(second copy stream), per chunk of 8 layers, overlapped; pinned host buffers"},
            "gpu_launches": launches_step * args.steps,
            "clocks": clk,
            "cpu_baseline": cb,
            "decode": {"tok_s": decode["tok_s"], "ms_per_token": decode["ms_per_token"],
                       "frac_of_peak": decode["frac_of_peak"], "launches": decode["launches_per_token"],
                       "tok_s_logits_32768_row_chunks": decode["tok_s_logits_32768_row_chunks"]},
            "decode_kv": {"tok_s": decode_kv["tok_s"], "positions": decode_kv["positions"]},
            "tp_decode": tp_decode,
            "roofline": {"bound": "hbm", "kernel": KERNEL_NAMES[dom_name],
                         "achieved": dom["GBps"], "peak": peak, "unit": "GB/s",
                         "frac": round(dom["GBps"] / peak, 4), "peak_source": peak_src,
                         "traffic": DRAM_BYTES.get(dom_name),
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch "
                                           "(profiles/gemv_kq_phi4_layer_shapes.md)"},
        }
        print(json.dumps(line), flush=True)
    model.close()
    ctx.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
