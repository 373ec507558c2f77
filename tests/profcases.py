"""Small, self-checking workloads for profiling one kernel at a time under ncu.

Each case builds its inputs on cuda:0, runs a few warm-up rounds and then the launches a
capture selects (`ncu -k regex:<kernel> -s <skip> -c <count>`), checks the context's
device error flag and prints "<case> ok". Sizes are the Phi-4-mini layer shapes, so the
DRAM figures of a capture are those of the bench's per-GEMV lines.

    python tests/profcases.py gemv            # 3 GEMV shapes x 6
    python tests/profcases.py decode --layers 32 [--max-seq 2048 --pos 1024]
    python tests/profcases.py gemm --m 256    # batched tcgen05 GEMM
    python tests/profcases.py attn --pos 1024 # RoPE + KV + attention
    python tests/profcases.py batched --m 64  # M-token decode step
    python tests/profcases.py timeline        # GEMV phase timeline (rrr_set_trace), no ncu
    python tests/profcases.py logits --m 64 --vocab 32768   # batched logits (tcgen05 3xTF32)
"""
import argparse
import ctypes
import importlib
import os
import sys
from ctypes import c_void_p

# run as a script from the repository root: the package directory sits one level up
sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

_PKG = "recursive-routing-racer-rs_b200"
BLOCK_BYTES = {12: 144, 13: 176, 14: 210}


def _weights(ctx, L, torch, qt, K, N, seed):
    nb = N * (K // 256)
    w = torch.empty(nb * BLOCK_BYTES[qt], dtype=torch.uint8, device="cuda")
    ctx.check(L.rrr_fill_kquant_random(ctx.h, qt, c_void_p(w.data_ptr()), nb, seed, None))
    return w


def case_gemv(ctx, L, torch, args):
    """gate_up Q4_K 16384x3072, o_proj Q4_K 3072x3072, down Q6_K 3072x8192; `rounds` rounds."""
    shapes = [(12, 3072, 16384), (12, 3072, 3072), (14, 8192, 3072)]
    bufs = []
    for qt, K, N in shapes:
        w = _weights(ctx, L, torch, qt, K, N, 7)
        bufs.append((qt, K, N, w, torch.randn(K, device="cuda"), torch.empty(N, device="cuda")))
    torch.cuda.synchronize()
    for _ in range(args.rounds):
        for qt, K, N, w, x, y in bufs:
            ctx.check(L.rrr_gemv_kq(ctx.h, qt, c_void_p(w.data_ptr()), c_void_p(x.data_ptr()),
                                    c_void_p(y.data_ptr()), K, N, None, None))


def case_decode(ctx, L, torch, args):
    """Eager decode steps of the synthetic Phi-4-mini model (136 launches per step at 32
    layers); --max-seq > 0: the KV-cache step at positions ending at --pos (169 launches)."""
    phi4 = importlib.import_module(_PKG + ".phi4")
    cfg = phi4.ModelConfig(n_layers=args.layers)
    m = phi4.SyntheticPhi4(ctx, cfg, seed=5)
    dec = phi4.Phi4Decoder(ctx, m, max_seq=args.max_seq)
    if args.max_seq:
        dec.set_position(max(0, args.pos - args.rounds))
    h = torch.randn(cfg.d_model, device="cuda")
    lg = torch.empty(cfg.vocab_size, device="cuda")
    am = torch.zeros(1, dtype=torch.int32, device="cuda")
    for _ in range(args.rounds):
        dec.forward(h.data_ptr(), lg.data_ptr(), am.data_ptr(), False)


def case_gemm(ctx, L, torch, args):
    """Batched GEMM, M = --m tokens, on gate_up Q4_K 16384x3072 and down Q6_K 3072x8192
    (--path: RRR_GEMM_* kernel choice, 0 = automatic)."""
    shapes = [(12, 3072, 16384), (14, 8192, 3072)]
    bufs = []
    for qt, K, N in shapes:
        w = _weights(ctx, L, torch, qt, K, N, 11)
        x = torch.randn(args.m, K, device="cuda").to(torch.bfloat16)
        bufs.append((qt, K, N, w, x, torch.empty(args.m, N, device="cuda")))
    torch.cuda.synchronize()
    for _ in range(args.rounds):
        for qt, K, N, w, x, y in bufs:
            ctx.check(L.rrr_gemm_kq_batched_path(ctx.h, qt, c_void_p(w.data_ptr()), c_void_p(x.data_ptr()),
                                                 c_void_p(y.data_ptr()), args.m, K, N, None, args.path, None))


def case_attn(ctx, L, torch, args):
    """Fused RoPE + f16 KV store + decode attention (Phi-4-mini heads: 24 query, 8 KV, 128)
    at position --pos of 8 layers' 2048-row caches, the position read from the device."""
    import ctypes
    ffi = importlib.import_module(_PKG + ".ffi")
    nh, nkv, hd, max_seq = 24, 8, 128, 2048
    kvs = nkv * hd
    a = ffi.AttnDesc(nh, nkv, hd, 96, 10000.0, 1.190238, None, 0, max_seq)
    caches = [(torch.randn(max_seq * kvs, device="cuda").half(), torch.randn(max_seq * kvs, device="cuda").half())
              for _ in range(8)]
    qkv = torch.randn((nh + 2 * nkv) * hd, device="cuda")
    out = torch.empty(nh * hd, device="cuda")
    dpos = torch.tensor([args.pos], dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    for _ in range(args.rounds):
        for kc, vc in caches:
            ctx.check(L.rrr_rope_attention_f16kv(ctx.h, ctypes.byref(a), c_void_p(qkv.data_ptr()), 0,
                                                 c_void_p(dpos.data_ptr()), c_void_p(kc.data_ptr()),
                                                 c_void_p(vc.data_ptr()), c_void_p(out.data_ptr()), None))


def case_batched(ctx, L, torch, args):
    """Eager M-token steps (--m) of the synthetic Phi-4-mini model through
    rrr_phi4_forward_batched at position 0: per layer RMSNorm -> bf16, 4 batched GEMMs,
    GQA-V / SiLU glue; batched logits and the row-wise argmax."""
    phi4 = importlib.import_module(_PKG + ".phi4")
    cfg = phi4.ModelConfig(n_layers=args.layers)
    m = phi4.SyntheticPhi4(ctx, cfg, seed=5)
    dec = phi4.Phi4Decoder(ctx, m)
    h = torch.randn(args.m, cfg.d_model, device="cuda")
    lg = torch.empty(args.m, cfg.vocab_size, device="cuda")
    am = torch.zeros(args.m, dtype=torch.int32, device="cuda")
    for _ in range(args.rounds):
        dec.forward_batched(h.data_ptr(), lg.data_ptr(), args.m, am.data_ptr(), False)


def case_logits(ctx, L, torch, args):
    """Batched F32 logits of --m tokens over --vocab rows of a 3072-wide f32 matrix
    (rrr_logits_f32_batched with the output RMSNorm: rmsnorm_kernel + logits_tc_kernel),
    `rounds` launches."""
    K, V, M = 3072, args.vocab, args.m
    W = torch.empty(V * K, device="cuda")
    ctx.check(L.rrr_fill_f32_normal(ctx.h, c_void_p(W.data_ptr()), V * K, 0.0, 0.02, 11, None))
    gamma = torch.rand(K, device="cuda") + 0.5
    x = torch.randn(M, K, device="cuda")
    xn = torch.empty(M, K, device="cuda")
    y = torch.empty(M, V, device="cuda")
    for _ in range(args.rounds):
        ctx.check(L.rrr_logits_f32_batched(ctx.h, c_void_p(W.data_ptr()), c_void_p(x.data_ptr()),
                                           c_void_p(xn.data_ptr()), c_void_p(y.data_ptr()), M, V, K,
                                           c_void_p(gamma.data_ptr()), ctypes.c_float(1e-5), None))


def case_timeline(ctx, L, torch, args):
    """The GEMV timeline (rrr_set_trace) of the graph-replayed decode step (--layers, position
    0, or the KV-cache step at --pos with --max-seq) and of the bench's table of independent
    GEMVs: per GEMV kind, the medians over the middle layers of each phase (us from the
    launch's first CTA start) and of the gap from the previous launch's last stored row."""
    import ctypes
    import json
    import numpy as np
    phi4 = importlib.import_module(_PKG + ".phi4")
    trace = importlib.import_module(_PKG + ".trace")
    cfg = phi4.ModelConfig(n_layers=args.layers)
    m = phi4.SyntheticPhi4(ctx, cfg, seed=5)
    names = ["qkv", "o_proj", "gate_up", "down"]

    def summarise(title, launches, per_layer):
        rows = []
        for i, name in enumerate(names):
            sel = [k for k in range(len(launches)) if k % per_layer == i
                   and 4 <= k // per_layer < args.layers - 4]
            if not sel:
                continue
            med = lambda key: round(float(np.median([launches[k][key] for k in sel])), 2)
            gap = [round((launches[k]["start_ns"] - (launches[k - 1]["start_ns"] + 1e3 * launches[k - 1]["end"])) / 1e3, 2)
                   for k in sel]
            rows.append({"gemv": name, "shape": "%s %dx%d" % (launches[sel[0]]["qtype"], launches[sel[0]]["N"],
                                                              launches[sel[0]]["K"]),
                         "ctas": launches[sel[0]]["ctas"], "last_start": med("last_start"),
                         "first_copy": med("first_copy"), "dependency": med("dependency"),
                         "prepared": med("prepared"), "prepared_last": med("prepared_last"),
                         "stored": med("stored"), "end": med("end"),
                         "gap_after_prev": float(np.median(gap))})
        span = (launches[-1]["start_ns"] + 1e3 * launches[-1]["end"] - launches[0]["start_ns"]) / 1e3
        print(json.dumps({"case": title, "launches": len(launches), "span_us": round(span, 1), "gemvs": rows}))

    # the decode step, replayed from its graph
    dec = phi4.Phi4Decoder(ctx, m, max_seq=args.max_seq)
    if args.max_seq:
        dec.set_position(max(0, args.pos - args.rounds - 2))
    h = torch.randn(cfg.d_model, device="cuda")
    lg = torch.empty(cfg.vocab_size, device="cuda")
    am = torch.zeros(1, dtype=torch.int32, device="cuda")
    tr = trace.GemvTrace(ctx, records=1 << 16)
    for _ in range(args.rounds + 2):
        dec.forward(h.data_ptr(), lg.data_ptr(), am.data_ptr(), True)
    torch.cuda.synchronize()
    # the last 4 * layers launches are the captured graph's (the first step ran eagerly)
    summarise("decode_step" + ("_kv_pos%d" % args.pos if args.max_seq else ""),
              tr.launches()[-4 * cfg.n_layers:], 4)
    tr.close()
    dec.close()
    # the GEMV table of the bench (independent inputs, one graph per replay)
    rrr = importlib.import_module(_PKG)
    X = torch.randn(cfg.n_layers * 16384, device="cuda")
    Y = torch.empty(cfg.n_layers * 4 * 16384, device="cuda")
    b = c_void_p()
    ctx.check(L.rrr_batch_create(ctx.h, ctypes.byref(b)))
    k = 0
    for l in range(cfg.n_layers):
        for name in names:
            p, qt, K, N = m.layers[l][name]
            bufs = (c_void_p * 3)(X.data_ptr() + 4 * l * 16384, p, Y.data_ptr() + 4 * k * 16384)
            sizes = (ctypes.c_uint64 * 3)(4 * K, cfg.weight_bytes(qt, K, N), 4 * N)
            push = ctypes.create_string_buffer(rrr.push_u32(K, N), 8)
            ctx.check(L.rrr_batch_add(b, {12: b"matmul_q4k", 13: b"matmul_q5k", 14: b"matmul_q6k"}[qt],
                                      bufs, sizes, 3, push, 8))
            k += 1
    tr = trace.GemvTrace(ctx, records=1 << 16)
    for _ in range(args.rounds + 2):
        ctx.check(L.rrr_batch_launch(b, None))
    torch.cuda.synchronize()
    summarise("gemv_table", tr.launches(), 4)
    tr.close()
    L.rrr_batch_destroy(b)


CASES = {"gemv": case_gemv, "decode": case_decode, "gemm": case_gemm, "attn": case_attn,
         "batched": case_batched, "timeline": case_timeline, "logits": case_logits}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--rounds", type=int, default=6)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--m", type=int, default=256)
    ap.add_argument("--pos", type=int, default=1024)
    ap.add_argument("--max-seq", type=int, default=0)
    ap.add_argument("--vocab", type=int, default=32768)
    ap.add_argument("--path", type=int, default=0)
    args = ap.parse_args(argv)
    import torch
    rrr = importlib.import_module(_PKG)
    L = rrr.ffi.lib()
    ctx = rrr.Context(0)
    CASES[args.case](ctx, L, torch, args)
    torch.cuda.synchronize()
    err = ctx.device_error()
    if err != 0:
        raise SystemExit("device error flag %d" % err)
    print("%s ok" % args.case)


if __name__ == "__main__":
    main()
