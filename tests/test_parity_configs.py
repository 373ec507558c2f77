"""Parity at the configurations BASELINE.json states, at their full sizes.

* the whole synthetic Phi-4-mini decode step (32 layers, hidden 3072, 24/8
  heads of 128, FFN 8192, 200,064-entry F32 logits) against the oracle's position-0 step
  (reference Phi4Model::forward_gpu, src/model/phi4.rs:1099-1196), eager and as a graph;
* the batched K-quant GEMM at its real shapes (gate_up Q4_K 16384x3072, down
  Q6_K 3072x8192) at M = 16, 64, 256 through the automatic choice and every kernel that
  serves the shape (reference forward_prefill_batched, phi4.rs:1257-1268, 1346-1391);
* the GEMV with heavy-tailed inputs (outlier channels 10^3-10^4x the rest, log-normal
  magnitudes), the activations real models produce, at the f32 bar;
* the tensor-parallel split emulated on one GPU at G = 2, 4, 8 against the oracle.

Weights come from the device generators; the K-quant blocks are regenerated on the host by
the oracle's copy of the generator (same bytes), the f32 norms and the sampled logits rows
are read back. Bars: f32 path 1e-4 relative L2; tensor-core path 1e-2 per token row.
"""
import ctypes
import importlib
import os
from ctypes import c_void_p

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

phi4 = importlib.import_module("recursive-routing-racer-rs_b200.phi4")
tp = importlib.import_module("recursive-routing-racer-rs_b200.tp")

TOL = 1e-4
THREADS = max(1, min(32, os.cpu_count() or 1))
GEMM_TCGEN05, GEMM_MMA, GEMM_MMA_I8 = 1, 2, 4
LAYER_KEYS = (("qkv", "w_qkv", "qkv_type"), ("o_proj", "w_o", "o_type"),
              ("gate_up", "w_gate_up", "gate_up_type"), ("down", "w_down", "down_type"))


def _d2h_f32(ctx, L, ptr, n, offset=0):
    out = np.empty(n, np.float32)
    ctx.check(L.rrr_d2h(ctx.h, c_void_p(out.ctypes.data), c_void_p(ptr + 4 * offset), 4 * n, None))
    ctx.check(L.rrr_sync(ctx.h, None))
    return out


def _oracle_model(ctx, L, oracle, m, rows):
    """The oracle's copy of SyntheticPhi4 `m`: K-quant blocks regenerated on the host from
    the same generator streams, norms read back, and the logits rows `rows` read back."""
    cfg = m.cfg
    layers = []
    for li, ent in enumerate(m.layers):
        lay = {}
        for name, wkey, tkey in LAYER_KEYS:
            _, qt, K, N = ent[name]
            lay[wkey] = oracle.fill_kquant_random(qt, N * (K // 256), phi4.tensor_seed(m.seed, li, name))
            lay[tkey] = qt
        lay["attn_norm"] = _d2h_f32(ctx, L, ent["attn_norm"], cfg.d_model)
        lay["ffn_norm"] = _d2h_f32(ctx, L, ent["ffn_norm"], cfg.d_model)
        layers.append(lay)
    onorm = _d2h_f32(ctx, L, m.output_norm, cfg.d_model)
    wrows = np.stack([_d2h_f32(ctx, L, m.w_out, cfg.d_model, int(r) * cfg.d_model) for r in rows])
    ocfg = dict(d_model=cfg.d_model, n_heads=cfg.n_heads, n_kv_heads=cfg.n_kv_heads,
                head_dim=cfg.head_dim, ffn_dim=cfg.ffn_dim, n_layers=cfg.n_layers,
                vocab=len(rows), eps=cfg.rms_eps)
    return ocfg, layers, onorm, wrows


def _sample_rows(V, n, seed):
    rng = np.random.default_rng(seed)
    rows = np.unique(np.concatenate([[0, V - 1], rng.choice(V, n, replace=False)]))
    return rows


# --------------------------------------------------------------------------- configs[2]
def test_decode_step_configs2_full_size(rrr, ctx, oracle):
    """32 layers at full shapes, the whole vocabulary computed on the GPU: the final hidden
    state in full and 514 sampled logits rows (the first and last included) within 1e-4 of
    the oracle, the argmax equal to the host argmax of the device logits."""
    import torch
    L = rrr.ffi.lib()
    cfg = phi4.ModelConfig()
    assert (cfg.n_layers, cfg.d_model, cfg.vocab_size) == (32, 3072, 200064)
    m = phi4.SyntheticPhi4(ctx, cfg, seed=31)
    dec = phi4.Phi4Decoder(ctx, m)
    rows = _sample_rows(cfg.vocab_size, 512, 8)
    ocfg, layers, onorm, wrows = _oracle_model(ctx, L, oracle, m, rows)
    h0 = np.random.default_rng(9).standard_normal(cfg.d_model).astype(np.float32)
    ref_h, ref_l = oracle.decode_step(ocfg, layers, onorm, wrows, h0, threads=THREADS)
    del layers
    for use_graph in (False, True, True):
        hid = torch.from_numpy(h0).cuda()
        lg = torch.full((cfg.vocab_size,), float("nan"), device="cuda")
        am = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        dec.forward(hid.data_ptr(), lg.data_ptr(), am.data_ptr(), use_graph)
        torch.cuda.synchronize()
        got_h, got_l = hid.cpu().numpy(), lg.cpu().numpy()
        assert np.isfinite(got_l).all()
        assert rel_l2(got_h, ref_h) < TOL, rel_l2(got_h, ref_h)
        assert rel_l2(got_l[rows], ref_l) < TOL, rel_l2(got_l[rows], ref_l)
        assert int(am.item()) == int(np.argmax(got_l))
    assert ctx.device_error() == 0
    dec.close()
    m.close()


# --------------------------------------------------------------------------- configs[3]
@pytest.mark.parametrize("name,qt,K,N", [("gate_up", 12, 3072, 16384), ("down", 14, 8192, 3072)])
def test_gemm_configs3_full_shapes(rrr, ctx, oracle, name, qt, K, N):
    """M = 16, 64, 256 tokens through the automatic choice (RRR_GEMM_AUTO) and each kernel
    that serves the shape (tcgen05 at every M, mma.sync at M <= 64): every token row within
    1e-2 of the f64 product of the oracle's dequantised weights and the bf16 activations,
    repeated calls bit-identical, the automatic result equal to its kernel's."""
    import torch
    L = rrr.ffi.lib()
    nb = N * (K // 256)
    seed = 4000 + qt
    w = torch.empty(nb * oracle.BLOCK_BYTES[qt], dtype=torch.uint8, device="cuda")
    ctx.check(L.rrr_fill_kquant_random(ctx.h, qt, c_void_p(w.data_ptr()), nb, seed, None))
    W = oracle.dequant(qt, oracle.fill_kquant_random(qt, nb, seed), N * K).reshape(N, K)
    Wt = np.ascontiguousarray(W.T.astype(np.float64))
    del W
    gen = torch.Generator().manual_seed(qt)
    for M in (16, 64, 256):
        X = torch.randn(M, K, generator=gen).to(torch.bfloat16)
        ref = X.float().numpy().astype(np.float64) @ Wt
        xd = X.cuda()
        paths = [0, GEMM_TCGEN05] + ([GEMM_MMA, GEMM_MMA_I8] if M <= 64 else [])
        outs = {}
        for path in paths:
            reps = []
            for _ in range(2):
                Y = torch.full((M, N), float("nan"), device="cuda")
                ctx.check(L.rrr_gemm_kq_batched_path(ctx.h, qt, c_void_p(w.data_ptr()), c_void_p(xd.data_ptr()),
                                                     c_void_p(Y.data_ptr()), M, K, N, None, path, None))
                torch.cuda.synchronize()
                reps.append(Y.cpu().numpy())
            assert ctx.device_error() == 0
            got = reps[0]
            assert np.isfinite(got).all(), (M, path)
            assert np.array_equal(reps[0], reps[1]), (M, path)
            for r in range(M):
                e = rel_l2(got[r], ref[r])
                assert e < 1e-2, (M, path, r, e)
            assert rel_l2(got.ravel(), ref.ravel()) < 5e-3, (M, path)
            outs[path] = got
        auto_kernel = GEMM_MMA if M <= 64 else GEMM_TCGEN05
        assert np.array_equal(outs[0], outs[auto_kernel]), M


# --------------------------------------------------------------------------- heavy tails
def _heavy_x(kind, K, rng):
    x = rng.standard_normal(K).astype(np.float32)
    if kind == "block_outliers":        # one 10^3x and one 10^4x element in every 256-block
        for b in range(K // 256):
            i, j = rng.choice(256, 2, replace=False)
            x[b * 256 + i] = np.float32(1e3 * np.sign(rng.standard_normal()))
            x[b * 256 + j] = np.float32(-1e4 * np.sign(rng.standard_normal()))
    elif kind == "outlier_channels":    # a few channels 10^3-10^4x the rest (LLM activations)
        ch = rng.choice(K, 6, replace=False)
        x[ch] = (rng.choice([-1.0, 1.0], 6) * np.array([1e3, 2e3, 5e3, 1e4, 3e3, 8e3])).astype(np.float32)
    elif kind == "lognormal":           # magnitudes exp(N(0, 2^2)), random signs
        x = (np.exp(rng.normal(0.0, 2.0, K)) * rng.choice([-1.0, 1.0], K)).astype(np.float32)
    elif kind == "tiny_blocks":         # blocks spread over 12 decades
        x *= (10.0 ** rng.uniform(-6, 6, K // 256)).repeat(256).astype(np.float32)
    return x


HEAVY = ["block_outliers", "outlier_channels", "lognormal", "tiny_blocks"]


@pytest.mark.parametrize("kind", HEAVY)
@pytest.mark.parametrize("qt,K,N", [(13, 3072, 5120), (12, 3072, 3072), (14, 8192, 3072)])
def test_gemv_heavy_tailed_x(rrr, ctx, oracle, kind, qt, K, N):
    """The GEMV's input digits are relative to a power-of-two scale per 256-block; inputs
    whose magnitudes span decades inside a block stay within the f32 bar."""
    import torch
    L = rrr.ffi.lib()
    rng = np.random.default_rng(abs(hash((kind, qt))) % 2**32)
    raw = oracle.random_blocks(qt, N * (K // 256), rng)
    x = _heavy_x(kind, K, rng)
    wd, xd = torch.from_numpy(raw).cuda(), torch.from_numpy(x).cuda()
    y = torch.empty(N, device="cuda")
    ctx.check(L.rrr_gemv_kq(ctx.h, qt, c_void_p(wd.data_ptr()), c_void_p(xd.data_ptr()),
                            c_void_p(y.data_ptr()), K, N, None, None))
    ref = oracle.gemv_kq(qt, raw, x, K, N, threads=THREADS)
    got = y.cpu().numpy()
    assert rel_l2(got, ref) < TOL, rel_l2(got, ref)


@pytest.mark.parametrize("kind", HEAVY)
@pytest.mark.parametrize("qt", [12, 13, 14])
def test_gemv_heavy_tailed_rmsnorm_prologue(rrr, ctx, oracle, kind, qt):
    """The same inputs through the fused RMSNorm prologue (the decode step's QKV and
    gate_up GEMVs): the GEMV input is rms_norm(x)*gamma."""
    import torch
    L = rrr.ffi.lib()
    K, N = 3072, 512
    rng = np.random.default_rng(abs(hash((kind, qt, "rms"))) % 2**32)
    raw = oracle.random_blocks(qt, N * (K // 256), rng)
    x = _heavy_x(kind, K, rng)
    gamma = rng.uniform(0.5, 1.5, K).astype(np.float32)
    wd, xd, gd = (torch.from_numpy(a).cuda() for a in (raw, x, gamma))
    y = torch.empty(N, device="cuda")
    pro = rrr.ffi.GemvPrologue(rrr.ffi.X_RMSNORM, gd.data_ptr(), 1e-5, 0, 0, 0)
    ctx.check(L.rrr_gemv_kq_ex(ctx.h, qt, c_void_p(wd.data_ptr()), c_void_p(xd.data_ptr()),
                               c_void_p(y.data_ptr()), K, N, None, ctypes.byref(pro), None))
    ref = oracle.gemv_kq(qt, raw, oracle.rms_norm(x, gamma, 1e-5), K, N, threads=THREADS)
    got = y.cpu().numpy()
    assert rel_l2(got, ref) < TOL, rel_l2(got, ref)


# --------------------------------------------------------------------------- configs[4]
@pytest.mark.parametrize("G", [2, 4, 8])
def test_tp_split_emulated_matches_oracle(rrr, ctx, oracle, G):
    """All G ranks' shards on this GPU (exchanges by torch ops), Phi-4-mini shapes with 2
    layers and the full vocabulary: every rank's hidden state and 514 sampled logits rows
    within 1e-4 of the oracle's step, every rank's argmax equal to the host argmax of its
    gathered logits. G = 8 cuts the O-projection's super-blocks (384 columns per rank)."""
    import torch
    L = rrr.ffi.lib()
    cfg = phi4.ModelConfig(n_layers=2)
    seed = 17
    m = phi4.SyntheticPhi4(ctx, cfg, seed=seed)          # read back for the oracle only
    rows = _sample_rows(cfg.vocab_size, 512, 3)
    ocfg, layers, onorm, wrows = _oracle_model(ctx, L, oracle, m, rows)
    m.close()
    h0 = np.random.default_rng(4).standard_normal(cfg.d_model).astype(np.float32)
    ref_h, ref_l = oracle.decode_step(ocfg, layers, onorm, wrows, h0, threads=THREADS)
    ws = [tp.SyntheticPhi4TP(ctx, cfg, tp.plan(cfg, G, g), seed=seed) for g in range(G)]
    decs = [tp.TPDecoder(ctx, w) for w in ws]
    hs = [torch.from_numpy(h0).cuda() for _ in range(G)]
    lgs = [torch.empty(cfg.vocab_size, device="cuda") for _ in range(G)]
    ams = [torch.zeros(1, dtype=torch.int32, device="cuda") for _ in range(G)]
    tp.emulate_step(decs, hs, lgs, ams)
    torch.cuda.synchronize()
    assert ctx.device_error() == 0
    for g in range(G):
        got_l = lgs[g].cpu().numpy()
        assert rel_l2(hs[g].cpu().numpy(), ref_h) < TOL, g
        assert rel_l2(got_l[rows], ref_l) < TOL, g
        assert int(ams[g].item()) == int(np.argmax(got_l))
    for w in ws:
        w.close()
