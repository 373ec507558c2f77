"""Decode glue at real positions: embedding rows, RoPE + f16 KV store, GQA decode
attention, and the KV-cache decode step (rrr_phi4_* with max_seq > 0).

CPU: the oracle's RoPE equals a direct restatement of apply_rope_cfg (phi4.rs:238-256)
(bit for bit where the f32 sin/cos agree with Python's double ones rounded to f32, else
within their last-bit difference); its attention equals a numpy softmax attention; its KV-cache step at
position 0 equals the position-0 step up to the f16 rounding of V.
GPU: embedding rows bit-exact against the oracle's dequantisers for every type of
dequant_tensor_f32; RoPE within 1 ulp-level (sin/cos are the only library calls), V
cache bit-exact, K cache within one f16 ulp; attention within 1e-5 relative L2 of the
oracle (f64) over 1..2048 positions; the KV-cache decode step within 1e-4 of the
oracle's step over several positions, eager and as a replayed CUDA graph."""
import ctypes
import math
from ctypes import c_void_p

import numpy as np
import pytest

from conftest import rel_l2

ROPE = dict(rope_dim=96, theta=10000.0, attn_factor=1.190238)


def _rope_direct(x, pos, nh, hd, rope_dim, theta, af, factors):
    """apply_rope_cfg written out with numpy f32 scalars (math.sin/cos on the f32 angle
    rounded back to f32)."""
    z = np.array(x, np.float32, copy=True)
    f32 = np.float32
    for h in range(nh):
        for i in range(rope_dim // 2):
            bf = f32(1.0) / f32(math.pow(f32(theta), f32(f32(2.0 * i) / f32(rope_dim))))
            fac = factors[i] if i < len(factors) else f32(1.0)
            ang = f32(f32(pos) * f32(bf / fac))
            s, c = f32(math.sin(ang)), f32(math.cos(ang))
            cs, ss = f32(c * f32(af)), f32(s * f32(af))
            x0, x1 = z[h * hd + 2 * i], z[h * hd + 2 * i + 1]
            z[h * hd + 2 * i] = f32(x0 * cs) - f32(x1 * ss)
            z[h * hd + 2 * i + 1] = f32(x0 * ss) + f32(x1 * cs)
    return z


@pytest.mark.parametrize("pos", [0, 1, 77, 2047])
def test_oracle_rope_matches_direct_restatement(oracle, pos):
    rng = np.random.default_rng(pos)
    x = rng.standard_normal(3 * 128).astype(np.float32)
    fac = rng.uniform(1.0, 1.5, 48).astype(np.float32)
    y = oracle.rope(x, pos, 3, 128, 96, 10000.0, 1.190238, fac)
    z = _rope_direct(x, pos, 3, 128, 96, 10000.0, 1.190238, fac)
    # glibc sinf / cosf (as Rust's f32 sin_cos) against math.sin / cos rounded to f32: the
    # same value or one ulp apart, so the rotated pairs agree to a few 1e-7
    assert np.allclose(y, z, rtol=0, atol=5e-7)
    if pos < 100:
        assert np.array_equal(y.view(np.uint32), z.view(np.uint32))
    # values past rope_dim are untouched; each rotated pair keeps its norm * attn_factor
    assert np.array_equal(y.reshape(3, 128)[:, 96:], x.reshape(3, 128)[:, 96:])
    n0 = np.hypot(x.reshape(3, 64, 2)[:, :48, 0], x.reshape(3, 64, 2)[:, :48, 1])
    n1 = np.hypot(y.reshape(3, 64, 2)[:, :48, 0], y.reshape(3, 64, 2)[:, :48, 1])
    assert np.allclose(n1, n0 * 1.190238, rtol=1e-5)


def test_oracle_attention_matches_numpy(oracle):
    rng = np.random.default_rng(3)
    nh, nkv, hd, S = 6, 2, 64, 37
    q = rng.standard_normal(nh * hd).astype(np.float32)
    kc = oracle.f32_to_f16_bits(rng.standard_normal((S, nkv * hd)))
    vc = oracle.f32_to_f16_bits(rng.standard_normal((S, nkv * hd)))
    out = oracle.attention_f16kv(q, kc, vc, S, nh, nkv, hd)
    K = kc.view(np.float16).astype(np.float64).reshape(S, nkv, hd)
    V = vc.view(np.float16).astype(np.float64).reshape(S, nkv, hd)
    ref = []
    for h in range(nh):
        g = h // (nh // nkv)
        s = K[:, g] @ q[h * hd:(h + 1) * hd].astype(np.float64) / math.sqrt(hd)
        p = np.exp(s - s.max())
        ref.append((p / p.sum()) @ V[:, g])
    assert rel_l2(out, np.concatenate(ref)) < 1e-6


SMALL = dict(d_model=768, n_heads=6, n_kv_heads=2, head_dim=128, ffn_dim=1024, n_layers=2,
             vocab=1000, eps=1e-5)
TYPES = dict(qkv_type=13, o_type=12, gate_up_type=12, down_type=14)


def _small_layers(oracle, seed):
    c = SMALL
    d, F = c["d_model"], c["ffn_dim"]
    qkv_dim = (c["n_heads"] + 2 * c["n_kv_heads"]) * c["head_dim"]
    rng = np.random.default_rng(seed)
    layers = []
    for l in range(c["n_layers"]):
        L = dict(TYPES)
        L["w_qkv"] = oracle.random_blocks(13, qkv_dim * d // 256, rng)
        L["w_o"] = oracle.random_blocks(12, d * d // 256, rng)
        L["w_gate_up"] = oracle.random_blocks(12, 2 * F * d // 256, rng)
        L["w_down"] = oracle.random_blocks(14, d * F // 256, rng)
        L["attn_norm"] = rng.uniform(0.5, 1.5, d).astype(np.float32)
        L["ffn_norm"] = rng.uniform(0.5, 1.5, d).astype(np.float32)
        layers.append(L)
    on = rng.uniform(0.5, 1.5, d).astype(np.float32)
    wo = (rng.standard_normal((c["vocab"], d)) * 0.02).astype(np.float32)
    return layers, on, wo


def test_oracle_kv_step_at_position_zero_is_the_v_stand_in(oracle):
    layers, on, wo = _small_layers(oracle, 4)
    c = SMALL
    h0 = np.random.default_rng(5).standard_normal(c["d_model"]).astype(np.float32)
    kvs = c["n_kv_heads"] * c["head_dim"]
    kc = np.zeros((c["n_layers"], 8, kvs), np.uint16)
    vc = np.zeros_like(kc)
    h1, lg1 = oracle.decode_step_kv(c, layers, on, wo, h0, 0, kc, vc, **ROPE)
    h2, lg2 = oracle.decode_step(c, layers, on, wo, h0)
    # identical except that V passes through the f16 cache
    assert rel_l2(h1, h2) < 2e-3 and rel_l2(lg1, lg2) < 2e-3
    assert np.any(kc[:, 0] != 0) and not np.any(kc[:, 1:])


# ------------------------------------------------------------------ GPU
def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _desc(rrr, nh, nkv, hd, max_seq, factors_dev=None, n_factors=0, rope_dim=96):
    return rrr.ffi.AttnDesc(nh, nkv, hd, min(rope_dim, hd), 10000.0, 1.190238,
                            factors_dev, n_factors, max_seq)


def _random_table(oracle, t, n_rows, d, rng):
    if t == 0:
        return rng.standard_normal(n_rows * d).astype(np.float32).view(np.uint8)
    if t == 1:
        return rng.standard_normal(n_rows * d).astype(np.float16).view(np.uint8)
    if t in (6, 8):
        bb = 22 if t == 6 else 34
        nb = n_rows * d // 32
        raw = rng.integers(0, 256, nb * bb, dtype=np.uint8).reshape(nb, bb)
        dd = rng.uniform(1e-4, 1e-2, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
        raw[:, :2] = dd
        return raw.reshape(-1)
    return oracle.random_blocks(t, n_rows * d // 256, rng)


@pytest.mark.gpu
@pytest.mark.parametrize("t", [0, 1, 6, 8, 12, 13, 14])
def test_embed_rows_bit_exact(rrr, ctx, oracle, t):
    import torch
    rng = np.random.default_rng(100 + t)
    n_rows, d = 50, 768
    raw = _random_table(oracle, t, n_rows, d, rng)
    tokens = np.array([0, 49, 7, 7, 23, 1], np.int32)
    tab, tok = _dev(torch, raw), _dev(torch, tokens)
    out = torch.empty(len(tokens), d, device="cuda")
    ctx.check(rrr.ffi.lib().rrr_embed_rows(ctx.h, t, c_void_p(tab.data_ptr()), n_rows, d,
                                           c_void_p(tok.data_ptr()), len(tokens),
                                           c_void_p(out.data_ptr()), None))
    torch.cuda.synchronize()
    full = oracle.dequant(t, raw, n_rows * d).reshape(n_rows, d) if t not in (0, 1) else \
        (raw.view(np.float32) if t == 0 else raw.view(np.float16).astype(np.float32)).reshape(n_rows, d)
    ref = full[tokens]
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.mark.gpu
def test_embed_rows_bad_token_and_shape(rrr, ctx, oracle):
    import torch
    rng = np.random.default_rng(9)
    raw = oracle.random_blocks(14, 10 * 512 // 256, rng)
    tab = _dev(torch, raw)
    tok = _dev(torch, np.array([3, 10, -1], np.int32))
    out = torch.full((3, 512), 7.0, device="cuda")
    ctx.check(rrr.ffi.lib().rrr_embed_rows(ctx.h, 14, c_void_p(tab.data_ptr()), 10, 512,
                                           c_void_p(tok.data_ptr()), 3, c_void_p(out.data_ptr()), None))
    assert ctx.device_error() == 6
    o = out.cpu().numpy()
    assert np.array_equal(o[0], oracle.dequant(14, raw, 10 * 512).reshape(10, 512)[3])
    assert not o[1:].any()
    L = rrr.ffi.lib()
    assert L.rrr_embed_rows(ctx.h, 14, c_void_p(tab.data_ptr()), 10, 500, c_void_p(tok.data_ptr()), 1,
                            c_void_p(out.data_ptr()), None) == -3
    assert L.rrr_embed_rows(ctx.h, 3, c_void_p(tab.data_ptr()), 10, 512, c_void_p(tok.data_ptr()), 1,
                            c_void_p(out.data_ptr()), None) == -2


def _f16_ulps(a_bits, b_bits):
    return np.abs(a_bits.astype(np.int32) - b_bits.astype(np.int32))


@pytest.mark.gpu
@pytest.mark.parametrize("rows,pos0,use_dpos", [(1, 0, False), (1, 1500, False), (5, 37, False),
                                                 (3, 2045, True)])
def test_rope_kv_store(rrr, ctx, oracle, rows, pos0, use_dpos):
    import torch
    nh, nkv, hd, max_seq = 24, 8, 128, 2048
    qkv_dim = (nh + 2 * nkv) * hd
    kvs = nkv * hd
    rng = np.random.default_rng(rows * 7 + pos0)
    qkv = rng.standard_normal((rows, qkv_dim)).astype(np.float32) * 3
    fac = rng.uniform(1.0, 1.5, 48).astype(np.float32)
    dq, df = _dev(torch, qkv), _dev(torch, fac)
    kc = torch.zeros(max_seq, kvs, dtype=torch.int16, device="cuda")
    vc = torch.zeros_like(kc)
    dpos = _dev(torch, np.array([pos0], np.int32))
    a = _desc(rrr, nh, nkv, hd, max_seq, c_void_p(df.data_ptr()), 48)
    ctx.check(rrr.ffi.lib().rrr_rope_kv_store(ctx.h, ctypes.byref(a), c_void_p(dq.data_ptr()), qkv_dim,
                                              rows, 0 if use_dpos else pos0,
                                              c_void_p(dpos.data_ptr()) if use_dpos else None,
                                              c_void_p(kc.data_ptr()), c_void_p(vc.data_ptr()), None))
    torch.cuda.synchronize()
    got = dq.cpu().numpy()
    K = kc.cpu().numpy().view(np.uint16)
    V = vc.cpu().numpy().view(np.uint16)
    for t in range(rows):
        pos = pos0 + t
        q = oracle.rope(qkv[t, :nh * hd], pos, nh, hd, 96, 10000.0, 1.190238, fac)
        k = oracle.rope(qkv[t, nh * hd:nh * hd + kvs], pos, nkv, hd, 96, 10000.0, 1.190238, fac)
        # sin / cos are the only library calls: CUDA's and glibc's may differ in the last bit
        assert np.allclose(got[t, :nh * hd], q, rtol=0, atol=4e-6 * 3 * 1.2)
        assert np.allclose(got[t, nh * hd:nh * hd + kvs], k, rtol=0, atol=4e-6 * 3 * 1.2)
        assert np.array_equal(got[t, nh * hd + kvs:], qkv[t, nh * hd + kvs:])
        assert _f16_ulps(K[pos], oracle.f32_to_f16_bits(k)).max() <= 1
        assert np.array_equal(V[pos], oracle.f32_to_f16_bits(qkv[t, nh * hd + kvs:]))
    touched = set(range(pos0, pos0 + rows))
    others = [r for r in range(max_seq) if r not in touched]
    assert not K[others].any() and not V[others].any()


@pytest.mark.gpu
@pytest.mark.parametrize("nh,nkv,hd", [(24, 8, 128), (8, 2, 64), (4, 4, 256)])
@pytest.mark.parametrize("seq,rows", [(1, 1), (2, 1), (129, 1), (1000, 4), (2048, 1)])
def test_attention_f16kv(rrr, ctx, oracle, nh, nkv, hd, seq, rows):
    import torch
    max_seq = 2048
    kvs = nkv * hd
    rng = np.random.default_rng(seq * 3 + hd + rows)
    pos0 = seq - rows   # row t sees positions 0 .. pos0 + t
    q = rng.standard_normal((rows, nh * hd + 16)).astype(np.float32)
    kc = oracle.f32_to_f16_bits(rng.standard_normal((max_seq, kvs)) * 2)
    vc = oracle.f32_to_f16_bits(rng.standard_normal((max_seq, kvs)))
    dq, dk, dv = _dev(torch, q), _dev(torch, kc.view(np.int16)), _dev(torch, vc.view(np.int16))
    out = torch.empty(rows, nh * hd, device="cuda")
    a = _desc(rrr, nh, nkv, hd, max_seq)
    for use_dpos in (False, True):
        dpos = _dev(torch, np.array([pos0], np.int32))
        out.fill_(float("nan"))
        ctx.check(rrr.ffi.lib().rrr_attention_f16kv(
            ctx.h, ctypes.byref(a), c_void_p(dq.data_ptr()), nh * hd + 16, rows,
            0 if use_dpos else pos0, c_void_p(dpos.data_ptr()) if use_dpos else None,
            c_void_p(dk.data_ptr()), c_void_p(dv.data_ptr()), c_void_p(out.data_ptr()), None))
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        for t in range(rows):
            ref = oracle.attention_f16kv(q[t, :nh * hd], kc, vc, pos0 + t + 1, nh, nkv, hd)
            assert rel_l2(got[t], ref) < 1e-5, (use_dpos, t, rel_l2(got[t], ref))


@pytest.mark.gpu
def test_attention_rejects_bad_positions(rrr, ctx):
    import torch
    L = rrr.ffi.lib()
    a = _desc(rrr, 24, 8, 128, 16)
    buf = torch.zeros(1 << 16, device="cuda")
    p = c_void_p(buf.data_ptr())
    assert L.rrr_attention_f16kv(ctx.h, ctypes.byref(a), p, 3072, 2, 15, None, p, p, p, None) == -3
    assert L.rrr_rope_kv_store(ctx.h, ctypes.byref(a), p, 5120, 1, 16, None, p, p, None) == -3
    bad = _desc(rrr, 24, 8, 96, 16)
    assert L.rrr_attention_f16kv(ctx.h, ctypes.byref(bad), p, 3072, 1, 0, None, p, p, p, None) == -3
    # a device position past the cache: nothing written, error flag set
    dpos = torch.tensor([16], dtype=torch.int32, device="cuda")
    ctx.check(L.rrr_rope_kv_store(ctx.h, ctypes.byref(a), p, 5120, 1, 0, c_void_p(dpos.data_ptr()),
                                  p, p, None))
    assert ctx.device_error() == 6


def _host_model(oracle, w, torch, phi4):
    """Full model tensors on the host (K-quant from the generator restatement, f32 by copy)."""
    cfg = w.cfg

    def f32(ptr, n):
        t = torch.empty(n, device="cuda")
        w.ctx.check(phi4.ffi.lib().rrr_d2d(w.ctx.h, c_void_p(t.data_ptr()), c_void_p(ptr), n * 4, None))
        torch.cuda.synchronize()
        return t.cpu().numpy()

    layers = []
    for l, e in enumerate(w.layers):
        L = dict(TYPES)
        for name, qt, K, N in cfg.layer_gemvs():
            key = {"qkv": "w_qkv", "o_proj": "w_o", "gate_up": "w_gate_up", "down": "w_down"}[name]
            L[key] = oracle.fill_kquant_random(qt, N * (K // 256), phi4.tensor_seed(w.seed, l, name))
        L["attn_norm"] = f32(e["attn_norm"], cfg.d_model)
        L["ffn_norm"] = f32(e["ffn_norm"], cfg.d_model)
        layers.append(L)
    return (layers, f32(w.output_norm, cfg.d_model),
            f32(w.w_out, cfg.vocab_size * cfg.d_model).reshape(cfg.vocab_size, cfg.d_model),
            f32(w.rope_factors, w.n_rope_factors))


@pytest.mark.gpu
def test_phi4_kv_decode_matches_oracle(rrr, ctx, oracle):
    import importlib
    import torch
    phi4 = importlib.import_module("recursive-routing-racer-rs_b200.phi4")
    c = SMALL
    cfg = phi4.ModelConfig(d_model=c["d_model"], n_heads=c["n_heads"], n_kv_heads=c["n_kv_heads"],
                           head_dim=c["head_dim"], ffn_dim=c["ffn_dim"], n_layers=c["n_layers"],
                           vocab_size=c["vocab"], rms_eps=c["eps"], **TYPES)
    w = phi4.SyntheticPhi4(ctx, cfg, seed=31)
    max_seq = 40
    dec_e = phi4.Phi4Decoder(ctx, w, max_seq=max_seq)
    dec_g = phi4.Phi4Decoder(ctx, w, max_seq=max_seq)
    assert dec_e.launches_per_step() == 5 * c["n_layers"] + 1 + 1
    layers, on, wo, fac = _host_model(oracle, w, torch, phi4)
    kvs = c["n_kv_heads"] * c["head_dim"]
    kc = np.zeros((c["n_layers"], max_seq, kvs), np.uint16)
    vc = np.zeros_like(kc)
    rng = np.random.default_rng(8)
    steps = list(range(6)) + [37, 38]   # 6 positions in a row, then a jump (set_position)
    lg = torch.empty(c["vocab"], device="cuda")
    am = torch.zeros(1, dtype=torch.int32, device="cuda")
    for i, pos in enumerate(steps):
        if i and pos != steps[i - 1] + 1:
            dec_e.set_position(pos)
            dec_g.set_position(pos)
            # the oracle's cache rows between are stale in both; fill them the same way
            for p in range(steps[i - 1] + 1, pos):
                hp = rng.standard_normal(c["d_model"]).astype(np.float32)
                oracle.decode_step_kv(c, layers, on, wo, hp, p, kc, vc, **ROPE, factors=fac)
                for dec in (dec_e, dec_g):
                    dec.set_position(p)
                    h = torch.from_numpy(hp).cuda()
                    dec.forward(h.data_ptr(), lg.data_ptr(), None, use_graph=dec is dec_g)
            torch.cuda.synchronize()
        assert dec_e.position == pos and dec_g.position == pos
        h0 = rng.standard_normal(c["d_model"]).astype(np.float32)
        h_ref, lg_ref = oracle.decode_step_kv(c, layers, on, wo, h0, pos, kc, vc, **ROPE, factors=fac)
        for dec in (dec_e, dec_g):
            h = torch.from_numpy(h0).cuda()
            dec.forward(h.data_ptr(), lg.data_ptr(), am.data_ptr(), use_graph=dec is dec_g)
            torch.cuda.synchronize()
            assert rel_l2(h.cpu().numpy(), h_ref) < 1e-4, (pos, dec is dec_g)
            assert rel_l2(lg.cpu().numpy(), lg_ref) < 1e-4
            assert int(am.item()) == int(np.argmax(lg_ref))
    assert ctx.device_error() == 0
    kd, vd = dec_g.kv_cache(1)
    K = torch.empty(max_seq * kvs, dtype=torch.int16, device="cuda")
    ctx.check(phi4.ffi.lib().rrr_d2d(ctx.h, c_void_p(K.data_ptr()), c_void_p(kd), max_seq * kvs * 2, None))
    Kh = K.cpu().numpy().view(np.float16).astype(np.float32).reshape(max_seq, kvs)
    # layer 1's K rows come from a GEMV whose input already differs by ~1e-5 (f32 order)
    assert rel_l2(Kh[:39], kc[1, :39].view(np.float16).astype(np.float32)) < 1e-3
    for dec in (dec_e, dec_g):
        dec.set_position(max_seq - 1)
        h = torch.from_numpy(h0).cuda()
        dec.forward(h.data_ptr(), lg.data_ptr(), None, use_graph=dec is dec_g)
        with pytest.raises(rrr.ffi.RRRError):
            dec.forward(h.data_ptr(), lg.data_ptr(), None, use_graph=dec is dec_g)
        dec.close()
    torch.cuda.synchronize()
    assert ctx.device_error() == 0
    w.close()


@pytest.mark.gpu
def test_named_dispatch_rope_kv_store_and_attention(rrr, ctx, oracle):
    """The reference's call pattern (forward_gpu / forward_dynamic): rope_kv_store (or the
    CPU RoPE + kv_store) and attention by shader name, bindings with byte sizes, push
    constants."""
    nh, nkv, hd, max_seq = 24, 8, 128, 64
    q_dim, kvs = nh * hd, nkv * hd
    eng = rrr.ComputeEngine.__new__(rrr.ComputeEngine)
    eng.ctx = ctx
    rng = np.random.default_rng(12)
    fac = rng.uniform(1.0, 1.5, 48).astype(np.float32)
    fbuf = eng.alloc_buffer(48 * 4)
    eng.upload(fbuf, fac)
    kbuf, vbuf = eng.alloc_buffer(max_seq * kvs * 2), eng.alloc_buffer(max_seq * kvs * 2)
    qkv_buf, qbuf, obuf = eng.alloc_buffer((q_dim + 2 * kvs) * 4), eng.alloc_buffer(q_dim * 4), \
        eng.alloc_buffer(q_dim * 4)
    kc = np.zeros((max_seq, kvs), np.uint16)
    vc = np.zeros_like(kc)
    out = np.empty(q_dim, np.float32)
    for pos in range(5):
        qkv = rng.standard_normal(q_dim + 2 * kvs).astype(np.float32)
        q = oracle.rope(qkv[:q_dim], pos, nh, hd, 96, 10000.0, 1.190238, fac)
        k = oracle.rope(qkv[q_dim:q_dim + kvs], pos, nkv, hd, 96, 10000.0, 1.190238, fac)
        kc[pos], vc[pos] = oracle.f32_to_f16_bits(k), oracle.f32_to_f16_bits(qkv[q_dim + kvs:])
        if pos % 2 == 0:   # GPU RoPE + KV store (forward_gpu)
            eng.upload(qkv_buf, qkv)
            eng.dispatch_by_name("rope_kv_store", [qkv_buf, fbuf, kbuf, vbuf],
                                 [(q_dim + 2 * kvs) * 4, 48 * 4, max_seq * kvs * 2, max_seq * kvs * 2],
                                 rrr.push_u32(pos, nh, nkv, hd, 96, q_dim, kvs))
            eng.sync()
            got = np.empty(q_dim + 2 * kvs, np.float32)
            eng.download(qkv_buf, got)
            assert np.allclose(got[:q_dim], q, rtol=0, atol=2e-5)
            q_in = got[:q_dim]
        else:              # CPU RoPE, then kv_store (forward_dynamic)
            eng.upload(qkv_buf, np.concatenate([q, k, qkv[q_dim + kvs:]]))
            eng.dispatch_by_name("kv_store", [qkv_buf, kbuf, vbuf],
                                 [(q_dim + 2 * kvs) * 4, max_seq * kvs * 2, max_seq * kvs * 2],
                                 rrr.push_u32(pos, q_dim, kvs))
            q_in = q
        eng.upload(qbuf, q_in)
        seq = pos + 1
        eng.dispatch_by_name("attention", [qbuf, kbuf, vbuf, obuf],
                             [q_dim * 4, seq * kvs * 2, seq * kvs * 2, q_dim * 4],
                             rrr.push_u32(seq, nkv, nh // nkv, hd))
        eng.sync()
        eng.download(obuf, out)
        assert rel_l2(out, oracle.attention_f16kv(q_in, kc, vc, seq, nh, nkv, hd)) < 1e-5
    with pytest.raises(rrr.RRRError) as e:
        eng.dispatch_by_name("attention", [qbuf, kbuf, vbuf, obuf], [q_dim * 4, 10, 10, q_dim * 4],
                             rrr.push_u32(3, nkv, nh // nkv, hd))
    assert e.value.code == -11
    with pytest.raises(rrr.RRRError) as e:
        eng.dispatch_by_name("rope", [qbuf, fbuf], [q_dim * 4, 48 * 4], rrr.push_u32(0, 0, 0, 0, 0))
    assert e.value.code == -9
    for b in (fbuf, kbuf, vbuf, qkv_buf, qbuf, obuf):
        b.free()


@pytest.mark.gpu
@pytest.mark.parametrize("pos,use_dpos", [(0, False), (1, True), (300, False), (2047, True)])
def test_fused_rope_attention_equals_two_kernels(rrr, ctx, oracle, pos, use_dpos):
    """rrr_rope_attention_f16kv (one launch) gives the same caches and output bits as
    rrr_rope_kv_store + rrr_attention_f16kv, and matches the oracle."""
    import torch
    nh, nkv, hd, max_seq = 24, 8, 128, 2048
    qkv_dim, kvs = (nh + 2 * nkv) * hd, nkv * hd
    rng = np.random.default_rng(pos + 5)
    fac = rng.uniform(1.0, 1.5, 48).astype(np.float32)
    df = _dev(torch, fac)
    a = _desc(rrr, nh, nkv, hd, max_seq, c_void_p(df.data_ptr()), 48)
    hist_k = oracle.f32_to_f16_bits(rng.standard_normal((max_seq, kvs)))
    hist_v = oracle.f32_to_f16_bits(rng.standard_normal((max_seq, kvs)))
    qkv = rng.standard_normal(qkv_dim).astype(np.float32) * 2
    dpos = _dev(torch, np.array([pos], np.int32))
    L = rrr.ffi.lib()
    outs, caches = [], []
    for fused in (True, False):
        kc, vc = _dev(torch, hist_k.view(np.int16)), _dev(torch, hist_v.view(np.int16))
        dq = _dev(torch, qkv)
        out = torch.empty(nh * hd, device="cuda")
        pp = (0, c_void_p(dpos.data_ptr())) if use_dpos else (pos, None)
        if fused:
            ctx.check(L.rrr_rope_attention_f16kv(ctx.h, ctypes.byref(a), c_void_p(dq.data_ptr()), pp[0], pp[1],
                                                 c_void_p(kc.data_ptr()), c_void_p(vc.data_ptr()),
                                                 c_void_p(out.data_ptr()), None))
        else:
            ctx.check(L.rrr_rope_kv_store(ctx.h, ctypes.byref(a), c_void_p(dq.data_ptr()), qkv_dim, 1, pp[0], pp[1],
                                          c_void_p(kc.data_ptr()), c_void_p(vc.data_ptr()), None))
            ctx.check(L.rrr_attention_f16kv(ctx.h, ctypes.byref(a), c_void_p(dq.data_ptr()), qkv_dim, 1, pp[0],
                                            pp[1], c_void_p(kc.data_ptr()), c_void_p(vc.data_ptr()),
                                            c_void_p(out.data_ptr()), None))
        torch.cuda.synchronize()
        outs.append(out.cpu().numpy())
        caches.append((kc.cpu().numpy(), vc.cpu().numpy()))
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    assert np.array_equal(caches[0][0], caches[1][0]) and np.array_equal(caches[0][1], caches[1][1])
    q = oracle.rope(qkv[:nh * hd], pos, nh, hd, 96, 10000.0, 1.190238, fac)
    k = oracle.rope(qkv[nh * hd:nh * hd + kvs], pos, nkv, hd, 96, 10000.0, 1.190238, fac)
    kc_ref, vc_ref = hist_k.copy(), hist_v.copy()
    kc_ref[pos], vc_ref[pos] = oracle.f32_to_f16_bits(k), oracle.f32_to_f16_bits(qkv[nh * hd + kvs:])
    assert rel_l2(outs[0], oracle.attention_f16kv(q, kc_ref, vc_ref, pos + 1, nh, nkv, hd)) < 1e-5
    rows = np.r_[0:pos, pos + 1:max_seq]
    assert np.array_equal(caches[0][0].view(np.uint16)[rows], hist_k[rows])
