"""The CPU oracle pinned before it is trusted: golden fixtures from gguf-py (independent
implementation), a live gguf-py cross-check, hand-derived known answers following the
reference's formulas (src/model/phi4.rs:444-542) and the f16 conversion edge cases."""
import os

import numpy as np
import pytest

from conftest import rel_l2
from edge_blocks import EDGE

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "kquant_golden.npz")


def _f16(bits):
    return np.array([bits], np.uint16).view(np.uint8)


def _bits_equal(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    nan = np.isnan(a) & np.isnan(b)
    return bool(np.all((a.view(np.uint32) == b.view(np.uint32)) | nan))


@pytest.mark.parametrize("qt", [12, 13, 14])
def test_oracle_matches_golden_fixtures(oracle, qt):
    g = np.load(GOLD)
    raw = g[f"raw_{qt}"]
    ref = g[f"deq_{qt}"]
    assert _bits_equal(oracle.dequant(qt, raw, ref.size), ref)


@pytest.mark.parametrize("qt", [12, 13, 14])
def test_oracle_gemv_matches_golden(oracle, qt):
    g = np.load(GOLD)
    y = oracle.gemv_kq(qt, g[f"gemv_w_{qt}"], g[f"gemv_x_{qt}"], 512, 6)
    assert rel_l2(y, g[f"gemv_y_{qt}"]) < 1e-6


@pytest.mark.parametrize("qt", [12, 13, 14])
def test_oracle_matches_gguf_py_live(oracle, qt):
    quants = pytest.importorskip("gguf.quants")
    from gguf import GGMLQuantizationType as T
    tt = {12: T.Q4_K, 13: T.Q5_K, 14: T.Q6_K}[qt]
    rng = np.random.default_rng(qt)
    bb = oracle.BLOCK_BYTES[qt]
    raw = np.concatenate([oracle.random_blocks(qt, 300, rng), EDGE[qt](),
                          rng.integers(0, 256, 50 * bb, dtype=np.uint8)])
    nb = raw.size // bb
    ref = quants.dequantize(raw.reshape(nb, bb), tt).reshape(-1)
    assert _bits_equal(oracle.dequant(qt, raw, nb * 256), ref)


def test_q6k_scale_index_known_answer(oracle):
    """README bug #8: is = g*8 + l/16 (phi4.rs:463). All q = 33 (q-32 = 1); scales[s] = s+1;
    d = 1 -> element e has value scales[e // 16]."""
    b = np.zeros(210, np.uint8)
    b[0:128] = 0x11            # every ql nibble = 1
    b[128:192] = 0xAA          # every qh 2-bit field = 2  ->  q = 1 | 2 << 4 = 33
    b[192:208] = np.arange(1, 17, dtype=np.int8).view(np.uint8)
    b[208:210] = _f16(0x3C00)
    out = oracle.dequant(14, b, 256)
    assert np.array_equal(out, (np.arange(256) // 16 + 1).astype(np.float32))
    assert out[16] == 2.0      # the buggy is = g*8 would give 1.0 here


def test_q4k_known_answer(oracle):
    """q * (d*sv) - (dmin*mv) with hand-computed scale/min unpacking (phi4.rs:492-505)."""
    b = np.zeros(144, np.uint8)
    b[0:2] = _f16(0x3C00)      # d = 1
    b[2:4] = _f16(0x3800)      # dmin = 0.5
    sc = b[4:16]
    sc[0] = 3                  # sub 0: sv = 3
    sc[4] = 2                  # sub 0: mv = 2
    sc[8] = 0x5F               # sub 4: sv = 0xF | (sc[0]>>6)<<4 = 15 ; mv = 5 | (sc[4]>>6)<<4 = 5
    sc[0] |= 0xC0              # sub 4 sv gains (3 << 4) -> 63 ; sub 0 keeps 3 (6-bit mask)
    b[16:144] = 0x21           # low nibble 1 (subs 0,2,4,6), high nibble 2 (subs 1,3,5,7)
    out = oracle.dequant(12, b, 256)
    assert out[0] == 1 * 3.0 - 0.5 * 2       # sub 0
    assert out[4 * 32] == 1 * 63.0 - 0.5 * 5  # sub 4
    assert out[32] == 0.0                      # sub 1: sv = 0, mv = 0


def test_q5k_high_bit_known_answer(oracle):
    """5th bit from qh[j] >> sub (phi4.rs:535)."""
    b = np.zeros(176, np.uint8)
    b[0:2] = _f16(0x3C00)
    b[4:8] = 1                 # sv = 1 for subs 0..3
    b[16 + 5] = 0b00000100     # qh[5] bit 2 -> sub 2, j = 5
    out = oracle.dequant(13, b, 256)
    expect = np.zeros(256, np.float32)
    expect[2 * 32 + 5] = 16.0
    assert np.array_equal(out, expect)


def test_f16_conversion(oracle):
    cases = {0x0000: 0.0, 0x3C00: 1.0, 0xC000: -2.0, 0x0001: 2.0 ** -24, 0x03FF: 1023 * 2.0 ** -24,
             0x0400: 2.0 ** -14, 0x7BFF: 65504.0}
    for bits, v in cases.items():
        assert oracle.f16_to_f32(bits) == np.float32(v)
    assert np.isinf(oracle.f16_to_f32(0x7C00)) and oracle.f16_to_f32(0xFC00) < 0
    assert np.isnan(oracle.f16_to_f32(0x7E00))
    allbits = np.arange(65536, dtype=np.uint16)
    ref = allbits.view(np.float16).astype(np.float32)
    got = np.array([oracle.f16_to_f32(int(h)) for h in allbits[::7]], np.float32)
    assert _bits_equal(got, ref[::7]) or np.allclose(got, ref[::7], equal_nan=True)


def test_rms_norm_and_silu(oracle):
    rng = np.random.default_rng(0)
    x = rng.standard_normal(3072).astype(np.float32)
    w = rng.uniform(0.5, 1.5, 3072).astype(np.float32)
    ref = w.astype(np.float64) * x / np.sqrt(np.mean(x.astype(np.float64) ** 2) + 1e-5)
    assert rel_l2(oracle.rms_norm(x, w, 1e-5), ref) < 1e-6
    gu = rng.standard_normal(2 * 64).astype(np.float32)
    g, u = gu[:64].astype(np.float64), gu[64:].astype(np.float64)
    assert rel_l2(oracle.silu_gate(gu), g / (1 + np.exp(-g)) * u) < 1e-6


def test_generator_distributions(oracle):
    """Synthetic blocks follow the benchmark config distributions."""
    for qt in (12, 13, 14):
        raw = oracle.fill_kquant_random(qt, 4000, 7).reshape(4000, -1)
        if qt == 14:
            d = raw[:, 208:210].copy().view(np.float16).astype(np.float32).ravel()
            sc = raw[:, 192:208].view(np.int8)
            assert sc.min() == -32 and sc.max() == 31
        else:
            d = raw[:, 0:2].copy().view(np.float16).astype(np.float32).ravel()
            dm = raw[:, 2:4].copy().view(np.float16).astype(np.float32).ravel()
            assert dm.min() >= 9.99e-5 and dm.max() <= 1.001e-2
        assert d.min() >= 9.99e-5 and d.max() <= 1.001e-2 and abs(d.mean() - 5.05e-3) < 3e-4
    a = oracle.fill_kquant_random(12, 10, 99)
    b = oracle.fill_kquant_random(12, 5, 99, block0=5)
    assert np.array_equal(a[5 * 144:], b)       # block i depends only on (seed, i)


def test_baseline_matches_checker(oracle):
    rng = np.random.default_rng(1)
    for qt, K, N in ((12, 512, 9), (14, 768, 5)):
        raw = oracle.random_blocks(qt, N * K // 256, rng)
        x = rng.standard_normal(K).astype(np.float32)
        y1 = oracle.gemv_kq(qt, raw, x, K, N)
        y2, td, tt = oracle.gemv_kq_baseline(qt, raw, x, K, N, threads=3)
        assert np.array_equal(y1, y2) and td >= 0 and tt >= 0


def test_decode_step_oracle_consistency(oracle):
    """The oracle's decode step equals its own building blocks composed by hand."""
    rng = np.random.default_rng(2)
    cfg = dict(d_model=256, n_heads=2, n_kv_heads=1, head_dim=128, ffn_dim=256, n_layers=1,
               vocab=10, eps=1e-5)
    d, F, hd = 256, 256, 128
    L = dict(qkv_type=12, o_type=12, gate_up_type=12, down_type=14,
             w_qkv=oracle.random_blocks(12, 4 * 128 * 256 // 256, rng),
             w_o=oracle.random_blocks(12, 256, rng), w_gate_up=oracle.random_blocks(12, 512, rng),
             w_down=oracle.random_blocks(14, 256, rng),
             attn_norm=rng.uniform(0.5, 1.5, d).astype(np.float32),
             ffn_norm=rng.uniform(0.5, 1.5, d).astype(np.float32))
    on = rng.uniform(0.5, 1.5, d).astype(np.float32)
    wo = rng.standard_normal((10, d)).astype(np.float32)
    h0 = rng.standard_normal(d).astype(np.float32)
    h1, logits = oracle.decode_step(cfg, [L], on, wo, h0)
    n = oracle.rms_norm(h0, L["attn_norm"])
    qkv = oracle.gemv_kq(12, L["w_qkv"], n, d, 4 * hd)
    v = qkv[3 * hd:]
    attn = np.concatenate([v, v])
    h = h0 + oracle.gemv_kq(12, L["w_o"], attn, d, d)
    gu = oracle.gemv_kq(12, L["w_gate_up"], oracle.rms_norm(h, L["ffn_norm"]), d, 2 * F)
    h = h + oracle.gemv_kq(14, L["w_down"], oracle.silu_gate(gu), F, d)
    assert np.array_equal(h, h1)
    assert np.array_equal(logits, oracle.gemv_f32(wo, oracle.rms_norm(h, on)))
