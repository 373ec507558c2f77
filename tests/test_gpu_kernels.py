"""GPU parity tests: every kernel through the C ABI against the CPU oracle on the same
seeded inputs. Bars: dequantised values bit-exact; f32 GEMV / RMSNorm / logits within
1e-4 relative L2 of the oracle's f32 result (the reference's CPU arithmetic)."""
import ctypes
from ctypes import c_void_p

import numpy as np
import pytest

from conftest import rel_l2
from edge_blocks import EDGE

pytestmark = pytest.mark.gpu

TOL = 1e-4          # f32 path (north star: 1e-4 relative L2)
QTYPES = [12, 13, 14]


@pytest.fixture(scope="module")
def G(torch_cuda):
    import gpu_util
    return gpu_util


def vp(t):
    return c_void_p(t.data_ptr())


def test_mma_fragment_layout(rrr, ctx):
    ok = ctypes.c_int(0)
    ctx.check(rrr.ffi.lib().rrr_selftest_mma(ctx.h, ctypes.byref(ok)))
    assert ok.value == 1


def _bits_equal(a: np.ndarray, b: np.ndarray) -> bool:
    ua, ub = a.view(np.uint32), b.view(np.uint32)
    nan = np.isnan(a) & np.isnan(b)
    return bool(np.all((ua == ub) | nan))


@pytest.mark.parametrize("qt", QTYPES)
def test_dequant_bit_exact_random(rrr, ctx, oracle, G, qt):
    rng = np.random.default_rng(100 + qt)
    nb = 777
    raw = oracle.random_blocks(qt, nb, rng)
    out = G.empty_f32(nb * 256)
    rd = G.dev(raw)
    ctx.check(rrr.ffi.lib().rrr_dequant_kq(ctx.h, qt, vp(rd), vp(out), nb, None))
    got = G.host(out)
    ref = oracle.dequant(qt, raw, nb * 256)
    assert _bits_equal(got, ref)


@pytest.mark.parametrize("qt", QTYPES)
def test_dequant_bit_exact_edge_blocks(rrr, ctx, oracle, G, qt):
    raw = EDGE[qt]()
    nb = raw.size // oracle.BLOCK_BYTES[qt]
    out = G.empty_f32(nb * 256)
    rd = G.dev(raw)
    ctx.check(rrr.ffi.lib().rrr_dequant_kq(ctx.h, qt, vp(rd), vp(out), nb, None))
    assert _bits_equal(G.host(out), oracle.dequant(qt, raw, nb * 256))


def _gemv(rrr, ctx, G, qt, raw, x, K, N, residual=None, pro=None):
    # device tensors are held in locals until the result is read back (a temporary freed
    # before the launch could be reused by the next allocation)
    y = G.empty_f32(N)
    r = G.dev(residual) if residual is not None else None
    wd, xd = G.dev(raw), G.dev(x)
    L = rrr.ffi.lib()
    if pro is None:
        ctx.check(L.rrr_gemv_kq(ctx.h, qt, vp(wd), vp(xd), vp(y), K, N,
                                vp(r) if r is not None else None, None))
    else:
        ctx.check(L.rrr_gemv_kq_ex(ctx.h, qt, vp(wd), vp(xd), vp(y), K, N,
                                   vp(r) if r is not None else None, ctypes.byref(pro), None))
    out = G.host(y)
    del wd, xd, r
    return out


@pytest.mark.parametrize("qt", QTYPES)
@pytest.mark.parametrize("K,N", [(256, 1), (256, 7), (512, 16), (768, 17), (1024, 33),
                                 (3072, 100), (2304, 45), (4096, 64)])
def test_gemv_small(rrr, ctx, oracle, G, qt, K, N):
    rng = np.random.default_rng(K * 1000 + N + qt)
    raw = oracle.random_blocks(qt, N * (K // 256), rng)
    x = rng.standard_normal(K).astype(np.float32)
    got = _gemv(rrr, ctx, G, qt, raw, x, K, N)
    ref = oracle.gemv_kq(qt, raw, x, K, N)
    assert rel_l2(got, ref) < TOL
    assert np.all(np.isfinite(got))


@pytest.mark.parametrize("name,qt,K,N", [("qkv", 13, 3072, 5120), ("o_proj", 12, 3072, 3072),
                                         ("gate_up", 12, 3072, 16384), ("down", 14, 8192, 3072)])
def test_gemv_config_shapes(rrr, ctx, oracle, G, name, qt, K, N):
    """Benchmark config 1 at full size (numpy-generated blocks)."""
    rng = np.random.default_rng(abs(hash(name)) % 2**32)
    raw = oracle.random_blocks(qt, N * (K // 256), rng)
    x = rng.standard_normal(K).astype(np.float32)
    got = _gemv(rrr, ctx, G, qt, raw, x, K, N)
    ref = oracle.gemv_kq(qt, raw, x, K, N, threads=8)
    assert rel_l2(got, ref) < TOL


@pytest.mark.parametrize("qt", QTYPES)
def test_gemv_device_generator_matches_oracle_bytes(rrr, ctx, oracle, G, qt):
    """The device block generator writes the oracle generator's bytes (full-size benches
    can then be checked on any row range)."""
    nb = 1000
    import torch
    buf = torch.empty(nb * oracle.BLOCK_BYTES[qt], dtype=torch.uint8, device="cuda")
    ctx.check(rrr.ffi.lib().rrr_fill_kquant_random(ctx.h, qt, vp(buf), nb, 1234, None))
    assert np.array_equal(G.host(buf), oracle.fill_kquant_random(qt, nb, 1234))


@pytest.mark.parametrize("qt", QTYPES)
def test_gemv_residual_and_alias(rrr, ctx, oracle, G, qt):
    K, N = 1024, 40
    rng = np.random.default_rng(7 + qt)
    raw = oracle.random_blocks(qt, N * (K // 256), rng)
    x = rng.standard_normal(K).astype(np.float32)
    res = rng.standard_normal(N).astype(np.float32)
    got = _gemv(rrr, ctx, G, qt, raw, x, K, N, residual=res)
    ref = res + oracle.gemv_kq(qt, raw, x, K, N)
    assert rel_l2(got, ref) < TOL
    # y aliasing residual (the decode step's h += W x)
    import torch
    h, wd, xd = G.dev(res), G.dev(raw), G.dev(x)
    ctx.check(rrr.ffi.lib().rrr_gemv_kq(ctx.h, qt, vp(wd), vp(xd), vp(h), K, N, vp(h), None))
    assert rel_l2(G.host(h), ref) < TOL


@pytest.mark.parametrize("qt", QTYPES)
def test_gemv_prologue_rmsnorm(rrr, ctx, oracle, G, qt):
    K, N = 3072, 64
    rng = np.random.default_rng(11 + qt)
    raw = oracle.random_blocks(qt, N * (K // 256), rng)
    h = (rng.standard_normal(K) * 3).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, K).astype(np.float32)
    gd = G.dev(gamma)
    pro = rrr.ffi.GemvPrologue(rrr.ffi.X_RMSNORM, gd.data_ptr(), 1e-5, 0, 0, 0)
    got = _gemv(rrr, ctx, G, qt, raw, h, K, N, pro=pro)
    ref = oracle.gemv_kq(qt, raw, oracle.rms_norm(h, gamma, 1e-5), K, N)
    assert rel_l2(got, ref) < TOL


@pytest.mark.parametrize("qt", QTYPES)
def test_gemv_prologue_silu_gate(rrr, ctx, oracle, G, qt):
    F, N = 2048, 48
    rng = np.random.default_rng(13 + qt)
    raw = oracle.random_blocks(qt, N * (F // 256), rng)
    gu = (rng.standard_normal(2 * F) * 2).astype(np.float32)
    pro = rrr.ffi.GemvPrologue(rrr.ffi.X_SILU_GATE, None, 0.0, 0, 0, 0)
    got = _gemv(rrr, ctx, G, qt, raw, gu, F, N, pro=pro)
    ref = oracle.gemv_kq(qt, raw, oracle.silu_gate(gu), F, N)
    assert rel_l2(got, ref) < TOL


@pytest.mark.parametrize("qt", QTYPES)
def test_gemv_prologue_gqa_v(rrr, ctx, oracle, G, qt):
    nq, nkv, hd = 24, 8, 128
    K, N = nq * hd, 32
    rng = np.random.default_rng(17 + qt)
    raw = oracle.random_blocks(qt, N * (K // 256), rng)
    qkv = rng.standard_normal((nq + 2 * nkv) * hd).astype(np.float32)
    pro = rrr.ffi.GemvPrologue(rrr.ffi.X_GQA_V, None, 0.0, nq, nkv, hd)
    got = _gemv(rrr, ctx, G, qt, raw, qkv, K, N, pro=pro)
    v = qkv[(nq + nkv) * hd:]
    attn = np.concatenate([v[(h // (nq // nkv)) * hd:(h // (nq // nkv) + 1) * hd] for h in range(nq)])
    ref = oracle.gemv_kq(qt, raw, attn, K, N)
    assert rel_l2(got, ref) < TOL


@pytest.mark.parametrize("qt", QTYPES)
@pytest.mark.parametrize("K,F,norm", [(3072, 8192, True), (512, 40, False), (256, 17, True)])
def test_gemv_swiglu_epilogue(rrr, ctx, oracle, G, qt, K, F, norm):
    """gate_up GEMV with silu(gate)*up fused (W rows [gate; up])."""
    rng = np.random.default_rng(K + F + qt)
    raw = oracle.random_blocks(qt, 2 * F * (K // 256), rng)
    h = (rng.standard_normal(K) * 2).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, K).astype(np.float32)
    gd, hd, y = G.dev(gamma), G.dev(h), G.empty_f32(F)
    wd = G.dev(raw)
    pro = rrr.ffi.GemvPrologue(rrr.ffi.X_RMSNORM if norm else rrr.ffi.X_PLAIN, gd.data_ptr(), 1e-5, 0, 0, 0)
    ctx.check(rrr.ffi.lib().rrr_gemv_kq_swiglu(ctx.h, qt, vp(wd), vp(hd), vp(y), K, F, ctypes.byref(pro), None))
    x = oracle.rms_norm(h, gamma, 1e-5) if norm else h
    ref = oracle.silu_gate(oracle.gemv_kq(qt, raw, x, K, 2 * F, threads=8))
    assert rel_l2(G.host(y), ref) < TOL


def test_gemv_error_codes(rrr, ctx, oracle, G):
    L = rrr.ffi.lib()
    raw = G.dev(oracle.random_blocks(12, 4, np.random.default_rng(0)))  # held for the test
    x = G.empty_f32(512)
    y = G.empty_f32(2)
    assert L.rrr_gemv_kq(ctx.h, 11, vp(raw), vp(x), vp(y), 512, 2, None, None) == -2
    assert L.rrr_gemv_kq(ctx.h, 12, vp(raw), vp(x), vp(y), 300, 2, None, None) == -3
    assert L.rrr_gemv_kq(ctx.h, 12, vp(raw), vp(x), vp(y), 512, 0, None, None) == -3
    assert L.rrr_gemv_kq(ctx.h, 12, c_void_p(raw.data_ptr() + 4), vp(x), vp(y), 512, 2, None, None) == -4
    assert "aligned" in rrr.ffi.last_error(ctx.h)
    assert L.rrr_gemv_kq(ctx.h, 12, None, vp(x), vp(y), 512, 2, None, None) == -1
    assert L.rrr_gemv_kq(None, 12, vp(raw), vp(x), vp(y), 512, 2, None, None) == -1
    assert L.rrr_gemv_kq(ctx.h, 12, vp(raw), vp(x), c_void_p(x.data_ptr()), 512, 2, None, None) == -1
    assert "overlap" in rrr.ffi.last_error(ctx.h)


def test_rmsnorm(rrr, ctx, oracle, G):
    rng = np.random.default_rng(3)
    for rows, d in [(1, 3072), (5, 3072), (3, 100), (1, 1)]:
        x = (rng.standard_normal(rows * d) * 2).astype(np.float32)
        g = rng.uniform(0.5, 1.5, d).astype(np.float32)
        y = G.empty_f32(rows * d)
        xd, gd = G.dev(x), G.dev(g)
        ctx.check(rrr.ffi.lib().rrr_rmsnorm(ctx.h, vp(xd), vp(gd), vp(y), rows, d, 1e-5, None))
        got = G.host(y).reshape(rows, d)
        for r in range(rows):
            assert rel_l2(got[r], oracle.rms_norm(x[r * d:(r + 1) * d], g, 1e-5)) < 1e-6


@pytest.mark.parametrize("V,K,chunk", [(1000, 3072, 0), (1000, 3072, 256), (4097, 512, 1000),
                                       (3, 4, 0)])
def test_logits_f32(rrr, ctx, oracle, G, V, K, chunk):
    rng = np.random.default_rng(V + K)
    W = (rng.standard_normal((V, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal(K).astype(np.float32)
    y = G.empty_f32(V)
    Wd, xd = G.dev(W), G.dev(x)
    ctx.check(rrr.ffi.lib().rrr_logits_f32(ctx.h, vp(Wd), vp(xd), vp(y), V, K, chunk,
                                           None, 0.0, None))
    assert rel_l2(G.host(y), oracle.gemv_f32(W, x)) < TOL


def test_logits_fused_norm_full_vocab(rrr, ctx, oracle, G):
    """Full 200064 x 3072 logits with the output norm fused; W generated on the device,
    checked on 512 sampled rows against the oracle (size-independent property)."""
    import torch
    V, K = 200064, 3072
    W = torch.empty(V * K, dtype=torch.float32, device="cuda")
    L = rrr.ffi.lib()
    ctx.check(L.rrr_fill_f32_normal(ctx.h, vp(W), V * K, 0.0, 0.02, 99, None))
    rng = np.random.default_rng(5)
    h = (rng.standard_normal(K) * 2).astype(np.float32)
    g = rng.uniform(0.5, 1.5, K).astype(np.float32)
    gd = G.dev(g)
    y = G.empty_f32(V)
    hd = G.dev(h)
    ctx.check(L.rrr_logits_f32(ctx.h, vp(W), vp(hd), vp(y), V, K, 32768, vp(gd), 1e-5, None))
    got = G.host(y)
    rows = np.sort(rng.choice(V, 512, replace=False))
    rows[-1] = V - 1
    Wr = W.view(V, K)[torch.from_numpy(rows).cuda()].cpu().numpy()
    ref = oracle.gemv_f32(Wr, oracle.rms_norm(h, g, 1e-5))
    assert rel_l2(got[rows], ref) < TOL
    del W


def test_argmax(rrr, ctx, G):
    L = rrr.ffi.lib()
    import torch
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    rng = np.random.default_rng(1)
    cases = []
    x = rng.standard_normal(200064).astype(np.float32)
    cases.append((x, int(np.argmax(x))))
    t = np.zeros(1000, np.float32); t[[10, 500]] = 5.0
    cases.append((t, 10))                                   # first maximum wins
    t = np.full(77, np.nan, np.float32); t[40] = -3.0
    cases.append((t, 40))                                   # NaN never selected
    cases.append((np.full(9, -np.inf, np.float32), 0))      # nothing > -inf
    t = np.zeros(8, np.float32); t[0] = -0.0; t[3] = 0.0
    cases.append((t, 0))                                    # -0 == +0: first index
    for arr, want in cases:
        ad = G.dev(arr)
        ctx.check(L.rrr_argmax_f32(ctx.h, vp(ad), arr.size, vp(out), None))
        assert int(G.host(out)[0]) == want


def test_silu_gate_and_residual(rrr, ctx, oracle, G):
    L = rrr.ffi.lib()
    rng = np.random.default_rng(2)
    F = 8192
    gu = (rng.standard_normal(2 * F) * 3).astype(np.float32)
    out = G.empty_f32(F)
    gd = G.dev(gu)
    ctx.check(L.rrr_silu_gate(ctx.h, vp(gd), vp(out), F, None))
    assert rel_l2(G.host(out), oracle.silu_gate(gu)) < 1e-6
    a = rng.standard_normal(3072).astype(np.float32)
    b = rng.standard_normal(3072).astype(np.float32)
    o = G.empty_f32(3072)
    ad, bd = G.dev(a), G.dev(b)
    ctx.check(L.rrr_residual_add(ctx.h, vp(ad), vp(bd), vp(o), 3072, None))
    assert np.array_equal(G.host(o), a + b)


def test_matmul_f32_transposed_chunk(rrr, ctx, oracle, G):
    rng = np.random.default_rng(4)
    for M, K, N in [(1, 3072, 8192), (3, 64, 33), (17, 40, 5)]:
        A = rng.standard_normal((M, K)).astype(np.float32)
        B = rng.standard_normal((K, N)).astype(np.float32)
        C = G.empty_f32(M * N)
        Ad, Bd = G.dev(A), G.dev(B)
        ctx.check(rrr.ffi.lib().rrr_matmul_f32(ctx.h, vp(Ad), vp(Bd), vp(C), M, K, N, None))
        assert rel_l2(G.host(C).reshape(M, N), oracle.matmul_f32(A, B)) < TOL


def test_dispatch_by_name_and_batch(rrr, ctx, oracle, G):
    """The reference call pattern: gpu_matmul_kquant / gpu_rmsnorm / a prebuilt table."""
    eng = rrr.ComputeEngine.__new__(rrr.ComputeEngine)
    eng.ctx = ctx
    rng = np.random.default_rng(8)
    K, N = 3072, 256
    raw = oracle.random_blocks(13, N * (K // 256), rng)
    a = rng.standard_normal(K).astype(np.float32)
    buf_a, buf_c = eng.alloc_buffer(K * 4), eng.alloc_buffer(N * 4)
    wbuf = eng.alloc_buffer(raw.nbytes)
    eng.upload(wbuf, raw)
    c = np.empty(N, np.float32)
    rrr.gpu_matmul_kquant(eng, buf_a, wbuf, buf_c, rrr.QType.Q5K, a, c, K, N)
    assert rel_l2(c, oracle.gemv_kq(13, raw, a, K, N)) < TOL
    # rmsnorm through its shader name
    gam = rng.uniform(0.5, 1.5, K).astype(np.float32)
    gbuf, nout = eng.alloc_buffer(K * 4), eng.alloc_buffer(K * 4)
    eng.upload(gbuf, gam)
    out = np.empty(K, np.float32)
    rrr.gpu_rmsnorm(eng, buf_a, gbuf, nout, a, out)
    assert rel_l2(out, oracle.rms_norm(a, gam, 1e-5)) < 1e-6
    # errors: unknown name, too-small binding, repacked layout
    with pytest.raises(rrr.RRRError):
        eng.dispatch_by_name("nope", [buf_a], [4], b"")
    with pytest.raises(rrr.RRRError) as e:
        eng.dispatch_by_name("matmul_q5k", [buf_a, wbuf, buf_c], [K * 4, 10, N * 4], rrr.push_u32(K, N))
    assert e.value.code == -11
    with pytest.raises(rrr.RRRError) as e:
        eng.dispatch_by_name("matmul_gpuq5", [buf_a, wbuf, buf_c], [K * 4, raw.nbytes, N * 4], rrr.push_u32(K, N))
    assert e.value.code == -9
    # prebuilt table: rmsnorm -> matmul_q5k, replayed as a graph twice
    b = eng.prebuilt_batch()
    b.add("rmsnorm", [buf_a, gbuf, nout], [K * 4] * 3, rrr.push_u32(1, K))
    b.add(*rrr.kquant_dispatch(nout, wbuf, buf_c, rrr.QType.Q5K, K, N)[:4])
    assert len(b) == 2
    for _ in range(2):
        b.launch()
        eng.sync()
        eng.download(buf_c, c)
        assert rel_l2(c, oracle.gemv_kq(13, raw, oracle.rms_norm(a, gam, 1e-5), K, N)) < TOL
    b.close()
    for bb in (buf_a, buf_c, wbuf, gbuf, nout):
        bb.free()


def test_prebuilt_table_dependent_gemvs(rrr, ctx, oracle, G):
    """A prebuilt table of consecutive matmul_q{4,5,6}k dispatches where each GEMV reads what
    the previous one wrote (stream order is the reference's barrier after each dispatch): a
    dependent run of mixed quant types with K up to 4096 and a ragged row count, an rmsnorm
    dispatch, then 70 more GEMVs, some of whose inputs no dispatch writes (those prepare
    their input before the grid dependency wait). Replayed twice with different inputs;
    every output against the oracle applied to the device's own inputs."""
    eng = rrr.ComputeEngine.__new__(rrr.ComputeEngine)
    eng.ctx = ctx
    rng = np.random.default_rng(81)
    bufs = []

    def buf(n_bytes):
        b = eng.alloc_buffer(n_bytes)
        bufs.append(b)
        return b

    def weight(qt, K, N):
        raw = oracle.random_blocks(qt, N * (K // 256), rng)
        w = buf(raw.nbytes)
        eng.upload(w, raw)
        return raw, w

    x0 = rng.standard_normal(3072).astype(np.float32)
    bx = buf(3072 * 4)
    eng.upload(bx, x0)
    # (qtype, K, N, input buffer index or "x0")
    spec = [(13, 3072, 2048), (14, 2048, 4096), (14, 4096, 768), (12, 768, 1000), (12, 768, 512)]
    tbl = eng.prebuilt_batch()
    ins, outs, raws = [], [], []
    prev = bx
    for i, (qt, K, N) in enumerate(spec):
        raw, w = weight(qt, K, N)
        out = buf(N * 4)
        src = prev if i != 4 else outs[2]          # the ragged GEMV and the next both read y[2]
        tbl.add(*rrr.kquant_dispatch(src, w, out, rrr.QType(qt), K, N)[:4])
        ins.append(src)
        outs.append(out)
        raws.append(raw)
        prev = out
    gam = rng.uniform(0.5, 1.5, 512).astype(np.float32)
    bg, bn = buf(512 * 4), buf(512 * 4)
    eng.upload(bg, gam)
    tbl.add("rmsnorm", [outs[4], bg, bn], [512 * 4] * 3, rrr.push_u32(1, 512))
    raw5, w5 = weight(13, 512, 256)
    many, odd = [], {}
    for j in range(70):
        out = buf(256 * 4)
        if j % 2 == 0:
            tbl.add(*rrr.kquant_dispatch(bn, w5, out, rrr.QType(13), 512, 256)[:4])
        else:
            odd[j], w = weight(12, 3072, 256)
            tbl.add(*rrr.kquant_dispatch(bx, w, out, rrr.QType(12), 3072, 256)[:4])
        many.append(out)
    host = lambda b, n: (lambda a: (eng.download(b, a), a)[1])(np.empty(n, np.float32))

    def check(x_in):
        for i, (qt, K, N) in enumerate(spec):
            # stages 1-4 read the buffer an earlier stage wrote in this replay
            xi = x_in if i == 0 else host(ins[i], K)
            assert rel_l2(host(outs[i], N), oracle.gemv_kq(qt, raws[i], xi, K, N)) < TOL, i
        normed = host(bn, 512)
        assert rel_l2(normed, oracle.rms_norm(host(outs[4], 512), gam, 1e-5)) < 1e-6
        ref5 = oracle.gemv_kq(13, raw5, normed, 512, 256)
        for j in range(70):
            ref = ref5 if j % 2 == 0 else oracle.gemv_kq(12, odd[j], x_in, 3072, 256)
            assert rel_l2(host(many[j], 256), ref) < TOL, j

    # replay, then replay again with a new input: every stage, the dependent ones included,
    # must follow it (a stage that read its input before the preceding stage wrote it would
    # still hold the first replay's values)
    tbl.launch()
    eng.sync()
    assert ctx.device_error() == 0
    check(x0)
    first = host(outs[3], 1000)
    x1 = rng.standard_normal(3072).astype(np.float32)
    eng.upload(bx, x1)
    tbl.launch()
    eng.sync()
    assert ctx.device_error() == 0
    check(x1)
    assert not np.array_equal(first, host(outs[3], 1000))
    tbl.close()
    for b in bufs:
        b.free()


@pytest.mark.parametrize("qt", QTYPES)
@pytest.mark.parametrize("M", [1, 5, 16, 37])
def test_gemm_batched(rrr, ctx, oracle, G, qt, M):
    """Batched-token GEMM, bf16 activations: within 1e-2 relative L2 (north star)."""
    import torch
    K, N = 2048, 96
    rng = np.random.default_rng(M * 10 + qt)
    raw = oracle.random_blocks(qt, N * (K // 256), rng)
    X = torch.randn(M, K, dtype=torch.bfloat16)
    Y = G.empty_f32(M * N)
    wd, xd = G.dev(raw), X.cuda()
    ctx.check(rrr.ffi.lib().rrr_gemm_kq_batched(ctx.h, qt, vp(wd), vp(xd), vp(Y), M, K, N, None))
    got = G.host(Y).reshape(M, N)
    Xf = X.float().numpy()
    for m in range(M):
        assert rel_l2(got[m], oracle.gemv_kq(qt, raw, Xf[m], K, N)) < 1e-2


GEMM_TCGEN05, GEMM_MMA, GEMM_PER_TOKEN, GEMM_MMA_I8 = 1, 2, 3, 4   # RRR_GEMM_* of rrr_gemm_kq_batched_path


def _gemm_tc_case(rrr, ctx, oracle, G, qt, M, K, N, seed, repeats=1, path=GEMM_TCGEN05):
    """Runs the batched GEMM kernel `path` `repeats` times; returns (outputs, f32 reference)."""
    import torch
    rng = np.random.default_rng(seed)
    raw = oracle.random_blocks(qt, N * (K // 256), rng)
    X = torch.randn(M, K, dtype=torch.bfloat16)
    W = oracle.dequant(qt, raw, N * K).reshape(N, K).astype(np.float64)
    ref = (X.float().numpy().astype(np.float64) @ W.T).astype(np.float32)
    wd, xd = G.dev(raw), X.cuda()
    outs = []
    for _ in range(repeats):
        Y = G.empty_f32(M * N)
        Y.fill_(float("nan"))
        ctx.check(rrr.ffi.lib().rrr_gemm_kq_batched_path(ctx.h, qt, vp(wd), vp(xd), vp(Y), M, K, N, None,
                                                         path, None))
        outs.append(G.host(Y).reshape(M, N))
    assert ctx.device_error() == 0
    return outs, ref


# Tensor-core tile path (M >= 16): split-K (tile grid smaller than the GPU) and single
# split (more than 148 row tiles), ragged row and token tiles, Q6_K rows that are not
# 16-byte aligned (K = 768: 630-byte rows), two token tiles (M > 256).
TC_SHAPES = [
    (16, 2048, 96),      # 1 tile, split-K 4
    (64, 3072, 200),     # ragged row tile, split-K 6
    (37, 768, 130),      # ragged token tile (TN 48), odd-aligned Q6_K rows
    (256, 1024, 384),    # TN 256
    (300, 512, 256),     # 2 token tiles of 160
    (16, 512, 19000),    # 149 row tiles: no split
]


@pytest.mark.parametrize("qt", QTYPES)
@pytest.mark.parametrize("M,K,N", TC_SHAPES)
def test_gemm_tc(rrr, ctx, oracle, G, qt, M, K, N):
    """tcgen05 batched GEMM vs the f32 product of the oracle's dequantised weights and the
    bf16 activations: within 1e-2 relative L2 per token row (north star)."""
    (got,), ref = _gemm_tc_case(rrr, ctx, oracle, G, qt, M, K, N, seed=M * 7 + K + N + qt)
    assert np.isfinite(got).all()
    for m in range(M):
        assert rel_l2(got[m], ref[m]) < 1e-2, (m, rel_l2(got[m], ref[m]))
    assert rel_l2(got.ravel(), ref.ravel()) < 5e-3


@pytest.mark.parametrize("qt", QTYPES)
def test_gemm_tc_repeat_deterministic(rrr, ctx, oracle, G, qt):
    """Split-K partial sums are added in split order by the last CTA of each tile, and the
    tile counters are left at zero: repeated calls give identical bits."""
    outs, ref = _gemm_tc_case(rrr, ctx, oracle, G, qt, 48, 4096, 256, seed=99 + qt, repeats=3)
    assert rel_l2(outs[0].ravel(), ref.ravel()) < 5e-3
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])


# mma.sync path (16 <= M <= 64): split-K clusters of up to 8, one tile, ragged rows and
# tokens, many row tiles (no split), the down-projection shape.
MMA_SHAPES = [
    (16, 2048, 96),      # 1 row tile, split-K 4
    (64, 3072, 200),     # ragged row tile, split-K 6
    (37, 1024, 530),     # ragged token tile (TN 48), 3 row tiles
    (48, 512, 19000),    # 75 row tiles: split-K 1
    (20, 8192, 3072),    # down-projection shape, 12 tiles x split-K 8
    (3, 3072, 1000),     # 3 tokens in a 16-token tile (rows 3-15 zero-filled), ragged rows
    (1, 2048, 256),      # one token (the forced path; the automatic choice runs a GEMV)
    (9, 8192, 3072),     # down-projection shape below 16 tokens
]


@pytest.mark.parametrize("qt", QTYPES)
@pytest.mark.parametrize("M,K,N", MMA_SHAPES)
def test_gemm_mma(rrr, ctx, oracle, G, qt, M, K, N):
    """mma.sync batched GEMM (weights dequantised into A fragments in registers) vs the f32
    product of the oracle's dequantised weights and the bf16 activations: within 1e-2
    relative L2 per token row (north star), repeat calls bit-identical."""
    if (K // 256) * {12: 144, 13: 176, 14: 210}[qt] % 16:
        pytest.skip("rows not a multiple of 16 bytes: the tcgen05 kernel serves this shape")
    outs, ref = _gemm_tc_case(rrr, ctx, oracle, G, qt, M, K, N, seed=M * 5 + K + N + qt, repeats=2,
                              path=GEMM_MMA)
    got = outs[0]
    assert np.isfinite(got).all()
    for m in range(M):
        assert rel_l2(got[m], ref[m]) < 1e-2, (m, rel_l2(got[m], ref[m]))
    assert rel_l2(got.ravel(), ref.ravel()) < 5e-3
    assert np.array_equal(outs[1], got)


@pytest.mark.parametrize("qt", QTYPES)
@pytest.mark.parametrize("M,K,N", MMA_SHAPES)
def test_gemm_mma_i8(rrr, ctx, oracle, G, qt, M, K, N):
    """Integer mma.sync batched GEMM (raw quants against int8 digits of X, 16-token tiles) vs
    the f32 product of the oracle's dequantised weights and the bf16 activations: within
    1e-2 relative L2 per token row (north star) and 1e-3 over the whole output (the weights
    are exact, X is represented to 2^-15 of its block maximum), repeat calls bit-identical."""
    if (K // 256) * {12: 144, 13: 176, 14: 210}[qt] % 16:
        pytest.skip("rows not a multiple of 16 bytes: the tcgen05 kernel serves this shape")
    outs, ref = _gemm_tc_case(rrr, ctx, oracle, G, qt, M, K, N, seed=M * 5 + K + N + qt, repeats=2,
                              path=GEMM_MMA_I8)
    got = outs[0]
    assert np.isfinite(got).all()
    for m in range(M):
        assert rel_l2(got[m], ref[m]) < 1e-2, (m, rel_l2(got[m], ref[m]))
    assert rel_l2(got.ravel(), ref.ravel()) < 1e-3, rel_l2(got.ravel(), ref.ravel())
    assert np.array_equal(outs[1], got)


@pytest.mark.parametrize("qt", QTYPES)
def test_gemm_mma_i8_residual_and_heavy_tails(rrr, ctx, oracle, G, qt):
    """The integer kernel with the residual epilogue (Y = X W^T + R, R equal to Y) on inputs
    with one 10^3x outlier per 256-block, and the tiles of a previous call's digits
    overwritten by the next call (two shapes back to back on the stream)."""
    import torch
    L = rrr.ffi.lib()
    rng = np.random.default_rng(77 + qt)
    for M, K, N in ((24, 4096, 512), (7, 2048, 300)):
        raw = oracle.random_blocks(qt, N * (K // 256), rng)
        X = torch.randn(M, K, dtype=torch.float32)
        for m in range(M):
            for b in range(K // 256):
                X[m, b * 256 + int(rng.integers(256))] = float(1e3 * rng.choice([-1.0, 1.0]))
        X = X.to(torch.bfloat16)
        R = rng.standard_normal((M, N)).astype(np.float32)
        W = oracle.dequant(qt, raw, N * K).reshape(N, K).astype(np.float64)
        ref = (X.float().numpy().astype(np.float64) @ W.T + R).astype(np.float32)
        wd, xd = G.dev(raw), X.cuda()
        Y = torch.from_numpy(R.copy()).cuda()
        ctx.check(L.rrr_gemm_kq_batched_path(ctx.h, qt, vp(wd), vp(xd), vp(Y), M, K, N, vp(Y),
                                             GEMM_MMA_I8, None))
        got = G.host(Y).reshape(M, N)
        assert ctx.device_error() == 0
        for m in range(M):
            assert rel_l2(got[m], ref[m]) < 1e-2, (M, m, rel_l2(got[m], ref[m]))
        assert rel_l2(got.ravel(), ref.ravel()) < 1e-3


@pytest.mark.parametrize("qt,K", [(12, 768), (13, 512), (14, 2048)])
def test_gemm_auto_short_rows_take_integer_kernel(rrr, ctx, oracle, G, qt, K):
    """The automatic choice runs the integer kernel for K <= 1024 at 3..64 tokens (the
    O-projection shard of a 4- or 8-way split) and the bf16 kernel above: identical bits to
    the forced path."""
    import torch
    L = rrr.ffi.lib()
    N, M = 3072, 64
    if (K // 256) * {12: 144, 13: 176, 14: 210}[qt] % 16:
        pytest.skip("rows not a multiple of 16 bytes")
    raw = oracle.random_blocks(qt, N * (K // 256), np.random.default_rng(K + qt))
    wd = G.dev(raw)
    X = torch.randn(M, K, dtype=torch.bfloat16).cuda()
    outs = {}
    for path in (0, GEMM_MMA, GEMM_MMA_I8):
        Y = G.empty_f32(M * N)
        ctx.check(L.rrr_gemm_kq_batched_path(ctx.h, qt, vp(wd), vp(X), vp(Y), M, K, N, None, path, None))
        outs[path] = G.host(Y)
    expect = GEMM_MMA_I8 if K <= 1024 else GEMM_MMA
    assert np.array_equal(outs[0], outs[expect])
    assert rel_l2(outs[GEMM_MMA_I8], outs[GEMM_MMA]) < 5e-3


def test_gemm_path_selection(rrr, ctx, oracle, G):
    """The mma.sync kernel rejects what it does not handle (M > 64, rows that are not a
    multiple of 16 bytes: Q6_K with K/256 not a multiple of 8); the tcgen05 kernel M < 16."""
    import torch
    L = rrr.ffi.lib()
    w = G.dev(oracle.random_blocks(14, 64 * 3, np.random.default_rng(1)))
    x = torch.zeros(128, 768, dtype=torch.bfloat16, device="cuda")
    y = G.empty_f32(128 * 64)
    assert L.rrr_gemm_kq_batched_path(ctx.h, 14, vp(w), vp(x), vp(y), 32, 768, 64, None, GEMM_MMA, None) == -3
    assert L.rrr_gemm_kq_batched_path(ctx.h, 14, vp(w), vp(x), vp(y), 128, 768, 64, None, GEMM_MMA, None) == -3
    assert L.rrr_gemm_kq_batched_path(ctx.h, 14, vp(w), vp(x), vp(y), 8, 768, 64, None, GEMM_TCGEN05, None) == -3
    assert L.rrr_gemm_kq_batched_path(ctx.h, 14, vp(w), vp(x), vp(y), 8, 768, 64, None, 7, None) == -1
    assert L.rrr_gemm_kq_batched_path(ctx.h, 14, vp(w), vp(x), vp(y), 32, 768, 64, None, GEMM_MMA_I8, None) == -3
    assert L.rrr_gemm_kq_batched_path(ctx.h, 14, vp(w), vp(x), vp(y), 128, 768, 64, None, GEMM_MMA_I8, None) == -3
    # automatic choice still serves the Q6_K shape (tcgen05 with per-row copies)
    ctx.check(L.rrr_gemm_kq_batched_path(ctx.h, 14, vp(w), vp(x), vp(y), 32, 768, 64, None, 0, None))
    torch.cuda.synchronize()
    assert ctx.device_error() == 0


@pytest.mark.parametrize("qt,K", [(12, 1024), (13, 1024), (14, 2048), (14, 1024)])
def test_gemm_auto_small_m(rrr, ctx, oracle, G, qt, K):
    """The automatic choice below 16 tokens: one GEMV per token for M <= 2 and for rows
    that are not a multiple of 16 bytes (Q6_K, K = 1024), from 3 tokens the integer
    mma.sync kernel for K <= 1024 and the bf16 one above; each result bit-identical to the
    forced kernel's."""
    import torch
    N = 512
    L = rrr.ffi.lib()
    w = G.dev(oracle.random_blocks(qt, N * (K // 256), np.random.default_rng(qt + K)))
    aligned = (K // 256) * {12: 144, 13: 176, 14: 210}[qt] % 16 == 0
    for M in (1, 2, 3, 8, 15):
        x = torch.randn(M, K, generator=torch.Generator().manual_seed(M)).to(torch.bfloat16).cuda()
        want = (GEMM_MMA_I8 if K <= 1024 else GEMM_MMA) if (M >= 3 and aligned) else GEMM_PER_TOKEN
        ys = []
        for path in (0, want):
            y = torch.full((M, N), float("nan"), device="cuda")
            ctx.check(L.rrr_gemm_kq_batched_path(ctx.h, qt, vp(w), vp(x), vp(y), M, K, N, None, path, None))
            ys.append(y.cpu().numpy())
        assert ctx.device_error() == 0
        assert np.isfinite(ys[0]).all()
        assert np.array_equal(ys[0], ys[1]), (M, want)


@pytest.mark.parametrize("qt", QTYPES)
@pytest.mark.parametrize("M,K,N,inplace", [(16, 1024, 768, True), (40, 1024, 768, True),
                                            (40, 768, 2048, False), (3, 512, 256, True),
                                            (300, 512, 256, True)])
def test_gemm_tc_residual(rrr, ctx, oracle, G, qt, M, K, N, inplace):
    """rrr_gemm_kq_batched_ex: Y = X W^T + R with R == Y (in place) or separate, on the
    split-K cluster path, the single-split path, both mma.sync paths (bf16 and integer)
    and the per-token path."""
    import torch
    rng = np.random.default_rng(M + K + N + qt)
    raw = oracle.random_blocks(qt, N * (K // 256), rng)
    X = torch.randn(M, K, dtype=torch.bfloat16)
    R = torch.randn(M, N) * 10
    W = oracle.dequant(qt, raw, N * K).reshape(N, K).astype(np.float64)
    ref = (X.float().numpy().astype(np.float64) @ W.T + R.numpy()).astype(np.float32)
    wd, xd = G.dev(raw), X.cuda()
    Y = R.clone().cuda()
    Rd = Y if inplace else R.clone().cuda()
    if not inplace:
        Y = torch.full((M, N), float("nan"), device="cuda")
    Y0 = Y.clone()
    R0 = Rd.clone()
    aligned_rows = (K // 256) * {12: 144, 13: 176, 14: 210}[qt] % 16 == 0
    paths = [0] + ([GEMM_TCGEN05] if M >= 16 else []) + \
        ([GEMM_MMA, GEMM_MMA_I8] if M <= 64 and aligned_rows else [])
    if M < 16:
        paths.append(GEMM_PER_TOKEN)
    for path in paths:
        Y.copy_(Y0)
        Rd.copy_(R0)
        ctx.check(rrr.ffi.lib().rrr_gemm_kq_batched_path(ctx.h, qt, vp(wd), vp(xd), vp(Y), M, K, N, vp(Rd),
                                                         path, None))
        got = G.host(Y).reshape(M, N)
        assert ctx.device_error() == 0
        for m in range(M):
            assert rel_l2(got[m], ref[m]) < 1e-2, (path, m, rel_l2(got[m], ref[m]))


def test_decode_step_small(rrr, ctx, oracle, G):
    """A small Phi-4-shaped model (numpy weights): eager and graph decode steps against
    the oracle's position-0 decode step."""
    import torch
    cfg = dict(d_model=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=768, n_layers=3,
               vocab=1000, eps=1e-5)
    rng = np.random.default_rng(21)
    d, F = cfg["d_model"], cfg["ffn_dim"]
    qkv_dim = (cfg["n_heads"] + 2 * cfg["n_kv_heads"]) * cfg["head_dim"]
    types = dict(qkv_type=13, o_type=12, gate_up_type=12, down_type=14)
    layers, keep = [], []
    arr = (rrr.ffi.Phi4Layer * cfg["n_layers"])()
    for l in range(cfg["n_layers"]):
        L = dict(types)
        L["w_qkv"] = oracle.random_blocks(13, qkv_dim * d // 256, rng)
        L["w_o"] = oracle.random_blocks(12, d * d // 256, rng)
        L["w_gate_up"] = oracle.random_blocks(12, 2 * F * d // 256, rng)
        L["w_down"] = oracle.random_blocks(14, d * F // 256, rng)
        L["attn_norm"] = rng.uniform(0.5, 1.5, d).astype(np.float32)
        L["ffn_norm"] = rng.uniform(0.5, 1.5, d).astype(np.float32)
        layers.append(L)
        dv = {k: G.dev(v) for k, v in L.items() if isinstance(v, np.ndarray)}
        keep.append(dv)
        arr[l].w_qkv, arr[l].qkv_type = dv["w_qkv"].data_ptr(), 13
        arr[l].w_o, arr[l].o_type = dv["w_o"].data_ptr(), 12
        arr[l].w_gate_up, arr[l].gate_up_type = dv["w_gate_up"].data_ptr(), 12
        arr[l].w_down, arr[l].down_type = dv["w_down"].data_ptr(), 14
        arr[l].attn_norm, arr[l].ffn_norm = dv["attn_norm"].data_ptr(), dv["ffn_norm"].data_ptr()
    onorm = rng.uniform(0.5, 1.5, d).astype(np.float32)
    wout = (rng.standard_normal((cfg["vocab"], d)) * 0.02).astype(np.float32)
    on_d, wo_d = G.dev(onorm), G.dev(wout)
    desc = rrr.ffi.Phi4Desc(d, cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"], F, cfg["n_layers"],
                            cfg["vocab"], 1e-5, 300, ctypes.cast(arr, ctypes.POINTER(rrr.ffi.Phi4Layer)),
                            on_d.data_ptr(), wo_d.data_ptr())
    h = ctypes.c_void_p()
    ctx.check(rrr.ffi.lib().rrr_phi4_create(ctx.h, ctypes.byref(desc), ctypes.byref(h)))
    h0 = rng.standard_normal(d).astype(np.float32)
    ref_h, ref_logits = oracle.decode_step(cfg, layers, onorm, wout, h0)
    for use_graph in (0, 1, 1):
        hid = G.dev(h0)
        logits = G.empty_f32(cfg["vocab"])
        am = torch.zeros(1, dtype=torch.int32, device="cuda")
        ctx.check(rrr.ffi.lib().rrr_phi4_forward(h, vp(hid), vp(logits), vp(am), use_graph, None))
        got_h, got_l = G.host(hid), G.host(logits)
        assert rel_l2(got_h, ref_h) < TOL
        assert rel_l2(got_l, ref_logits) < TOL
        assert int(G.host(am)[0]) == int(np.argmax(got_l))
        if use_graph:
            # graph replays read the captured buffers: re-run on the same pointers
            hid.copy_(torch.from_numpy(h0).cuda())
            ctx.check(rrr.ffi.lib().rrr_phi4_forward(h, vp(hid), vp(logits), vp(am), 1, None))
            assert rel_l2(G.host(hid), ref_h) < TOL
    rrr.ffi.lib().rrr_phi4_destroy(h)


def test_no_device_errors(rrr, ctx):
    assert ctx.device_error() == 0


@pytest.mark.parametrize("M,V,K", [(1, 1000, 3072), (3, 4097, 512), (16, 1000, 3072), (64, 2000, 3072),
                                   (100, 777, 100), (130, 300, 256), (300, 257, 64)])
def test_logits_f32_batched_tensor_core(rrr, ctx, oracle, G, M, V, K):
    """Batched logits on the tcgen05 tensor cores (3xTF32): every token row within the f32
    bar (1e-4 relative L2) of the oracle's f32 GEMV, with and without the fused output
    RMSNorm; ragged vocabulary tiles, K not a multiple of the 32-wide stage, 1 to 3 token
    tiles; repeated calls bit-identical."""
    import torch
    rng = np.random.default_rng(M * 7 + V + K)
    W = (rng.standard_normal((V, K)) * 0.02).astype(np.float32)
    X = (rng.standard_normal((M, K)) * 2).astype(np.float32)
    g = rng.uniform(0.5, 1.5, K).astype(np.float32)
    Wd, Xd, gd = G.dev(W), G.dev(X), G.dev(g)
    xn = torch.empty(M * K, device="cuda")
    L = rrr.ffi.lib()
    for gamma in (None, gd):
        outs = []
        for _ in range(2):
            Y = torch.full((M, V), float("nan"), device="cuda")
            ctx.check(L.rrr_logits_f32_batched(ctx.h, vp(Wd), vp(Xd), vp(xn), vp(Y), M, V, K,
                                               vp(gamma) if gamma is not None else None, 1e-5, None))
            outs.append(G.host(Y).reshape(M, V))
        got = outs[0]
        assert np.array_equal(outs[0], outs[1])
        for m in range(M):
            xin = oracle.rms_norm(X[m], g, 1e-5) if gamma is not None else X[m]
            e = rel_l2(got[m], oracle.gemv_f32(W, xin))
            assert e < TOL, (m, e)
    assert ctx.device_error() == 0


def test_logits_f32_batched_full_vocab(rrr, ctx, oracle, G):
    """64 tokens over the full 200064 x 3072 matrix (generated on the device), output norm
    fused: 512 sampled vocabulary rows of every token within 1e-4 of the oracle."""
    import torch
    V, K, M = 200064, 3072, 64
    L = rrr.ffi.lib()
    W = torch.empty(V * K, dtype=torch.float32, device="cuda")
    ctx.check(L.rrr_fill_f32_normal(ctx.h, vp(W), V * K, 0.0, 0.02, 123, None))
    rng = np.random.default_rng(6)
    X = (rng.standard_normal((M, K)) * 2).astype(np.float32)
    g = rng.uniform(0.5, 1.5, K).astype(np.float32)
    Xd, gd = G.dev(X), G.dev(g)
    xn = torch.empty(M * K, device="cuda")
    Y = torch.empty((M, V), device="cuda")
    ctx.check(L.rrr_logits_f32_batched(ctx.h, vp(W), vp(Xd), vp(xn), vp(Y), M, V, K, vp(gd), 1e-5, None))
    got = G.host(Y)
    rows = np.unique(np.concatenate([[0, V - 1], rng.choice(V, 512, replace=False)]))
    Wr = W.view(V, K)[torch.from_numpy(rows).cuda()].cpu().numpy()
    for m in range(M):
        ref = oracle.gemv_f32(Wr, oracle.rms_norm(X[m], g, 1e-5))
        assert rel_l2(got[m, rows], ref) < TOL, m
    del W


def test_gemv_timeline_trace(rrr, ctx, oracle, G):
    """rrr_set_trace: one record per CTA of every GEMV launch with ordered phase stamps
    (start <= dependency <= prepared <= stored; start <= first copy <= last copy), the
    launch's shape and sequence number; tracing off assigns nothing; results unchanged."""
    import importlib
    import torch
    trace = importlib.import_module("recursive-routing-racer-rs_b200.trace")
    L = rrr.ffi.lib()
    rng = np.random.default_rng(17)
    shapes = [(12, 3072, 1000), (14, 2048, 300), (13, 512, 4096)]
    data = []
    for qt, K, N in shapes:
        raw = oracle.random_blocks(qt, N * (K // 256), rng)
        x = rng.standard_normal(K).astype(np.float32)
        data.append((qt, K, N, raw, G.dev(raw), G.dev(x), G.empty_f32(N), x))
    tr = trace.GemvTrace(ctx, records=4096)
    for qt, K, N, raw, wd, xd, y, x in data:
        ctx.check(L.rrr_gemv_kq(ctx.h, qt, vp(wd), vp(xd), vp(y), K, N, None, None))
    torch.cuda.synchronize()
    launches = tr.launches()
    assert [(l["qtype"], l["K"], l["N"]) for l in launches] == \
        [({12: "Q4_K", 13: "Q5_K", 14: "Q6_K"}[qt], K, N) for qt, K, N in shapes]
    nxt, n = tr.position()
    assert n == 3 and nxt == sum(l["ctas"] for l in launches)
    r = tr.records().astype(np.int64)
    assert len(r) == nxt
    assert (r[:, 0] <= r[:, 2]).all() and (r[:, 2] <= r[:, 3]).all() and (r[:, 3] <= r[:, 4]).all()
    has_copy = r[:, 1] > 0
    assert has_copy.any()
    assert (r[has_copy, 0] <= r[has_copy, 1]).all() and (r[has_copy, 1] <= r[has_copy, 5]).all()
    assert sorted((r[:, 7] & 0xFFFF).tolist()) == sorted(
        [c for l in launches for c in range(l["ctas"])])
    for qt, K, N, raw, wd, xd, y, x in data:
        assert rel_l2(G.host(y), oracle.gemv_kq(qt, raw, x, K, N)) < TOL
    tr.close()
    # off: nothing more is assigned
    ctx.check(L.rrr_gemv_kq(ctx.h, 12, vp(data[0][4]), vp(data[0][5]), vp(data[0][6]), 3072, 1000, None, None))
    torch.cuda.synchronize()
    nxt2, n2 = ctypes.c_int64(), ctypes.c_int64()
    ctx.check(L.rrr_trace_position(ctx.h, ctypes.byref(nxt2), ctypes.byref(n2)))
    assert n2.value == 0 and nxt2.value == 0
    assert ctx.device_error() == 0
