"""The bf16 glue of the batched step (csrc/batch_kernels.cu) through the C ABI, in both the
vector form (rows of a multiple of 4, aligned) and the scalar form: RMSNorm -> bf16
(phi4.rs:593-599), SiLU(gate) * up -> bf16 (phi4.rs:1368-1373), GQA-V -> bf16 and the
window copy. Each output is within one bf16 rounding step of the f32 value computed with
the reference's formulas (the RMS sum order differs between forms)."""
import ctypes
from ctypes import c_void_p

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_mod(torch_cuda):
    import torch
    return torch


def vp(t):
    return c_void_p(t.data_ptr())


def close_bf16(got, ref):
    # one bf16 step: 2^-8 relative (round to nearest: at most half of it, plus the
    # difference of the f32 inputs to the rounding)
    return np.all(np.abs(got - ref) <= np.abs(ref) * 2.0 ** -7 + 1e-30)


@pytest.mark.parametrize("rows,d", [(64, 3072), (5, 4096), (3, 770), (2, 4100)])
def test_rmsnorm_bf16(rrr, ctx, torch_mod, rows, d):
    torch = torch_mod
    g = torch.Generator(device="cuda").manual_seed(d)
    x = torch.randn(rows, d, device="cuda", generator=g) * 3
    gam = torch.rand(d, device="cuda", generator=g) + 0.5
    y = torch.empty(rows, d, dtype=torch.bfloat16, device="cuda")
    ctx.check(rrr.ffi.lib().rrr_rmsnorm_bf16(ctx.h, vp(x), vp(gam), vp(y), rows, d, 1e-5, None))
    torch.cuda.synchronize()
    xn, gn = x.cpu().numpy(), gam.cpu().numpy()
    inv = 1.0 / np.sqrt((xn.astype(np.float64) ** 2).mean(1, keepdims=True) + 1e-5)
    ref = (gn * xn) * inv
    assert close_bf16(y.float().cpu().numpy(), ref)


@pytest.mark.parametrize("rows,F", [(64, 8192), (7, 1026)])
def test_silu_gate_bf16(rrr, ctx, torch_mod, rows, F):
    torch = torch_mod
    g = torch.Generator(device="cuda").manual_seed(F)
    gu = torch.randn(rows, 2 * F, device="cuda", generator=g) * 2
    y = torch.empty(rows, F, dtype=torch.bfloat16, device="cuda")
    ctx.check(rrr.ffi.lib().rrr_silu_gate_bf16(ctx.h, vp(gu), vp(y), rows, F, None))
    torch.cuda.synchronize()
    a = gu.cpu().numpy().astype(np.float64)
    ref = a[:, :F] / (1.0 + np.exp(-a[:, :F])) * a[:, F:]
    assert close_bf16(y.float().cpu().numpy(), ref)


def test_gqa_v_and_window_bf16(rrr, ctx, torch_mod):
    torch = torch_mod
    nq, nkv, hd, rows = 24, 8, 128, 5
    qkv = torch.randn(rows, (nq + 2 * nkv) * hd, device="cuda")
    kwin, koff = nq * hd + 256, 128
    a = torch.empty(rows, kwin, dtype=torch.bfloat16, device="cuda")
    L = rrr.ffi.lib()
    ctx.check(L.rrr_gqa_v_bf16(ctx.h, vp(qkv), vp(a), rows, nq, nkv, hd, kwin, koff, None))
    x = torch.randn(rows, nq * hd, device="cuda")
    w = torch.empty(rows, kwin, dtype=torch.bfloat16, device="cuda")
    ctx.check(L.rrr_window_bf16(ctx.h, vp(x), vp(w), rows, nq * hd, kwin, koff, None))
    torch.cuda.synchronize()
    v = qkv.cpu().numpy()[:, (nq + nkv) * hd:]
    hpk = nq // nkv
    ref = np.zeros((rows, kwin), np.float32)
    for h in range(nq):
        ref[:, koff + h * hd:koff + (h + 1) * hd] = v[:, (h // hpk) * hd:(h // hpk + 1) * hd]
    got = a.float().cpu().numpy()
    assert np.array_equal(got, torch.from_numpy(ref).to(torch.bfloat16).float().numpy())
    refw = np.zeros((rows, kwin), np.float32)
    refw[:, koff:koff + nq * hd] = x.cpu().numpy()
    assert np.array_equal(w.float().cpu().numpy(), torch.from_numpy(refw).to(torch.bfloat16).float().numpy())
