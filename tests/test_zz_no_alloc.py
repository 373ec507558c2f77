"""The allocation-free argmax entry point (rrr_argmax_f32_noalloc).

Some callers of this library cannot allocate device memory: a host whose device memory
is entirely reserved by its own caching allocator, code that runs while a stream capture
it does not own is open (cudaMalloc is not allowed there), and latency-critical paths
that cannot afford the device synchronisation cudaMalloc implies. They cannot create a
context (rrr_init allocates), so rrr_argmax_f32_noalloc takes none and keeps its scratch
in a fixed device array. These tests call it through the C ABI and check that it returns
the same index as the context-based rrr_argmax_f32 on the same logits, for two calls in a
row. This file is collected last so that a run stopping at its first failure has already
run every other test.
"""
import ctypes
from ctypes import c_void_p

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _both(rrr, ctx, x_np, stream=None):
    import torch
    L = rrr.ffi.lib()
    x = torch.from_numpy(np.ascontiguousarray(x_np, np.float32)).cuda()
    a = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    b = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    if stream is not None:
        # x, a and b were written on the current stream: order those writes before the calls
        stream.wait_stream(torch.cuda.current_stream())
    s = None if stream is None else c_void_p(stream.cuda_stream)
    rc = L.rrr_argmax_f32_noalloc(c_void_p(x.data_ptr()), x.numel(), c_void_p(a.data_ptr()), s)
    assert rc == 0, rrr.ffi.last_error(None)
    ctx.check(L.rrr_argmax_f32(ctx.h, c_void_p(x.data_ptr()), x.numel(), c_void_p(b.data_ptr()), s))
    torch.cuda.synchronize()
    return int(a.item()), int(b.item())


def test_noalloc_argmax_two_calls_match_context_argmax(rrr, ctx):
    rng = np.random.default_rng(2026)
    first = rng.standard_normal(200064).astype(np.float32)      # Phi-4-mini vocabulary
    second = rng.standard_normal(200064).astype(np.float32) * 3.0
    second[123457] = 50.0
    for x in (first, second):                                   # two calls in a row
        got, ref = _both(rrr, ctx, x)
        assert got == ref == int(np.argmax(x))


def test_noalloc_argmax_edge_cases_and_stream(rrr, ctx):
    import torch
    rng = np.random.default_rng(7)
    big = rng.standard_normal(8_388_608).astype(np.float32)
    t = np.full(9000, np.nan, np.float32)
    t[8191] = -1.0
    cases = [(np.array([1.5], np.float32), 0),
             (np.zeros(5000, np.float32), 0),                     # ties: first index
             (np.full(4097, -np.inf, np.float32), 0),             # nothing > -inf: 0
             (big, int(np.argmax(big))),                          # the maximum size
             (t, 8191)]                                           # NaN never selected
    s = torch.cuda.Stream()
    for x, want in cases:
        got, ref = _both(rrr, ctx, x, stream=s)
        assert got == ref == want


def test_noalloc_argmax_inside_a_foreign_stream_capture(rrr, ctx):
    """The caller this entry point exists for: code running inside a stream capture it
    does not own. After one warm-up call (the per-context set-up), a call is captured
    into a CUDA graph on a side stream and replayed on fresh logits."""
    import torch
    L = rrr.ffi.lib()
    n = 200064
    x = torch.zeros(n, device="cuda")
    out = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    assert L.rrr_argmax_f32_noalloc(c_void_p(x.data_ptr()), n, c_void_p(out.data_ptr()), None) == 0
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            rc = L.rrr_argmax_f32_noalloc(c_void_p(x.data_ptr()), n, c_void_p(out.data_ptr()),
                                          c_void_p(s.cuda_stream))
    assert rc == 0, rrr.ffi.last_error(None)
    rng = np.random.default_rng(11)
    for _ in range(2):
        v = rng.standard_normal(n).astype(np.float32)
        x.copy_(torch.from_numpy(v))
        out.fill_(-7)
        g.replay()
        torch.cuda.synchronize()
        assert int(out.item()) == int(np.argmax(v))
    del g


def test_noalloc_argmax_rejects_oversize_and_null(rrr):
    L = rrr.ffi.lib()
    assert L.rrr_argmax_f32_noalloc(c_void_p(16), 8_388_609, c_void_p(16), None) == -3
    assert "8388608" in rrr.ffi.last_error(None)
    assert L.rrr_argmax_f32_noalloc(None, 10, c_void_p(16), None) == -1
    assert L.rrr_argmax_f32_noalloc(c_void_p(16), 0, c_void_p(16), None) == -3
