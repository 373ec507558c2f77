"""Device-side timeline of the K-quant GEMVs (rrr_set_trace): one record per CTA of every
traced launch, with %globaltimer stamps of the kernel's phases. The reference has no
tracing; this is how the per-launch latency of the decode step is taken apart.

    tr = GemvTrace(ctx, records=1 << 16)   # device buffer, tracing on
    ... run steps ...
    tr.launches()                          # one row per launch, phases in microseconds
    tr.close()                             # tracing off
"""
from __future__ import annotations

import ctypes
from ctypes import c_void_p

import numpy as np

from . import ffi

QNAMES = {12: "Q4_K", 13: "Q5_K", 14: "Q6_K"}


class GemvTrace:
    """Turns the context's GEMV timeline on over a device buffer of `records` records."""

    def __init__(self, ctx: ffi.Context, records: int = 1 << 16):
        import torch
        self.ctx = ctx
        self.buf = torch.zeros(records * 8, dtype=torch.int64, device=f"cuda:{ctx.device}")
        ctx.check(ffi.lib().rrr_set_trace(ctx.h, c_void_p(self.buf.data_ptr()), records * 64))

    def position(self) -> tuple[int, int]:
        """(next record, launches traced so far)."""
        nxt, n = ctypes.c_int64(), ctypes.c_int64()
        self.ctx.check(ffi.lib().rrr_trace_position(self.ctx.h, ctypes.byref(nxt), ctypes.byref(n)))
        return nxt.value, n.value

    def records(self) -> np.ndarray:
        """All written records as uint64 [n, 8] (rows with a zero start stamp dropped)."""
        import torch
        torch.cuda.synchronize(self.buf.device)
        r = self.buf.view(-1, 8).cpu().numpy().view(np.uint64)
        return r[r[:, 0] != 0]

    def launches(self) -> list[dict]:
        """One dict per traced launch in launch order: shape, CTAs and the phases in us,
        relative to the launch's first CTA start: the last CTA's start, the first weight copy,
        the grid dependency (median over CTAs), the input prepared (median and last), the rows
        stored (median and last)."""
        r = self.records()
        if len(r) == 0:
            return []
        seq = (r[:, 7] >> np.uint64(16)).astype(np.int64)
        out = []
        for s in np.unique(seq):
            g = r[seq == s].astype(np.float64)
            t0 = g[:, 0].min()
            us = lambda v: round((v - t0) / 1e3, 3)
            meta = int(r[seq == s][0, 6])
            out.append({"seq": int(s), "qtype": QNAMES.get(meta >> 56, str(meta >> 56)),
                        "K": (meta >> 28) & 0xFFFFFFF, "N": meta & 0xFFFFFFF, "ctas": len(g),
                        "start_ns": int(t0), "last_start": us(g[:, 0].max()),
                        "first_copy": us(g[:, 1][g[:, 1] > 0].min()) if (g[:, 1] > 0).any() else None,
                        "dependency": us(np.median(g[:, 2])), "prepared": us(np.median(g[:, 3])),
                        "prepared_last": us(g[:, 3].max()), "stored": us(np.median(g[:, 4])),
                        "end": us(g[:, 4].max())})
        return out

    def close(self) -> None:
        if self.buf is not None:
            self.ctx.check(ffi.lib().rrr_set_trace(self.ctx.h, None, 0))
            self.buf = None
