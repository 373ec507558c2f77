"""Host mirror of RRR's Vulkan ComputeEngine (src/gpu/engine.rs) and the weight-path
helpers of src/model/phi4.rs:612-697, over the CUDA C ABI.

Names and argument meaning follow the reference so call sites port one to one:
`ComputeEngine.alloc_buffer` (engine.rs:200), `dispatch_by_name` (engine.rs:476),
`pre_allocate` + `dispatch_batch` (engine.rs:244, 317), `upload` / `download`
(phi4.rs:616-626), `gpu_matmul_kquant` (phi4.rs:631), `gpu_matmul_f32` (phi4.rs:661),
`gpu_rmsnorm` (phi4.rs:680), `kquant_dispatch` (phi4.rs:1081), `QType` (phi4.rs:118-157).
Differences: buffers are device memory with explicit copies instead of host-mapped
memory, and every failure raises RRRError instead of panicking.
"""
from __future__ import annotations

import ctypes
import enum
import struct
from ctypes import c_uint64, c_void_p

import numpy as np

from . import ffi


class QType(enum.Enum):
    """phi4.rs:118-157. Only the raw GGUF layouts exist here (no GPUQ repack)."""
    Q4K = 12
    Q5K = 13
    Q6K = 14
    F32 = 0

    def shader_name(self) -> str:
        return {12: "matmul_q4k", 13: "matmul_q5k", 14: "matmul_q6k", 0: "matmul_tiled"}[self.value]

    def batch_shader_name(self) -> str:
        return {12: "matmul_q4k_batch", 13: "matmul_q5k_batch", 14: "matmul_q6k_batch",
                0: "matmul_tiled"}[self.value]

    def block_bytes(self) -> int:
        return {12: 144, 13: 176, 14: 210, 0: 1024}[self.value]

    def workgroups(self, n: int) -> int:
        return n

    @staticmethod
    def from_gguf(typ: int) -> "QType":
        return {12: QType.Q4K, 13: QType.Q5K, 14: QType.Q6K}.get(typ, QType.F32)


class GpuBuffer:
    """A device allocation (engine.rs:38-43); `ptr` is the device address."""

    def __init__(self, engine: "ComputeEngine", ptr: int, capacity: int):
        self.engine = engine
        self.ptr = ptr
        self.capacity = capacity

    def free(self) -> None:
        if self.ptr:
            self.engine.ctx.check(ffi.lib().rrr_free(self.engine.ctx.h, c_void_p(self.ptr)))
            self.ptr = 0


class PrebuiltBatch:
    """pre_allocate_desc_set + dispatch_batch_persistent_v2: a recorded table replayed as
    one CUDA graph."""

    def __init__(self, engine: "ComputeEngine"):
        self.engine = engine
        h = c_void_p()
        engine.ctx.check(ffi.lib().rrr_batch_create(engine.ctx.h, ctypes.byref(h)))
        self.h = h

    def add(self, name: str, buffers, sizes, push: bytes) -> None:
        bufs, szs = _bind(buffers, sizes)
        pb = ctypes.create_string_buffer(push, len(push)) if push else None
        self.engine.ctx.check(ffi.lib().rrr_batch_add(self.h, name.encode(), bufs, szs, len(buffers),
                                                      pb, len(push)))

    def launch(self, stream=None) -> None:
        self.engine.ctx.check(ffi.lib().rrr_batch_launch(self.h, _stream(stream)))

    def __len__(self) -> int:
        n = ctypes.c_int()
        self.engine.ctx.check(ffi.lib().rrr_batch_size(self.h, ctypes.byref(n)))
        return n.value

    def close(self) -> None:
        if self.h:
            ffi.lib().rrr_batch_destroy(self.h)
            self.h = None


def _ptr(b) -> int:
    if isinstance(b, GpuBuffer):
        return b.ptr
    if hasattr(b, "data_ptr"):
        return b.data_ptr()
    return int(b)


def _bind(buffers, sizes):
    bufs = (c_void_p * len(buffers))(*[_ptr(b) for b in buffers])
    szs = (c_uint64 * len(sizes))(*[int(s) for s in sizes])
    return bufs, szs


def _stream(stream):
    if stream is None:
        return None
    if hasattr(stream, "cuda_stream"):
        return c_void_p(stream.cuda_stream)
    return c_void_p(int(stream))


def push_u32(*vals: int) -> bytes:
    return struct.pack("<%dI" % len(vals), *vals)


class ComputeEngine:
    """engine.rs:15-29 over one rrr_ctx."""

    def __init__(self, device: int = 0):
        self.ctx = ffi.Context(device)

    def alloc_buffer(self, size: int) -> GpuBuffer:
        p = c_void_p()
        self.ctx.check(ffi.lib().rrr_alloc(self.ctx.h, size, ctypes.byref(p)))
        return GpuBuffer(self, p.value, size)

    def upload(self, buf: GpuBuffer, data: np.ndarray, stream=None) -> None:
        a = np.ascontiguousarray(data)
        self.ctx.check(ffi.lib().rrr_h2d(self.ctx.h, c_void_p(buf.ptr), a.ctypes.data, a.nbytes,
                                         _stream(stream)))
        if stream is None:
            self.sync()

    def download(self, buf: GpuBuffer, out: np.ndarray, stream=None) -> np.ndarray:
        assert out.flags["C_CONTIGUOUS"]
        self.ctx.check(ffi.lib().rrr_d2h(self.ctx.h, out.ctypes.data, c_void_p(buf.ptr), out.nbytes,
                                         _stream(stream)))
        self.sync(stream)
        return out

    def sync(self, stream=None) -> None:
        self.ctx.check(ffi.lib().rrr_sync(self.ctx.h, _stream(stream)))

    def dispatch_by_name(self, name: str, buffers, sizes, push: bytes, groups=None,
                         stream=None) -> None:
        """engine.rs:476. `groups` is accepted for call-site compatibility; the CUDA grid
        is chosen by the kernel's launcher."""
        bufs, szs = _bind(buffers, sizes)
        pb = ctypes.create_string_buffer(push, len(push)) if push else None
        self.ctx.check(ffi.lib().rrr_dispatch_by_name(self.ctx.h, name.encode(), bufs, szs,
                                                      len(buffers), pb, len(push), _stream(stream)))

    def prebuilt_batch(self) -> PrebuiltBatch:
        return PrebuiltBatch(self)

    def close(self) -> None:
        self.ctx.close()


# ------------------------------------------------------------------ phi4.rs:612-697
def upload(engine: ComputeEngine, buf: GpuBuffer, data: np.ndarray) -> None:
    engine.upload(buf, np.asarray(data, dtype=np.float32))


def download(engine: ComputeEngine, buf: GpuBuffer, out: np.ndarray) -> np.ndarray:
    return engine.download(buf, out)


def gpu_matmul_kquant(engine: ComputeEngine, buf_a: GpuBuffer, weight_buf: GpuBuffer,
                      buf_c: GpuBuffer, qtype: QType, a: np.ndarray, c: np.ndarray, k: int,
                      n: int) -> None:
    """phi4.rs:631-658: C[N] = A[K] @ W[N, K] on raw K-quant blocks."""
    upload(engine, buf_a, a)
    if qtype == QType.F32:
        engine.dispatch_by_name("matmul_tiled", [buf_a, weight_buf, buf_c],
                                [k * 4, k * n * 4, n * 4], push_u32(1, k, n))
    else:
        total = n * (k // 256) * qtype.block_bytes()
        engine.dispatch_by_name(qtype.shader_name(), [buf_a, weight_buf, buf_c],
                                [k * 4, total, n * 4], push_u32(k, n))
    download(engine, buf_c, c)


def gpu_matmul_f32(engine: ComputeEngine, buf_a: GpuBuffer, buf_b: GpuBuffer, buf_c: GpuBuffer,
                   a: np.ndarray, c: np.ndarray, m: int, k: int, n: int) -> None:
    """phi4.rs:661-678: C[M,N] = A[M,K] B[K,N] (B in the transposed chunk layout)."""
    upload(engine, buf_a, a)
    engine.dispatch_by_name("matmul_tiled", [buf_a, buf_b, buf_c],
                            [m * k * 4, k * n * 4, m * n * 4], push_u32(m, k, n))
    download(engine, buf_c, c)


def gpu_rmsnorm(engine: ComputeEngine, buf_in: GpuBuffer, weight_buf: GpuBuffer,
                buf_out: GpuBuffer, x: np.ndarray, out: np.ndarray) -> None:
    """phi4.rs:680-697 (d taken from x instead of the D_MODEL constant)."""
    d = x.size
    upload(engine, buf_in, x)
    engine.dispatch_by_name("rmsnorm", [buf_in, weight_buf, buf_out], [d * 4, d * 4, d * 4],
                            push_u32(1, d))
    download(engine, buf_out, out)


def kquant_dispatch(buf_in, weight_buf, buf_out, qtype: QType, k: int, n: int):
    """phi4.rs:1081-1096: the (name, buffers, sizes, push, groups) tuple of one GEMV."""
    total = n * (k // 256) * qtype.block_bytes()
    return (qtype.shader_name(), [buf_in, weight_buf, buf_out], [k * 4, total, n * 4],
            push_u32(k, n), [qtype.workgroups(n), 1, 1])
