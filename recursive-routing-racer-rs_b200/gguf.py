"""Host mirror of RRR's GGUF loader (src/model/gguf.rs) over the C++ reader in the C ABI
(rrr_gguf_*). `GGUFModel.load`, `tensor_infos`, `tensor_bytes` (zero-copy view of the
mapping), `tensor_f32`, `meta_u64`, `meta_str` keep the reference's names and meaning.
"""
from __future__ import annotations

import ctypes
from ctypes import c_char_p, c_float, c_int64, c_uint32, c_uint64, c_void_p
from dataclasses import dataclass

import numpy as np

from . import ffi


@dataclass
class TensorInfo:
    """gguf.rs:10-16 (shape in GGUF order: ne0 first)."""
    name: str
    shape: list
    typ: int
    offset: int
    n_bytes: int


class GGUFModel:
    def __init__(self, handle: c_void_p):
        self.h = handle
        n = c_int64()
        self._check(ffi.lib().rrr_gguf_n_tensors(self.h, ctypes.byref(n)))
        self.n_tensors = n.value
        v = c_uint32()
        self._check(ffi.lib().rrr_gguf_version(self.h, ctypes.byref(v)))
        self.version = v.value
        off = c_uint64()
        self._check(ffi.lib().rrr_gguf_data_offset(self.h, ctypes.byref(off)))
        self.data_offset = off.value
        self.tensor_infos = []
        for i in range(self.n_tensors):
            t = ffi.GGUFTensor()
            self._check(ffi.lib().rrr_gguf_tensor_at(self.h, i, ctypes.byref(t)))
            self.tensor_infos.append(TensorInfo(t.name.decode(), list(t.shape[:t.n_dims]), t.type,
                                                t.offset, t.n_bytes))

    @staticmethod
    def _check(rc: int) -> None:
        ffi.check(rc, None)

    @classmethod
    def load(cls, path: str) -> "GGUFModel":
        """gguf.rs:125-170."""
        h = c_void_p()
        ffi.check(ffi.lib().rrr_gguf_open(path.encode(), ctypes.byref(h)), None)
        return cls(h)

    def load_tensors(self, ctx: ffi.Context, names):
        """rrr_gguf_load: the named tensors into one device allocation through the file's
        pinned staging. Returns (device pointers, sizes, seconds); rrr_free of pointers[0]
        releases all of them."""
        n = len(names)
        arr = (ctypes.c_char_p * n)(*[nm.encode() for nm in names])
        ptrs = (ctypes.c_void_p * n)()
        sizes = (ctypes.c_uint64 * n)()
        secs = ctypes.c_double()
        ctx.check(ffi.lib().rrr_gguf_load(ctx.h, self.h, arr, n, ptrs, sizes, ctypes.byref(secs)))
        return [p for p in ptrs], [int(x) for x in sizes], secs.value

    def _find(self, name: str) -> ffi.GGUFTensor:
        t = ffi.GGUFTensor()
        self._check(ffi.lib().rrr_gguf_find_tensor(self.h, name.encode(), ctypes.byref(t)))
        return t

    def tensor_bytes(self, name: str) -> np.ndarray:
        """gguf.rs:173-195: raw bytes as a read-only uint8 view of the mapping."""
        t = self._find(name)
        buf = (ctypes.c_uint8 * t.n_bytes).from_address(t.data)
        a = np.frombuffer(buf, dtype=np.uint8)
        a.flags.writeable = False
        return a

    def tensor_f32(self, name: str) -> np.ndarray:
        """gguf.rs:198-206 (an F32 tensor viewed as floats)."""
        return self.tensor_bytes(name).view(np.float32)

    def meta_u64(self, key: str) -> int:
        """gguf.rs:208-210: 0 when missing."""
        v = c_uint64()
        return v.value if ffi.lib().rrr_gguf_meta_u64(self.h, key.encode(), ctypes.byref(v)) == 0 else 0

    def meta_f32(self, key: str) -> float:
        v = c_float()
        return v.value if ffi.lib().rrr_gguf_meta_f32(self.h, key.encode(), ctypes.byref(v)) == 0 else 0.0

    def meta_str(self, key: str) -> str:
        """gguf.rs:212-214: "" when missing."""
        v = c_char_p()
        return v.value.decode() if ffi.lib().rrr_gguf_meta_str(self.h, key.encode(), ctypes.byref(v)) == 0 else ""

    def upload(self, ctx: ffi.Context, name: str) -> tuple[int, int]:
        """Raw tensor bytes to a new device buffer (load_weight_gpu without the repack)."""
        p = c_void_p()
        n = c_uint64()
        ctx.check(ffi.lib().rrr_gguf_upload(ctx.h, self.h, name.encode(), ctypes.byref(p), ctypes.byref(n)))
        return p.value, n.value

    def close(self) -> None:
        if self.h:
            ffi.lib().rrr_gguf_close(self.h)
            self.h = None
