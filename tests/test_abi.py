"""The C ABI surface without a GPU: the library loads, exports every function the header
declares (and ffi.py binds all of them), and argument validation returns the documented
status codes instead of crashing. No compute call is made."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "rrr_cuda.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\**\s*(rrr_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_interface():
    names = declared_functions()
    for must in ("rrr_init", "rrr_gemv_kq", "rrr_gemm_kq_batched", "rrr_rmsnorm", "rrr_logits_f32",
                 "rrr_dispatch_by_name", "rrr_gguf_open", "rrr_phi4_forward", "rrr_last_error"):
        assert must in names
    assert len(names) >= 50


def test_library_exports_every_declared_symbol(rrr):
    L = rrr.ffi.lib()
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, missing


def test_ffi_binds_every_declared_symbol(rrr):
    unbound = [n for n in declared_functions() if n not in rrr.ffi.PROTOS]
    assert not unbound, unbound


def _header_params(name):
    """Parameter count of a declared function (comments stripped)."""
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    m = re.search(r"\b" + name + r"\s*\(([^;]*?)\)\s*;", text, flags=re.S)
    args = [a for a in m.group(1).split(",") if a.strip() and a.strip() != "void"]
    return len(args)


def test_rust_binding_in_integration_doc_matches_header():
    """The Rust extern block of the integration guide (the binding a maintainer adds to
    the reference crate) declares every header function with the same number of
    parameters."""
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    block = doc[doc.index("```rust"):]
    block = block[:block.index("```", 7)]
    rust = {}
    for m in re.finditer(r"pub fn (rrr_\w+)\((.*?)\)\s*->", block, flags=re.S):
        params = [p for p in m.group(2).split(",") if p.strip()]
        rust[m.group(1)] = len(params)
    declared = declared_functions()
    assert sorted(rust) == declared, sorted(set(declared) ^ set(rust))
    for name in declared:
        assert rust[name] == _header_params(name), name


def test_status_strings_and_version(rrr):
    L = rrr.ffi.lib()
    assert L.rrr_abi_version() == 1
    for code, name in rrr.ffi.STATUS.items():
        assert L.rrr_status_string(code).decode() == name


def test_null_context_is_an_error_not_a_crash(rrr):
    L = rrr.ffi.lib()
    assert L.rrr_gemv_kq(None, 12, None, None, None, 256, 1, None, None) == -1
    assert L.rrr_rmsnorm(None, None, None, None, 1, 1, 1e-5, None) == -1
    assert L.rrr_logits_f32(None, None, None, None, 1, 4, 0, None, 0.0, None) == -1
    assert L.rrr_dispatch_by_name(None, b"rmsnorm", None, None, 0, None, 0, None) == -1
    assert L.rrr_destroy(None) == -1
    assert "null context" in rrr.ffi.last_error(None)


def test_init_without_gpu_reports_cuda_error(rrr):
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    h = ctypes.c_void_p()
    rc = rrr.ffi.lib().rrr_init(0, ctypes.byref(h))
    assert rc == -5 and not h.value
    assert "CUDA" in rrr.ffi.last_error(None) or "device" in rrr.ffi.last_error(None)
    with pytest.raises(rrr.RRRError):
        rrr.Context(0)


def test_package_fails_loudly_without_library(rrr, monkeypatch, tmp_path):
    ffi = rrr.ffi
    monkeypatch.setattr(ffi, "_lib", None)
    monkeypatch.setattr(ffi, "LIB_PATH", str(tmp_path / "missing.so"))
    with pytest.raises(RuntimeError, match="no fallback"):
        ffi.lib()


def test_qtype_table_matches_reference(rrr):
    Q = rrr.QType
    assert [Q.from_gguf(t) for t in (12, 13, 14, 0)] == [Q.Q4K, Q.Q5K, Q.Q6K, Q.F32]
    assert [q.block_bytes() for q in (Q.Q4K, Q.Q5K, Q.Q6K)] == [144, 176, 210]
    assert Q.Q6K.shader_name() == "matmul_q6k" and Q.Q4K.batch_shader_name() == "matmul_q4k_batch"
    name, bufs, sizes, push, groups = rrr.kquant_dispatch(1, 2, 3, Q.Q5K, 3072, 5120)
    assert name == "matmul_q5k" and sizes == [3072 * 4, 5120 * 12 * 176, 5120 * 4]
    assert push == rrr.push_u32(3072, 5120) and groups == [5120, 1, 1]


def test_model_config_bytes(rrr):
    cfg = rrr.ModelConfig()
    shapes = {n: (q, K, N) for n, q, K, N in cfg.layer_gemvs()}
    assert shapes == {"qkv": (13, 3072, 5120), "o_proj": (12, 3072, 3072),
                      "gate_up": (12, 3072, 16384), "down": (14, 8192, 3072)}
    layer = sum(cfg.weight_bytes(q, K, N) for q, K, N in shapes.values())
    assert layer == 65_077_248
    assert cfg.step_bytes() == 4_541_657_088
