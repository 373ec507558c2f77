"""The GGUF reader (rrr_gguf_*, replaces GGUFModel, src/model/gguf.rs) against files written
by gguf-py's GGUFWriter: header, metadata of every value type, tensor infos, zero-copy
tensor bytes and the data-section alignment; malformed files return RRR_ERR_IO.
No GPU needed (host code in the same library)."""
import ctypes
import os

import numpy as np
import pytest

gguf = pytest.importorskip("gguf")


def _write(path, rng, extra_kv=True):
    from gguf import GGMLQuantizationType as T
    w = gguf.GGUFWriter(path, "phi3")
    w.add_uint32("phi3.embedding_length", 512)
    w.add_uint32("phi3.attention.head_count", 4)
    w.add_uint32("phi3.attention.head_count_kv", 2)
    w.add_uint32("phi3.feed_forward_length", 768)
    w.add_uint32("phi3.block_count", 1)
    w.add_float32("phi3.attention.layer_norm_rms_epsilon", 1e-5)
    if extra_kv:
        # every scalar type, including the 1-byte ones the reference misreads
        w.add_uint8("test.u8", 200)
        w.add_int8("test.i8", -5)
        w.add_uint16("test.u16", 65000)
        w.add_int16("test.i16", -30000)
        w.add_int32("test.i32", -7)
        w.add_uint64("test.u64", 1 << 40)
        w.add_int64("test.i64", -(1 << 40))
        w.add_float64("test.f64", 2.5)
        w.add_bool("test.bool", True)
        w.add_string("test.str", "hello")
        w.add_array("test.arr", [1, 2, 3])
        w.add_uint8("test.u8_after", 7)   # parsed correctly only if u8 is one byte
    import oracle
    tensors = {}
    for name, qt, K, N in [("blk.0.attn_qkv.weight", T.Q5_K, 512, 1024),
                           ("blk.0.ffn_down.weight", T.Q6_K, 768, 512),
                           ("blk.0.attn_output.weight", T.Q4_K, 512, 512)]:
        raw = oracle.random_blocks(int(qt), N * K // 256, rng).reshape(N, -1)
        w.add_tensor(name, raw, raw_dtype=qt)
        tensors[name] = (int(qt), K, N, raw.reshape(-1))
    emb = rng.standard_normal((10, 512)).astype(np.float32)
    w.add_tensor("token_embd.weight", emb)
    tensors["token_embd.weight"] = (0, 512, 10, emb.reshape(-1).view(np.uint8))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return tensors


@pytest.fixture(scope="module")
def gfile(tmp_path_factory, oracle):
    p = str(tmp_path_factory.mktemp("gguf") / "tiny.gguf")
    tensors = _write(p, np.random.default_rng(3))
    return p, tensors


def test_reader_matches_writer(rrr, gfile):
    path, tensors = gfile
    g = rrr.GGUFModel.load(path)
    ref = gguf.GGUFReader(path)
    assert g.version == 3
    assert g.n_tensors == len(ref.tensors) == 4
    assert g.data_offset == ref.data_offset
    names = {t.name for t in g.tensor_infos}
    assert names == set(tensors)
    for t in g.tensor_infos:
        qt, K, N, raw = tensors[t.name]
        assert t.typ == qt and t.shape == [K, N]
        got = g.tensor_bytes(t.name)
        assert got.nbytes == raw.nbytes and np.array_equal(got, raw)
    # tensor_f32 on the F32 tensor
    assert np.array_equal(g.tensor_f32("token_embd.weight"), tensors["token_embd.weight"][3].view(np.float32))
    g.close()


def test_metadata_types(rrr, gfile):
    path, _ = gfile
    g = rrr.GGUFModel.load(path)
    assert g.meta_str("general.architecture") == "phi3"
    assert g.meta_u64("phi3.embedding_length") == 512
    assert abs(g.meta_f32("phi3.attention.layer_norm_rms_epsilon") - 1e-5) < 1e-12
    assert g.meta_u64("test.u8") == 200
    assert g.meta_u64("test.u16") == 65000
    assert g.meta_u64("test.u64") == 1 << 40
    assert g.meta_u64("test.i8") == (-5) & 0xFFFFFFFFFFFFFFFF    # as_u64 of a signed value
    assert g.meta_u64("test.u8_after") == 7                       # the 1-byte read kept sync
    assert g.meta_f32("test.f64") == 2.5
    assert g.meta_str("test.str") == "hello"
    assert g.meta_u64("missing.key") == 0 and g.meta_str("missing.key") == ""
    cfg = rrr.ModelConfig.from_gguf(g)
    assert (cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim, cfg.n_layers,
            cfg.vocab_size) == (512, 4, 2, 128, 768, 1, 10)
    g.close()


def test_missing_tensor_and_bad_files(rrr, gfile, tmp_path):
    path, _ = gfile
    g = rrr.GGUFModel.load(path)
    with pytest.raises(rrr.RRRError):
        g.tensor_bytes("nope.weight")
    g.close()
    data = open(path, "rb").read()
    bad = tmp_path / "bad_magic.gguf"
    bad.write_bytes(b"XXXX" + data[4:])
    with pytest.raises(rrr.RRRError) as e:
        rrr.GGUFModel.load(str(bad))
    assert e.value.code == -10
    for cut in (10, 100, len(data) // 2, len(data) - 3):
        trunc = tmp_path / f"trunc{cut}.gguf"
        trunc.write_bytes(data[:cut])
        with pytest.raises(rrr.RRRError) as e:
            rrr.GGUFModel.load(str(trunc))
        assert e.value.code == -10
    with pytest.raises(rrr.RRRError):
        rrr.GGUFModel.load(str(tmp_path / "does_not_exist.gguf"))


@pytest.mark.gpu
def test_upload_and_gemv_from_gguf(rrr, ctx, oracle, gfile):
    """load_weight_gpu without the repack: raw tensor bytes -> device -> GEMV."""
    import torch
    from ctypes import c_void_p
    path, tensors = gfile
    g = rrr.GGUFModel.load(path)
    L = rrr.ffi.lib()
    for name in ("blk.0.attn_qkv.weight", "blk.0.ffn_down.weight", "blk.0.attn_output.weight"):
        qt, K, N, raw = tensors[name]
        dptr, nbytes = g.upload(ctx, name)
        assert nbytes == raw.nbytes
        x = torch.randn(K, device="cuda")
        y = torch.empty(N, device="cuda")
        ctx.check(L.rrr_gemv_kq(ctx.h, qt, c_void_p(dptr), c_void_p(x.data_ptr()), c_void_p(y.data_ptr()),
                                K, N, None, None))
        torch.cuda.synchronize()
        ref = oracle.gemv_kq(qt, raw, x.cpu().numpy(), K, N)
        got = y.cpu().numpy()
        assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-4
        ctx.check(L.rrr_free(ctx.h, c_void_p(dptr)))
    g.close()


@pytest.mark.gpu
def test_gguf_load_many_tensors_through_pinned_staging(rrr, ctx, tmp_path):
    """rrr_gguf_load: several tensors, one of 100 MB (four 32 MB staging chunks, both pinned
    buffers reused twice) and several not multiples of the chunk, into one device
    allocation; every byte on the device equals the file's, twice in a row (the staging is
    reused by the second call)."""
    import torch
    from ctypes import c_char_p, c_double, c_uint64, c_void_p
    from gguf import GGMLQuantizationType as T
    path = str(tmp_path / "load.gguf")
    rng = np.random.default_rng(9)
    w = gguf.GGUFWriter(path, "phi3")
    data = {}
    for name, rows, nb in [("a.weight", 3, 1), ("big.weight", 2048 * 2, 171),   # 100.9 MB Q4_K
                           ("c.weight", 77, 5), ("d.weight", 1, 12)]:
        raw = rng.integers(0, 256, size=(rows, nb * 144), dtype=np.uint8)
        w.add_tensor(name, raw, raw_dtype=T.Q4_K)
        data[name] = raw.reshape(-1)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    g = rrr.GGUFModel.load(path)
    L = rrr.ffi.lib()
    names = list(data)
    arr = (c_char_p * len(names))(*[n.encode() for n in names])
    for _ in range(2):
        ptrs = (c_void_p * len(names))()
        sizes = (c_uint64 * len(names))()
        secs = c_double()
        ctx.check(L.rrr_gguf_load(ctx.h, g.h, arr, len(names), ptrs, sizes, ctypes.byref(secs)))
        assert ptrs[0] is not None and all(p % 256 == 0 for p in ptrs)
        for i, n in enumerate(names):
            assert sizes[i] == data[n].nbytes
            host = np.empty(data[n].nbytes, np.uint8)
            ctx.check(L.rrr_d2h(ctx.h, c_void_p(host.ctypes.data), c_void_p(ptrs[i]), host.nbytes, None))
            ctx.check(L.rrr_sync(ctx.h, None))
            assert np.array_equal(host, data[n]), n
        assert secs.value > 0
        ctx.check(L.rrr_free(ctx.h, c_void_p(ptrs[0])))
    g.close()
