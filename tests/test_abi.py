"""CPU-side checks of the C ABI: the library loads, exports every symbol that
include/nq8.h declares, and its host-only logic (GGUF parsing, argument
validation) behaves without a GPU."""
import ctypes
import os
import re

import numpy as np
import pytest

from nspeech_b200 import lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "nq8.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(nq_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = L.load()
    names = declared_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
        assert n in L.SIGNATURES, f"{n} has no ctypes signature"
    assert set(L.SIGNATURES) == set(names)
    assert lib.nq_version().startswith(b"nq8")


def test_null_arguments_are_rejected_without_device_work():
    lib = L.load()
    out = ctypes.c_void_p()
    assert lib.nq_weight_from_q8_0(None, 4, 32, 0, ctypes.byref(out)) == L.NQ_ERR_ARG
    assert "null" in L.last_error()
    assert lib.nq_linear(None, None, 0, 1, 32, None, 0, None, 0, 32, None) == L.NQ_ERR_ARG
    assert lib.nq_set_wait_limit(0) == L.NQ_ERR_ARG
    for bad in (-1, 1, 32, 100, 192, 1024):
        assert lib.nq_set_gemm_unit_tokens(bad) == L.NQ_ERR_ARG, bad
    assert lib.nq_set_gemm_unit_tokens(512) == L.NQ_ERR_ARG
    for ok in (64, 128, 256, 0):
        assert lib.nq_set_gemm_unit_tokens(ok) == L.NQ_OK, ok
    for bad in (-1, 17):
        assert lib.nq_set_gemm_tail_split(bad) == L.NQ_ERR_ARG, bad
    for ok in (1, 2, 16, 0):
        assert lib.nq_set_gemm_tail_split(ok) == L.NQ_OK, ok
    for bad in (-1, 2):
        assert lib.nq_set_attention_kernel(bad) == L.NQ_ERR_ARG, bad
    for ok in (L.NQ_ATTENTION_MMA_SYNC, L.NQ_ATTENTION_TCGEN05):
        assert lib.nq_set_attention_kernel(ok) == L.NQ_OK, ok
    for bad in (-1, 3):
        assert lib.nq_set_gemv_path(bad) == L.NQ_ERR_ARG, bad
    for ok in (L.NQ_GEMV_SPLIT, L.NQ_GEMV_CLUSTER, L.NQ_GEMV_AUTO):
        assert lib.nq_set_gemv_path(ok) == L.NQ_OK, ok
    for bad in (-1, 2):
        assert lib.nq_set_conv_path(bad) == L.NQ_ERR_ARG, bad
    for ok in (L.NQ_CONV_IM2COL, L.NQ_CONV_AUTO):
        assert lib.nq_set_conv_path(ok) == L.NQ_OK, ok
    buf = ctypes.create_string_buffer(8)
    n = lib.nq_last_error(buf, len(buf))
    assert n > 0 and len(buf.value) == min(n, 7)


def _write_gguf(path, oracle, n=40, k=96):
    gguf = pytest.importorskip("gguf")
    w = oracle.normal(11, (n, k), 0.0, 0.02)
    q = oracle.quantize_q8_0(w)
    wr = gguf.GGUFWriter(str(path), arch="parakeet")
    wr.add_uint32("general.alignment", 64)
    wr.add_string("general.name", "synthetic")
    wr.add_array("tokenizer.ggml.tokens", ["a", "b", "c"])
    wr.add_tensor("enc.w", q, raw_dtype=gguf.GGMLQuantizationType.Q8_0)
    wr.add_tensor("enc.b", oracle.normal(12, (n,), 0.0, 0.01))
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    return q


def test_gguf_tensor_info(tmp_path, oracle):
    p = tmp_path / "m.gguf"
    _write_gguf(p, oracle)
    lib = L.load()
    t, n, k = ctypes.c_int(), ctypes.c_int64(), ctypes.c_int64()
    rc = lib.nq_gguf_tensor_info(str(p).encode(), b"enc.w", ctypes.byref(t), ctypes.byref(n), ctypes.byref(k))
    assert rc == L.NQ_OK, L.last_error()
    assert (t.value, n.value, k.value) == (8, 40, 96)
    rc = lib.nq_gguf_tensor_info(str(p).encode(), b"enc.b", ctypes.byref(t), ctypes.byref(n), ctypes.byref(k))
    assert rc == L.NQ_ERR_SHAPE and t.value == 0  # f32, 1-D
    assert lib.nq_gguf_tensor_info(str(p).encode(), b"nope", None, None, None) == L.NQ_ERR_ARG
    assert lib.nq_gguf_tensor_info(str(tmp_path / "missing.gguf").encode(), b"enc.w", None, None, None) == L.NQ_ERR_IO


def test_gguf_rejects_corrupt_files(tmp_path, oracle):
    p = tmp_path / "m.gguf"
    _write_gguf(p, oracle)
    raw = p.read_bytes()
    lib = L.load()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"XXXX" + raw[4:])
    assert lib.nq_gguf_tensor_info(str(bad).encode(), b"enc.w", None, None, None) == L.NQ_ERR_FORMAT
    assert "magic" in L.last_error()
    for cut in (10, 30, 100, 200):
        bad.write_bytes(raw[:cut])
        assert lib.nq_gguf_tensor_info(str(bad).encode(), b"enc.w", None, None, None) in (L.NQ_ERR_FORMAT, L.NQ_ERR_ARG)
    bad.write_bytes(raw[:4] + (7).to_bytes(4, "little") + raw[8:])
    assert lib.nq_gguf_tensor_info(str(bad).encode(), b"enc.w", None, None, None) == L.NQ_ERR_FORMAT


def test_q8_0_blob_layout_matches_gguf(tmp_path, oracle):
    """The bytes a GGUF file stores for a Q8_0 tensor are the oracle's blocks."""
    gguf = pytest.importorskip("gguf")
    p = tmp_path / "m.gguf"
    q = _write_gguf(p, oracle)
    r = gguf.GGUFReader(str(p))
    t = [t for t in r.tensors if t.name == "enc.w"][0]
    assert np.array_equal(np.asarray(t.data).reshape(q.shape), q)
