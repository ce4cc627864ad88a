"""ctypes front-end of the CPU oracle (``oracle/nq8_oracle.c``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, by ``__graft_entry__.smoke()``
as the checker and by ``bench.py``'s CPU-baseline leg.  The shipped library
(``nspeech_b200``) never imports this module.

Each function names the reference code it restates (paths relative to the
dropbox/nspeech source tree); see the header of ``nq8_oracle.c``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libnq8_oracle.so")
_lib = None

QK = 32
BLOCK_BYTES = 34

EPI_NONE, EPI_SILU, EPI_GELU_ERF, EPI_GLU_SIGMOID, EPI_GLU_SILU = range(5)

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_i64 = ctypes.c_int64


def build() -> str:
    """Compile the oracle with its Makefile (gcc) if it is missing or stale."""
    src = os.path.join(_HERE, "nq8_oracle.c")
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        L.oq_f32_to_f16.argtypes = [ctypes.c_float]
        L.oq_f32_to_f16.restype = ctypes.c_uint16
        L.oq_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.oq_f16_to_f32.restype = ctypes.c_float
        L.oq_f32_to_bf16.argtypes = [ctypes.c_float]
        L.oq_f32_to_bf16.restype = ctypes.c_uint16
        L.oq_quantize_q8_0.argtypes = [_f32p, _i64, _i64, _u8p]
        L.oq_dequant_q8_0.argtypes = [_u8p, _i64, _i64, _f32p]
        L.oq_dequant_q8_0_t.argtypes = [_u8p, _i64, _i64, _f32p]
        L.oq_pack_bf16.argtypes = [_f32p, _i64, _u16p]
        L.oq_matmul_fbgemm_bf16.argtypes = [_f32p, _i64, _i64, _u8p, _i64, _f32p]
        L.oq_matmul_qtiled.argtypes = [_f32p, _i64, _i64, _u8p, _i64, _f32p]
        L.oq_matmul_exact_f64.argtypes = [_f32p, _i64, _i64, _u8p, _i64, _f64p]
        L.oq_epilogue_f64.argtypes = [_f64p, _i64, _i64, ctypes.c_void_p, ctypes.c_int, _f64p]
        L.oq_max_rel_err.argtypes = [_f32p, _f64p, _i64, _i64, ctypes.c_double]
        L.oq_max_rel_err.restype = ctypes.c_double
        L.oq_fill_normal.argtypes = [ctypes.c_uint64, _f32p, _i64, ctypes.c_float, ctypes.c_float]
        L.oq_fill_uniform.argtypes = [ctypes.c_uint64, _f32p, _i64, ctypes.c_float, ctypes.c_float]
        _lib = L
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ----------------------------------------------------------------- generators
def normal(seed: int, shape, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(int(np.prod(shape)), dtype=np.float32)
    lib().oq_fill_normal(seed, out, out.size, mean, std)
    return out.reshape(shape)


def uniform(seed: int, shape, lo: float, hi: float) -> np.ndarray:
    out = np.empty(int(np.prod(shape)), dtype=np.float32)
    lib().oq_fill_uniform(seed, out, out.size, lo, hi)
    return out.reshape(shape)


# ----------------------------------------------------------------------- Q8_0
def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    """[n, k] f32 -> [n, k/32*34] uint8 GGUF Q8_0 blocks (ggml semantics)."""
    w = _f32(w)
    n, k = w.shape
    if k % QK:
        raise ValueError(f"k={k} is not a multiple of {QK}")
    out = np.empty((n, k // QK * BLOCK_BYTES), dtype=np.uint8)
    lib().oq_quantize_q8_0(w, n, k, out)
    return out


def dequant_q8_0(blocks: np.ndarray, n: int, k: int) -> np.ndarray:
    out = np.empty((n, k), dtype=np.float32)
    lib().oq_dequant_q8_0(np.ascontiguousarray(blocks, dtype=np.uint8), n, k, out)
    return out


def dequant_q8_0_t(blocks: np.ndarray, n: int, k: int) -> np.ndarray:
    out = np.empty((k, n), dtype=np.float32)
    lib().oq_dequant_q8_0_t(np.ascontiguousarray(blocks, dtype=np.uint8), n, k, out)
    return out


def pack_bf16(w: np.ndarray) -> np.ndarray:
    w = _f32(w)
    out = np.empty(w.shape, dtype=np.uint16)
    lib().oq_pack_bf16(w.reshape(-1), w.size, out.reshape(-1))
    return out


def f32_to_f16_bits(v: float) -> int:
    return int(lib().oq_f32_to_f16(v))


def f32_to_bf16_bits(v: float) -> int:
    return int(lib().oq_f32_to_bf16(v))


# ------------------------------------------------------------------- matmuls
def matmul_fbgemm_bf16(x: np.ndarray, blocks: np.ndarray, n: int) -> np.ndarray:
    """REF_FBGEMM_BF16 (src/fast_matmul.rs:138-167): y = x . bf16(W)^T in f32."""
    x = _f32(x)
    m, k = x.shape
    y = np.empty((m, n), dtype=np.float32)
    lib().oq_matmul_fbgemm_bf16(x, m, k, np.ascontiguousarray(blocks, dtype=np.uint8), n, y)
    return y


def matmul_qtiled(x: np.ndarray, blocks: np.ndarray, n: int) -> np.ndarray:
    """REF_QTILED (src/fast_matmul.rs:30-62): Q8_0 x Q8_0 per-block dot."""
    x = _f32(x)
    m, k = x.shape
    y = np.empty((m, n), dtype=np.float32)
    lib().oq_matmul_qtiled(x, m, k, np.ascontiguousarray(blocks, dtype=np.uint8), n, y)
    return y


def matmul_exact(x: np.ndarray, blocks: np.ndarray, n: int) -> np.ndarray:
    """REF_EXACT: y = x . dequant(W)^T in f64 (the tolerance anchor)."""
    x = _f32(x)
    m, k = x.shape
    y = np.empty((m, n), dtype=np.float64)
    lib().oq_matmul_exact_f64(x, m, k, np.ascontiguousarray(blocks, dtype=np.uint8), n, y)
    return y


def epilogue(y: np.ndarray, bias, epi: int) -> np.ndarray:
    """Bias + activation on a raw f64 product (GLU: first half * act(second))."""
    y = np.ascontiguousarray(y, dtype=np.float64)
    m, n = y.shape
    n_out = n // 2 if epi in (EPI_GLU_SIGMOID, EPI_GLU_SILU) else n
    out = np.empty((m, n_out), dtype=np.float64)
    b = None
    if bias is not None:
        b = _f32(bias)
    lib().oq_epilogue_f64(y, m, n, None if b is None else b.ctypes.data, epi, out)
    return out


def linear_exact(x, blocks, n, bias=None, epi=EPI_NONE) -> np.ndarray:
    """f64 reference of act(x . dequant(W)^T + bias)."""
    return epilogue(matmul_exact(x, blocks, n), bias, epi)


def max_rel_err(y: np.ndarray, yref: np.ndarray, tau: float = 1e-3) -> float:
    """max |y - yref| / max(|yref|, tau * rms(yref row)) over all elements."""
    y = _f32(y)
    yref = np.ascontiguousarray(yref, dtype=np.float64)
    if y.shape != yref.shape:
        raise ValueError(f"shape mismatch {y.shape} vs {yref.shape}")
    m = y.shape[0] if y.ndim > 1 else 1
    n = y.shape[-1]
    return float(lib().oq_max_rel_err(y.reshape(-1), yref.reshape(-1), m, n, tau))
