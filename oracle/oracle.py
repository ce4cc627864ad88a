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

EPI_NONE, EPI_SILU, EPI_GELU_ERF, EPI_GLU_SIGMOID, EPI_GLU_SILU, EPI_RELU = range(6)

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_i64 = ctypes.c_int64


def build() -> str:
    """Compile the oracle with its Makefile (gcc) if it is missing or stale."""
    srcs = [os.path.join(_HERE, s) for s in ("nq8_oracle.c", "encoder_oracle.c", "fbgemm_cpu.c", "Makefile")]
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < max(os.path.getmtime(s) for s in srcs):
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
        L.ofb_matmul_q8_0.argtypes = [_f32p, _i64, _i64, _u8p, _i64, ctypes.c_int, _f32p]
        L.ofb_isa.restype = ctypes.c_int
        L.ofb_force_isa.argtypes = [ctypes.c_int]
        L.ofb_set_threads.argtypes = [ctypes.c_int]
        L.ofb_max_threads.restype = ctypes.c_int
        L.ofb_pack_q8_0.argtypes = [_u8p, _i64, _i64, ctypes.c_int]
        L.ofb_pack_q8_0.restype = ctypes.c_void_p
        L.ofb_free.argtypes = [ctypes.c_void_p]
        L.ofb_linear.argtypes = [ctypes.c_void_p, _f32p, _i64, _i64, ctypes.c_void_p, _f32p, _i64]
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


def matmul_fbgemm_packed(x: np.ndarray, blocks: np.ndarray, n: int, bf16: bool = True) -> np.ndarray:
    """The same product through fbgemm_cpu.c's packed AVX-512 / AVX2 kernels
    (weights packed to bf16 once, FbgemmBf16Op's structure); bit-identical to
    matmul_fbgemm_bf16 for bf16=True, exact f32 weights for bf16=False."""
    x = _f32(x)
    m, k = x.shape
    y = np.empty((m, n), dtype=np.float32)
    lib().ofb_matmul_q8_0(x, m, k, np.ascontiguousarray(blocks, dtype=np.uint8), n, 1 if bf16 else 0, y)
    return y


class PackedWeight:
    """A Q8_0 weight dequantized and packed to bf16 once (MatMul::from_tensor,
    src/fast_matmul.rs:191-208), multiplied by the packed CPU kernels
    (FbgemmBf16Op::cpu_fwd, :138-167).  The CPU baseline's linear."""

    def __init__(self, blocks: np.ndarray, n: int, k: int, bf16: bool = True):
        self.n, self.k = n, k
        self._h = lib().ofb_pack_q8_0(np.ascontiguousarray(blocks, dtype=np.uint8), n, k, 1 if bf16 else 0)

    def __call__(self, x: np.ndarray, bias=None, out=None) -> np.ndarray:
        x = _f32(x)
        m = x.shape[0]
        y = np.empty((m, self.n), np.float32) if out is None else out
        b = None if bias is None else _f32(bias)
        lib().ofb_linear(self._h, x, m, x.shape[1], None if b is None else b.ctypes.data, y, self.n)
        return y

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.ofb_free(self._h)
            self._h = None


def set_threads(n: int) -> None:
    """OpenMP threads of the CPU kernels (the CPU baseline's core count)."""
    lib().ofb_set_threads(int(n))


def max_threads() -> int:
    return int(lib().ofb_max_threads())


def cpu_isa() -> int:
    """512 when the packed kernels run AVX-512, 256 for AVX2 + FMA."""
    return int(lib().ofb_isa())


def force_isa(isa: int) -> None:
    lib().ofb_force_isa(int(isa))


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


def resadd_layernorm(y, res_in, gamma, beta=None, eps: float = 1e-5):
    """Decoder-step residual add + LayerNorm, in f64: r = res_in + y and
    out = (r - mean) / sqrt(var + eps) * gamma (+ beta), biased variance over
    the row.  Restates residual_add and LayerNorm::forward of
    src/moonshine/decoder.rs:41-50,67-74 (weight-only LayerNorm, eps 1e-5),
    the CPU form of the fused reduce + residual + LayerNorm of
    kernels/moonshine_kernels.py:1109-1146.  Returns (r, out)."""
    r = np.asarray(res_in, dtype=np.float64) + np.asarray(y, dtype=np.float64)
    mean = r.mean(axis=1, keepdims=True)
    c = r - mean
    var = (c * c).mean(axis=1, keepdims=True)
    out = c / np.sqrt(var + eps) * np.asarray(gamma, dtype=np.float64)[None, :]
    if beta is not None:
        out = out + np.asarray(beta, dtype=np.float64)[None, :]
    return r, out


def max_rel_err(y: np.ndarray, yref: np.ndarray, tau: float = 1e-3) -> float:
    """max |y - yref| / max(|yref|, tau * rms(yref row)) over all elements."""
    y = _f32(y)
    yref = np.ascontiguousarray(yref, dtype=np.float64)
    if y.shape != yref.shape:
        raise ValueError(f"shape mismatch {y.shape} vs {yref.shape}")
    m = y.shape[0] if y.ndim > 1 else 1
    n = y.shape[-1]
    return float(lib().oq_max_rel_err(y.reshape(-1), yref.reshape(-1), m, n, tau))


# ---------------------------------------------------------------- encoder
class _EncCfg(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("feat_in", "d_model", "n_heads", "ff_mult", "n_layers",
                                             "conv_kernel", "sub_channels", "scale_input")]


_U8P = ctypes.POINTER(ctypes.c_uint8)
_F32P = ctypes.POINTER(ctypes.c_float)


class _EncLayer(ctypes.Structure):
    _fields_ = ([(n, _U8P) for n in ("ff1_w1", "ff1_w2", "ff2_w1", "ff2_w2", "q", "k", "v", "o", "rel", "pw1", "pw2")]
                + [(n, _F32P) for n in ("ff1_b1", "ff1_b2", "ff2_b1", "ff2_b2", "q_b", "k_b", "v_b", "o_b", "pw1_b",
                                        "pw2_b", "bias_u", "bias_v", "dw_w", "dw_b", "bn_g", "bn_b", "bn_mean",
                                        "bn_var")]
                + [("ln_g", _F32P * 5), ("ln_b", _F32P * 5)])


class _EncWeights(ctypes.Structure):
    _fields_ = ([(n, _F32P) for n in ("c0_w", "c0_b", "dw2_w", "dw2_b", "dw5_w", "dw5_b", "pw3_b", "pw6_b", "lin_b")]
                + [(n, _U8P) for n in ("pw3", "pw6", "lin")] + [("layers", ctypes.POINTER(_EncLayer))])


class EncoderModel:
    """Batch-1 FastConformer encoder (encoder_oracle.c) with every linear packed
    once, as the reference packs at load time; ``__call__`` runs one segment.

    ``tensors``: name -> f32 array for vectors, uint8 Q8_0 blocks [n, k/32*34]
    for the rank-2 / pointwise matrices (the names of remap_nemo_tensor_name).
    weight_mode 0: bf16-rounded dequantized weights (fast_matmul semantics);
    1: exact dequantized f32 weights (candle Linear).
    """

    def __init__(self, cfg: dict, tensors: dict, weight_mode: int = 0):
        L = lib()
        L.oq_encoder_prepare.argtypes = [ctypes.POINTER(_EncCfg), ctypes.POINTER(_EncWeights), ctypes.c_int]
        L.oq_encoder_prepare.restype = ctypes.c_void_p
        L.oq_encoder_run.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int, _f32p]
        L.oq_encoder_run.restype = ctypes.c_int
        L.oq_encoder_release.argtypes = [ctypes.c_void_p]
        self.cfg = dict(cfg)
        self._keep, self._c, self._w = _encoder_structs(cfg, tensors)
        self._h = L.oq_encoder_prepare(ctypes.byref(self._c), ctypes.byref(self._w), int(weight_mode))

    def __call__(self, mel: np.ndarray) -> np.ndarray:
        mel = _f32(mel)
        t_mel = mel.shape[0]
        t3 = t_mel
        for _ in range(3):
            t3 = (t3 - 1) // 2 + 1
        out = np.empty((t3, self.cfg["d_model"]), np.float32)
        got = lib().oq_encoder_run(self._h, mel.reshape(-1), t_mel, out.reshape(-1))
        assert got == t3
        return out

    def close(self):
        if getattr(self, "_h", None):
            lib().oq_encoder_release(self._h)
            self._h = None

    def __del__(self):
        if _lib is not None:
            self.close()


def encoder_forward(cfg: dict, tensors: dict, mel: np.ndarray, weight_mode: int = 0) -> np.ndarray:
    """One-shot batch-1 encoder forward -> [T3, d_model] (see EncoderModel)."""
    m = EncoderModel(cfg, tensors, weight_mode)
    try:
        return m(mel)
    finally:
        m.close()


def _encoder_structs(cfg: dict, tensors: dict):
    """ctypes config and weight table over the caller's arrays (kept alive by
    the returned list)."""
    keep = []

    def f(name, default=None):
        a = tensors.get(name)
        if a is None:
            a = default
        a = np.ascontiguousarray(a, dtype=np.float32)
        keep.append(a)
        return a.ctypes.data_as(_F32P)

    def q(name):
        a = np.ascontiguousarray(tensors[name], dtype=np.uint8)
        keep.append(a)
        return a.ctypes.data_as(_U8P)

    d = cfg["d_model"]
    ones, zeros = np.ones(d, np.float32), np.zeros(d, np.float32)
    c = _EncCfg(**{n: int(cfg[n]) for n, _ in _EncCfg._fields_})
    layers = (_EncLayer * cfg["n_layers"])()
    for i in range(cfg["n_layers"]):
        p = f"encoder.layers.{i}."
        Ly = layers[i]
        Ly.ff1_w1, Ly.ff1_w2 = q(p + "feed_forward1.linear1.weight"), q(p + "feed_forward1.linear2.weight")
        Ly.ff2_w1, Ly.ff2_w2 = q(p + "feed_forward2.linear1.weight"), q(p + "feed_forward2.linear2.weight")
        Ly.q, Ly.k = q(p + "self_attn.q_proj.weight"), q(p + "self_attn.k_proj.weight")
        Ly.v, Ly.o = q(p + "self_attn.v_proj.weight"), q(p + "self_attn.o_proj.weight")
        Ly.rel = q(p + "self_attn.relative_k_proj.weight")
        Ly.pw1, Ly.pw2 = q(p + "conv.pointwise_conv1.weight"), q(p + "conv.pointwise_conv2.weight")
        ff = d * cfg["ff_mult"]
        Ly.ff1_b1 = f(p + "feed_forward1.linear1.bias", np.zeros(ff, np.float32))
        Ly.ff1_b2 = f(p + "feed_forward1.linear2.bias", zeros)
        Ly.ff2_b1 = f(p + "feed_forward2.linear1.bias", np.zeros(ff, np.float32))
        Ly.ff2_b2 = f(p + "feed_forward2.linear2.bias", zeros)
        Ly.q_b, Ly.k_b = f(p + "self_attn.q_proj.bias", zeros), f(p + "self_attn.k_proj.bias", zeros)
        Ly.v_b, Ly.o_b = f(p + "self_attn.v_proj.bias", zeros), f(p + "self_attn.o_proj.bias", zeros)
        Ly.pw1_b = f(p + "conv.pointwise_conv1.bias", np.zeros(2 * d, np.float32))
        Ly.pw2_b = f(p + "conv.pointwise_conv2.bias", zeros)
        Ly.bias_u, Ly.bias_v = f(p + "self_attn.bias_u"), f(p + "self_attn.bias_v")
        Ly.dw_w, Ly.dw_b = f(p + "conv.depthwise_conv.weight"), f(p + "conv.depthwise_conv.bias", zeros)
        Ly.bn_g, Ly.bn_b = f(p + "conv.norm.weight", ones), f(p + "conv.norm.bias", zeros)
        Ly.bn_mean, Ly.bn_var = f(p + "conv.norm.running_mean", zeros), f(p + "conv.norm.running_var", ones)
        for j, nm in enumerate(("norm_feed_forward1", "norm_self_att", "norm_conv", "norm_feed_forward2", "norm_out")):
            Ly.ln_g[j] = f(p + nm + ".weight", ones)
            Ly.ln_b[j] = f(p + nm + ".bias", zeros)
    sp = "encoder.subsampling."
    C = cfg["sub_channels"]
    zc = np.zeros(C, np.float32)
    W = _EncWeights(c0_w=f(sp + "layers.0.weight"), c0_b=f(sp + "layers.0.bias", zc),
                    dw2_w=f(sp + "layers.2.weight"), dw2_b=f(sp + "layers.2.bias", zc),
                    dw5_w=f(sp + "layers.5.weight"), dw5_b=f(sp + "layers.5.bias", zc),
                    pw3_b=f(sp + "layers.3.bias", zc), pw6_b=f(sp + "layers.6.bias", zc),
                    lin_b=f(sp + "linear.bias", zeros), pw3=q(sp + "layers.3.weight"), pw6=q(sp + "layers.6.weight"),
                    lin=q(sp + "linear.weight"), layers=layers)
    keep.append(layers)
    return keep, c, W


# ------------------------------------------------------------ Kokoro convs
def _leaky(x: np.ndarray, slope: float) -> np.ndarray:
    return np.where(x >= 0, x, x * slope)


def conv1d_ref(x, w, bias=None, stride: int = 1, padding: int = 0, dilation: int = 1, x_leaky: float = 1.0):
    """Conv1d of one NCW sequence in float64 (candle Tensor::conv1d as the
    Kokoro decoder calls it, src/kokoro/decoder.rs:154-773; the Triton conv1d_k
    / im2col_conv1d of kernels/kokoro_kernels.py:182,426):
    y[co, t] = bias[co] + sum_{ci, j} w[co, ci, j] * leaky(x)[ci, t*stride - padding + j*dilation],
    zero padding.  x [C_in, T_in], w [C_out, C_in, K] -> [C_out, T_out]."""
    x = _leaky(np.asarray(x, np.float64), x_leaky)
    w = np.asarray(w, np.float64)
    c_in, t_in = x.shape
    c_out, _, k = w.shape
    t_out = (t_in + 2 * padding - dilation * (k - 1) - 1) // stride + 1
    xp = np.zeros((c_in, t_in + 2 * padding + stride), np.float64)
    xp[:, padding:padding + t_in] = x
    cols = np.stack([xp[:, j * dilation: j * dilation + (t_out - 1) * stride + 1: stride] for j in range(k)], axis=1)
    y = np.einsum("oik,ikt->ot", w, cols)
    if bias is not None:
        y = y + np.asarray(bias, np.float64)[:, None]
    return y


def conv_transpose1d_ref(x, w, bias=None, stride: int = 1, padding: int = 0, output_padding: int = 0,
                         x_leaky: float = 1.0):
    """ConvTranspose1d (groups 1) of one NCW sequence in float64 (candle
    Tensor::conv_transpose1d, the generator upsampling of src/kokoro/
    decoder.rs:432-470,752): every input frame ti adds w[ci, co, :] * x[ci, ti]
    at output frames ti*stride - padding + j.  x [C_in, T_in], w [C_in, C_out, K]
    -> [C_out, (T_in - 1)*stride - 2*padding + K + output_padding]."""
    x = _leaky(np.asarray(x, np.float64), x_leaky)
    w = np.asarray(w, np.float64)
    c_in, t_in = x.shape
    _, c_out, k = w.shape
    t_out = (t_in - 1) * stride - 2 * padding + k + output_padding
    full = np.zeros((c_out, (t_in - 1) * stride + k + output_padding), np.float64)
    contrib = np.einsum("it,iok->tok", x, w)  # [T_in, C_out, K]
    for ti in range(t_in):
        full[:, ti * stride: ti * stride + k] += contrib[ti]
    y = full[:, padding: padding + t_out]
    if bias is not None:
        y = y + np.asarray(bias, np.float64)[:, None]
    return y
