"""Kokoro conv1d / conv_transpose1d on the B200 library (C ABI nq_conv*).

Mirrors the conv entries of ``KokoroGpuBackend`` (src/kokoro/gpu_backend.rs:
59-110: ``conv1d``, ``conv1d_k``, ``conv1d_lrelu001``, ``conv_transpose1d``,
``conv_transpose1d_lrelu``; Triton kernels ``conv1d_k`` and ``im2col_conv1d``,
kernels/kokoro_kernels.py:182,426) for one sequence in NCW layout: x is
[C_in, T_in], the output [C_out, T_out].  A conv1d weight is a ``QWeight`` of
the GGUF 2-D form [C_out, C_in * K] (Q8_0, or kept at bf16 precision when
C_in * K is not a multiple of 32); a conv_transpose1d weight comes from its
[C_in, C_out, K] values (``ConvTransposeWeight``).  The library lowers both
to its tensor-core GEMMs (im2col / col2im around the GEMM).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np
import torch

from . import lib as _l
from .fast_matmul import MatMulError, QWeight, _dtype_code, _stream_ptr

_P = ctypes.c_void_p


def conv1d_out_len(t_in: int, k: int, stride: int = 1, padding: int = 0, dilation: int = 1) -> int:
    t = int(_l.load().nq_conv1d_out_len(t_in, k, stride, padding, dilation))
    if t < 0:
        raise MatMulError(f"conv1d of {t_in} frames, kernel {k}, stride {stride}, padding {padding}: no output")
    return t


def conv_transpose1d_out_len(t_in: int, k: int, stride: int, padding: int = 0, output_padding: int = 0) -> int:
    t = int(_l.load().nq_conv_transpose1d_out_len(t_in, k, stride, padding, output_padding))
    if t < 0:
        raise MatMulError("conv_transpose1d: no output frames")
    return t


def _check_x(x: torch.Tensor) -> None:
    if x.dim() != 2 or x.stride(1) != 1 or not x.is_cuda:
        raise MatMulError("x must be a CUDA tensor [C_in, T_in] with unit time stride")


def conv1d(x: torch.Tensor, w: QWeight, bias: Optional[torch.Tensor], k: int, stride: int = 1, padding: int = 0,
           dilation: int = 1, x_leaky: float = 1.0, epilogue: int = _l.NQ_EPI_NONE, out: Optional[torch.Tensor] = None,
           out_dtype: Optional[torch.dtype] = None, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """y[co, t] = act(bias[co] + sum_{ci, j} W[co, ci*k + j] * leaky(x[ci, t*stride - padding + j*dilation]))."""
    _check_x(x)
    c_in, t_in = x.shape
    t_out = conv1d_out_len(t_in, k, stride, padding, dilation)
    if out is None:
        out = torch.empty((w.n, t_out), device=x.device, dtype=out_dtype or x.dtype)
    _l.check(_l.load().nq_conv1d(w.handle, x.data_ptr(), _dtype_code(x), c_in, t_in, x.stride(0), k, stride, padding,
                                 dilation, float(x_leaky), bias.data_ptr() if bias is not None else None, epilogue,
                                 out.data_ptr(), _dtype_code(out), out.stride(0), _stream_ptr(stream)))
    return out


def conv1d_lrelu001(x, w, bias, k, stride=1, padding=0, dilation=1, **kw) -> torch.Tensor:
    """leaky_relu(0.01) on the input, then conv1d (KokoroGpuBackend::conv1d_lrelu001)."""
    return conv1d(x, w, bias, k, stride, padding, dilation, x_leaky=0.01, **kw)


class ConvTransposeWeight(QWeight):
    """A conv_transpose1d weight: [C_in, C_out, K] values stored transposed as
    a bf16-only GEMM weight [C_out * K, C_in]."""

    @classmethod
    def from_f32(cls, w: np.ndarray, device: int = 0) -> "ConvTransposeWeight":
        cls._ensure(device)
        w = np.ascontiguousarray(w, dtype=np.float32)
        if w.ndim != 3:
            raise MatMulError("conv_transpose1d weight must be [C_in, C_out, K]")
        c_in, c_out, k = w.shape
        h = _P()
        _l.check(_l.load().nq_conv_transpose1d_weight(w.ctypes.data, c_in, c_out, k, ctypes.byref(h)))
        obj = cls(h.value, c_out * k, c_in, 0, device)
        obj.kernel = k
        return obj


def conv_transpose1d(x: torch.Tensor, w: ConvTransposeWeight, bias: Optional[torch.Tensor], stride: int,
                     padding: int = 0, output_padding: int = 0, x_leaky: float = 1.0,
                     epilogue: int = _l.NQ_EPI_NONE, out: Optional[torch.Tensor] = None,
                     out_dtype: Optional[torch.dtype] = None,
                     stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """y[co, t] = act(bias[co] + sum over (ci, ti, j) with t = ti*stride - padding + j of W[ci, co, j] * x[ci, ti])."""
    _check_x(x)
    c_in, t_in = x.shape
    k = w.kernel
    t_out = conv_transpose1d_out_len(t_in, k, stride, padding, output_padding)
    if out is None:
        out = torch.empty((w.n // k, t_out), device=x.device, dtype=out_dtype or x.dtype)
    _l.check(_l.load().nq_conv_transpose1d(w.handle, x.data_ptr(), _dtype_code(x), c_in, t_in, x.stride(0), k, stride,
                                           padding, output_padding, float(x_leaky),
                                           bias.data_ptr() if bias is not None else None, epilogue, out.data_ptr(),
                                           _dtype_code(out), out.stride(0), _stream_ptr(stream)))
    return out


def conv_transpose1d_lrelu(x, w, bias, stride, padding=0, output_padding=0, **kw) -> torch.Tensor:
    """leaky_relu(0.1) on the input, then conv_transpose1d (conv_transpose1d_lrelu)."""
    return conv_transpose1d(x, w, bias, stride, padding, output_padding, x_leaky=0.1, **kw)
