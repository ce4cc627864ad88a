"""Decode chain: the dependent M = 1 projections of one decoder token as a
single cooperative launch (``nq_chain_*`` in include/nq8.h).

The reference runs a Moonshine decoder token as a sequence of separate
backend calls -- ``DecoderBackend::gemv`` for the projections and
``gemv_resadd_ln`` for the residual add + LayerNorm after each block
(src/moonshine/decoder.rs, src/moonshine/gpu_decoder.rs:67-70) -- each one
its own GPU dispatch.  ``DecodeChain`` records the same calls once, binding
their buffers, and ``run()`` executes all of them in one persistent kernel.
Every step computes the corresponding ``QWeight.linear`` /
``QWeight.gemv_resadd_ln`` call with one row (the same bf16 weight products,
f32 sums in another fixed order, deterministic).
"""
from __future__ import annotations

import ctypes
from typing import List, Optional

import torch

from . import lib as _l
from .fast_matmul import MatMulError, QWeight, _dtype_code, _stream_ptr


def _vec(t: torch.Tensor, name: str, n: int, dtypes) -> None:
    if not t.is_cuda or t.dtype not in dtypes:
        raise MatMulError(f"{name} must be a CUDA tensor of {', '.join(str(d) for d in dtypes)}")
    if t.numel() < n or not t.is_contiguous():
        raise MatMulError(f"{name} must be contiguous with at least {n} elements")


class DecodeChain:
    """Recorded M = 1 GEMV steps of a decoder token, run as one launch.

    Steps bind tensors by address: keep them allocated (the chain holds
    references) and write new inputs into them between runs."""

    def __init__(self, device: int = 0):
        QWeight._ensure(device)
        h = ctypes.c_void_p()
        _l.check(_l.load().nq_chain_create(ctypes.byref(h)))
        self._h = h.value
        self._keep: List[object] = []

    def linear(self, w: QWeight, x: torch.Tensor, out: torch.Tensor, bias: Optional[torch.Tensor] = None,
               epilogue: int = _l.NQ_EPI_NONE) -> torch.Tensor:
        """out = act(w . x + bias) for one bf16 row x [K] (nq_chain_linear)."""
        glu = epilogue in (_l.NQ_EPI_GLU_SIGMOID, _l.NQ_EPI_GLU_SILU)
        _vec(x, "x", w.k, (torch.bfloat16,))
        _vec(out, "out", w.n // 2 if glu else w.n, (torch.float32, torch.bfloat16))
        if bias is not None:
            _vec(bias, "bias", w.n, (torch.float32,))
        _l.check(_l.load().nq_chain_linear(self._h, w.handle, x.data_ptr(),
                                           bias.data_ptr() if bias is not None else None, epilogue,
                                           out.data_ptr(), _dtype_code(out)))
        self._keep += [w, x, out, bias]
        return out

    def gemv_resadd_ln(self, w: QWeight, x: torch.Tensor, residual_in: torch.Tensor, gamma: torch.Tensor,
                       beta: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None, eps: float = 1e-5,
                       residual_out: Optional[torch.Tensor] = None,
                       out: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
        """residual_out = residual_in + w . x + bias; out = LayerNorm(residual_out)
        * gamma + beta in bf16 (nq_chain_gemv_resadd_ln).  residual_out may be
        residual_in; out may be None when nothing reads it."""
        _vec(x, "x", w.k, (torch.bfloat16,))
        for name, t in (("residual_in", residual_in), ("gamma", gamma), ("beta", beta), ("bias", bias)):
            if t is not None:
                _vec(t, name, w.n, (torch.float32,))
        if residual_out is None:
            residual_out = residual_in
        _vec(residual_out, "residual_out", w.n, (torch.float32,))
        if out is not None:
            _vec(out, "out", w.n, (torch.bfloat16,))
        _l.check(_l.load().nq_chain_gemv_resadd_ln(
            self._h, w.handle, x.data_ptr(), bias.data_ptr() if bias is not None else None, residual_in.data_ptr(),
            residual_out.data_ptr(), gamma.data_ptr(), beta.data_ptr() if beta is not None else None, float(eps),
            out.data_ptr() if out is not None else None))
        self._keep += [w, x, residual_in, residual_out, gamma, beta, bias, out]
        return out

    @property
    def steps(self) -> int:
        return int(_l.load().nq_chain_steps(self._h))

    def run(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        """One launch of every recorded step, in order, on `stream`."""
        _l.check(_l.load().nq_chain_run(self._h, _stream_ptr(stream)))

    def close(self) -> None:
        if self._h:
            _l.load().nq_chain_free(self._h)
            self._h = None
            self._keep = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
