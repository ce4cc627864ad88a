"""Parakeet FastConformer encoder on the B200 library (C ABI nq_encoder_*).

Mirrors ``FastConformerEncoder`` (src/parakeet/fast_conformer.rs:1040-1104)
and ``TransducerModel::run_encoder`` (src/parakeet/transducer.rs:387-404),
extended to batches of padded VAD segments.  The forward runs natively in
libnq8 (C++ host code, CUDA kernels); Python only passes pointers.
"""
from __future__ import annotations

import ctypes
import os
from typing import Dict, Optional, Sequence, Tuple

import numpy as np
import torch

from . import lib as _l
from .synthetic import EncoderSpec

_P = ctypes.c_void_p


def out_frames(t_mel: int) -> int:
    return int(_l.load().nq_encoder_out_frames(int(t_mel)))


class ParakeetEncoder:
    def __init__(self, spec: EncoderSpec = EncoderSpec(), device: int = 0):
        torch.cuda.set_device(device)
        _l.init(device)
        self.spec = spec
        self.device = device
        cfg = _l.EncoderConfig(**spec.as_dict())
        h = _P()
        _l.check(_l.load().nq_encoder_create(ctypes.byref(cfg), ctypes.byref(h)))
        self._h = h.value

    # ------------------------------------------------------------- weights
    def set_tensor(self, name: str, data: np.ndarray, q8_0_dims: Optional[Sequence[int]] = None) -> None:
        """F32 array (any tensor), or Q8_0 blocks (uint8) with their logical dims."""
        if q8_0_dims is not None:
            blob = np.ascontiguousarray(data, dtype=np.uint8)
            dims = list(q8_0_dims)
            gtype = 8
        else:
            blob = np.ascontiguousarray(data, dtype=np.float32)
            dims = list(blob.shape)
            gtype = 0
        d = (ctypes.c_int64 * len(dims))(*dims)
        _l.check(_l.load().nq_encoder_set_tensor(self._h, name.encode(), gtype, blob.ctypes.data, d, len(dims)))

    def load_tensors(self, tensors: Dict[str, Tuple[np.ndarray, bool]]) -> "ParakeetEncoder":
        for name, (arr, _q8) in tensors.items():
            self.set_tensor(name, arr)
        return self

    def load_gguf(self, path: str) -> "ParakeetEncoder":
        _l.check(_l.load().nq_encoder_load_gguf(self._h, os.fsencode(path)))
        return self

    def finalize(self) -> "ParakeetEncoder":
        _l.check(_l.load().nq_encoder_finalize(self._h))
        return self

    # ------------------------------------------------------------- forward
    def forward(self, mel: torch.Tensor, lengths: Optional[Sequence[int]] = None,
                out: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, list]:
        """mel: CUDA f32 [B, T_mel, feat_in] -> ([B, T, d_model] f32, encoder lengths)."""
        if mel.dim() != 3 or mel.dtype != torch.float32 or not mel.is_contiguous() or not mel.is_cuda:
            raise ValueError("mel must be a contiguous CUDA f32 tensor [B, T, F]")
        B, T, F = mel.shape
        if F != self.spec.feat_in:
            raise ValueError(f"mel has {F} bins, encoder expects {self.spec.feat_in}")
        To = out_frames(T)
        if out is None:
            out = torch.empty((B, To, self.spec.d_model), device=mel.device, dtype=torch.float32)
        lens = (ctypes.c_int32 * B)(*(lengths if lengths is not None else [T] * B))
        olens = (ctypes.c_int32 * B)()
        stream = torch.cuda.current_stream().cuda_stream
        _l.check(_l.load().nq_encoder_forward(self._h, mel.data_ptr(), lens, B, T, out.data_ptr(), olens, stream))
        return out, list(olens)

    __call__ = forward

    def forward_host(self, mel: np.ndarray, lengths: Optional[Sequence[int]] = None,
                     out: Optional[np.ndarray] = None, stream: int = 0) -> Tuple[np.ndarray, list]:
        """Host buffers in and out (copies on `stream`, synchronized on return)."""
        mel = np.ascontiguousarray(mel, dtype=np.float32)
        B, T, _ = mel.shape
        if out is None:
            out = np.empty((B, out_frames(T), self.spec.d_model), np.float32)
        lens = (ctypes.c_int32 * B)(*(lengths if lengths is not None else [T] * B))
        olens = (ctypes.c_int32 * B)()
        _l.check(_l.load().nq_encoder_forward_host(self._h, mel.ctypes.data, lens, B, T, out.ctypes.data, olens,
                                                   _P(stream)))
        return out, list(olens)

    def forward_host_async(self, mel: np.ndarray, lengths: Optional[Sequence[int]], out: np.ndarray,
                           stream: int = 0) -> list:
        """Queue a forward with pinned host buffers (mel in, out back); see wait()."""
        B, T, _ = mel.shape
        lens = (ctypes.c_int32 * B)(*(lengths if lengths is not None else [T] * B))
        olens = (ctypes.c_int32 * B)()
        _l.check(_l.load().nq_encoder_forward_host_async(self._h, mel.ctypes.data, lens, B, T, out.ctypes.data,
                                                         olens, _P(stream)))
        return list(olens)

    def wait(self) -> None:
        """Block until every queued forward_host_async output is in host memory."""
        _l.check(_l.load().nq_encoder_wait(self._h))

    def launch_count(self, batch: int, t_mel: int) -> int:
        return int(_l.load().nq_encoder_launch_count(self._h, batch, t_mel))

    def free(self) -> None:
        if self._h:
            _l.load().nq_encoder_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
