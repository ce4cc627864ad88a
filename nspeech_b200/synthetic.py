"""Seeded random-init weights and inputs for the Parakeet FastConformer encoder.

No checkpoint can be downloaded here, so benchmarks and tests use random
weights of the reference architecture (FastConformerConfig defaults of the
Parakeet TDT 0.6B model: d_model 1024, 8 heads, 24 layers, FFN x4, conv
kernel 9, 256 subsampling channels, 128 mel bins) under the tensor names of
``remap_nemo_tensor_name`` (src/parakeet/transducer.rs:1279-1302).

Every rank-2 linear and pointwise convolution is a Q8_0 matrix ("q8" in the
returned spec); the generator returns f32 values, which the library quantizes
with ggml semantics (or a caller quantizes first and passes Q8_0 blocks).
"""
from __future__ import annotations

from dataclasses import dataclass, asdict
from typing import Dict, Tuple

import numpy as np


@dataclass
class EncoderSpec:
    feat_in: int = 128
    d_model: int = 1024
    n_heads: int = 8
    ff_mult: int = 4
    n_layers: int = 24
    conv_kernel: int = 9
    sub_channels: int = 256
    scale_input: int = 1

    def as_dict(self) -> dict:
        return asdict(self)


PARAKEET_TDT_0_6B = EncoderSpec()


Init = Tuple[str, float]  # ("normal", std) | ("one_plus", std) | ("zeros", 0) | ("ones", 0)


def tensor_shapes(spec: EncoderSpec) -> Dict[str, Tuple[Tuple[int, ...], bool, Init]]:
    """name -> (shape, is_q8_matrix, init) for every encoder tensor."""
    d, C, K = spec.d_model, spec.sub_channels, spec.conv_kernel
    ff = d * spec.ff_mult
    hd = d // spec.n_heads
    out: Dict[str, Tuple[Tuple[int, ...], bool, Init]] = {}
    N = lambda std: ("normal", float(std))  # noqa: E731
    sp = "encoder.subsampling."
    out[sp + "layers.0.weight"] = ((C, 1, 3, 3), False, N(0.3))
    out[sp + "layers.0.bias"] = ((C,), False, N(0.05))
    out[sp + "layers.2.weight"] = ((C, 1, 3, 3), False, N(0.3))
    out[sp + "layers.2.bias"] = ((C,), False, N(0.05))
    out[sp + "layers.3.weight"] = ((C, C), True, N(1.0 / np.sqrt(C)))
    out[sp + "layers.3.bias"] = ((C,), False, N(0.05))
    out[sp + "layers.5.weight"] = ((C, 1, 3, 3), False, N(0.3))
    out[sp + "layers.5.bias"] = ((C,), False, N(0.05))
    out[sp + "layers.6.weight"] = ((C, C), True, N(1.0 / np.sqrt(C)))
    out[sp + "layers.6.bias"] = ((C,), False, N(0.05))
    flat = C * (spec.feat_in // 8)
    out[sp + "linear.weight"] = ((d, flat), True, N(0.02))
    out[sp + "linear.bias"] = ((d,), False, N(0.01))
    for i in range(spec.n_layers):
        p = f"encoder.layers.{i}."
        for ffn in ("feed_forward1", "feed_forward2"):
            out[p + ffn + ".linear1.weight"] = ((ff, d), True, N(0.02))
            out[p + ffn + ".linear1.bias"] = ((ff,), False, N(0.01))
            out[p + ffn + ".linear2.weight"] = ((d, ff), True, N(0.02))
            out[p + ffn + ".linear2.bias"] = ((d,), False, N(0.01))
        for proj in ("q_proj", "k_proj", "v_proj", "o_proj"):
            out[p + f"self_attn.{proj}.weight"] = ((d, d), True, N(0.02))
            out[p + f"self_attn.{proj}.bias"] = ((d,), False, N(0.01))
        out[p + "self_attn.relative_k_proj.weight"] = ((d, d), True, N(0.02))
        out[p + "self_attn.bias_u"] = ((spec.n_heads, hd), False, N(0.02))
        out[p + "self_attn.bias_v"] = ((spec.n_heads, hd), False, N(0.02))
        out[p + "conv.pointwise_conv1.weight"] = ((2 * d, d), True, N(0.02))
        out[p + "conv.pointwise_conv1.bias"] = ((2 * d,), False, N(0.01))
        out[p + "conv.depthwise_conv.weight"] = ((d, 1, K), False, N(0.1))
        out[p + "conv.depthwise_conv.bias"] = ((d,), False, N(0.01))
        out[p + "conv.pointwise_conv2.weight"] = ((d, d), True, N(0.02))
        out[p + "conv.pointwise_conv2.bias"] = ((d,), False, N(0.01))
        for nm in ("norm_feed_forward1", "norm_self_att", "norm_conv", "norm_feed_forward2", "norm_out"):
            out[p + nm + ".weight"] = ((d,), False, ("one_plus", 0.1))
            out[p + nm + ".bias"] = ((d,), False, N(0.02))
        out[p + "conv.norm.weight"] = ((d,), False, ("one_plus", 0.1))
        out[p + "conv.norm.bias"] = ((d,), False, N(0.02))
        out[p + "conv.norm.running_mean"] = ((d,), False, ("zeros", 0.0))
        out[p + "conv.norm.running_var"] = ((d,), False, ("ones", 0.0))
    return out


def encoder_tensors(spec: EncoderSpec, seed: int = 1) -> Dict[str, Tuple[np.ndarray, bool]]:
    """name -> (f32 array, is_q8_matrix), seeded (numpy PCG64)."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, (shape, q8, (kind, std)) in tensor_shapes(spec).items():
        if kind == "ones":
            a = np.ones(shape, np.float32)
        elif kind == "zeros":
            a = np.zeros(shape, np.float32)
        elif kind == "one_plus":
            a = (1.0 + std * rng.standard_normal(shape, dtype=np.float32)).astype(np.float32)
        else:
            a = (std * rng.standard_normal(shape, dtype=np.float32)).astype(np.float32)
        out[name] = (a, q8)
    return out


def segment_lengths_s(n: int = 1024, lo: float = 2.0, hi: float = 30.0, seed: int = 4) -> np.ndarray:
    """Config-5 VAD segment durations in seconds, uniform in [lo, hi]."""
    return np.random.default_rng(seed).uniform(lo, hi, n)


def mel_frames(seconds: float, hop_s: float = 0.01) -> int:
    """10 ms hop log-mel frames of a segment."""
    return max(1, int(round(seconds / hop_s)))
