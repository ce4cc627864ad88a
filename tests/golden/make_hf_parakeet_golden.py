"""Golden outputs of an independent FastConformer implementation for the
encoder oracle (``oracle/encoder_oracle.c``).

Run from the repository root:  python tests/golden/make_hf_parakeet_golden.py

The reference's encoder (src/parakeet/fast_conformer.rs:69-1104, dropbox/
nspeech) is a Rust port of NVIDIA NeMo's FastConformer; the reference cannot
be built here.  transformers 5.5.0 ships a separate port of the same model,
``transformers.models.parakeet.modeling_parakeet.ParakeetEncoder``.  This
script loads the seeded synthetic weights of ``nspeech_b200.synthetic``
(Q8_0-quantized, then dequantized exactly: the f32 values candle's Linear
multiplies on the reference's Linux path, src/parakeet/transducer.rs:
1841-1865) into that module, runs it in float64 on the CPU and stores its
output.  tests/test_oracle_vs_parakeet.py checks the oracle against the
stored outputs (and against a live transformers run when it is importable).

Per case the fixture holds the HF output [T3, d_model] (f64 -> f32); the
weights and the mel input are regenerated from their seeds (CASES).
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, spec kwargs, weight seed, mel frames, mel seed)
CASES = [
    ("d256_h4_l2", dict(feat_in=128, d_model=256, n_heads=4, n_layers=2, sub_channels=64), 21, 400, 31),
    ("d512_h8_l1_f80", dict(feat_in=80, d_model=512, n_heads=8, n_layers=1, sub_channels=32), 22, 333, 32),
]


def hf_encoder(spec, tensors_q):
    """transformers ParakeetEncoder (eval, float64) holding the given weights.

    tensors_q: name -> (f32 array, is_q8) with Q8_0 matrices already replaced by
    their exact dequantization."""
    import torch
    from transformers.models.parakeet.configuration_parakeet import ParakeetEncoderConfig
    from transformers.models.parakeet.modeling_parakeet import ParakeetEncoder

    cfg = ParakeetEncoderConfig(hidden_size=spec.d_model, num_hidden_layers=spec.n_layers,
                                num_attention_heads=spec.n_heads, intermediate_size=spec.d_model * spec.ff_mult,
                                conv_kernel_size=spec.conv_kernel, subsampling_conv_channels=spec.sub_channels,
                                num_mel_bins=spec.feat_in, scale_input=bool(spec.scale_input), dropout=0.0,
                                dropout_positions=0.0, layerdrop=0.0, activation_dropout=0.0, attention_dropout=0.0)
    model = ParakeetEncoder(cfg).double().eval()
    sd = model.state_dict()
    new = {}
    for name, ref in sd.items():
        if name.endswith("num_batches_tracked"):
            new[name] = ref
            continue
        src = tensors_q["encoder." + name]
        new[name] = torch.from_numpy(np.asarray(src, np.float64).reshape(tuple(ref.shape)))
    missing = set(sd) - set(new)
    assert not missing, missing
    model.load_state_dict(new, strict=True)
    return model


def dequantized_tensors(spec, seed):
    from nspeech_b200 import synthetic as S
    from oracle import oracle as O
    out, blocks = {}, {}
    for name, (v, q8) in S.encoder_tensors(spec, seed).items():
        if q8:
            m = v.reshape(v.shape[0], -1)
            q = O.quantize_q8_0(m)
            blocks[name] = q
            out[name] = O.dequant_q8_0(q, m.shape[0], m.shape[1]).reshape(v.shape)
        else:
            out[name] = v
            blocks[name] = v
    return out, blocks


def hf_forward(spec, seed, mel):
    import torch
    deq, _ = dequantized_tensors(spec, seed)
    model = hf_encoder(spec, deq)
    with torch.no_grad():
        y = model(torch.from_numpy(mel.astype(np.float64))[None]).last_hidden_state[0]
    return y.numpy()


def main() -> None:
    import transformers
    from nspeech_b200 import synthetic as S
    from oracle import oracle as O
    out = {"transformers_version": np.array(transformers.__version__)}
    for name, kw, wseed, frames, mseed in CASES:
        spec = S.EncoderSpec(**kw)
        mel = O.normal(mseed, (frames, spec.feat_in))
        y = hf_forward(spec, wseed, mel)
        out[f"{name}_hf"] = y.astype(np.float32)
        print(name, y.shape, float(np.abs(y).max()))
    np.savez_compressed(os.path.join(HERE, "encoder_hf_parakeet.npz"), **out)


if __name__ == "__main__":
    main()
