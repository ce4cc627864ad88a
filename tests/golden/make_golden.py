"""Generate the committed golden fixtures under tests/golden/.

Run from the repository root:  python tests/golden/make_golden.py

Two fixture families:

* ``q8_0_ggufpy.npz`` -- Q8_0 quantization goldens produced by gguf-py 0.19.0
  (``gguf.quants.quantize(..., GGMLQuantizationType.Q8_0)``, quants.py:378-401),
  the bit-exact Python restatement of ggml-quants.c ``quantize_row_q8_0_ref``
  that candle's ``QTensor::quantize`` follows (used by the reference at
  tools/quantize-parakeet/src/main.rs:108).  Includes hand-built known-answer
  blocks (all 127, all zero, +-0.5 rounding ties, f16-subnormal scale,
  negative maximum) and seeded N(0, 0.02) weights.
* ``matmul_small.npz`` -- seeded small matmul cases with the CPU oracle's three
  semantics (fbgemm-bf16, QTiled, f64 exact), pinning the oracle against
  regressions and giving the GPU tests ready-made expected outputs.

gguf-py is only needed to (re)generate; the tests read the .npz files.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def kat_blocks() -> np.ndarray:
    rows = []
    rows.append(np.full(32, 127.0, np.float32))                      # d = 1, q = 127
    rows.append(np.zeros(32, np.float32))                            # d = 0, q = 0
    tie = np.zeros(32, np.float32)
    tie[0] = 127.0                                                   # d = 1, id = 1
    tie[1:9] = [0.5, -0.5, 1.5, -1.5, 2.5, -2.5, 126.5, -126.5]      # half away from zero
    rows.append(tie)
    rows.append(np.linspace(-1e-4, 1e-4, 32).astype(np.float32))     # subnormal f16 d
    neg = np.linspace(-3.0, 2.0, 32).astype(np.float32)               # negative maximum
    rows.append(neg)
    big = np.linspace(-60000.0, 65000.0, 32).astype(np.float32)       # large magnitude
    rows.append(big)
    return np.stack(rows)


def main() -> None:
    from gguf.constants import GGMLQuantizationType
    from gguf.quants import quantize

    kat = kat_blocks()
    rnd = O.normal(20240, (48, 256), 0.0, 0.02)
    wide = O.normal(20241, (8, 4096), 0.0, 1.0)
    np.savez_compressed(
        os.path.join(HERE, "q8_0_ggufpy.npz"),
        kat_x=kat,
        kat_q=quantize(kat, GGMLQuantizationType.Q8_0),
        rnd_x=rnd,
        rnd_q=quantize(rnd, GGMLQuantizationType.Q8_0),
        wide_x=wide,
        wide_q=quantize(wide, GGMLQuantizationType.Q8_0),
    )

    cases = {}
    # (m, n, k, seed): ragged and tiny shapes the GPU tests also use.
    for (m, n, k, seed) in [(1, 64, 64, 1), (3, 130, 96, 2), (17, 128, 256, 3), (33, 200, 160, 4),
                            (64, 256, 512, 5), (129, 96, 64, 6)]:
        x = O.normal(100 + seed, (m, k), 0.0, 1.0)
        w = O.normal(200 + seed, (n, k), 0.0, 0.02)
        q = O.quantize_q8_0(w)
        tag = f"m{m}_n{n}_k{k}"
        cases[f"{tag}_x"] = x
        cases[f"{tag}_q"] = q
        cases[f"{tag}_fbgemm"] = O.matmul_fbgemm_bf16(x, q, n)
        cases[f"{tag}_qtiled"] = O.matmul_qtiled(x, q, n)
        cases[f"{tag}_exact"] = O.matmul_exact(x, q, n)
    np.savez_compressed(os.path.join(HERE, "matmul_small.npz"), **cases)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
