"""Time Q8_0 linear shapes on the GPU through the C ABI (nq_linear).

    python -m nspeech_b200.gemm_bench --shape 12000x1024x4096 --shape 1x640x640 [--x bf16] [--iters 20]

Each shape is M x K x N (tokens x in-features x out-features).  Random Q8_0
weights are rotated over enough copies to exceed the 126 MB L2, so weight
reads come from HBM; times are CUDA events over `iters` back-to-back calls
(host launch overhead included for small shapes).  Prints one JSON line per
shape with TFLOP/s and algorithmic GB/s (N*K*34/32 + M*K*sx + M*N*sy bytes).
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from . import lib
from .fast_matmul import QWeight


def _weights(n: int, k: int, copies: int, rng) -> list:
    out = []
    for _ in range(copies):
        q = rng.integers(-127, 128, size=(n, k // 32, 34), dtype=np.int64).astype(np.uint8)
        d = (rng.random((n, k // 32)) * 1e-3 + 1e-4).astype(np.float16)
        q[:, :, :2] = d.view(np.uint8).reshape(n, k // 32, 2)
        out.append(QWeight.from_q8_0(q.reshape(n, -1), n, k))
    return out


def time_shape(m: int, k: int, n: int, x_dtype=torch.bfloat16, y_dtype=torch.bfloat16, iters: int = 20,
               epilogue: int = lib.NQ_EPI_NONE, seed: int = 0) -> dict:
    rng = np.random.default_rng(seed)
    wbytes = n * k * 34 / 32
    copies = int(min(32, max(1, np.ceil(300e6 / wbytes))))
    ws = _weights(n, k, copies, rng)
    x = torch.randn(m, k, device="cuda").to(x_dtype)
    y = torch.empty(m, n, device="cuda", dtype=y_dtype)
    for i in range(3):
        ws[i % copies].linear(x, out=y, epilogue=epilogue)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(iters):
        ws[i % copies].linear(x, out=y, epilogue=epilogue)
    e1.record()
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / iters / 1e3
    if lib.status() != 0:
        raise RuntimeError("device status reported a timeout")
    byts = wbytes + m * k * x.element_size() + m * n * y.element_size()
    return {"m": m, "k": k, "n": n, "x": str(x_dtype).split(".")[-1], "us": round(t * 1e6, 2),
            "tflops": round(2 * m * n * k / t / 1e12, 1), "gbs": round(byts / t / 1e9, 1)}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", action="append", required=True, help="MxKxN")
    ap.add_argument("--x", choices=["bf16", "f32"], default="bf16")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--device", type=int, default=0)
    a = ap.parse_args()
    torch.cuda.set_device(a.device)
    lib.init(a.device)
    xd = torch.bfloat16 if a.x == "bf16" else torch.float32
    for s in a.shape:
        m, k, n = (int(v) for v in s.lower().split("x"))
        print(json.dumps(time_shape(m, k, n, x_dtype=xd, iters=a.iters)), flush=True)


if __name__ == "__main__":
    main()
