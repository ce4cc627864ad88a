"""Time Q8_0 linear shapes on the GPU through the C ABI (nq_linear).

    python -m nspeech_b200.gemm_bench --shape 12000x1024x4096 --shape 1x640x640 [--x bf16] [--iters 20]
    python -m nspeech_b200.gemm_bench --cfg1-sweep [--graph]

Each shape is M x K x N (tokens x in-features x out-features).  Random Q8_0
weights are rotated over enough copies to exceed the 126 MB L2, so weight
reads come from HBM; times are CUDA events over `iters` back-to-back calls
(host launch overhead included for small shapes), or with --graph the
device time per call of a CUDA graph of those calls.  Prints one JSON line
per shape with TFLOP/s and algorithmic GB/s (N*K*34/32 + M*K*sx + M*N*sy
bytes), and the fraction of the bound that applies (HBM for M <= 125, where
the arithmetic intensity is below the ridge; tensor otherwise) against the
measured peaks in MEASURED_PEAKS.json when present.

--cfg1-sweep: the configs[0] block (K -> N: 1024->4096, 4096->1024,
1024->3072, 1024->1024, 1024->2048, 1024->1024) at M in {1, 2, 4, 8, 16,
125, 1024, 2048, 4096, 12000}; f32 activations in and out, or
bf16 with --sweep-dtype bf16 (the encoder's activations); --sweep-m picks a
subset of M.  --keep-bf16 gives every weight a kept bf16 copy, as the
encoder does, so M >= 128 GEMMs skip the per-call dequantize pass.
"""
from __future__ import annotations

import argparse
import json
import os

import numpy as np
import torch

from . import lib
from .fast_matmul import QWeight


def _weights(n: int, k: int, copies: int, rng, keep_bf16: bool = False) -> list:
    out = []
    for _ in range(copies):
        q = rng.integers(-127, 128, size=(n, k // 32, 34), dtype=np.int64).astype(np.uint8)
        d = (rng.random((n, k // 32)) * 1e-3 + 1e-4).astype(np.float16)
        q[:, :, :2] = d.view(np.uint8).reshape(n, k // 32, 2)
        w = QWeight.from_q8_0(q.reshape(n, -1), n, k)
        out.append(w.keep_bf16() if keep_bf16 else w)
    return out


CFG1_KN = [(1024, 4096), (4096, 1024), (1024, 3072), (1024, 1024), (1024, 2048), (1024, 1024)]
CFG1_M = [1, 2, 4, 8, 16, 125, 1024, 2048, 4096, 12000]


def _peaks() -> dict:
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def time_shape(m: int, k: int, n: int, x_dtype=torch.bfloat16, y_dtype=torch.bfloat16, iters: int = 20,
               epilogue: int = lib.NQ_EPI_NONE, seed: int = 0, graph: bool = False, keep_bf16: bool = False) -> dict:
    rng = np.random.default_rng(seed)
    wbytes = n * k * 34 / 32
    # weights stream past L2 (the kept bf16 copy, when kept, is what the GEMM reads)
    copies = int(min(32, max(1, np.ceil(300e6 / (n * k * 2 if keep_bf16 else wbytes)))))
    ws = _weights(n, k, copies, rng, keep_bf16)
    x = torch.randn(m, k, device="cuda").to(x_dtype)
    y = torch.empty(m, n, device="cuda", dtype=y_dtype)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i in range(max(3, copies)):  # also sizes the stream's workspace before any capture
            ws[i % copies].linear(x, out=y, epilogue=epilogue)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(iters):
                ws[i % copies].linear(x, out=y, epilogue=epilogue)
        g.replay()
        torch.cuda.synchronize()
        reps = 5
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / (reps * iters) / 1e3
        del g
    else:
        e0.record()
        for i in range(iters):
            ws[i % copies].linear(x, out=y, epilogue=epilogue)
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / iters / 1e3
    if lib.status() != 0:
        raise RuntimeError("device status reported a timeout")
    byts = wbytes + m * k * x.element_size() + m * n * y.element_size()
    pk = _peaks()
    tflops, gbs = 2 * m * n * k / t / 1e12, byts / t / 1e9
    bound = "hbm" if m <= 125 else "tensor"
    frac = gbs / pk["hbm_gbs"] if bound == "hbm" else tflops / pk["bf16_tflops"]
    return {"m": m, "k": k, "n": n, "x": str(x_dtype).split(".")[-1], "y": str(y_dtype).split(".")[-1],
            "us": round(t * 1e6, 2), "tflops": round(tflops, 1), "gbs": round(gbs, 1), "bound": bound,
            "frac": round(frac, 3), "peak_source": pk["source"], "timing": "graph" if graph else "calls",
            "weights": "kept bf16 copy" if keep_bf16 else "q8_0"}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", action="append", default=[], help="MxKxN")
    ap.add_argument("--cfg1-sweep", action="store_true", help="the configs[0] block over the M sweep")
    ap.add_argument("--sweep-dtype", choices=["f32", "bf16"], default="f32",
                    help="activations in and out for --cfg1-sweep (f32: configs[0]; bf16: the encoder's)")
    ap.add_argument("--x", choices=["bf16", "f32"], default="bf16")
    ap.add_argument("--y", choices=["bf16", "f32"], default="bf16")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--graph", action="store_true", help="time a CUDA graph of the calls (device time)")
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--keep-bf16", action="store_true",
                    help="give every weight a kept bf16 copy (nq_weight_keep_bf16), as the encoder does")
    ap.add_argument("--sweep-m", default="", help="comma-separated subset of the sweep's M values")
    ap.add_argument("--unit-tokens", default="0",
                    help="comma-separated GEMM unit widths to time each shape with (nq_set_gemm_unit_tokens; 0 = default)")
    a = ap.parse_args()
    torch.cuda.set_device(a.device)
    lib.init(a.device)
    dt = {"bf16": torch.bfloat16, "f32": torch.float32}
    jobs = [(tuple(int(v) for v in s.lower().split("x")), dt[a.x], dt[a.y]) for s in a.shape]
    if a.cfg1_sweep:
        sd = dt[a.sweep_dtype]
        ms = [int(v) for v in a.sweep_m.split(",")] if a.sweep_m else CFG1_M
        jobs += [((m, k, n), sd, sd) for m in ms for k, n in CFG1_KN]
    if not jobs:
        ap.error("give --shape or --cfg1-sweep")
    units = [int(v) for v in a.unit_tokens.split(",")]
    for (m, k, n), xd, yd in jobs:
        for u in units:
            lib.check(lib.load().nq_set_gemm_unit_tokens(u))
            r = time_shape(m, k, n, x_dtype=xd, y_dtype=yd, iters=a.iters, graph=a.graph, keep_bf16=a.keep_bf16)
            r["unit_tokens"] = u
            print(json.dumps(r), flush=True)
    lib.check(lib.load().nq_set_gemm_unit_tokens(0))


if __name__ == "__main__":
    main()
