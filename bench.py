#!/usr/bin/env python
"""Parakeet FastConformer encoder RTFx on B200 through the nspeech Q8_0 path.

Workload (the metric's multi-GPU configuration): ONE job
of 1024 synthetic VAD segments with durations U[2, 30] s (seed 4), as 128-bin
log-mel N(0, 1) at a 10 ms hop (segment j's features from its own seed), through
the full 24-layer encoder (configs[1] architecture, random-init Q8_0 weights).
The job is cut into length buckets of <= 32 padded segments, and the buckets
are split over the ranks by greedy longest-processing-time on the estimated
bucket cost (nspeech_b200/shard.py): one process per GPU, no collective on the
data path, strong scaling.  One step = every bucket of this rank once.
`--shard weak` instead gives every rank its own 1024 segments (seed 4 + rank).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference] [--shard lpt|weak]
    python bench.py --gemv [--gemv-shapes MxKxN,...] [--gemv-plain CALLS]
    python bench.py --linear (--shape MxKxN ... | --cfg1-sweep) [--graph] [--keep-bf16] ...

Prints one JSON line (rank 0).  `value`: RTFx = audio seconds of all ranks /
max-over-ranks device time of K steps, inputs resident in HBM.  `e2e`: the
same through the public host-buffer entry point (H2D of the mel features and
D2H of the encoder output inside the timed region), over K steps.
`cpu_baseline` (N = 1): the CPU restatement of the reference's path
(oracle/encoder_oracle.c over oracle/fbgemm_cpu.c: weights packed to bf16 once,
f32 activations, AVX-512 FMA, OpenMP) on a stratified sample of the same
segments, at all host cores and at one core, plus the configs[0] linear set.
`--impl reference` times that CPU path on the same sample per step.

`--gemv` times the Q8_0 GEMV (M <= 16, the decode-step projections) alone:
per shape, a CUDA graph of back-to-back nq_linear calls over enough weight
copies to stream past L2, reported as device time per call and HBM GB/s
(weight + x + y bytes) against the measured peak, and the configs[2] decode
step; one JSON line.  `--gemv-plain CALLS` only makes CALLS plain calls per
shape (for ncu).

`--linear` times nq_linear per shape (M x K x N), one JSON line per shape:
random Q8_0 weights rotated over enough copies to exceed the 126 MB L2, CUDA
events over --iters back-to-back calls, or with --graph the device time per
call of a CUDA graph of those calls; TFLOP/s and algorithmic GB/s
(N*K*34/32 + M*K*sx + M*N*sy) against the bound that applies (HBM for
M <= 125, tensor above).  --cfg1-sweep: the configs[0] block (K -> N:
1024->4096, 4096->1024, 1024->3072, 1024->1024, 1024->2048, 1024->1024) at
M in {1, 2, 4, 8, 16, 125, 1024, 2048, 4096, 12000}, f32 in and out, or bf16
with --sweep-dtype bf16; --keep-bf16 gives every weight a kept bf16 copy as
the encoder does; --kokoro adds the configs[3] Kokoro linears at M = 200.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Parakeet encoder RTFx (audio s/s) at 1/2/4/8 B200; Q8_0 GEMM % of peak"
UNIT = "audio s/s"
# libnq8 kernel classes timed by its event profiler (include/nq8.h NQ_KCLASS_*).
KCLASSES = {"gemm": 0, "gemv": 1, "dequant": 2, "reduce": 3, "attention": 4, "layernorm": 5}
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--segments", type=int, default=1024)
    ap.add_argument("--max-batch", type=int, default=32)
    ap.add_argument("--shard", choices=["weak", "lpt"], default="lpt",
                    help="lpt: one job of --segments split over the ranks (strong scaling); "
                         "weak: each rank runs its own --segments")
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--e2e-steps", type=int, default=0, help="steps of the e2e timing (0: --steps)")
    ap.add_argument("--streams", type=int, default=2, help="CUDA streams the buckets of a step alternate over")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-segments", type=int, default=16,
                    help="segments of the CPU sample (stratified by length over the job) at all host cores")
    ap.add_argument("--cpu-segments-one-core", type=int, default=2, help="segments of the one-core CPU sample")
    ap.add_argument("--cpu-threads", type=int, default=0, help="CPU threads (0: all the host offers)")
    ap.add_argument("--gemv", action="store_true", help="time the Q8_0 GEMV alone instead of the encoder")
    ap.add_argument("--gemv-shapes", default="1x640x640,1x640x2560,1x2560x640,1x4096x4096,1x8192x8192,"
                    "1x640x32768,8x4096x4096,16x4096x4096,1x16384x16384")
    ap.add_argument("--gemv-plain", type=int, default=0, help="only make this many plain calls per shape")
    ap.add_argument("--gemv-path", type=int, default=0, choices=(0, 1, 2),
                    help="--gemv: GEMV form (nq_set_gemv_path: 0 auto, 1 split + reduce, 2 cluster where it applies)")
    ap.add_argument("--no-decode-step", action="store_true", help="--gemv without the configs[2] decode step")
    ap.add_argument("--linear", action="store_true", help="time nq_linear per shape instead of the encoder")
    ap.add_argument("--shape", action="append", default=[], help="--linear: MxKxN")
    ap.add_argument("--cfg1-sweep", action="store_true", help="--linear: the configs[0] block over the M sweep")
    ap.add_argument("--kokoro", action="store_true", help="--linear: the configs[3] Kokoro linears at M = 200")
    ap.add_argument("--sweep-dtype", choices=["f32", "bf16"], default="f32",
                    help="--linear: activations in and out of the sweeps (f32: configs[0]; bf16: the encoder's)")
    ap.add_argument("--x", choices=["bf16", "f32"], default="bf16", help="--linear: activation dtype of --shape")
    ap.add_argument("--y", choices=["bf16", "f32"], default="bf16", help="--linear: output dtype of --shape")
    ap.add_argument("--iters", type=int, default=20, help="--linear: calls per timing")
    ap.add_argument("--graph", action="store_true", help="--linear: time a CUDA graph of the calls")
    ap.add_argument("--keep-bf16", action="store_true", help="--linear: kept bf16 weight copies (as the encoder)")
    ap.add_argument("--sweep-m", default="", help="--linear: comma-separated subset of the sweep's M values")
    ap.add_argument("--unit-tokens", default="0",
                    help="GEMM unit width (nq_set_gemm_unit_tokens; 0 = the cost model's choice); "
                         "--linear: comma-separated widths to time each shape with")
    ap.add_argument("--qtiled", action="store_true", help="--linear: weights with QTiled semantics (from_qtensor)")
    ap.add_argument("--conv", action="store_true",
                    help="time the Kokoro generator's conv1d / conv_transpose1d shapes (nq_conv*) instead")
    ap.add_argument("--conv-frames", type=int, default=300, help="--conv: decoder frames (80 Hz) of the utterance")
    ap.add_argument("--conv-only", default=None,
                    help="--conv: time only the convs whose name contains this text (e.g. 'k11 d5')")
    ap.add_argument("--tail-split", type=int, default=0,
                    help="nq_set_gemm_tail_split mode of the GEMMs (0 cost model, 1 off, >= 2 pieces)")
    ap.add_argument("--attention", choices=["tcgen05", "mma_sync"], default="tcgen05",
                    help="encoder attention kernel (nq_set_attention_kernel)")
    return ap.parse_args()


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        d["source"] = "measured"
        return d
    return dict(FALLBACK_PEAKS)


# ------------------------------------------------------------------ workload
def job_segments(n_segments: int, seed: int = 4):
    """Mel frame counts of the configs[4] job: durations U[2, 30] s."""
    from nspeech_b200 import synthetic as S
    return [S.mel_frames(s) for s in S.segment_lengths_s(n_segments, 2.0, 30.0, seed=seed)]


def segment_mel(j: int, frames: int, feat: int, rank_seed: int = 0) -> np.ndarray:
    """Log-mel features of segment j (its own seed: independent of the split)."""
    return np.random.default_rng(100000 + 1000003 * rank_seed + j).standard_normal((frames, feat), dtype=np.float32)


def plan_buckets(rank: int, world: int, n_segments: int, max_batch: int, shard: str):
    """This rank's buckets as (segment indices, mel frame counts), and their mel seed.

    shard "lpt": one job of n_segments (seed 4) split over the ranks by
    nspeech_b200.shard (length buckets, greedy LPT on the estimated bucket
    cost).  shard "weak": the rank's own n_segments (seed 4 + rank),
    length-bucketed.
    """
    from nspeech_b200 import shard as SH
    if shard == "lpt":
        frames = job_segments(n_segments, 4)
        parts = SH.shard_segments(frames, max_batch, world, rank)
        return [(idx, [int(frames[j]) for j in idx]) for idx in parts], 0
    frames = job_segments(n_segments, 4 + rank)
    return [(idx, [int(frames[j]) for j in idx]) for idx in SH.length_buckets(frames, max_batch)], rank


def materialize(plan, feat: int, rank_seed: int):
    """Padded bucket tensors [(mel [B, T, feat], lengths)] of a plan."""
    out = []
    for idx, lens in plan:
        mel = np.zeros((len(idx), max(lens), feat), np.float32)
        for r, (j, L) in enumerate(zip(idx, lens)):
            mel[r, :L] = segment_mel(j, L, feat, rank_seed)
        out.append((mel, lens))
    return out


def make_buckets(rank: int, n_segments: int, max_batch: int, feat: int, shard: str = "weak", world: int = 1):
    """This rank's padded buckets [(mel [B, T, feat], lengths)] and their audio seconds."""
    plan, rank_seed = plan_buckets(rank, world, n_segments, max_batch, shard)
    buckets = materialize(plan, feat, rank_seed)
    return buckets, float(sum(L for _, ls in buckets for L in ls)) * 0.01


def workload_config(args, world: int, plan, spec) -> dict:
    """The line's `config` (both arms report the same one)."""
    from nspeech_b200.shard import encoder_frames
    audio_s = sum(L for _, ls in plan for L in ls) * 0.01
    segs = sum(len(ls) for _, ls in plan)
    return {
        "workload": (f"configs[4]: one job of {args.segments} VAD segments split over {world} GPU(s) "
                     "(length buckets, greedy LPT)" if args.shard == "lpt" else
                     f"configs[4]: {args.segments} VAD segments/GPU") +
                    f", U[2,30] s, length-bucketed batches <= {args.max_batch}, "
                    f"full {spec.n_layers}-layer encoder (configs[1] architecture)",
        "model": f"Parakeet TDT 0.6B FastConformer encoder ({spec.n_layers} layers, d {spec.d_model}, "
                 f"{spec.n_heads} heads, FFN {spec.d_model * spec.ff_mult}, conv {spec.conv_kernel})",
        "segments_per_gpu": segs, "shard": args.shard, "max_batch": args.max_batch, "audio_s_per_gpu": audio_s,
        "buckets": len(plan), "streams": max(1, args.streams), "attention": args.attention,
        "gemm_unit_tokens": int(args.unit_tokens.split(",")[0]) or "auto",
        "seq_len": max(encoder_frames(max(ls)) for _, ls in plan),
        "global_batch": args.segments if args.shard == "lpt" else args.segments * world,
        "parallelism": f"dp{world} (segment-sharded, no collective on the data path)",
        "l2": "inputs larger than L2: 0.64 GB of Q8_0 weights stream per pass; activations up to 1.6 GB",
    }


def make_encoder(spec, seed=1, timings=None):
    """The GPU encoder with seeded random weights; `timings` (dict) receives the
    wall seconds of generating the f32 tensors, staging them (the library
    quantizes them to Q8_0 with ggml's rule) and nq_encoder_finalize (repack,
    upload, kept bf16 copies)."""
    from nspeech_b200 import synthetic as S
    from nspeech_b200.encoder import ParakeetEncoder
    t0 = time.perf_counter()
    enc = ParakeetEncoder(spec, device=int(os.environ.get("LOCAL_RANK", 0)))
    tensors = S.encoder_tensors(spec, seed)
    t1 = time.perf_counter()
    enc.load_tensors(tensors)
    t2 = time.perf_counter()
    enc.finalize()
    t3 = time.perf_counter()
    if timings is not None:
        timings.update({"generate_s": t1 - t0, "stage_and_quantize_s": t2 - t1, "finalize_s": t3 - t2})
    return enc, tensors


# -------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while timing."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.device)], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        if self.path and os.path.exists(self.path):
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                    rows.append(parts)
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


# ------------------------------------------------------------- CPU baseline
def cpu_info() -> dict:
    from oracle import oracle as O
    model = ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"nproc": os.cpu_count(), "cpu_model": model, "isa": "avx512f" if O.cpu_isa() == 512 else "avx2+fma"}


def cpu_sample(n_segments: int, n_take: int):
    """n_take segments of the configs[4] job (seed 4), stratified by length:
    the (i + 1/2) / n_take quantiles of the sorted durations."""
    frames = job_segments(n_segments, 4)
    order = sorted(range(len(frames)), key=lambda j: (frames[j], j))
    return [(order[int((i + 0.5) * len(order) / n_take)], None) for i in range(n_take)], frames


def cpu_model(spec, tensors):
    """The CPU path restating the reference's Linux encoder with fast_matmul
    linears: every Q8_0 weight dequantized and packed to bf16 once
    (src/fast_matmul.rs:191-208), f32 activations (oracle/encoder_oracle.c,
    oracle/fbgemm_cpu.c)."""
    from oracle import oracle as O
    q = {k: (O.quantize_q8_0(v.reshape(v.shape[0], -1)) if q8 else v) for k, (v, q8) in tensors.items()}
    return O.EncoderModel(spec.as_dict(), q, weight_mode=0)


def cpu_encoder_pass(model, picks, frames, feat: int) -> tuple:
    """Encode each picked segment (batch 1, as the reference): (audio s, wall s)."""
    audio, wall = 0.0, 0.0
    for j, _ in picks:
        mel = segment_mel(j, frames[j], feat)
        t0 = time.perf_counter()
        model(mel)
        wall += time.perf_counter() - t0
        audio += frames[j] * 0.01
    return audio, wall


def cpu_linear_set(threads: int, reps: int = 10) -> dict:
    """configs[0] on the CPU path: the six linears of one block at M = 125,
    f32 x ~ N(0, 1) (seed 0), Q8_0 weights N(0, 0.02), f32 bias N(0, 0.01);
    3 warm-up and `reps` timed passes of the whole set (median, min, max)."""
    from oracle import oracle as O
    O.set_threads(threads)
    m = 125
    ws = []
    for i, (k, n) in enumerate(CFG1_KN):
        q = O.quantize_q8_0(O.normal(300 + i, (n, k), 0.0, 0.02))
        ws.append((O.PackedWeight(q, n, k), O.normal(400 + i, (m, k)), O.normal(500 + i, (n,), 0.0, 0.01),
                   np.empty((m, n), np.float32)))
    flops = sum(2.0 * m * n * k for k, n in CFG1_KN)
    times = []
    for it in range(3 + reps):
        t0 = time.perf_counter()
        for w, x, b, y in ws:
            w(x, b, out=y)
        if it >= 3:
            times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"threads": threads, "m": m, "gflops": flops / med / 1e9, "ms_median": 1e3 * med,
            "ms_min": 1e3 * min(times), "ms_max": 1e3 * max(times)}


def cpu_baseline(args, spec, tensors) -> dict:
    """RTFx of the CPU path on a stratified sample of the job at all host
    cores and at one core, and the configs[0] linear set at both (BASELINE
    CPU plan: pre-packed bf16 weights, f32 activations, AVX-512 widening + FMA,
    OpenMP over 128-column tiles)."""
    from oracle import oracle as O
    threads = args.cpu_threads or O.max_threads()
    model = cpu_model(spec, tensors)
    picks, frames = cpu_sample(args.segments, args.cpu_segments)
    O.set_threads(threads)
    model(segment_mel(0, 200, spec.feat_in))  # warm-up
    audio, wall = cpu_encoder_pass(model, picks, frames, spec.feat_in)
    one = None
    if args.cpu_segments_one_core > 0:
        picks1, _ = cpu_sample(args.segments, args.cpu_segments_one_core)
        O.set_threads(1)
        a1, w1 = cpu_encoder_pass(model, picks1, frames, spec.feat_in)
        one = {"value": a1 / w1, "cores": 1, "sample": f"{len(picks1)} segments, {a1:.1f} audio s"}
    lin = [cpu_linear_set(threads), cpu_linear_set(1)]
    O.set_threads(threads)
    model.close()
    return {"value": audio / wall, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{len(picks)} of the job's {args.segments} segments, stratified by length "
                      f"({audio:.1f} audio s), batch 1, full {spec.n_layers}-layer encoder",
            "path": "oracle/encoder_oracle.c + oracle/fbgemm_cpu.c: Q8_0 weights dequantized and packed to bf16 "
                    "once, f32 activations, bf16 widened in registers + FMA (k-sequential f32 sums), OpenMP over "
                    "48-row x 128-column tiles; attention as f32 GEMMs per (head, 32-query block)",
            "one_core": one, "cfg1_linear_set": lin, **cpu_info()}


def run_reference(args, rank: int, world: int) -> None:
    """The reference's CPU path (the port; the Rust build is unavailable) on
    the stratified sample of this arm's job, all host cores, per step."""
    if rank != 0:
        return
    from oracle import oracle as O
    from nspeech_b200 import synthetic as S
    spec = S.EncoderSpec(n_layers=args.layers)
    tensors = S.encoder_tensors(spec, 1)
    plan, _ = plan_buckets(0, world, args.segments, args.max_batch, args.shard)
    threads = args.cpu_threads or O.max_threads()
    model = cpu_model(spec, tensors)
    del tensors
    picks, frames = cpu_sample(args.segments, args.cpu_segments)
    O.set_threads(threads)
    for _ in range(args.warmup):
        cpu_encoder_pass(model, picks, frames, spec.feat_in)
    audio_step, t_total = 0.0, 0.0
    for _ in range(args.steps):
        a, w = cpu_encoder_pass(model, picks, frames, spec.feat_in)
        audio_step, t_total = a, t_total + w
    value = args.steps * audio_step / t_total
    one = None
    if args.cpu_segments_one_core > 0:
        picks1, _ = cpu_sample(args.segments, args.cpu_segments_one_core)
        O.set_threads(1)
        a1, w1 = cpu_encoder_pass(model, picks1, frames, spec.feat_in)
        one = {"value": a1 / w1, "cores": 1, "sample": f"{len(picks1)} segments, {a1:.1f} audio s"}
        O.set_threads(threads)
    model.close()
    sample = (f"{len(picks)} of the job's {args.segments} segments per step, stratified by length "
              f"({audio_step:.1f} audio s), batch 1 (the reference's run_encoder), all host cores")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * t_total / args.steps, "higher_is_better": True,
        "scaling": "strong" if args.shard == "lpt" else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded N(0,1) log-mel features, random-init Q8_0 weights",
        "config": workload_config(args, world, plan, spec),
        "audio_s_per_step": audio_step,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample,
                         "one_core": one, **cpu_info()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------- ours
def reduce_over_ranks(t_s: float, t_e2e: float, audio_s: float, dist, device: str):
    """Whole-job figures: the slowest rank's device and e2e times, the audio of all ranks.

    Every rank calls it once after its timed regions (two all-reduces, same
    order on every rank); with dist None (one process) it returns its inputs.
    """
    if not dist:
        return t_s, t_e2e, audio_s
    import torch
    vals = torch.tensor([t_s, t_e2e, audio_s], dtype=torch.float64, device=device)
    mx = vals.clone()
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    tot = vals.clone()
    dist.all_reduce(tot, op=dist.ReduceOp.SUM)
    return float(mx[0]), float(mx[1]), float(tot[2])


def run_ours(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    from nspeech_b200 import lib, synthetic as S
    from nspeech_b200.encoder import out_frames

    dist = None
    if world > 1:
        import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    lib.init(local_rank)
    lib.check(lib.load().nq_set_gemm_tail_split(args.tail_split))
    lib.check(lib.load().nq_set_attention_kernel(
        lib.NQ_ATTENTION_TCGEN05 if args.attention == "tcgen05" else lib.NQ_ATTENTION_MMA_SYNC))
    lib.check(lib.load().nq_set_gemm_unit_tokens(int(args.unit_tokens.split(",")[0])))
    spec = S.EncoderSpec(n_layers=args.layers)
    load_t = {}
    enc, tensors = make_encoder(spec, timings=load_t)
    plan, rank_seed = plan_buckets(rank, world, args.segments, args.max_batch, args.shard)
    if not plan:
        raise SystemExit(f"rank {rank}: no buckets (--shard lpt needs at least one bucket per rank)")
    buckets = materialize(plan, spec.feat_in, rank_seed)
    audio_s = sum(L for _, ls in buckets for L in ls) * 0.01

    mel_dev, out_dev = [], []
    for mel, lens in buckets:
        mel_dev.append(torch.from_numpy(mel).cuda())
        out_dev.append(torch.empty((mel.shape[0], out_frames(mel.shape[1]), spec.d_model), device="cuda"))
    launches_per_step = sum(enc.launch_count(m.shape[0], m.shape[1]) for m, _ in buckets)

    # Buckets alternate over `--streams` streams (each has its own activation
    # arena in the library): one bucket's forward fills the SMs that the
    # other's kernels leave idle (GEMM wave tails, memory-bound phases).
    streams = [torch.cuda.Stream() for _ in range(max(1, args.streams))]

    def step(n_streams=len(streams)):
        cur = torch.cuda.current_stream()
        for s in streams[:n_streams]:
            s.wait_stream(cur)
        for j, ((mel, lens), md, od) in enumerate(zip(buckets, mel_dev, out_dev)):
            with torch.cuda.stream(streams[j % n_streams]):
                enc.forward(md, lens, out=od)
        for s in streams[:n_streams]:
            cur.wait_stream(s)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if lib.status() != 0:
        raise RuntimeError("device status reported a timeout during warm-up")
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = lib.launch_counter()
    with ClockSampler(local_rank) as clk:
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t_s = e0.elapsed_time(e1) / 1e3
    launches_timed = lib.launch_counter() - launches0

    # ---- roofline pass: the same K steps again with the library's per-launch
    # CUDA-event timer on (events on each kernel's own stream), on one stream
    # so that a kernel's event time is its own and not shared with the other
    # stream's kernels.  Kept out of the timed region above: an event recorded
    # between two kernels ends the programmatic-launch overlap of the second
    # with the first, which costs ~10% of the step.
    for kc in KCLASSES.values():
        lib.profile_read(kc, reset=True)
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    lib.profile_enable(True)
    p0.record()
    for _ in range(args.steps):
        step(1)
    p1.record()
    torch.cuda.synchronize()
    lib.profile_enable(False)
    t_prof = p0.elapsed_time(p1) / 1e3
    kern = {name: lib.profile_read(kc) for name, kc in KCLASSES.items()}
    gemm = kern["gemm"]
    if lib.status() != 0:
        raise RuntimeError("device status reported a timeout during the timed region")

    # ---- e2e: host buffers through nq_encoder_forward_host_async (pinned
    # memory), K steps: each step's mel goes in and its encoder output comes
    # back to host memory inside the timed region.
    host_in = [torch.from_numpy(m).pin_memory() for m, _ in buckets]
    host_out = [torch.empty(tuple(o.shape), dtype=torch.float32).pin_memory() for o in out_dev]
    torch.cuda.synchronize()
    handles = [s.cuda_stream for s in streams]

    def e2e_step():
        for j, ((mel, lens), hi, ho) in enumerate(zip(buckets, host_in, host_out)):
            enc.forward_host_async(hi.numpy(), lens, ho.numpy(), handles[j % len(handles)])
        enc.wait()  # every output of the step is in host memory

    e2e_steps = args.e2e_steps or args.steps
    e2e_step()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    t_e2e = time.perf_counter() - t0
    h2d = sum(m.nbytes for m, _ in buckets)
    d2h = sum(o.numel() * 4 for o in out_dev)

    # ---- single 30 s segment latency, for reference
    mel30 = torch.from_numpy(np.random.default_rng(1).standard_normal((1, 3000, spec.feat_in),
                                                                       dtype=np.float32)).cuda()
    o30 = torch.empty((1, out_frames(3000), spec.d_model), device="cuda")
    for _ in range(3):
        enc.forward(mel30, None, out=o30)
    torch.cuda.synchronize()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record()
    for _ in range(10):
        enc.forward(mel30, None, out=o30)
    a1.record()
    torch.cuda.synchronize()
    cfg2_ms = a0.elapsed_time(a1) / 10

    # ---- max over ranks
    t_max, te2e_max, audio_total = reduce_over_ranks(t_s, t_e2e, audio_s, dist, "cuda")

    if rank == 0:
        pk = peaks()
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(args, spec, tensors)
        achieved = gemm["flops"] / (gemm["ms"] / 1e3) / 1e12 if gemm["ms"] > 0 else 0.0
        peak_t = pk.get("bf16_tflops_sustained", pk.get("bf16_tflops"))
        traffic, traffic_src = None, None
        tpath = os.path.join(ROOT, "profiles", "gemm_bf16_sm100_traffic.json")
        if os.path.exists(tpath):
            with open(tpath) as f:
                tj = json.load(f)
            traffic, traffic_src = tj.get("traffic_bytes_per_launch"), tj.get("source")
            if traffic is None and tj.get("traffic_bytes_per_gflop") and gemm["launches"]:
                # scaled to this run's average launch by its algorithmic GFLOP
                traffic = tj["traffic_bytes_per_gflop"] * gemm["flops"] / gemm["launches"] / 1e9
        line = {
            "metric": METRIC,
            "value": args.steps * audio_total / t_max,
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": 1e3 * t_max / args.steps,
            "higher_is_better": True,
            "scaling": "strong" if args.shard == "lpt" else "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic: seeded N(0,1) log-mel features, random-init Q8_0 weights",
            "config": workload_config(args, world, plan, spec),
            "e2e": {"value": e2e_steps * audio_total / te2e_max, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                    "api": "nq_encoder_forward_host_async per bucket (buckets alternating over the streams) + "
                           "nq_encoder_wait per step (pinned host buffers); wall clock, max over ranks"},
            "roofline": {"kernel": "gemm_bf16_sm100_kernel (GEMM class; M < 128 calls use gemm_q8_sm100_kernel)",
                         "bound": "tensor", "achieved": achieved, "peak": peak_t,
                         "unit": "TFLOP/s", "frac": achieved / peak_t if peak_t else None, "traffic": traffic,
                         "traffic_source": traffic_src,
                         "peak_source": f"{pk['source']} bf16_tflops_sustained",
                         "launches": gemm["launches"], "avg_launch_us": 1e3 * gemm["ms"] / max(1, gemm["launches"]),
                         "algorithmic_gflop_per_launch": gemm["flops"] / max(1, gemm["launches"]) / 1e9,
                         "share_of_step": gemm["ms"] / 1e3 / t_prof if t_prof else None,
                         "measured_in": "profiled repetition of the timed steps on one stream (per-launch CUDA "
                                        "events; share_of_step is of that one-stream step)",
                         "profiled_ms_per_step": 1e3 * t_prof / args.steps},
            "kernels": kern,
            "cpu_baseline": cpu,
            "clocks": clk.summary(),
            "gpu_launches": launches_timed,
            "gpu_launches_expected": launches_per_step * args.steps,
            "cfg2_single_30s": {"ms": cfg2_ms, "rtfx": 30.0 / (cfg2_ms / 1e3)},
            "load": dict(load_t, note="per process, before the timed region; excluded from value"),
        }
        print(json.dumps(line), flush=True)


# -------------------------------------------------------------------- linear
CFG1_KN = [(1024, 4096), (4096, 1024), (1024, 3072), (1024, 1024), (1024, 2048), (1024, 1024)]
CFG1_M = [1, 2, 4, 8, 16, 125, 1024, 2048, 4096, 12000]
# configs[3] Kokoro linears (K -> N) at M = 200 phonemes: ALBERT Q/K/V/dense,
# FFN and FFN output (src/kokoro/albert.rs:126-149), bert_encoder 768 -> 512
# (src/kokoro/model.rs:84-87).
KOKORO_KN = [(768, 768), (768, 2048), (2048, 768), (768, 512)]


def _linear_weights(n: int, k: int, copies: int, rng, keep_bf16: bool = False, qtiled: bool = False) -> list:
    from nspeech_b200 import lib
    from nspeech_b200.fast_matmul import QWeight
    out = []
    for _ in range(copies):
        q = rng.integers(-127, 128, size=(n, k // 32, 34), dtype=np.int64).astype(np.uint8)
        d = (rng.random((n, k // 32)) * 1e-3 + 1e-4).astype(np.float16)
        q[:, :, :2] = d.view(np.uint8).reshape(n, k // 32, 2)
        w = QWeight.from_q8_0(q.reshape(n, -1), n, k, flags=lib.NQ_MODE_QTILED if qtiled else 0)
        out.append(w.keep_bf16() if keep_bf16 else w)
    return out


def time_linear(m: int, k: int, n: int, x_dtype, y_dtype, iters: int = 20, seed: int = 0, graph: bool = False,
                keep_bf16: bool = False, qtiled: bool = False) -> dict:
    """Device time per nq_linear call of one shape (see the module docstring)."""
    import torch
    from nspeech_b200 import lib
    rng = np.random.default_rng(seed)
    wbytes = n * k * 34 / 32
    # weights stream past L2 (the kept bf16 copy, when kept, is what the GEMM reads)
    copies = int(min(32, max(1, np.ceil(300e6 / (n * k * 2 if keep_bf16 else wbytes)))))
    ws = _linear_weights(n, k, copies, rng, keep_bf16, qtiled)
    x = torch.randn(m, k, device="cuda").to(x_dtype)
    y = torch.empty(m, n, device="cuda", dtype=y_dtype)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i in range(max(3, copies)):  # also sizes the stream's workspace before any capture
            ws[i % copies].linear(x, out=y)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(iters):
                ws[i % copies].linear(x, out=y)
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
        with torch.cuda.stream(stream):
            e0.record()
            for i in range(iters):
                ws[i % copies].linear(x, out=y)
            e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / iters / 1e3
    if lib.status() != 0:
        raise RuntimeError("device status reported a timeout")
    byts = wbytes + m * k * x.element_size() + m * n * y.element_size()
    pk = peaks()
    tflops, gbs = 2 * m * n * k / t / 1e12, byts / t / 1e9
    bound = "hbm" if m <= 125 else "tensor"
    frac = gbs / pk["hbm_gbs"] if bound == "hbm" else tflops / pk["bf16_tflops"]
    return {"m": m, "k": k, "n": n, "x": str(x_dtype).split(".")[-1], "y": str(y_dtype).split(".")[-1],
            "us": round(t * 1e6, 2), "tflops": round(tflops, 1), "gbs": round(gbs, 1), "bound": bound,
            "frac": round(frac, 3), "peak_source": pk["source"], "timing": "graph" if graph else "calls",
            "weights": ("qtiled " if qtiled else "") + ("kept bf16 copy" if keep_bf16 else "q8_0")}


def run_linear(args) -> None:
    import torch
    from nspeech_b200 import lib
    torch.cuda.set_device(0)
    lib.init(0)
    dt = {"bf16": torch.bfloat16, "f32": torch.float32}
    jobs = [(tuple(int(v) for v in s.lower().split("x")), dt[args.x], dt[args.y]) for s in args.shape]
    sd = dt[args.sweep_dtype]
    if args.cfg1_sweep:
        ms = [int(v) for v in args.sweep_m.split(",")] if args.sweep_m else CFG1_M
        jobs += [((m, k, n), sd, sd) for m in ms for k, n in CFG1_KN]
    if args.kokoro:
        jobs += [((200, k, n), sd, sd) for k, n in KOKORO_KN]
    if not jobs:
        raise SystemExit("--linear needs --shape, --cfg1-sweep or --kokoro")
    units = [int(v) for v in args.unit_tokens.split(",")]
    lib.check(lib.load().nq_set_gemm_tail_split(args.tail_split))
    for (m, k, n), xd, yd in jobs:
        for u in units:
            lib.check(lib.load().nq_set_gemm_unit_tokens(u))
            r = time_linear(m, k, n, xd, yd, iters=args.iters, graph=args.graph, keep_bf16=args.keep_bf16,
                            qtiled=args.qtiled)
            r["unit_tokens"] = u
            r["tail_split"] = args.tail_split
            print(json.dumps(r), flush=True)
    lib.check(lib.load().nq_set_gemm_unit_tokens(0))
    lib.check(lib.load().nq_set_gemm_tail_split(0))


# configs[3] Kokoro ISTFTNet generator convolutions for an utterance of F
# decoder frames (upsample rates 10 and 6; src/kokoro/decoder.rs generator):
# (name, kind, c_in, c_out, K, stride, padding, dilation, T_in as a multiple of F)
KOKORO_CONVS = [
    ("ups.0", "t", 512, 256, 20, 10, 5, 1, 1),
    ("resblock 256 k3 d1", "c", 256, 256, 3, 1, 1, 1, 10),
    ("resblock 256 k7 d3", "c", 256, 256, 7, 1, 9, 3, 10),
    ("resblock 256 k11 d5", "c", 256, 256, 11, 1, 25, 5, 10),
    ("ups.1", "t", 256, 128, 12, 6, 3, 1, 10),
    ("resblock 128 k3 d1", "c", 128, 128, 3, 1, 1, 1, 60),
    ("resblock 128 k11 d5", "c", 128, 128, 11, 1, 25, 5, 60),
    ("conv_post", "c", 128, 22, 7, 1, 3, 1, 60),
]


def run_conv_sweep(args) -> None:
    """Device time per nq_conv1d / nq_conv_transpose1d call (CUDA graph of
    back-to-back calls, bf16 NCW input and output, seeded weights: Q8_0 for
    conv1d, the [C_in, C_out, K] values for conv_transpose1d), with the
    convolution's FLOPs (2 * C_out * C_in * K * T_out, conv_transpose:
    2 * C_in * C_out * K * T_in) against the measured bf16 peak."""
    import torch
    from nspeech_b200 import conv as C, lib
    from nspeech_b200.fast_matmul import QWeight
    torch.cuda.set_device(0)
    lib.init(0)
    pk = peaks()
    rng = np.random.default_rng(0)
    rows = []
    for name, kind, cin, cout, k, stride, pad, dil, tmul in KOKORO_CONVS:
        if args.conv_only and args.conv_only not in name:
            continue
        t_in = args.conv_frames * tmul
        x = torch.randn(cin, t_in, device="cuda").to(torch.bfloat16)
        if kind == "c":
            if (cin * k) % 32 == 0:  # random Q8_0 blocks of the GGUF form [C_out, C_in * K]
                w = _linear_weights(cout, cin * k, 1, rng, keep_bf16=True)[0]
            else:  # left in f32 by the quantizer: kept at bf16 precision
                w = QWeight.from_f32((rng.standard_normal((cout, cin * k)) * 0.05).astype(np.float32))
            t_out = C.conv1d_out_len(t_in, k, stride, pad, dil)
            flops = 2.0 * cout * cin * k * t_out
            call = lambda: C.conv1d(x, w, None, k, stride, pad, dil, out=y)  # noqa: E731
        else:
            w = C.ConvTransposeWeight.from_f32((rng.standard_normal((cin, cout, k)) * 0.05).astype(np.float32))
            t_out = C.conv_transpose1d_out_len(t_in, k, stride, pad)
            flops = 2.0 * cin * cout * k * t_in
            call = lambda: C.conv_transpose1d(x, w, None, stride, pad, out=y)  # noqa: E731
        y = torch.empty(cout, t_out, device="cuda", dtype=torch.bfloat16)
        implicit = (kind == "c" and stride == 1 and cin % 64 == 0 and t_out > 16) or (kind == "t" and cin % 64 == 0)

        def graph_us():
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                call()  # scratch sized (and the weight's tap-major copy built) before capture
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            iters = 10
            with torch.cuda.graph(g, stream=s):
                for _ in range(iters):
                    call()
            g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(5):
                g.replay()
            e1.record()
            torch.cuda.synchronize()
            del g
            return e0.elapsed_time(e1) * 1e3 / (5 * iters)

        us = graph_us()
        row = {"conv": name, "c_in": cin, "c_out": cout, "k": k, "stride": stride, "t_in": t_in,
               "t_out": t_out, "path": "implicit" if implicit else ("im2col" if kind == "c" else "col2im"),
               "us": round(us, 2), "tflops": round(flops / us / 1e6, 1),
               "frac_bf16_peak": round(flops / us / 1e6 / pk["bf16_tflops"], 3)}
        if implicit:  # the same call through the im2col / column-GEMM lowering, for comparison
            lib.check(lib.load().nq_set_conv_path(lib.NQ_CONV_IM2COL))
            try:
                row["us_im2col" if kind == "c" else "us_col2im"] = round(graph_us(), 2)
            finally:
                lib.check(lib.load().nq_set_conv_path(lib.NQ_CONV_AUTO))
        rows.append(row)
    if lib.status() != 0:
        raise RuntimeError("device status bits set after the conv sweep")
    print(json.dumps({"metric": "Kokoro generator conv1d / conv_transpose1d (nq_conv*), bf16 NCW",
                      "frames": args.conv_frames, "peak_bf16_tflops": pk["bf16_tflops"],
                      "peak_source": pk.get("source", "measured"), "convs": rows}), flush=True)


def run_gemv_sweep(args) -> None:
    """Graph-timed Q8_0 GEMV per shape (synthetic Q8_0 weights, bf16 x and y)."""
    import torch
    from nspeech_b200 import lib
    from nspeech_b200.fast_matmul import QWeight
    torch.cuda.set_device(0)
    lib.init(0)
    lib.check(lib.load().nq_set_gemv_path(args.gemv_path))
    pk = peaks()
    rng = np.random.default_rng(0)
    rows = []
    for shp in args.gemv_shapes.split(","):
        m, k, n = (int(v) for v in shp.split("x"))
        q = rng.integers(0, 256, size=(n, k // 32, 34), dtype=np.uint8)
        q[:, :, :2] = (rng.random((n, k // 32)) * 1e-3 + 1e-4).astype(np.float16).view(np.uint8).reshape(n, k // 32, 2)
        blocks = np.ascontiguousarray(q.reshape(n, -1))
        wbytes = n * k * 34 / 32
        copies = 1 if args.gemv_plain else int(min(64, max(2, np.ceil(400e6 / wbytes))))
        ws = [QWeight.from_q8_0(blocks, n, k) for _ in range(copies)]
        x = torch.randn(m, k, device="cuda").bfloat16()
        y = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        if args.gemv_plain:
            for _ in range(args.gemv_plain):
                ws[0].linear(x, out=y)
            torch.cuda.synchronize()
            continue
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            for w in ws:
                w.linear(x, out=y)  # workspace sized before capture
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for w in ws:
                w.linear(x, out=y)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        reps = max(3, 200 // copies)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
        byts = wbytes + m * k * 2 + m * n * 2
        rows.append({"m": m, "k": k, "n": n, "us": round(us, 2), "gbs": round(byts / us / 1e3, 1),
                     "frac_hbm": round(byts / us / 1e3 / pk["hbm_gbs"], 3)})
        del g, ws
        torch.cuda.empty_cache()
    decode = None if args.gemv_plain or args.no_decode_step else decode_step(rng, pk)
    if lib.status() != 0:
        raise RuntimeError("device status bits set after the GEMV sweep")
    if not args.gemv_plain:
        print(json.dumps({"metric": "Q8_0 GEMV HBM GB/s (graph of back-to-back calls, weights past L2)",
                          "peak_hbm_gbs": pk["hbm_gbs"], "peak_source": pk.get("source", "measured"),
                          "shapes": rows, "decode_step": decode}), flush=True)


def decode_step(rng, pk) -> dict:
    """configs[2] decoder: the Q8_0 contractions of one greedy token (M = 1), as
    a chain where each call's input is an earlier call's output: per layer the
    fused Q/K/V (640 -> 3 x 640), the self-attention O projection with
    residual + LayerNorm, the cross-attention Q projection, its O projection
    with residual + LayerNorm, fc1 (640 -> 2 x 2560, GLU-SiLU) and fc2
    (2560 -> 640) with residual + LayerNorm; 14 layers, then the lm_head
    (640 -> 32768).  131.95 MB of Q8_0 weights per token (the cross K/V are
    computed once per utterance).  The attention kernels between the
    projections are not part of this path and are left out.  Timed as a CUDA
    graph of 8 tokens over distinct weight copies (more than L2)."""
    import torch
    from nspeech_b200 import lib
    from nspeech_b200.fast_matmul import QWeight

    d, ff, layers, vocab = 640, 2560, 14, 32768

    def qw(n, k, flags=0):
        q = rng.integers(0, 256, size=(n, k // 32, 34), dtype=np.uint8)
        q[:, :, :2] = (rng.random((n, k // 32)) * 1e-3 + 1e-4).astype(np.float16).view(np.uint8).reshape(n, k // 32, 2)
        return QWeight.from_q8_0(np.ascontiguousarray(q.reshape(n, -1)), n, k, flags=flags)

    copies = 2  # 2 x 132 MB > L2: consecutive tokens read their weights from HBM
    nets = []
    for _ in range(copies):
        lay = [dict(qkv=qw(3 * d, d), o=qw(d, d), cq=qw(d, d), co=qw(d, d), fc1=qw(2 * ff, d, lib.NQ_PACK_GLU),
                    fc2=qw(d, ff)) for _ in range(layers)]
        nets.append((lay, qw(vocab, d)))
    wbytes = sum(w.n * w.k * 34 / 32 for L in nets[0][0] for w in L.values()) + nets[0][1].n * nets[0][1].k * 34 / 32
    x = torch.randn(1, d, device="cuda").bfloat16()
    res = torch.randn(1, d, device="cuda")
    g = torch.ones(d, device="cuda")
    qkv = torch.empty(1, 3 * d, device="cuda", dtype=torch.bfloat16)
    h = torch.empty(1, d, device="cuda", dtype=torch.bfloat16)
    t = torch.empty(1, ff, device="cuda", dtype=torch.bfloat16)
    logits = torch.empty(1, vocab, device="cuda", dtype=torch.bfloat16)

    def token(net):
        lay, head = net
        for L in lay:
            L["qkv"].linear(x, out=qkv)
            L["o"].gemv_resadd_ln(qkv[:, :d], res, g, residual_out=res, out=h)  # attention output stands in
            L["cq"].linear(h, out=qkv[:, :d])
            L["co"].gemv_resadd_ln(qkv[:, :d], res, g, residual_out=res, out=h)
            L["fc1"].linear(h, epilogue=lib.NQ_EPI_GLU_SILU, out=t)
            L["fc2"].gemv_resadd_ln(t, res, g, residual_out=res, out=x)
        head.linear(x, out=logits)

    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for net in nets:
            token(net)
    torch.cuda.synchronize()
    lib.launch_counter(reset=True)
    with torch.cuda.stream(s):
        token(nets[0])
    torch.cuda.synchronize()
    launches_op = lib.launch_counter(reset=True)
    tokens = 8
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=s):
        for i in range(tokens):
            token(nets[i % copies])
    for _ in range(2):
        gr.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 5
    e0.record()
    for _ in range(reps):
        gr.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * tokens)
    del gr
    floor_us = wbytes / pk["hbm_gbs"] / 1e3
    calls = layers * 6 + 1

    # The same token as one decode-chain launch (nq_chain_*): the same calls
    # recorded once per weight copy, then a graph of 8 chain runs.
    from nspeech_b200.decode import DecodeChain
    chains = []
    for lay, head in nets:
        c = DecodeChain(0)
        for L in lay:
            c.linear(L["qkv"], x[0], qkv[0])
            c.gemv_resadd_ln(L["o"], qkv[0, :d], res[0], g, residual_out=res[0], out=h[0])
            c.linear(L["cq"], h[0], qkv[0, :d])
            c.gemv_resadd_ln(L["co"], qkv[0, :d], res[0], g, residual_out=res[0], out=h[0])
            c.linear(L["fc1"], h[0], t[0], epilogue=lib.NQ_EPI_GLU_SILU)
            c.gemv_resadd_ln(L["fc2"], t[0], res[0], g, residual_out=res[0], out=x[0])
        c.linear(head, x[0], logits[0])
        chains.append(c)
    with torch.cuda.stream(s):
        for c in chains:
            c.run(s)  # uploads
    torch.cuda.synchronize()
    gc = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gc, stream=s):
        for i in range(tokens):
            chains[i % copies].run(s)
    for _ in range(2):
        gc.replay()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        gc.replay()
    e1.record()
    torch.cuda.synchronize()
    us_chain = e0.elapsed_time(e1) * 1e3 / (reps * tokens)
    del gc
    for c in chains:
        c.close()
    if lib.status() != 0:
        raise RuntimeError("device status bits set after the decode chain")
    return {"config": "configs[2] Moonshine decoder, M = 1, 14 layers + lm_head", "weight_mb_per_token":
            round(wbytes / 1e6, 2), "hbm_floor_us": round(floor_us, 1), "gemv_calls_per_token": calls,
            "op_by_op": {"us_per_token": round(us, 1), "frac_of_floor": round(floor_us / us, 3),
                         "launches_per_token": launches_op},
            "chain": {"us_per_token": round(us_chain, 1), "frac_of_floor": round(floor_us / us_chain, 3),
                      "launches_per_token": 1}}


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.gemv:
        run_gemv_sweep(args)
        return
    if args.linear:
        run_linear(args)
        return
    if args.conv:
        run_conv_sweep(args)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        # stdout carries exactly one JSON line: NCCL prints its version banner
        # to fd 1 when the first communicator comes up, so create it (the
        # barrier) with fd 1 pointing at stderr.
        sys.stdout.flush()
        saved_fd = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local_rank))
            dist.barrier()
        finally:
            sys.stdout.flush()
            os.dup2(saved_fd, 1)
            os.close(saved_fd)
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
