"""bench.py contract pieces that need no GPU.

`--impl reference` times the CPU restatement of the reference encoder
(oracle/encoder_oracle.c over oracle/fbgemm_cpu.c) on a stratified sample of
the configs[4] job. The checks:
- rank 0 prints exactly one JSON line with the keys the driver reads;
- other ranks print nothing and exit 0;
- --help lists the sharding modes.
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(args, env_extra=None, timeout=600):
    env = dict(os.environ)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        env.pop(k, None)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, "bench.py", *args], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=timeout)


def test_reference_arm_prints_one_json_line():
    r = _run(["--impl", "reference", "--steps", "2", "--warmup", "1", "--layers", "2", "--cpu-segments", "3",
              "--cpu-segments-one-core", "1"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference"
    assert d["steps"] == 2 and d["warmup"] == 1 and d["n_gpus"] == 1
    assert d["higher_is_better"] is True and d["value"] > 0
    assert d["value"] * d["ms_per_step"] / 1e3 == pytest.approx(d["audio_s_per_step"], rel=1e-6)
    assert 3 * 2.0 <= d["audio_s_per_step"] <= 3 * 30.0  # three segments of U[2, 30] s
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] == "port"
    assert cb["one_core"]["cores"] == 1 and cb["one_core"]["value"] > 0
    assert cb["nproc"] >= 1 and cb["cpu_model"] and cb["isa"] in ("avx512f", "avx2+fma")
    assert d["config"]["shard"] == "lpt" and d["scaling"] == "strong"
    assert d["config"]["segments_per_gpu"] == 1024
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_are_silent():
    r = _run(["--impl", "reference", "--steps", "1", "--warmup", "0", "--layers", "1", "--cpu-segments", "1"],
             {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_help_lists_shard_modes():
    r = _run(["--help"], timeout=120)
    assert r.returncode == 0
    assert "--shard" in r.stdout and "lpt" in r.stdout


def test_cpu_sample_is_stratified_over_the_job():
    sys.path.insert(0, ROOT)
    import bench
    picks, frames = bench.cpu_sample(1024, 16)
    lens = sorted(frames[j] for j, _ in picks)
    assert len(set(j for j, _ in picks)) == 16
    srt = sorted(frames)
    assert lens[0] <= srt[len(srt) // 16] and lens[-1] >= srt[-len(srt) // 16]
    # the CPU sample's features are the GPU job's own segments
    plan, seed = bench.plan_buckets(0, 1, 1024, 32, "lpt")
    assert seed == 0 and sum(len(i) for i, _ in plan) == 1024
    j, L = picks[3][0], frames[picks[3][0]]
    mel = bench.materialize([([j], [L])], 128, 0)[0][0][0]
    assert (mel == bench.segment_mel(j, L, 128)).all()
