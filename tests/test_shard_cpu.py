"""Splitting one encoder job over GPUs (nspeech_b200/shard.py, bench.py --shard lpt), on CPU.

Segments are independent through the encoder (the reference encodes them
batch 1, src/parakeet/transducer.rs:387). So the split is pure host logic:
- length buckets;
- a deterministic greedy LPT assignment that every rank computes alone;
- a gather of per-segment results after the job (gloo, world size 2).
"""
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from nspeech_b200 import shard as SH  # noqa: E402
from nspeech_b200 import synthetic as S  # noqa: E402


def _job(n=1024):
    return [S.mel_frames(s) for s in S.segment_lengths_s(n, 2.0, 30.0, seed=4)]


def test_encoder_frames_matches_library():
    from nspeech_b200 import lib
    f = lib.load().nq_encoder_out_frames
    for t in [1, 2, 3, 7, 8, 9, 15, 16, 17, 200, 2999, 3000, 3001]:
        assert SH.encoder_frames(t) == f(t), t


def test_length_buckets_sorted_bounded_and_complete():
    frames = _job(100)
    buckets = SH.length_buckets(frames, 32)
    assert [len(b) for b in buckets] == [32, 32, 32, 4]
    flat = [i for b in buckets for i in b]
    assert sorted(flat) == list(range(100))
    lens = [frames[i] for i in flat]
    assert lens == sorted(lens)
    assert SH.length_buckets([], 4) == []
    with pytest.raises(ValueError):
        SH.length_buckets(frames, 0)


def test_bucket_cost_terms():
    frames = [800, 400, 3000]
    t = SH.encoder_frames(3000)
    assert SH.bucket_cost(frames, [0, 2]) == pytest.approx(2 * t * (1 + SH.ATTN_PER_FRAME * t))
    assert SH.bucket_cost(frames, [0, 2], attn_per_frame=0.0) == 2 * t
    assert SH.bucket_cost(frames, []) == 0.0


def test_assign_lpt_known_answer():
    # 5 -> r0; 4 -> r1; 3 -> r1 (4 < 5); 3 -> r0 (5 < 7); 2 -> r1 (7 < 8); 2 -> r0 (8 < 9)
    assert SH.assign_lpt([5, 4, 3, 3, 2, 2], 2) == [[0, 3, 5], [1, 2, 4]]
    # equal costs: lower bucket index first, ties to the lower rank
    assert SH.assign_lpt([1, 1, 1, 1], 3) == [[0, 3], [1], [2]]
    assert SH.assign_lpt([3, 1], 1) == [[0, 1]]
    assert SH.assign_lpt([], 2) == [[], []]
    with pytest.raises(ValueError):
        SH.assign_lpt([1.0], 0)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_configs4_job_splits_balanced_and_disjoint(world):
    frames = _job()
    parts = [SH.shard_segments(frames, 32, world, r) for r in range(world)]
    segs = [i for p in parts for b in p for i in b]
    assert sorted(segs) == list(range(len(frames)))  # every segment exactly once
    assert all(len(b) <= 32 for p in parts for b in p)
    assert SH.imbalance(frames, 32, world) < 1.01
    # deterministic: recomputing gives the same split
    assert parts == [SH.shard_segments(frames, 32, world, r) for r in range(world)]
    with pytest.raises(ValueError):
        SH.shard_segments(frames, 32, world, world)


def test_bench_lpt_buckets_do_not_depend_on_world_size():
    import bench
    n, mb, feat = 40, 8, 16
    frames = _job(n)
    one, audio1 = bench.make_buckets(0, n, mb, feat, "lpt", 1)
    rows1 = {}
    for (mel, lens), idx in zip(one, SH.shard_segments(frames, mb, 1, 0)):
        for r, j in enumerate(idx):
            rows1[j] = mel[r, :lens[r]]
            assert not mel[r, lens[r]:].any()  # padding is zero
    audio = 0.0
    for rank in range(3):
        part, a = bench.make_buckets(rank, n, mb, feat, "lpt", 3)
        audio += a
        for (mel, lens), idx in zip(part, SH.shard_segments(frames, mb, 3, rank)):
            for r, j in enumerate(idx):
                np.testing.assert_array_equal(mel[r, :lens[r]], rows1[j])
    assert audio == pytest.approx(audio1)
    assert audio1 == pytest.approx(sum(frames) * 0.01)


def test_gather_without_process_group_is_identity():
    res = {3: np.arange(4), 1: "x"}
    out = SH.gather_segments(res, None)
    assert out == res and out is not res


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import datetime
    import pickle
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import bench
        from nspeech_b200 import shard as SHr
        frames = _job(64)
        mine = SHr.shard_segments(frames, 8, world, rank)
        # per-segment "results": a small array derived from the segment index
        res = {j: np.full(3, j, np.int32) for b in mine for j in b}
        merged = SHr.gather_segments(res, dist)
        _, audio = bench.make_buckets(rank, 64, 8, 4, "lpt", world)
        t_max, _, audio_total = bench.reduce_over_ranks(1.0 + rank, 1.0, audio, dist, "cpu")
        dup = None
        try:
            SHr.gather_segments({0: 1}, dist)  # every rank claims segment 0
        except ValueError as e:
            dup = str(e)
        with open(os.path.join(out_dir, f"rank{rank}.pkl"), "wb") as f:
            pickle.dump({"merged": merged, "audio_total": audio_total, "t_max": t_max, "dup": dup}, f)
    finally:
        dist.destroy_process_group()


def test_gather_and_totals_over_two_ranks(tmp_path):
    import pickle
    torch = pytest.importorskip("torch")
    import torch.multiprocessing as mp
    assert torch is not None
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    r = []
    for i in range(world):
        with open(os.path.join(tmp_path, f"rank{i}.pkl"), "rb") as f:
            r.append(pickle.load(f))
    frames = _job(64)
    assert r[1]["merged"] is None
    merged = r[0]["merged"]
    assert sorted(merged) == list(range(64))
    assert all((v == k).all() for k, v in merged.items())
    for x in r:  # the whole job's audio once, the slowest rank's time
        assert float(x["audio_total"]) == pytest.approx(sum(frames) * 0.01)
        assert float(x["t_max"]) == 2.0
    assert "segment 0 produced by two ranks" in r[0]["dup"]
    assert r[1]["dup"] is None
