"""Multi-rank host logic of bench.py on CPU (gloo, world size 2).

bench.py shards the configs[4] workload by segments: every rank draws its
own segment set (seed 4 + rank), runs it with no collective on the data path,
and after the timed region the ranks agree on the slowest rank's times and
the total audio (reduce_over_ranks).  This runs exactly that host code in two
processes over gloo and checks the sharding and the reduction.
"""
import os
import socket
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import datetime
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import bench
        buckets, audio_s = bench.make_buckets(rank, 16, 8, 128)
        lens = sorted(L for _, ls in buckets for L in ls)
        t_dev, t_e2e = 1.0 + rank, 10.0 - rank
        t_max, te2e_max, audio_total = bench.reduce_over_ranks(t_dev, t_e2e, audio_s, dist, "cpu")
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), lens=np.array(lens), audio=audio_s, t_max=t_max,
                 te2e_max=te2e_max, audio_total=audio_total,
                 shapes=np.array([m.shape for m, _ in buckets]))
    finally:
        dist.destroy_process_group()


def test_segment_sharding_and_rank_reduction(tmp_path):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    r = [np.load(os.path.join(tmp_path, f"rank{i}.npz")) for i in range(world)]
    # each rank holds its own 16 segments, in length-sorted buckets of <= 8
    for x in r:
        assert len(x["lens"]) == 16
        assert (x["shapes"][:, 0] <= 8).all() and x["shapes"][:, 2].tolist() == [128] * len(x["shapes"])
        assert float(x["audio"]) == pytest.approx(float(x["lens"].sum()) * 0.01)
    assert not np.array_equal(r[0]["lens"], r[1]["lens"])  # different seeds, different segments
    # whole-job figures agree on every rank: slowest times, summed audio
    for x in r:
        assert float(x["t_max"]) == 2.0
        assert float(x["te2e_max"]) == 10.0
        assert float(x["audio_total"]) == pytest.approx(float(r[0]["audio"]) + float(r[1]["audio"]))


def test_single_process_reduction_is_identity():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.reduce_over_ranks(1.5, 2.5, 30.0, None, "cpu") == (1.5, 2.5, 30.0)
