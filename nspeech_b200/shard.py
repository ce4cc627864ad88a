"""Splitting one batched-encoder job over GPUs, one process per GPU.

VAD segments are independent through the encoder: the reference encodes
them one at a time, batch 1 (src/parakeet/transducer.rs:387). So a job of
segments splits over GPUs with no exchange on the data path:

1. ``length_buckets`` sorts the segments by frame count (stable) and cuts
   runs of at most ``max_batch``. Each bucket is padded to its longest
   member, as ``nq_encoder_forward`` takes it.
2. ``bucket_cost`` estimates a bucket's device time:
   B x T x (1 + ATTN_PER_FRAME x T), with T the padded encoder frames.
   - The first term is the per-token work: Q8_0 GEMMs, LayerNorm, convs.
   - The second is attention, which grows as T^2.
   - ``ATTN_PER_FRAME`` comes from one B200 step of the configs[4] workload
     with the tcgen05 attention kernel: attention ~40 ms of 447 ms, with
     sum(B T) = 216,032 and sum(B T^2) = 56.0 M.
3. ``assign_lpt`` is greedy longest-processing-time. Buckets go out in
   decreasing cost, each to the rank with the least cost so far; ties go to
   the lower rank, and equal costs keep the lower bucket index first. It is
   deterministic, so every rank computes the same assignment from the same
   segment list without talking to the others.
4. ``gather_segments`` moves the per-segment results (encoder frames or
   argmax tokens) to one rank over ``torch.distributed`` after the job. This
   is the only cross-rank traffic.
"""
from __future__ import annotations

import heapq
from typing import Dict, List, Optional, Sequence

ATTN_PER_FRAME = 3.8e-4


def encoder_frames(mel_frames: int) -> int:
    """Encoder frames of a segment of ``mel_frames`` log-mel frames.

    There are three stride-2 convs (kernel 3, pad 1); this matches
    ``nq_encoder_out_frames``.
    """
    t = int(mel_frames)
    for _ in range(3):
        t = (t - 1) // 2 + 1
    return t


def length_buckets(frames: Sequence[int], max_batch: int) -> List[List[int]]:
    """Segment indices in length-sorted runs of at most ``max_batch``."""
    if max_batch < 1:
        raise ValueError("max_batch must be >= 1")
    order = sorted(range(len(frames)), key=lambda i: (int(frames[i]), i))
    return [order[i:i + max_batch] for i in range(0, len(order), max_batch)]


def bucket_cost(frames: Sequence[int], bucket: Sequence[int], attn_per_frame: float = ATTN_PER_FRAME) -> float:
    """Estimated device time of one padded bucket, in per-token-work units."""
    if not bucket:
        return 0.0
    t = encoder_frames(max(int(frames[i]) for i in bucket))
    return len(bucket) * t * (1.0 + attn_per_frame * t)


def assign_lpt(costs: Sequence[float], n_ranks: int) -> List[List[int]]:
    """Bucket indices per rank; greedy longest-processing-time, deterministic."""
    if n_ranks < 1:
        raise ValueError("n_ranks must be >= 1")
    out: List[List[int]] = [[] for _ in range(n_ranks)]
    heap = [(0.0, r) for r in range(n_ranks)]  # (assigned cost, rank)
    for b in sorted(range(len(costs)), key=lambda i: (-float(costs[i]), i)):
        load, r = heapq.heappop(heap)
        out[r].append(b)
        heapq.heappush(heap, (load + float(costs[b]), r))
    return out


def shard_segments(frames: Sequence[int], max_batch: int, n_ranks: int, rank: int,
                   attn_per_frame: float = ATTN_PER_FRAME) -> List[List[int]]:
    """This rank's buckets (lists of segment indices), in bucket order."""
    if not 0 <= rank < n_ranks:
        raise ValueError("rank out of range")
    buckets = length_buckets(frames, max_batch)
    costs = [bucket_cost(frames, b, attn_per_frame) for b in buckets]
    mine = sorted(assign_lpt(costs, n_ranks)[rank])
    return [buckets[i] for i in mine]


def imbalance(frames: Sequence[int], max_batch: int, n_ranks: int,
              attn_per_frame: float = ATTN_PER_FRAME) -> float:
    """Largest rank cost / mean rank cost of the assignment (1.0 = balanced)."""
    buckets = length_buckets(frames, max_batch)
    costs = [bucket_cost(frames, b, attn_per_frame) for b in buckets]
    loads = [sum(costs[i] for i in part) for part in assign_lpt(costs, n_ranks)]
    mean = sum(loads) / n_ranks
    return max(loads) / mean if mean > 0 else 1.0


def gather_segments(results: Dict[int, object], dist=None, dst: int = 0) -> Optional[Dict[int, object]]:
    """Per-segment results of every rank, merged on rank ``dst``.

    ``results`` maps segment index -> result (any picklable object, e.g. a
    numpy array of encoder frames or argmax tokens). Rank ``dst`` gets the
    union and every other rank gets None. A segment index produced by two
    ranks raises ValueError on ``dst``. Without a process group (``dist`` None
    or not initialised), the input comes back as is.
    """
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return dict(results)
    world, rank = dist.get_world_size(), dist.get_rank()
    parts = [None] * world if rank == dst else None
    dist.gather_object(dict(results), parts, dst=dst)
    if rank != dst:
        return None
    merged: Dict[int, object] = {}
    for part in parts:
        for k, v in part.items():
            if k in merged:
                raise ValueError(f"segment {k} produced by two ranks")
            merged[k] = v
    return merged
