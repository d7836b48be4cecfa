"""Utterance sharding across GPUs (one process per GPU, no collective on the
data path).

Utterances are independent, so a multi-GPU job partitions them: each rank
runs its share through its own context (itts_cfm_run_batch buckets them by
length) and keeps its outputs. The partition balances the sampler's
algorithmic cost per utterance, F(T) = 294.09e6*T + 53,248*T^2 FLOP per
guided step, with a deterministic longest-processing-time assignment so that
every rank computes the same partition without communicating.
"""
from __future__ import annotations

from typing import Callable, Sequence


def utterance_cost(T: int) -> float:
    """Algorithmic FLOPs of one guided CFM step for an utterance of T frames."""
    return 2 * 2 * 73_523_200.0 * T + 2 * 13 * 4 * 512.0 * T * T


def shard(lengths: Sequence[int], world: int) -> list[list[int]]:
    """Assign utterance indices to `world` ranks, balancing utterance_cost.

    Longest-processing-time first: utterances sorted by cost (ties by index)
    go to the currently least-loaded rank (ties by rank id). Within a rank,
    indices are returned sorted by length so its buckets are contiguous.
    """
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(lengths)), key=lambda i: (-utterance_cost(lengths[i]), i))
    load = [0.0] * world
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        parts[r].append(i)
        load[r] += utterance_cost(lengths[i])
    return [sorted(p, key=lambda i: (lengths[i], i)) for p in parts]


def imbalance(lengths: Sequence[int], parts: list[list[int]]) -> float:
    """max rank cost / mean rank cost (1.0 = perfect balance)."""
    costs = [sum(utterance_cost(lengths[i]) for i in p) for p in parts]
    mean = sum(costs) / len(costs)
    return max(costs) / mean if mean else 1.0


def run_sharded(utts: Sequence[dict], rank: int, world: int, run_batch: Callable[[list[dict]], list]) -> dict[int, object]:
    """Run this rank's share with `run_batch` (e.g. Context.run_batch bound to
    steps/cfg) and return {utterance index: output} for the local share."""
    mine = shard([u["noise"].shape[0] for u in utts], world)[rank]
    if not mine:
        return {}
    outs = run_batch([utts[i] for i in mine])
    return dict(zip(mine, outs))
