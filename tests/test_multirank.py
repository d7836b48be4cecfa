"""Multi-rank host logic on CPU: utterance sharding with world_size 2 over the
gloo backend (the path bench.py takes under torchrun, minus the GPU work)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

import shard
import workloads as W


def test_shard_partition_is_exact_and_balanced():
    lengths = [u.T for u in W.config_utterances(3)]
    for world in (1, 2, 4, 8):
        parts = shard.shard(lengths, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(len(lengths)))
        assert shard.imbalance(lengths, parts) < 1.05
    assert shard.shard([800] * 1024, 8) == shard.shard([800] * 1024, 8)  # deterministic
    assert all(len(p) == 128 for p in shard.shard([800] * 1024, 8))


def test_run_sharded_maps_outputs_to_indices():
    utts = [dict(noise=np.zeros((t, 80), np.float32)) for t in (30, 10, 20, 40, 50)]
    got = {}
    for rank in range(2):
        got.update(shard.run_sharded(utts, rank, 2, lambda us: [u["noise"].shape[0] for u in us]))
    assert got == {i: u["noise"].shape[0] for i, u in enumerate(utts)}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lengths = [u.T for u in W.config_utterances(3)]
    mine = shard.shard(lengths, world)[rank]
    # every rank derives the same partition independently; check by gathering
    got = [None] * world
    dist.all_gather_object(got, mine)
    # max-over-ranks timing reduction used by bench.py
    t = torch.tensor([float(rank + 1)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, got, float(t.item())))


@pytest.mark.timeout(120)
def test_gloo_two_ranks_agree_on_partition():
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=110) for _ in range(2)]
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    lengths = [u.T for u in W.config_utterances(3)]
    want = shard.shard(lengths, 2)
    for rank, got, tmax in res:
        assert got == want
        assert tmax == 2.0
