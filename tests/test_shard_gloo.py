"""Multi-process host logic on CPU (gloo, world size 2): batch shares cover the batch
exactly once, and the reported time is the max over ranks."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from krea2_svdquant_b200.shard import max_over_ranks, shard_range


def test_shard_range_partitions():
    for total in (0, 1, 7, 8, 9, 33):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for r in range(world):
                s, c = shard_range(total, world, r)
                seen += list(range(s, s + c))
            assert seen == list(range(total))
            counts = [shard_range(total, world, r)[1] for r in range(world)]
            assert max(counts) - min(counts) <= 1
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


def test_max_over_ranks_single_process():
    assert max_over_ranks(3.5) == 3.5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        start, count = shard_range(8, world, rank)
        images = torch.arange(8)[start:start + count]
        # each rank "processes" its images: a per-rank time that differs between ranks
        t = max_over_ranks(10.0 + rank)
        total = torch.tensor([int(images.numel())])
        dist.all_reduce(total)
        out.put((rank, images.tolist(), t, int(total.item())))
    finally:
        dist.destroy_process_group()


def test_gloo_world2_shards_and_max():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][1] == [0, 1, 2, 3] and res[1][1] == [4, 5, 6, 7]
    assert all(r[2] == 11.0 for r in res)
    assert all(r[3] == 8 for r in res)
