"""The multi-GPU host logic on CPU: contiguous sequence shards cover the job exactly once, the job time is the slowest
rank's, and the generated tokens gather back in sequence order. Two gloo ranks stand in for two GPUs."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tempo_compiler_b200.sharding import gather_tokens, max_over_ranks, shard


@pytest.mark.parametrize(("total", "world"), [(512, 1), (512, 2), (512, 8), (7, 3), (3, 4)])
def test_shards_cover_every_sequence_once(total: int, world: int) -> None:
    owned = []
    for rank in range(world):
        first, count = shard(total, world, rank)
        owned.extend(range(first, first + count))
    assert owned == list(range(total))
    with pytest.raises(ValueError):
        shard(total, world, world)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, total: int, results) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        first, count = shard(total, world, rank)
        # each rank's "generated tokens" are a function of the global sequence index
        tokens = torch.stack([torch.arange(5, dtype=torch.int32) + 100 * s for s in range(first, first + count)])
        slowest = max_over_ranks(1.5 + rank)
        gathered = gather_tokens(tokens, total)
        if rank == 0:
            results["slowest"] = slowest
            results["gathered"] = gathered.tolist()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("total", [8, 7])
def test_two_gloo_ranks_time_and_gather(total: int) -> None:
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, total, results), nprocs=2, join=True, start_method="spawn")
    assert results["slowest"] == 2.5
    expected = [[100 * s + i for i in range(5)] for s in range(total)]
    assert results["gathered"] == expected
