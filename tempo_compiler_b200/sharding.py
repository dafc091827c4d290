"""Sequence sharding across GPUs: independent sequences, full weight replicas, no collective on the data path.

The batched workload is 512 independent sequences. Rank r of N takes a contiguous run of them; the only
communication is timing (a barrier and a max over ranks) and, optionally, gathering the generated tokens on rank 0
at the end. The same functions run on NCCL (one process per GPU) and on gloo (the CPU tests).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard(total: int, world: int, rank: int) -> tuple[int, int]:
    """The [first, first + count) sequences rank `rank` of `world` owns; the first `total % world` ranks take one
    extra, so every sequence is owned exactly once."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    base, extra = divmod(total, world)
    count = base + (1 if rank < extra else 0)
    first = rank * base + min(rank, extra)
    return first, count


def max_over_ranks(value: float, device: torch.device | str = "cpu") -> float:
    """The maximum of `value` over all ranks (the job's time is the slowest rank's)."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_tokens(tokens: torch.Tensor, total: int, device: torch.device | str = "cpu") -> torch.Tensor | None:
    """Collects every rank's [count, steps] token block into one [total, steps] tensor on rank 0 (None elsewhere).

    Blocks are padded to the largest shard for the collective and trimmed afterwards."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return tokens
    world, rank = dist.get_world_size(), dist.get_rank()
    widest = shard(total, world, 0)[1]
    padded = torch.zeros((widest, tokens.shape[1]), dtype=tokens.dtype, device=device)
    padded[: tokens.shape[0]] = tokens.to(device)
    blocks = [torch.empty_like(padded) for _ in range(world)] if rank == 0 else None
    dist.gather(padded, blocks, dst=0)
    if rank != 0:
        return None
    return torch.cat([blocks[r][: shard(total, world, r)[1]] for r in range(world)])
