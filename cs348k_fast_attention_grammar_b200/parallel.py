"""Batch x head data parallelism over the GPUs of one node.

(batch, head) pairs are independent, so the flattened ``B*H`` range is split
into contiguous, equal blocks, one per rank; each rank generates its own shard
from the seed (``inputs.make_qkv``), runs the kernel on it with no collective
in the data path, and only afterwards

* ``gather_shards`` collects the O shards on rank 0 (NCCL gather), and
* ``reduce_error_stats`` combines the per-rank verification statistics
  (MAX of max-abs-error, SUM of abs-error sum and element count).

The reference has no multi-GPU code; this is the sharding BASELINE asks for.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(num_pairs: int, world: int, rank: int) -> range:
    """Contiguous block of flattened pairs owned by ``rank``."""
    if num_pairs % world != 0:
        base, extra = divmod(num_pairs, world)
        start = rank * base + min(rank, extra)
        return range(start, start + base + (1 if rank < extra else 0))
    per = num_pairs // world
    return range(rank * per, (rank + 1) * per)


def owner_of(pair: int, num_pairs: int, world: int) -> int:
    for r in range(world):
        if pair in shard_range(num_pairs, world, r):
            return r
    raise ValueError(pair)


def verify_pairs(num_pairs: int, count: int, seed: int = 1234) -> list[int]:
    """Seeded random subset of pairs checked against the fp32 reference."""
    g = torch.Generator().manual_seed(seed)
    count = min(count, num_pairs)
    return sorted(torch.randperm(num_pairs, generator=g)[:count].tolist())


def gather_shards(local: torch.Tensor, world: int, rank: int, num_pairs: int):
    """Gather every rank's ``[1, pairs_r, S, D]`` shard into one
    ``[1, num_pairs, S, D]`` tensor on rank 0 (None elsewhere)."""
    if world == 1:
        return local
    sizes = [len(shard_range(num_pairs, world, r)) for r in range(world)]
    if len(set(sizes)) != 1:
        raise ValueError("gather_shards needs equal shard sizes")
    if rank == 0:
        bufs = [torch.empty_like(local) for _ in range(world)]
        dist.gather(local, gather_list=bufs, dst=0)
        return torch.cat(bufs, dim=1)
    dist.gather(local, dst=0)
    return None


def reduce_error_stats(max_abs: float, sum_abs: float, count: int, device) -> dict:
    """All-reduce (MAX, SUM, SUM) of per-rank verification statistics."""
    mx = torch.tensor([max_abs], dtype=torch.float64, device=device)
    sc = torch.tensor([sum_abs, float(count)], dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(sc, op=dist.ReduceOp.SUM)
    n = sc[1].item()
    return {"max_abs": mx.item(), "mean_abs": (sc[0].item() / n) if n else 0.0,
            "elements": int(n)}
