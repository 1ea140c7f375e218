"""Sharding draft requests across GPUs (one process per GPU).

The draft forward has no cross-request dependency. Every rank therefore holds
a full weight replica and drafts its own sequences, and nothing is exchanged on
the data path. Weights fit easily (about 3.5 GB at 27B dims), and tensor
parallelism would add two all-reduces per layer for no gain.

Collectives appear only around the data path:
- the max of per-rank device times, which gives whole-job throughput;
- host-side gathering of per-request results (acceptance lengths, ids).

This matches the reference's serving loop, which handles requests
independently (mirror_sd/generate.py).

``shard_requests`` is deterministic. Every rank computes the same plan with no
communication: longest context first, each request to the least-loaded rank,
where load is context rows plus block rows.
"""
from typing import List, Optional, Sequence

import torch
import torch.distributed as dist


def shard_requests(ctx_lens: Sequence[int], world: int, rank: int, block: int = 0) -> List[int]:
    """Indices of the requests rank ``rank`` drafts, in ascending order.

    Each request costs ``ctx + block`` rows (fc + context K/V GEMMs scale with
    ctx, the block path with block).  Longest-processing-time greedy: requests
    sorted by cost (descending, ties by index) go to the least-loaded rank
    (ties to the lowest rank).  Every request lands on exactly one rank."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    order = sorted(range(len(ctx_lens)), key=lambda i: (-(int(ctx_lens[i]) + block), i))
    load = [0] * world
    mine = []
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        load[r] += int(ctx_lens[i]) + block
        if r == rank:
            mine.append(i)
    return sorted(mine)


def _reduce_device():
    if dist.is_initialized() and dist.get_backend() == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def max_over_ranks(value: float) -> float:
    """Max of ``value`` over all ranks (the step time that bounds the job);
    ``value`` itself without an initialised process group."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=_reduce_device())
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_to_rank0(obj) -> Optional[list]:
    """Host-side gather of per-rank results (list in rank order on rank 0,
    None elsewhere)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return [obj]
    out = [None] * dist.get_world_size() if dist.get_rank() == 0 else None
    dist.gather_object(obj, out, dst=0)
    return out


def job_throughput(tokens_per_rank: Sequence[int], step_ms_max: float) -> float:
    """Whole-job draft tokens per second: all ranks' tokens over the slowest
    rank's step time (weak scaling: per-rank work is fixed)."""
    return float(sum(tokens_per_rank)) / (step_ms_max / 1e3)
