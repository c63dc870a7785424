"""Multi-GPU plumbing: one process per GPU, independent inferences per rank.

The lowered-op path has no cross-inference reduction, so N GPUs run N full
weight replicas on disjoint work ("replicas only"): either whole
inferences per rank (weak scaling, what the benchmark does) or contiguous
batch rows of one inference per rank through ``emx_b200_run``'s
``batch_begin/batch_count`` (strong scaling).  No collective touches the data
path; ``torch.distributed`` (NCCL on GPUs, gloo in the CPU tests) is used only
for barriers and for reducing timings.
"""
from __future__ import annotations

import hashlib
import os


def world() -> tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def shard_rows(batch: int, world_size: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced split of `batch` rows: (batch_begin, batch_count)."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError("bad rank/world")
    base, extra = divmod(batch, world_size)
    begin = rank * base + min(rank, extra)
    return begin, base + (1 if rank < extra else 0)


def replica_seed(rank: int, base: int = 0) -> int:
    """Input seed of a rank's independent inferences."""
    return base + rank


def plan_digest(plan_bytes: bytes, weight_bytes: bytes) -> str:
    return hashlib.sha256(plan_bytes + b"|" + weight_bytes).hexdigest()


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank scalar (timing) across the default process group."""
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def check_same_plan(plan_bytes: bytes, weight_bytes: bytes, device=None) -> bool:
    """True when every rank emitted a byte-identical plan (replicas must agree)."""
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return True
    d = int(plan_digest(plan_bytes, weight_bytes)[:15], 16)
    t = torch.tensor([d, -d], dtype=torch.int64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return int(t[0].item()) == d and int(t[1].item()) == -d
