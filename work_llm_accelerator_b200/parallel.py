"""Sequence-level data parallelism: one process per GPU, independent sequences per rank, and the single
collective of the design -- an all-gather of each step's next-token ids (NCCL over NVLink on the GPU box;
gloo in the CPU tests). The reference has no parallel runtime; this is the "independent sequences are
partitioned across GPUs" part of the target.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, stop) share of `total` sequences for `rank` (earlier ranks take the remainder)."""
    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError("bad shard request")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather_tokens(local: torch.Tensor, world: int) -> torch.Tensor:
    """All-gather equally sized int32 token vectors from every rank into [world * n] (rank-major)."""
    if world == 1:
        return local.clone()
    out = torch.empty(world * local.numel(), dtype=local.dtype, device=local.device)
    if dist.get_backend() == "nccl":
        dist.all_gather_into_tensor(out, local.contiguous())
    else:
        parts = list(out.chunk(world))
        dist.all_gather(parts, local.contiguous())
        out = torch.cat(parts)
    return out


def max_over_ranks(values: list[float], device: torch.device | str = "cpu") -> list[float]:
    """Element-wise maximum over ranks (timings are reported as the slowest rank)."""
    t = torch.tensor(values, dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t]
