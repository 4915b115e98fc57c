"""Sequence-level data parallelism: one process and one engine per GPU, each holding a full replica of the
weights and the KV cache of its own share of the independent sequences. The only collective is the per-step
all-gather of next-token ids, issued by the engine itself from C++ (qwen_engine_gather_tokens: ncclAllGather
on the engine's stream, over NVLink / NVSwitch). This module is the host-side bootstrap around it:
- shard_range: which sequences a rank owns;
- connect_engine: the NCCL communicator id made on rank 0 and handed to every rank's engine through the
  launcher's torch.distributed group (the bootstrap only: no data-path traffic goes through torch);
- max_over_ranks: multi-GPU timings are reported as the slowest rank.
The reference has no parallel runtime; this is the "independent sequences are partitioned across GPUs" part
of the target.
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


def broadcast_bytes(data: bytes | None, src: int = 0, device: torch.device | str = "cpu") -> bytes:
    """`data` from rank `src` on every rank, over the default torch.distributed group (gloo or nccl)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        if data is None:
            raise ValueError("single rank: nothing to receive")
        return data
    n = torch.tensor([len(data) if dist.get_rank() == src else 0], dtype=torch.int64, device=device)
    dist.broadcast(n, src)
    buf = torch.zeros(int(n.item()), dtype=torch.uint8, device=device)
    if dist.get_rank() == src:
        buf.copy_(torch.frombuffer(bytearray(data), dtype=torch.uint8))
    dist.broadcast(buf, src)
    return bytes(buf.cpu().tolist())


def connect_engine(engine, world: int, rank: int, device: torch.device | str = "cpu") -> bytes:
    """Give `engine` (host.Engine) its token-exchange communicator: rank 0 makes the NCCL id, every rank joins.
    Returns the id (for tests)."""
    from . import host

    uid = host.nccl_unique_id() if rank == 0 else None
    uid = broadcast_bytes(uid, 0, device)
    if engine is not None:
        engine.nccl_init(uid, world, rank)
    return uid


def max_over_ranks(values: list[float], device: torch.device | str = "cpu") -> list[float]:
    """Element-wise maximum over ranks (timings are reported as the slowest rank)."""
    t = torch.tensor(values, dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t]
