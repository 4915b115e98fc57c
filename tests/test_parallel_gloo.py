"""World-size-2 gloo tests (CPU) of the multi-GPU host logic: sequence sharding, the bootstrap of the engines'
NCCL token-exchange communicator (rank 0's id reaches every rank intact), max-over-ranks timing, and a rank
that fails before joining a step. The all-gather itself is NCCL on the GPUs (qwen_engine_gather_tokens) and is
exercised by bench.py --gpus N and the 2-GPU test in tests/test_gpu_multi.py."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from work_llm_accelerator_b200.parallel import connect_engine, max_over_ranks, shard_range


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank: int, world: int, port: int, mode: str, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        if mode == "gather":
            start, stop = shard_range(8, world, rank)
            uid = connect_engine(None, world, rank)  # the NCCL id made on rank 0, as every rank receives it
            slow = max_over_ranks([1.0 + rank, 5.0 - rank])
            q.put((rank, (start, stop), uid, slow))
        elif mode == "fail":
            if rank == 1:
                raise SystemExit(3)  # leaves before the step's collective
            try:
                max_over_ranks([1.0])
                q.put((rank, "no-error"))
            except Exception as exc:  # the peer's absence surfaces as an error, not a hang
                q.put((rank, type(exc).__name__))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _run(mode: str, world: int = 2, timeout: float = 90.0):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    for p in procs:
        p.join(timeout)
    for p in procs:
        if p.is_alive():
            p.kill()
    while not q.empty():
        results.append(q.get())
    return procs, results


def test_shard_range_covers_everything():
    for total in (0, 1, 7, 64):
        for world in (1, 2, 3, 8):
            spans = [shard_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_id_exchange_and_max_world2():
    procs, results = _run("gather")
    assert all(p.exitcode == 0 for p in procs)
    results = dict((r[0], r[1:]) for r in results)
    assert results[0][0] == (0, 4) and results[1][0] == (4, 8)
    assert len(results[0][1]) == 128 and results[0][1] == results[1][1]
    for rank in (0, 1):
        assert results[rank][2] == [2.0, 5.0]


def test_rank_failure_is_an_error_not_a_hang():
    procs, results = _run("fail", timeout=120.0)
    assert procs[1].exitcode == 3
    survivors = [r for r in results if r[0] == 0]
    assert procs[0].exitcode is not None  # did not hang past the join timeout
    if survivors:
        assert survivors[0][1] != "no-error"
