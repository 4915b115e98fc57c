"""The engines' NCCL token exchange (qwen_engine_nccl_init / qwen_engine_gather_tokens) on GPUs.

- One GPU: a one-rank communicator; the gather copies the step's ids through NCCL unchanged.
- Two GPUs (when the box has them): one process and one engine per GPU, each decoding its own sequence; after
  every step the engines all-gather the next-token ids and both ranks must see [rank 0's id, rank 1's id], each
  equal to what that rank decoded. NVLS is off (NCCL_NVLS_ENABLE=0), no kernel of the engine touches a peer's
  memory.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def host(built_libs, gpu_available):
    if not gpu_available:
        pytest.fail("no CUDA device: the -m gpu suite must run on a B200")
    from work_llm_accelerator_b200 import host as h

    return h


def test_single_rank_gather(host):
    import torch

    eng = host.Engine(0, 8, max_seqs=1, max_len=64)
    try:
        eng.nccl_init(host.nccl_unique_id(), 1, 0)
        eng.init_synthetic(3)
        first = eng.prefill(0, [1, 2, 3, 4])
        cur = torch.tensor([first], dtype=torch.int32, device="cuda")
        nxt = torch.zeros(1, dtype=torch.int32, device="cuda")
        allv = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        eng.decode_device([0], cur.data_ptr(), nxt.data_ptr())
        eng.gather_tokens(nxt.data_ptr(), 1, allv.data_ptr())
        torch.cuda.synchronize()
        assert int(allv.item()) == int(nxt.item())
        with pytest.raises(host.EngineError):
            eng.nccl_init(host.nccl_unique_id(), 1, 0)  # one communicator per engine
    finally:
        eng.close()


def test_single_rank_async_gather(host):
    """The side-stream gather (qwen_engine_gather_tokens_async) beside the following steps, with the batch-1
    kernel on 146 CTAs (two SMs free): after the join, every step's gathered id equals the id the step wrote,
    and the tokens equal the synchronous loop's."""
    import torch

    def run(async_gather: bool):
        eng = host.Engine(0, 8, max_seqs=1, max_len=64)
        try:
            eng.nccl_init(host.nccl_unique_id(), 1, 0)
            eng.init_synthetic(3)
            if async_gather:
                eng.set_option("bs1_ctas", 146)
            first = eng.prefill(0, [1, 2, 3, 4])
            bufs = [torch.tensor([first], dtype=torch.int32, device="cuda"), torch.zeros(1, dtype=torch.int32, device="cuda")]
            seen = torch.full((6,), -1, dtype=torch.int32, device="cuda")
            stream = torch.cuda.ExternalStream(eng.stream())
            with torch.cuda.stream(stream):
                for i in range(6):
                    eng.decode_device([0], bufs[i % 2].data_ptr(), bufs[(i + 1) % 2].data_ptr())
                    if async_gather:
                        eng.gather_tokens_async(bufs[(i + 1) % 2].data_ptr(), 1, seen[i:].data_ptr())
                    else:
                        eng.gather_tokens(bufs[(i + 1) % 2].data_ptr(), 1, seen[i:].data_ptr())
                if async_gather:
                    eng.gather_join()
            torch.cuda.synchronize()
            assert host.kernel_error(reset=True) == 0
            return seen.cpu().tolist()
        finally:
            torch.cuda.synchronize()
            eng.close()

    assert run(True) == run(False)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank: int, world: int, port: int, q) -> None:
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    os.environ["QWEN_B200_DEVICE"] = str(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from work_llm_accelerator_b200 import host
    from work_llm_accelerator_b200.parallel import connect_engine

    eng = host.Engine(rank, 8, max_seqs=1, max_len=64)
    try:
        connect_engine(eng, world, rank)
        eng.init_synthetic(7)
        first = eng.prefill(0, [10 + rank, 20, 30, 40, 50 + 3 * rank])
        cur = torch.tensor([first], dtype=torch.int32, device="cuda")
        nxt = torch.zeros(1, dtype=torch.int32, device="cuda")
        allv = torch.zeros(world, dtype=torch.int32, device="cuda")
        own, seen = [], []
        for _ in range(4):
            eng.decode_device([0], cur.data_ptr(), nxt.data_ptr())
            eng.gather_tokens(nxt.data_ptr(), 1, allv.data_ptr())
            torch.cuda.synchronize()
            own.append(int(nxt.item()))
            seen.append(allv.cpu().tolist())
            cur.copy_(nxt)
        # the side-stream gathers beside the steps (the bench's multi-GPU loop), batch-1 kernel on 146 CTAs
        eng.set_option("bs1_ctas", 146)
        bufs = [cur.clone(), torch.zeros(1, dtype=torch.int32, device="cuda")]
        allk = torch.full((4, world), -1, dtype=torch.int32, device="cuda")
        stream = torch.cuda.ExternalStream(eng.stream())
        with torch.cuda.stream(stream):
            for i in range(4):
                eng.decode_device([0], bufs[i % 2].data_ptr(), bufs[(i + 1) % 2].data_ptr())
                own.append(None)  # filled below
                eng.gather_tokens_async(bufs[(i + 1) % 2].data_ptr(), 1, allk[i].data_ptr())
            eng.gather_join()
        torch.cuda.synchronize()
        seen += allk.cpu().tolist()
        q.put((rank, own, seen))
    finally:
        torch.cuda.synchronize()
        eng.close()
        dist.destroy_process_group()


def test_two_gpu_token_gather(host):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs)
    res = {}
    while not q.empty():
        r, own, seen = q.get()
        res[r] = (own, seen)
    assert sorted(res) == [0, 1]
    for step in range(4):
        want = [res[0][0][step], res[1][0][step]]
        assert res[0][1][step] == want and res[1][1][step] == want
    # asynchronous gathers: both ranks see the same ids, each rank's own id in its column
    for step in range(4, 8):
        assert res[0][1][step] == res[1][1][step]
        assert all(v >= 0 for v in res[0][1][step])
