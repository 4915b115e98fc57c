"""GPU test of the device-pointer operator API (include/qwen_b200_ops.h) against a plain PyTorch fp32
reference of the same op: softmax(q k^T / sqrt(128)) v per query head, 6 query heads per KV head."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-5


def torch_reference(q, k, v):
    import torch

    L = k.numel() // 256
    qh = q.view(12, 128).double()
    kh = k.view(L, 2, 128).double()
    vh = v.view(L, 2, 128).double()
    out = torch.empty(12, 128, dtype=torch.float64, device=q.device)
    for h in range(12):
        g = h // 6
        s = (kh[:, g, :] @ qh[h]) * np.float32(1.0 / np.sqrt(128.0))
        p = torch.softmax(s, dim=0)
        out[h] = p @ vh[:, g, :]
    return out.view(-1).float()


@pytest.mark.parametrize("seq_len", [1, 63, 64, 65, 513, 2048, 4096, 32768])  # 32768: the maximum (512 chunks)
def test_decode_attention_op_matches_torch(built_libs, gpu_available, seq_len):
    import torch

    if not gpu_available:
        pytest.fail("no CUDA device")
    from work_llm_accelerator_b200 import host

    g = torch.Generator(device="cpu").manual_seed(seq_len)
    q = torch.randn(1536, generator=g).cuda()
    k = torch.randn(seq_len * 256, generator=g).cuda()
    v = torch.randn(seq_len * 256, generator=g).cuda()
    ctx = torch.zeros(1536, device="cuda")
    host.decode_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), seq_len, ctx.data_ptr(),
                          torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ref = torch_reference(q, k, v)
    err = float((ctx - ref).norm() / ref.norm())
    assert err <= TOL, err


def test_decode_attention_op_rejects_host_memory(built_libs, gpu_available):
    if not gpu_available:
        pytest.fail("no CUDA device")
    from work_llm_accelerator_b200 import host

    a = np.zeros(1536 * 4, np.float32)
    with pytest.raises(host.EngineError):
        host.decode_attention(a.ctypes.data, a.ctypes.data, a.ctypes.data, 2, a.ctypes.data)
