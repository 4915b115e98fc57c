"""The allocation-free decode attention entry point (qwen_b200_decode_attention_noalloc) against the
allocating one (qwen_b200_decode_attention), through the C-ABI, on two calls in a row.

Some host programs cannot call cudaMalloc when they run attention: runtimes that reserve all GPU memory in
their own pool at start-up, or latency-critical loops where an allocation would synchronise the device.
The no-allocation entry point serves them from a fixed scratch array inside the library, limited to
histories of 8192 tokens. This file sorts last so that a run stopping at the first failure has already run
every other test; it also passes on its own in a fresh process.
"""
from __future__ import annotations

import ctypes

import pytest

pytestmark = pytest.mark.gpu



def _entry_points():
    from work_llm_accelerator_b200 import host

    lib = host.core_lib()
    fn = lib.qwen_b200_decode_attention_noalloc
    fn.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return host, lib.qwen_b200_decode_attention, fn


def test_noalloc_matches_allocating_entry_point(built_libs, gpu_available):
    import torch

    if not gpu_available:
        pytest.fail("no CUDA device: the -m gpu suite must run on a B200")
    host, alloc_fn, noalloc_fn = _entry_points()
    stream = torch.cuda.current_stream().cuda_stream
    # calls in a row: the history limit itself (the scratch array is sized exactly for it), then shorter
    # histories, so leftovers of an earlier call would show
    for seq_len, seed in ((8192, 3), (700, 1), (65, 2)):
        g = torch.Generator(device="cpu").manual_seed(seed)
        q = torch.randn(1536, generator=g).cuda()
        k = torch.randn(seq_len * 256, generator=g).cuda()
        v = torch.randn(seq_len * 256, generator=g).cuda()
        ctx_alloc = torch.zeros(1536, device="cuda")
        ctx_noalloc = torch.full((1536,), float("nan"), device="cuda")
        assert alloc_fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), seq_len, ctx_alloc.data_ptr(), stream) == 0, \
            host.last_error()
        assert noalloc_fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), seq_len, ctx_noalloc.data_ptr(), stream) == 0, \
            host.last_error()
        torch.cuda.synchronize()
        assert host.kernel_error(reset=True) == 0  # no bounded wait gave up
        # the same kernel on the same inputs: identical results, not merely close ones
        assert torch.equal(ctx_noalloc, ctx_alloc), (seq_len, float((ctx_noalloc - ctx_alloc).abs().max()))


def test_noalloc_rejects_histories_beyond_its_scratch(built_libs, gpu_available):
    import torch

    if not gpu_available:
        pytest.fail("no CUDA device: the -m gpu suite must run on a B200")
    host, _, noalloc_fn = _entry_points()
    q = torch.zeros(1536, device="cuda")
    k = torch.zeros(8193 * 256, device="cuda")
    ctx = torch.zeros(1536, device="cuda")
    st = noalloc_fn(q.data_ptr(), k.data_ptr(), k.data_ptr(), 8193, ctx.data_ptr(),
                    torch.cuda.current_stream().cuda_stream)
    assert st == 1
    assert "8192" in host.last_error()
    # a misaligned buffer is an argument error that names the buffer
    st = noalloc_fn(q.data_ptr() + 4, k.data_ptr(), k.data_ptr(), 16, ctx.data_ptr(),
                    torch.cuda.current_stream().cuda_stream)
    assert st == 1 and "q is not 16-byte aligned" in host.last_error()
