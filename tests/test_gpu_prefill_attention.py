"""GPU tests of the tensor-core prefill attention (include/qwen_b200_ops.h qwen_b200_prefill_attention).

The reference's prefill context (hls/prefill_only/qwen_prefill_attention_kernel.cpp:204-289) is two passes
over the causal keys with approx_exp. The CUDA-core kernel (mode 1) keeps its serial fp32 scores; the
tensor-core kernel (mode 0) computes scores and context from fp16 (hi, lo) operand pairs with fp32
accumulation. Checked here:
  - mode 0 against mode 1 and against a float64 restatement of the reference's algorithm, over ragged
    lengths (tile edges at 64 keys and 128 queries) up to 4096 tokens;
  - the fallback: inputs the fp16 split cannot hold give exactly the CUDA-core result;
  - the exponential the kernels evaluate (approx_exp with exact divisions by constants, no branches) is
    bit-identical to the reference's approx_exp for every float in [-16, 0], every positive finite float,
    and on samples below -16 and the special values.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HEADS, KV_HEADS, HEAD_DIM, HIDDEN, KV_WIDTH = 12, 2, 128, 1536, 256
SCALING = np.float32(0.08838834764831845)
TOL = 1e-5


@pytest.fixture(scope="module")
def cuda(built_libs, gpu_available):
    if not gpu_available:
        pytest.fail("no CUDA device")
    import torch

    return torch


def approx_exp_torch(torch, v):
    """The reference's approx_exp (oracle/qwen_oracle.c, hls/prefill_only/qwen_prefill_attention_kernel.cpp:
    47-110) as float32 tensor operations: each op rounds once (IEEE), divisions are tensor / tensor."""
    live = v > -16.0
    s = v.clone()
    steps = torch.zeros_like(v, dtype=torch.int32)
    for _ in range(5):
        m = s < -1.0
        s = torch.where(m, s * 0.5, s)
        steps += m.to(torch.int32)
    term = torch.ones_like(v)
    series = torch.ones_like(v)
    for d in range(1, 7):
        term = term * (s / torch.full_like(s, float(d)))
        series = series + term
    for i in range(1, 5):
        series = torch.where(steps >= i, series * series, series)
    series = torch.where(series > 0.0, series, torch.zeros_like(series))
    return torch.where(live, series, torch.zeros_like(series))


def approx_exp_np(v: np.ndarray) -> np.ndarray:
    """Same function with numpy float32 arrays (IEEE single, elementwise)."""
    F = np.float32
    v = v.astype(F)
    s = v.copy()
    steps = np.zeros(v.shape, np.int32)
    for _ in range(5):
        m = s < F(-1.0)
        s = np.where(m, s * F(0.5), s).astype(F)
        steps += m
    term = np.ones_like(v)
    series = np.ones_like(v)
    for d in range(1, 7):
        term = (term * (s / F(d))).astype(F)
        series = (series + term).astype(F)
    for i in range(1, 5):
        series = np.where(steps >= i, series * series, series).astype(F)
    series = np.where(series > F(0.0), series, F(0.0)).astype(F)
    return np.where(v > F(-16.0), series, F(0.0)).astype(F)


def reference_context(q: np.ndarray, k: np.ndarray, v: np.ndarray, S: int) -> np.ndarray:
    """The reference's two-pass causal context in float64 (approx_exp on the float32 argument), vectorised
    per query head."""
    qh = q.reshape(S, HEADS, HEAD_DIM).astype(np.float64)
    kh = k.reshape(S, KV_HEADS, HEAD_DIM).astype(np.float64)
    vh = v.reshape(S, KV_HEADS, HEAD_DIM).astype(np.float64)
    out = np.zeros((S, HEADS, HEAD_DIM), np.float64)
    causal = np.tril(np.ones((S, S), bool))
    for h in range(HEADS):
        g = h // (HEADS // KV_HEADS)
        ss = (qh[:, h, :] @ kh[:, g, :].T).astype(np.float32) * SCALING
        ss = np.where(causal, ss, np.float32(-np.inf))
        mx = ss.max(axis=1, keepdims=True)
        e = np.where(causal, approx_exp_np(np.where(causal, ss - mx, 0.0)), 0.0).astype(np.float64)
        den = e.sum(axis=1, keepdims=True)
        out[:, h, :] = (e @ vh[:, g, :]) / den
    return out.reshape(S, HIDDEN)


def run_attention(torch, q, k, v, S, mode):
    from work_llm_accelerator_b200 import host

    ctx = torch.full((S, HIDDEN), float("nan"), device="cuda")
    host.prefill_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), S, ctx.data_ptr(), mode,
                           torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert host.kernel_error(True) == 0
    return ctx


def inputs(torch, S, seed, q_scale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = (torch.randn(S, HIDDEN, generator=g) * q_scale).cuda()
    k = torch.randn(S, KV_WIDTH, generator=g).cuda()
    v = torch.randn(S, KV_WIDTH, generator=g).cuda()
    return q, k, v


def rel(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm())


@pytest.mark.parametrize("S", [1, 5, 63, 64, 65, 127, 128, 129, 200, 383, 1000])
def test_tensor_core_matches_cuda_core_and_reference(cuda, S):
    torch = cuda
    q, k, v = inputs(torch, S, 1000 + S)
    tc = run_attention(torch, q, k, v, S, 0)
    simt = run_attention(torch, q, k, v, S, 1)
    assert torch.isfinite(tc).all()
    assert rel(tc, simt) <= TOL
    ref = torch.from_numpy(reference_context(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), S))
    assert rel(tc.cpu(), ref) <= TOL
    assert rel(simt.cpu(), ref) <= TOL


@pytest.mark.parametrize("S,q_scale", [(2048, 1.0), (4096, 4.0)])
def test_tensor_core_long_sequences(cuda, S, q_scale):
    """Up to the 4096-token prefill config; q_scale 4 makes the softmax peaked (scores spread over tens)."""
    torch = cuda
    q, k, v = inputs(torch, S, S, q_scale)
    tc = run_attention(torch, q, k, v, S, 0)
    simt = run_attention(torch, q, k, v, S, 1)
    assert torch.isfinite(tc).all()
    assert rel(tc, simt) <= TOL
    # per-row check as well: no query row may be off (a row error would hide in a global norm)
    row_err = ((tc - simt).norm(dim=1) / simt.norm(dim=1)).max().item()
    assert row_err <= 1e-4


def test_values_outside_the_split_fall_back_to_cuda_cores(cuda):
    torch = cuda
    S = 150
    q, k, v = inputs(torch, S, 7)
    k[3, 17] = 40000.0  # |x| >= 32768 cannot be held by the fp16 (hi, lo) pair
    tc = run_attention(torch, q, k, v, S, 0)
    simt = run_attention(torch, q, k, v, S, 1)
    assert torch.equal(tc, simt)
    # and a split-safe input again afterwards (the flag is per call)
    k[3, 17] = 1.0
    tc = run_attention(torch, q, k, v, S, 0)
    simt = run_attention(torch, q, k, v, S, 1)
    assert not torch.equal(tc, simt) and rel(tc, simt) <= TOL


def test_prefill_attention_op_rejects_bad_arguments(cuda):
    torch = cuda
    from work_llm_accelerator_b200 import host

    q = torch.zeros(4, HIDDEN, device="cuda")
    kv = torch.zeros(4, KV_WIDTH, device="cuda")
    ctx = torch.zeros(4, HIDDEN, device="cuda")
    with pytest.raises(host.EngineError):
        host.prefill_attention(q.data_ptr(), kv.data_ptr(), kv.data_ptr(), 4, ctx.data_ptr(), 2)
    with pytest.raises(host.EngineError):
        host.prefill_attention(q.data_ptr(), kv.data_ptr(), kv.data_ptr(), 0, ctx.data_ptr(), 0)
    a = np.zeros(HIDDEN * 4, np.float32)
    with pytest.raises(host.EngineError):
        host.prefill_attention(a.ctypes.data, a.ctypes.data, a.ctypes.data, 2, a.ctypes.data, 0)


def test_kernel_exponential_bit_identical_exhaustive(cuda):
    """approx_exp as the kernel evaluates it (divisions by 3, 5, 6 as multiply + FMA correction) against
    the reference's function restated with IEEE divisions: every float in [-16, 0] and every positive
    finite float, bit for bit. The torch restatement itself is pinned to numpy and to the oracle's C
    approx_exp on samples first."""
    torch = cuda
    import qwen_oracle as qo
    from work_llm_accelerator_b200 import host

    rng = np.random.default_rng(5)
    sample = np.concatenate([rng.uniform(-20, 13, 200_000), -np.exp(rng.uniform(-90, 2.8, 50_000)),
                             [-16.0, -15.999999, -8.0, -4.0, -2.0, -1.0, -0.0, 0.0, 1e-40, -1e-40, 88.0, 1e30,
                              -1e30, np.inf, -np.inf, np.nan], -rng.uniform(16, 1e6, 5000)])
    sample = sample.astype(np.float32)
    xs = torch.from_numpy(sample).cuda()
    t_ref = approx_exp_torch(torch, xs).cpu().numpy()
    with np.errstate(all="ignore"):
        assert t_ref.tobytes() == approx_exp_np(sample).tobytes()
    for x in np.concatenate([sample[:: 997], sample[-5021:-5000]]):
        with np.errstate(all="ignore"):
            assert np.float32(qo.approx_exp(float(x))).tobytes() == approx_exp_np(np.array([x]))[0].tobytes(), x
    # the kernel's function on the same sample, special values included (inf, -inf, nan, below -16)
    y = torch.empty_like(xs)
    host.prefill_approx_exp(xs.data_ptr(), y.data_ptr(), xs.numel(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert y.cpu().numpy().tobytes() == t_ref.tobytes()

    def check(lo_bits: int, hi_bits: int) -> None:
        chunk = 1 << 26
        for start in range(lo_bits, hi_bits, chunk):
            stop = min(start + chunk, hi_bits)
            bits = torch.arange(start, stop, dtype=torch.int64, device="cuda")
            x = (bits - (1 << 32) * (bits >= (1 << 31))).to(torch.int32).view(torch.float32)
            y = torch.empty_like(x)
            host.prefill_approx_exp(x.data_ptr(), y.data_ptr(), x.numel(), torch.cuda.current_stream().cuda_stream)
            ref = approx_exp_torch(torch, x)
            bad = (y.view(torch.int32) != ref.view(torch.int32)).nonzero()
            assert bad.numel() == 0, (hex(start + int(bad[0])), float(x[bad[0]]), float(y[bad[0]]), float(ref[bad[0]]))

    check(0x80000000, 0xC1800001)  # -0 .. -16
    check(0x00000000, 0x7F800000)  # +0 .. largest finite
