"""Greedy-token identity with the reference host libraries (north_star: "greedy token sequences are identical
over the decode run") through the engine's "exact" option.

In that option every layer and the LM head compute in the reference host code's arithmetic order: serial fp32
sums per output (no FMA), the double decode RMSNorm, the libm decode RoPE table, the prefill approximations, and
for the decode softmax and SiLU the host C library's expf restated on the GPU. The 28-layer W4 engine then
reproduces, free-running, the reference library's tokens and the sha256 of every layer's bf16 hidden state
recorded in tests/golden/golden.json (made by tests/golden/make_golden.py from oracle/_ref, the reference's own
host libraries): `full_model_w4` (8-token prompt, 4 greedy steps) and `full_model_w4_long` (32-token prompt,
16 greedy steps). The W8 engine in the same option equals the C restatement run with int8 codes, bit for bit.
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

import qwen_oracle as qo
from qwen_full_model import OracleModel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def host(built_libs, gpu_available):
    if not gpu_available:
        pytest.fail("no CUDA device: the -m gpu suite must run on a B200")
    from work_llm_accelerator_b200 import host as h

    return h


def digest(rows) -> str:
    h = hashlib.sha256()
    for r in rows:
        h.update(np.ascontiguousarray(r, np.float32).tobytes())
    return h.hexdigest()


def test_exact_expf_matches_host_c_library(host):
    """The exact option's expf equals this machine's C library expf (the reference host library's std::exp on
    floats) bit for bit: one bit pattern in 64 over all 2^32 (shifted by a random offset), every special value,
    and the decode softmax's range [-30, 0] densely."""
    import torch

    rng = np.random.default_rng(0)
    off = int(rng.integers(0, 64))
    bits = (np.arange(0, 1 << 32, 64, dtype=np.uint64) + off).astype(np.uint32)
    dense = np.linspace(-30.0, 0.0, 1 << 22, dtype=np.float32).view(np.uint32)
    special = np.array([0x00000000, 0x80000000, 0x7f800000, 0xff800000, 0x7fc00000, 0x00000001, 0x80000001,
                        0x42b17218, 0x42b17217, 0xc2cff1b5, 0xc2cff1b4, 0xc2ce8ed0, 0x42b00000, 0xc2b00000],
                       dtype=np.uint32)
    x = np.concatenate([bits, dense, special]).view(np.float32)
    want = qo.host_expf(x)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty_like(xd)
    host.exact_expf(xd.data_ptr(), yd.data_ptr(), x.size)
    got = yd.cpu().numpy()
    nan_w, nan_g = np.isnan(want), np.isnan(got)
    assert np.array_equal(nan_w, nan_g)
    bad = np.flatnonzero(got.view(np.uint32)[~nan_w] != want.view(np.uint32)[~nan_w])
    assert bad.size == 0, f"{bad.size} mismatches, first x = {x[~nan_w][bad[:5]]}"


def _run_engine(host, wbits: int, seed: int, prompt, steps: int):
    """Free-running exact-mode greedy run: (tokens, per-call sha256 of the 28 layer outputs)."""
    eng = host.Engine(0, wbits, max_seqs=1, max_len=len(prompt) + steps + 8)
    try:
        eng.init_synthetic(seed)
        eng.set_option("exact", 1)
        eng.set_option("dump_hidden", 1)
        toks, shas, hidden = [eng.prefill(0, prompt)], [], []
        h = eng.read_hidden(1)[:, 0]
        shas.append(digest(h))
        hidden.append(h)
        for _ in range(steps):
            toks.append(int(eng.decode([0], [toks[-1]])[0]))
            h = eng.read_hidden(1)[:, 0]
            shas.append(digest(h))
            hidden.append(h)
        assert host.kernel_error(reset=True) == 0
        return toks, shas, hidden
    finally:
        eng.close()


@pytest.mark.parametrize("kind", ["full_model_w4", "full_model_w4_long"])
def test_exact_w4_reproduces_reference_tokens_and_hidden_states(host, golden, kind):
    case = next(c for c in golden["cases"] if c["kind"] == kind)
    steps = len(case["tokens"]) - 1
    toks, shas, hidden = _run_engine(host, 4, case["seed"], case["prompt"], steps)
    # the first divergence, if any, names the call and whether the layers or only the LM head differ
    for i, (sha, want) in enumerate(zip(shas, case["hidden_sha"])):
        assert sha == want, f"{kind}: hidden states differ from the reference at call {i} (0 = prefill)"
    assert toks == case["tokens"]
    assert [float(v) for v in hidden[-1][-1][:8]] == case["final_hidden_head"]


def test_exact_w8_matches_restatement_bit_for_bit(host):
    """W8 codes (no reference library takes them): the exact option equals the C restatement run with int8
    codes -- every layer's hidden state of every call and every token."""
    seed = 41
    prompt = [int(t) for t in np.random.default_rng(seed).integers(0, qo.VOCAB, 9)]
    steps = 3
    toks, _, hidden = _run_engine(host, 8, seed, prompt, steps)
    ora = OracleModel(seed, 8)
    want = [ora.prefill(prompt)]
    assert all(np.array_equal(hidden[0][l], ora.hidden_trace[l]) for l in range(qo.LAYERS))
    for i in range(steps):
        want.append(ora.decode(want[-1]))
        assert all(np.array_equal(hidden[i + 1][l], ora.hidden_trace[l]) for l in range(qo.LAYERS)), i
    assert toks == want


def test_exact_option_graph_replay_and_switching(host):
    """Captured exact steps replay to the same tokens as eager ones, and switching the option off returns
    the engine to its tensor-core path (a different, valid greedy run on the same weights)."""
    seed, prompt = 43, [3, 1, 4, 1, 5, 9, 2, 6]
    runs = []
    for graphs in (0, 1):
        eng = host.Engine(0, 4, max_seqs=1, max_len=64)
        try:
            eng.init_synthetic(seed)
            eng.set_option("exact", 1)
            eng.set_option("graphs", graphs)
            toks = [eng.prefill(0, prompt)]
            for _ in range(5):
                toks.append(int(eng.decode([0], [toks[-1]])[0]))
            runs.append(toks)
            eng.set_option("exact", 0)
            eng.reset(0)
            assert 0 <= eng.prefill(0, prompt) < qo.VOCAB
        finally:
            eng.close()
    assert runs[0] == runs[1]
