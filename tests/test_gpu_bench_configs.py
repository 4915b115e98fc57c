"""The benchmarked GPU paths compared directly with the oracle at the benchmark configurations' shapes.

- Config 2: every layer of the persistent 28-layer decode kernel (`decode_bs1_kernel`, the bench line's
  kernel; the tensor-core `decode_stack_kernel` gives bit-identical layers) at history 517 after a 512-token
  prompt. Each layer's input (the engine's own previous-layer output)
  and K/V history go to the oracle's decode layer (W8). The oracle's bf16-rounded output must match the
  engine's per element within one bf16 unit in the last place plus 1e-5 of the row's RMS, every layer within
  north_star's 1e-3 relative L2, and the new K/V rows within 1e-5.
- Configs 1, 2 and 4: the W8 drop-in prefill layer against the oracle at 128 tokens (stock capacity), and at
  512 and 4096 tokens (capacity raised, as the reference rebuilt with kDefaultPrefillSeqTile = 4096). These
  exercise the CTA-pair and cluster split-K GEMM forms and their fp32 epilogues (bias, RoPE up to position
  4095, SiLU * up, residual).
- The tensor-core prefill attention at 2048 and 4096 tokens against the float64 restatement of the
  reference's two-pass context.

Per-layer criterion: north_star's 1e-3 relative L2. The tests assert the tighter 1e-5 (fp32 reordering only)
where no bf16 rounding intervenes.
"""
from __future__ import annotations

import numpy as np
import pytest

import qwen_oracle as qo
from qwen_full_model import OracleModel

pytestmark = pytest.mark.gpu

TOL = 1e-5


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def bf16_excess(a: np.ndarray, b: np.ndarray, rel_floor: float = 1e-5) -> float:
    """Largest |a - b| beyond what the tolerance allows, per element: one bf16 unit in the last place of b (a
    rounding flip) plus rel_floor times the row's RMS (fp32 reordering is relative to the row, so elements
    near zero may differ by several of their own ulps). <= 0 means every element is within tolerance."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    mag = np.maximum(np.abs(b), np.finfo(np.float32).tiny)
    ulp = 2.0 ** (np.floor(np.log2(mag)) - 7)
    allow = ulp + rel_floor * float(np.sqrt(np.mean(b * b)))
    return float((np.abs(a - b) - allow).max())


@pytest.fixture(scope="module")
def host(built_libs, gpu_available):
    if not gpu_available:
        pytest.fail("no CUDA device: the -m gpu suite must run on a B200")
    from work_llm_accelerator_b200 import host as h

    return h


def test_persistent_decode_kernel_layers_match_oracle_at_config2(host):
    seed, prompt_len, steps = 2024, 512, 5
    eng = host.Engine(0, 8, max_seqs=1, max_len=prompt_len + steps + 16)
    try:
        eng.init_synthetic(seed)
        prompt = [int(t) for t in np.random.default_rng(seed).integers(0, qo.VOCAB, prompt_len)]
        tok = eng.prefill(0, prompt)
        for _ in range(steps):
            tok = int(eng.decode([0], [tok])[0])
        past = eng.seq_len(0)
        assert past == prompt_len + steps
        eng.set_option("dump_hidden", 1)  # eager launches of the same persistent kernel
        nxt = int(eng.decode([0], [tok])[0])
        hidden = eng.read_hidden(1)[:, 0]
        kvs = [eng.read_kv(0, l, past + 1) for l in range(qo.LAYERS)]
        assert host.kernel_error(reset=True) == 0
    finally:
        eng.close()
    ora = OracleModel(seed, 8, layers=qo.LAYERS)
    x = ora.embed_rows([tok]).reshape(-1)
    worst_kv, worst_excess, worst_rel = 0.0, -1.0, 0.0
    for l in range(qo.LAYERS):
        k_e, v_e = kvs[l]
        kc = np.zeros((past + 1) * qo.KV_WIDTH, np.float32)
        vc = kc.copy()
        kc[:past * qo.KV_WIDTH] = k_e[:past * qo.KV_WIDTH]
        vc[:past * qo.KV_WIDTH] = v_e[:past * qo.KV_WIDTH]
        st, out = qo.decode_layer(ora.params[l], x, past, kc, vc)
        assert st == 0
        row = slice(past * qo.KV_WIDTH, (past + 1) * qo.KV_WIDTH)
        worst_kv = max(worst_kv, rel_l2(k_e[row], kc[row]), rel_l2(v_e[row], vc[row]))
        want = qo.round_bf16(out)
        worst_excess = max(worst_excess, bf16_excess(hidden[l], want))
        worst_rel = max(worst_rel, rel_l2(hidden[l], want))
        x = hidden[l]  # the engine's own input to the next layer
    assert worst_kv <= TOL
    assert worst_rel <= 1e-3, worst_rel  # north_star per-layer bound
    assert worst_excess <= 0.0, (worst_excess, worst_rel)
    # the LM head + argmax of the engine's final hidden state
    assert nxt == qo.lm_head_argmax(hidden[-1], ora.final_norm, ora.embed)


def layer_args(p):
    return (p["input_layernorm"], p["post_attention_layernorm"], p["q_w"], p["k_w"], p["v_w"], p["o_w"], p["gate_w"],
            p["up_w"], p["down_w"], p["q_bias"], p["k_bias"], p["v_bias"], p["q_s"], p["k_s"], p["v_s"], p["o_s"],
            p["gate_s"], p["up_s"], p["down_s"])


@pytest.mark.parametrize("S", [128, 512, 4096])
def test_w8_prefill_layer_matches_oracle_at_config_lengths(host, S):
    pre = host.load_prefill_lib()
    seed = 60 + S % 97
    p = qo.synth_layer(seed, 3, 8)
    x = qo.synth(seed, qo.STREAM_ACT, S * qo.HIDDEN)
    k_or = np.zeros(S * qo.KV_WIDTH, np.float32)
    v_or = k_or.copy()
    st, out_or = qo.prefill_layer(p, x, S, k_or, v_or)
    assert st == 0
    kc, vc, out = np.zeros_like(k_or), np.zeros_like(v_or), np.zeros(S * qo.HIDDEN, np.float32)
    old = host.prefill_seq_capacity()
    try:
        host.set_prefill_seq_capacity(max(128, S))
        assert pre.qwen_prefill_layer_smoke_forward_w8(x, S, *qo.tiles_tuple(), *layer_args(p), kc, vc, out) == 0
    finally:
        host.set_prefill_seq_capacity(old)
    assert host.kernel_error(reset=True) == 0
    assert rel_l2(out, out_or) <= TOL
    assert rel_l2(kc, k_or) <= TOL and rel_l2(vc, v_or) <= TOL
    # per token as well: a wrong tile or RoPE position would hide in a global norm
    o, w = out.reshape(S, qo.HIDDEN).astype(np.float64), out_or.reshape(S, qo.HIDDEN).astype(np.float64)
    assert float((np.linalg.norm(o - w, axis=1) / np.linalg.norm(w, axis=1)).max()) <= 1e-4
    k, kw = kc.reshape(S, qo.KV_WIDTH).astype(np.float64), k_or.reshape(S, qo.KV_WIDTH).astype(np.float64)
    assert float((np.linalg.norm(k - kw, axis=1) / np.linalg.norm(kw, axis=1)).max()) <= 1e-4


@pytest.mark.parametrize("S,q_scale", [(2048, 1.0), (4096, 4.0)])
def test_tensor_core_attention_long_against_reference_context(host, S, q_scale):
    import torch
    from test_gpu_prefill_attention import HIDDEN, inputs, reference_context, rel

    q, k, v = inputs(torch, S, 7 * S, q_scale)
    ctx = torch.full((S, HIDDEN), float("nan"), device="cuda")
    host.prefill_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), S, ctx.data_ptr(), 0,
                           torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert host.kernel_error(True) == 0
    ref = torch.from_numpy(reference_context(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), S))
    got = ctx.cpu()
    assert torch.isfinite(got).all()
    assert rel(got, ref) <= TOL
    row_err = ((got.double() - ref).norm(dim=1) / ref.norm(dim=1)).max().item()
    assert row_err <= 1e-4
