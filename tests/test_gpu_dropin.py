"""GPU parity of the drop-in C-ABI (libqwen_decode_stub.so / libqwen_prefill_stub.so built by this repo)
against the oracle (the C restatement, itself pinned bit-for-bit to the reference's host libraries by
tests/golden/golden.json) on seeded synthetic inputs.

Tolerances: the projections sum in a different order than the reference's serial fp32 loop and apply
the per-channel scale after the sum, so results differ by rounding only. Single layer: relative L2
error <= 1e-5 on outputs and new KV rows (the product target for hidden states is 1e-3 after 28
layers); integer/layout paths (top == layer, glue == layer, stubs) are exact.
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

import qwen_oracle as qo

pytestmark = pytest.mark.gpu

TOL = 1e-5


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


@pytest.fixture(scope="module")
def libs(built_libs, gpu_available):
    if not gpu_available:
        pytest.fail("no CUDA device: the -m gpu suite must run on a B200")
    from work_llm_accelerator_b200 import host

    return host.load_decode_lib(), host.load_prefill_lib()


def kv_hist(seed, past, size):
    k = np.zeros(size, np.float32)
    v = np.zeros(size, np.float32)
    k[:past * qo.KV_WIDTH] = qo.synth(seed, qo.STREAM_ACT + 1, past * qo.KV_WIDTH)
    v[:past * qo.KV_WIDTH] = qo.synth(seed, qo.STREAM_ACT + 2, past * qo.KV_WIDTH)
    return k, v


def layer_args(p):
    return (p["input_layernorm"], p["post_attention_layernorm"], p["q_w"], p["k_w"], p["v_w"], p["o_w"], p["gate_w"],
            p["up_w"], p["down_w"], p["q_bias"], p["k_bias"], p["v_bias"], p["q_s"], p["k_s"], p["v_s"], p["o_s"],
            p["gate_s"], p["up_s"], p["down_s"])


@pytest.mark.parametrize("seed,past", [(11, 128), (12, 5), (13, 0), (14, 2047)])
@pytest.mark.parametrize("wbits", [4, 8])
def test_decode_layer_matches_oracle(libs, golden, seed, past, wbits):
    dec, _ = libs
    p = qo.synth_layer(seed, 0, wbits)
    x = qo.synth(seed, qo.STREAM_ACT, qo.HIDDEN)
    kc, vc = kv_hist(seed, past, (past + 1) * qo.KV_WIDTH)
    k_or, v_or = kc.copy(), vc.copy()
    st, out_or = qo.decode_layer(p, x, past, k_or, v_or)
    assert st == 0
    if wbits == 4:  # the oracle itself is pinned to the reference's digests
        for case in golden["cases"]:
            if case["kind"] == "decode_layer" and case["seed"] == seed and case["past"] == past:
                assert sha(out_or) == case["out_sha"]
    out = np.zeros(qo.HIDDEN, np.float32)
    fn = dec.qwen_decode_layer_smoke_forward if wbits == 4 else dec.qwen_decode_layer_smoke_forward_w8
    assert fn(x, past, *layer_args(p), kc, vc, out) == 0
    row = slice(past * qo.KV_WIDTH, (past + 1) * qo.KV_WIDTH)
    assert rel_l2(out, out_or) <= TOL
    assert rel_l2(kc[row], k_or[row]) <= TOL and rel_l2(vc[row], v_or[row]) <= TOL
    # history rows untouched
    assert np.array_equal(kc[:past * qo.KV_WIDTH], k_or[:past * qo.KV_WIDTH])


@pytest.mark.parametrize("wbits", [4, 8])
def test_decode_top_equals_layer_and_halves(libs, wbits):
    """top (descriptor + DDR address decode) == layer smoke, and attention + MLP smokes compose to it
    (the reference's validate_decode_top_wrapper_regression.py check)."""
    dec, _ = libs
    seed, past = 15, 37
    p = qo.synth_layer(seed, 3, wbits)
    x = qo.synth(seed, qo.STREAM_ACT, qo.HIDDEN)
    kc, vc = kv_hist(seed, past, (past + 1) * qo.KV_WIDTH)
    out_layer = np.zeros(qo.HIDDEN, np.float32)
    k1, v1 = kc.copy(), vc.copy()
    fn = dec.qwen_decode_layer_smoke_forward if wbits == 4 else dec.qwen_decode_layer_smoke_forward_w8
    assert fn(x, past, *layer_args(p), k1, v1, out_layer) == 0

    wd, sd = p.ddr()
    base_w, base_s = 3 * 1024, 3 * 1024  # non-zero bases exercise the address decode
    wbuf = np.zeros(wd.size + base_w, np.uint8)
    wbuf[base_w:] = wd
    sbuf = np.zeros(sd.size + base_s // 4, np.float32)
    sbuf[base_s // 4:] = sd
    kv = np.concatenate([kc, vc])
    act = np.zeros(3 * qo.HIDDEN, np.float32)
    act[qo.HIDDEN:2 * qo.HIDDEN] = x
    top = dec.qwen_decode_top_smoke_forward if wbits == 4 else dec.qwen_decode_top_smoke_forward_w8
    st = top(3, past, qo.HIDDEN * 4, 2 * qo.HIDDEN * 4, base_w, base_s, 0, kc.size * 4, wbuf, sbuf, kv, act,
             *qo.sram_ports())
    assert st == 0
    assert np.array_equal(act[2 * qo.HIDDEN:], out_layer)
    assert np.array_equal(kv[:kc.size], k1) and np.array_equal(kv[kc.size:], v1)
    if wbits == 4:
        a = np.zeros(qo.HIDDEN, np.float32)
        k2, v2 = kc.copy(), vc.copy()
        assert dec.qwen_decode_attention_smoke_forward(x, past, p["input_layernorm"], p["q_w"], p["k_w"], p["v_w"],
                                                       p["o_w"], p["q_bias"], p["k_bias"], p["v_bias"], p["q_s"],
                                                       p["k_s"], p["v_s"], p["o_s"], k2, v2, a) == 0
        m = np.zeros(qo.HIDDEN, np.float32)
        assert dec.qwen_decode_mlp_smoke_forward(a, p["post_attention_layernorm"], p["gate_w"], p["up_w"],
                                                 p["down_w"], p["gate_s"], p["up_s"], p["down_s"], m) == 0
        assert np.array_equal(m, out_layer)


def test_decode_attention_smoke_kat(libs):
    """verification/validate_decode_attention_smoke.py: one-hot input, unit weights on (0,0)."""
    dec, _ = libs
    H, KV = qo.HIDDEN, qo.KV_WIDTH
    x = np.zeros(H, np.float32)
    x[0] = 1.0
    qw = np.zeros(H * H // 2, np.uint8)
    kw = np.zeros(KV * H // 2, np.uint8)
    vw = np.zeros(KV * H // 2, np.uint8)
    ow = np.zeros(H * H // 2, np.uint8)
    for w in (qw, kw, vw, ow):
        w[0] = 1
    ones = lambda n: np.ones(n, np.float32)  # noqa: E731
    zeros = lambda n: np.zeros(n, np.float32)  # noqa: E731
    kc, vc, out = zeros(KV), zeros(KV), zeros(H)
    assert dec.qwen_decode_attention_smoke_forward(x, 0, ones(H), qw, kw, vw, ow, zeros(H), zeros(KV), zeros(KV),
                                                   ones(H), ones(KV), ones(KV), ones(H), kc, vc, out) == 0
    expected = 1.0 / np.sqrt((1.0 / H) + 1.0e-6)
    assert np.isclose(kc[0], expected, atol=1e-5) and np.isclose(vc[0], expected, atol=1e-5)
    assert np.isclose(out[0], expected, atol=1e-5)
    assert np.count_nonzero(out[1:]) == 0


def test_decode_stub_is_zero(libs):
    dec, _ = libs
    x = qo.synth(3, qo.STREAM_ACT, qo.HIDDEN)
    out = np.full(qo.HIDDEN, 7.0, np.float32)
    assert dec.qwen_decode_stub_forward(x, 4, out) == 0
    assert np.count_nonzero(out) == 0


@pytest.mark.parametrize("seed,S", [(21, 16), (22, 7), (23, 1)])
@pytest.mark.parametrize("wbits", [4, 8])
def test_prefill_layer_matches_oracle(libs, golden, seed, S, wbits):
    _, pre = libs
    p = qo.synth_layer(seed, 0, wbits)
    x = qo.synth(seed, qo.STREAM_ACT, S * qo.HIDDEN)
    k_or = np.zeros(S * qo.KV_WIDTH, np.float32)
    v_or = k_or.copy()
    st, out_or = qo.prefill_layer(p, x, S, k_or, v_or)
    assert st == 0
    if wbits == 4:
        for case in golden["cases"]:
            if case["kind"] == "prefill_layer" and case["seed"] == seed and case["seq_len"] == S:
                assert sha(out_or) == case["out_sha"] and sha(k_or, v_or) == case["kv_sha"]
    kc = np.zeros_like(k_or)
    vc = np.zeros_like(v_or)
    out = np.zeros(S * qo.HIDDEN, np.float32)
    fn = pre.qwen_prefill_layer_smoke_forward if wbits == 4 else pre.qwen_prefill_layer_smoke_forward_w8
    assert fn(x, S, *qo.tiles_tuple(), *layer_args(p), kc, vc, out) == 0
    assert rel_l2(out, out_or) <= TOL
    assert rel_l2(kc, k_or) <= TOL and rel_l2(vc, v_or) <= TOL


def test_prefill_top_glue_equal_layer(libs):
    """The reference's own self-consistency pins: top == layer (validate_prefill_top_wrapper_regression.py)
    and glue == layer (validate_prefill_glue_smoke.py)."""
    _, pre = libs
    seed, S = 25, 11
    p = qo.synth_layer(seed, 1, 4)
    x = qo.synth(seed, qo.STREAM_ACT, S * qo.HIDDEN)
    kc, vc, out = (np.zeros(S * qo.KV_WIDTH, np.float32), np.zeros(S * qo.KV_WIDTH, np.float32),
                   np.zeros(S * qo.HIDDEN, np.float32))
    assert pre.qwen_prefill_layer_smoke_forward(x, S, *qo.tiles_tuple(), *layer_args(p), kc, vc, out) == 0
    kg, vg, og = np.zeros_like(kc), np.zeros_like(vc), np.zeros_like(out)
    assert pre.qwen_prefill_glue_smoke_forward(x, S, *qo.tiles_tuple(), *layer_args(p), kg, vg, og) == 0
    assert np.array_equal(og, out) and np.array_equal(kg, kc) and np.array_equal(vg, vc)
    wd, sd = p.ddr()
    act = np.zeros(3 * S * qo.HIDDEN, np.float32)
    act[:S * qo.HIDDEN] = x
    kv = np.zeros(2 * S * qo.KV_WIDTH, np.float32)
    st = pre.qwen_prefill_top_smoke_forward(1, S, *qo.tiles_tuple(), 0, S * qo.HIDDEN * 4, 0, 0, 0,
                                            S * qo.KV_WIDTH * 4, wd, sd, kv, act, *qo.sram_ports())
    assert st == 0
    assert np.array_equal(act[S * qo.HIDDEN:2 * S * qo.HIDDEN], out)
    assert np.array_equal(kv[:S * qo.KV_WIDTH], kc) and np.array_equal(kv[S * qo.KV_WIDTH:], vc)
    # the scratch slot holds the attention output, as in the reference
    a = np.zeros(S * qo.HIDDEN, np.float32)
    k3, v3 = np.zeros_like(kc), np.zeros_like(vc)
    assert pre.qwen_prefill_attention_smoke_forward(x, S, *qo.tiles_tuple()[:8], p["input_layernorm"], p["q_w"],
                                                    p["k_w"], p["v_w"], p["o_w"], p["q_bias"], p["k_bias"],
                                                    p["v_bias"], p["q_s"], p["k_s"], p["v_s"], p["o_s"], k3, v3,
                                                    a) == 0
    assert np.array_equal(act[2 * S * qo.HIDDEN:], a)


def test_prefill_long_sequence_capacity_4096(libs, golden):
    """S = 130 > the stock capacity: rejected (20) at the default capacity like the stock reference, and
    computed like the reference rebuilt with kDefaultPrefillSeqTile = 4096 once the capacity is raised."""
    from work_llm_accelerator_b200 import host

    _, pre = libs
    seed, S = 24, 130
    p = qo.synth_layer(seed, 0, 4)
    x = qo.synth(seed, qo.STREAM_ACT, S * qo.HIDDEN)
    wd, sd = p.ddr()
    act = np.zeros(3 * S * qo.HIDDEN, np.float32)
    act[:S * qo.HIDDEN] = x
    kv = np.zeros(2 * S * qo.KV_WIDTH, np.float32)
    args = (0, S, *qo.tiles_tuple(), 0, S * qo.HIDDEN * 4, 0, 0, 0, S * qo.KV_WIDTH * 4, wd, sd, kv, act,
            *qo.sram_ports())
    old = host.prefill_seq_capacity()
    try:
        host.set_prefill_seq_capacity(128)
        assert pre.qwen_prefill_top_smoke_forward(*args) == 20
        host.set_prefill_seq_capacity(4096)
        assert pre.qwen_prefill_top_smoke_forward(*args) == 0
    finally:
        host.set_prefill_seq_capacity(old)
    k_or = np.zeros(S * qo.KV_WIDTH, np.float32)
    v_or = k_or.copy()
    st, out_or = qo.prefill_layer(p, x, S, k_or, v_or)
    for case in golden["cases"]:
        if case["kind"] == "prefill_layer" and case["seq_len"] == S:
            assert sha(out_or) == case["out_sha"]
    assert rel_l2(act[S * qo.HIDDEN:2 * S * qo.HIDDEN], out_or) <= TOL
    assert rel_l2(kv[:S * qo.KV_WIDTH], k_or) <= TOL


def test_prefill_stub_is_zero(libs):
    _, pre = libs
    S = 5
    x = qo.synth(4, qo.STREAM_ACT, S * qo.HIDDEN)
    out = np.full(S * qo.HIDDEN, 3.0, np.float32)
    assert pre.qwen_prefill_stub_forward(x, S, *qo.tiles_tuple(), out) == 0
    assert np.count_nonzero(out) == 0


def test_status_codes_match_reference_on_gpu(libs, ref_libs):
    """Error paths that need the GPU to reach (MLP-stage errors after the attention stage ran)."""
    _, pre = libs
    S = 4
    lay = qo.layer_layout(4)
    w = np.zeros(lay["total"], np.uint8)
    s = np.zeros(lay["total"] // 4, np.float32)
    for tiles in (qo.tiles_tuple({"mlp_ff": 1280}), qo.tiles_tuple({"mlp_hidden": 512})):
        got = []
        for lib in (pre, ref_libs.prefill):
            x = np.zeros(3 * S * qo.HIDDEN, np.float32)
            kv = np.zeros(2 * S * qo.KV_WIDTH, np.float32)
            got.append(lib.qwen_prefill_top_smoke_forward(0, S, *tiles, 0, S * qo.HIDDEN * 4, 0, 0, 0,
                                                          S * qo.KV_WIDTH * 4, w, s, kv, x, *qo.sram_ports()))
        assert got[0] == got[1] == 1
