"""The fp32 golden "layer0 reference" entry points (qwen_decode_layer0_reference_forward,
qwen_prefill_layer0_reference_forward[_with_cache]) on the GPU against the reference's own host libraries
(oracle/_ref, built from hls/decode_only/qwen_decode_layer0_reference_wrapper.cpp and
hls/prefill_only/qwen_prefill_layer0_reference_wrapper.cpp) on the same seeded fp32 weights and inputs.

The GPU layers restate the reference's arithmetic operation for operation (double accumulation in its order,
bf16 roundings, the host C library's expf for the SiLU). The softmax exponential is double precision, where
CUDA's exp may differ from the host's in the last bit of a probability; once the context is stored as float
and every linear output rounded to bf16, that can only move an output by the rounding of one element, so the
test requires bit-identity for all but a vanishing fraction of elements and every element within one bf16
unit in the last place.
"""
from __future__ import annotations

import numpy as np
import pytest

import qwen_oracle as qo

pytestmark = pytest.mark.gpu

H, KV, I = 1536, 256, 8960
EPS = np.float32(1e-6)


@pytest.fixture(scope="module")
def libs(built_libs, gpu_available, ref_libs):
    if not gpu_available:
        pytest.fail("no CUDA device: the -m gpu suite must run on a B200")
    from work_llm_accelerator_b200 import host

    return host.load_decode_lib(), host.load_prefill_lib(), ref_libs


def weights(seed: int, with_bias: bool):
    rng = np.random.default_rng(seed)

    def n(*shape, mean=0.0, sd=0.02):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(sd) + np.float32(mean)).astype(np.float32)

    w = dict(in_ln=n(H, mean=1.0), q_w=n(H, H), q_b=n(H), k_w=n(KV, H), k_b=n(KV), v_w=n(KV, H), v_b=n(KV),
             o_w=n(H, H), o_b=n(H) if with_bias else None, post_ln=n(H, mean=1.0), gate_w=n(I, H),
             gate_b=n(I) if with_bias else None, up_w=n(I, H), up_b=n(I) if with_bias else None, down_w=n(H, I),
             down_b=n(H) if with_bias else None)
    return w


def ptr(a):
    return None if a is None else a.ctypes.data


def wargs(w):
    return [ptr(w[k]) for k in ("in_ln", "q_w", "q_b", "k_w", "k_b", "v_w", "v_b", "o_w", "o_b", "post_ln", "gate_w",
                                "gate_b", "up_w", "up_b", "down_w", "down_b")]


def assert_matches(got: np.ndarray, want: np.ndarray, what: str) -> None:
    got, want = got.reshape(-1), want.reshape(-1)
    diff = np.flatnonzero(got.view(np.uint32) != want.view(np.uint32))
    assert diff.size <= max(1, want.size // 10000), f"{what}: {diff.size} of {want.size} elements differ"
    if diff.size:
        rel = np.abs(got[diff].astype(np.float64) - want[diff]) / np.maximum(np.abs(want[diff]), 1e-30)
        assert rel.max() <= 2.0 ** -7, f"{what}: element off by {rel.max():.3g} relative"


@pytest.mark.parametrize("past,with_bias", [(0, True), (9, False), (70, True)])
def test_decode_layer0_matches_reference(libs, past, with_bias):
    dec, _, ref = libs
    w = weights(100 + past, with_bias)
    rng = np.random.default_rng(past)
    x = rng.standard_normal(H, dtype=np.float32)
    pk = rng.standard_normal(2 * past * 128, dtype=np.float32)
    pv = rng.standard_normal(2 * past * 128, dtype=np.float32)
    outs = []
    for lib in (dec, ref.decode):
        out = np.zeros(H, np.float32)
        nk = np.zeros(2 * (past + 1) * 128, np.float32)
        nv = np.zeros_like(nk)
        st = lib.qwen_decode_layer0_reference_forward(ptr(x), past, ptr(pk) if past else None,
                                                      ptr(pv) if past else None, *wargs(w), EPS, ptr(out), ptr(nk),
                                                      ptr(nv))
        assert st == 0
        outs.append((out, nk, nv))
    (o, k, v), (o_r, k_r, v_r) = outs
    assert_matches(k, k_r, "next K cache")
    assert_matches(v, v_r, "next V cache")
    assert_matches(o, o_r, "output")


@pytest.mark.parametrize("S,with_bias", [(1, False), (6, True)])
def test_prefill_layer0_matches_reference(libs, S, with_bias):
    _, pre, ref = libs
    w = weights(200 + S, with_bias)
    x = np.random.default_rng(S).standard_normal(S * H, dtype=np.float32)
    res = []
    for lib in (pre, ref.prefill):
        out = np.zeros(S * H, np.float32)
        kc = np.zeros(2 * S * 128, np.float32)
        vc = np.zeros_like(kc)
        assert lib.qwen_prefill_layer0_reference_forward_with_cache(ptr(x), S, *wargs(w), EPS, ptr(out), ptr(kc),
                                                                    ptr(vc)) == 0
        out2 = np.zeros(S * H, np.float32)
        assert lib.qwen_prefill_layer0_reference_forward(ptr(x), S, *wargs(w), EPS, ptr(out2)) == 0
        assert np.array_equal(out, out2)
        res.append((out, kc, vc))
    (o, k, v), (o_r, k_r, v_r) = res
    assert_matches(k, k_r, "K cache")
    assert_matches(v, v_r, "V cache")
    assert_matches(o, o_r, "output")


def test_layer0_status_codes_match_reference(libs):
    dec, pre, ref = libs
    w = weights(7, True)
    x = np.zeros(4 * H, np.float32)
    out = np.zeros(4 * H, np.float32)
    kc = np.zeros(2 * 5 * 128, np.float32)
    for lib in (dec, ref.decode):
        assert lib.qwen_decode_layer0_reference_forward(None, 0, None, None, *wargs(w), EPS, ptr(out), ptr(kc),
                                                        ptr(kc)) == 1
        assert lib.qwen_decode_layer0_reference_forward(ptr(x), -1, None, None, *wargs(w), EPS, ptr(out), ptr(kc),
                                                        ptr(kc)) == 1
        assert lib.qwen_decode_layer0_reference_forward(ptr(x), 0, None, None, *wargs(w), EPS, ptr(out), None,
                                                        ptr(kc)) == 1
    for lib in (pre, ref.prefill):
        assert lib.qwen_prefill_layer0_reference_forward(ptr(x), 0, *wargs(w), EPS, ptr(out)) == 1
        assert lib.qwen_prefill_layer0_reference_forward(ptr(x), 32769, *wargs(w), EPS, ptr(out)) == 1
        assert lib.qwen_prefill_layer0_reference_forward(None, 2, *wargs(w), EPS, ptr(out)) == 1
        assert lib.qwen_prefill_layer0_reference_forward_with_cache(ptr(x), 2, *wargs(w), EPS, ptr(out), ptr(kc),
                                                                    None) == 1
