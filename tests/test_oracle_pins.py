"""CPU tests of the oracle (the checker): pinned to the reference's own host libraries through the golden
digests (always) and directly (when oracle/_ref is built), plus restatement cross-checks of its
elementwise arithmetic."""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

import qwen_oracle as qo


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def kv_hist(seed, past, size):
    k = np.zeros(size, np.float32)
    v = np.zeros(size, np.float32)
    k[:past * qo.KV_WIDTH] = qo.synth(seed, qo.STREAM_ACT + 1, past * qo.KV_WIDTH)
    v[:past * qo.KV_WIDTH] = qo.synth(seed, qo.STREAM_ACT + 2, past * qo.KV_WIDTH)
    return k, v


def test_golden_decode_cases(golden):
    n = 0
    for case in golden["cases"]:
        if not case["kind"].startswith("decode"):
            continue
        seed, past = case["seed"], case["past"]
        p = qo.synth_layer(seed, 0, 4)
        x = qo.synth(seed, qo.STREAM_ACT, qo.HIDDEN)
        kc, vc = kv_hist(seed, past, (past + 1) * qo.KV_WIDTH)
        if case["kind"] == "decode_layer":
            st, out = qo.decode_layer(p, x, past, kc, vc)
            row = slice(past * qo.KV_WIDTH, (past + 1) * qo.KV_WIDTH)
            assert st == 0 and sha(out) == case["out_sha"] and sha(kc[row], vc[row]) == case["kv_sha"]
        elif case["kind"] == "decode_attention":
            st, a = qo.decode_attention(p, x, past, kc, vc)
            assert st == 0 and sha(a) == case["out_sha"]
        n += 1
    assert n >= 6


def test_golden_prefill_cases(golden):
    n = 0
    for case in golden["cases"]:
        if case["kind"] != "prefill_layer":
            continue
        seed, S = case["seed"], case["seq_len"]
        p = qo.synth_layer(seed, 0, 4)
        x = qo.synth(seed, qo.STREAM_ACT, S * qo.HIDDEN)
        kc = np.zeros(S * qo.KV_WIDTH, np.float32)
        vc = kc.copy()
        st, out = qo.prefill_layer(p, x, S, kc, vc)
        assert st == 0 and sha(out) == case["out_sha"] and sha(kc, vc) == case["kv_sha"]
        n += 1
    assert n >= 3


@pytest.mark.slow
def test_golden_full_model_w4(golden):
    from qwen_full_model import OracleModel

    case = next(c for c in golden["cases"] if c["kind"] == "full_model_w4")
    m = OracleModel(case["seed"], 4)
    toks = [m.prefill(case["prompt"])]
    hs = [sha(*m.hidden_trace)]
    for _ in range(len(case["tokens"]) - 1):
        toks.append(m.decode(toks[-1]))
        hs.append(sha(*m.hidden_trace))
    assert toks == case["tokens"]
    assert hs == case["hidden_sha"]


def test_port_bit_exact_vs_reference_libs(ref_libs):
    """Fresh seeds (not in the golden file): decode + prefill halves and layers, bit-for-bit."""
    seed, past, S = 77, 9, 5
    p = qo.synth_layer(seed, 2, 4)
    x = qo.synth(seed, qo.STREAM_ACT, qo.HIDDEN)
    kc, vc = kv_hist(seed, past, (past + 1) * qo.KV_WIDTH)
    k2, v2 = kc.copy(), vc.copy()
    st, out = qo.decode_layer(p, x, past, kc, vc)
    out2 = np.zeros(qo.HIDDEN, np.float32)
    args = (p["input_layernorm"], p["post_attention_layernorm"], p["q_w"], p["k_w"], p["v_w"], p["o_w"], p["gate_w"],
            p["up_w"], p["down_w"], p["q_bias"], p["k_bias"], p["v_bias"], p["q_s"], p["k_s"], p["v_s"], p["o_s"],
            p["gate_s"], p["up_s"], p["down_s"])
    assert ref_libs.decode.qwen_decode_layer_smoke_forward(x, past, *args, k2, v2, out2) == 0
    assert np.array_equal(out, out2) and np.array_equal(kc, k2) and np.array_equal(vc, v2)
    xs = qo.synth(seed, qo.STREAM_ACT + 5, S * qo.HIDDEN)
    kc = np.zeros(S * qo.KV_WIDTH, np.float32)
    vc, k2, v2 = kc.copy(), kc.copy(), kc.copy()
    st, out = qo.prefill_layer(p, xs, S, kc, vc)
    out2 = np.zeros(S * qo.HIDDEN, np.float32)
    assert ref_libs.prefill.qwen_prefill_layer_smoke_forward(xs, S, *qo.tiles_tuple(), *args, k2, v2, out2) == 0
    assert np.array_equal(out, out2) and np.array_equal(kc, k2) and np.array_equal(vc, v2)


def test_decode_history_regression_kat():
    """verification/validate_decode_attention_history_regression.py: sparse weights over a 2-token
    history, against its numpy reference with the int4 decoder done in int32 (the committed decoder
    subtracts 16 from a uint8 and wraps under NumPy 2)."""
    H, HD, KV = qo.HIDDEN, qo.HEAD_DIM, qo.KV_WIDTH

    def setw(packed, in_dim, o, i, val):
        flat = o * in_dim + i
        nib = val & 0xF
        if flat % 2 == 0:
            packed[flat // 2] = (packed[flat // 2] & 0xF0) | nib
        else:
            packed[flat // 2] = (packed[flat // 2] & 0x0F) | (nib << 4)

    x = np.zeros(H, np.float32)
    x[:4] = [1.0, -0.75, 0.5, 0.25]
    p = qo.LayerParams(4)
    qw, kw = np.zeros(H * H // 2, np.uint8), np.zeros(KV * H // 2, np.uint8)
    vw, ow = np.zeros(KV * H // 2, np.uint8), np.zeros(H * H // 2, np.uint8)
    setw(qw, H, 0, 0, 1)
    setw(qw, H, HD, 1, -1)
    setw(qw, H, 6 * HD, 2, 1)
    setw(qw, H, 7 * HD, 3, 1)
    setw(kw, H, 0, 0, 1)
    setw(kw, H, HD, 1, -1)
    setw(vw, H, 0, 0, 1)
    setw(vw, H, HD, 2, 1)
    setw(ow, H, 0, 0, 1)
    setw(ow, H, 1, HD, 1)
    setw(ow, H, 2, 6 * HD, 1)
    setw(ow, H, 3, 7 * HD, 1)
    p.tensors.update(q_w=qw, k_w=kw, v_w=vw, o_w=ow, q_s=np.ones(H, np.float32), k_s=np.ones(KV, np.float32),
                     v_s=np.ones(KV, np.float32), o_s=np.ones(H, np.float32), q_bias=np.zeros(H, np.float32),
                     k_bias=np.zeros(KV, np.float32), v_bias=np.zeros(KV, np.float32),
                     input_layernorm=np.ones(H, np.float32))
    kc = np.zeros(KV * 3, np.float32)
    vc = np.zeros(KV * 3, np.float32)
    for t in range(2):
        kc[t * KV] = 0.25 * (t + 1)
        kc[t * KV + HD] = -0.5 * (t + 1)
        vc[t * KV] = 1.25 * (t + 1)
        vc[t * KV + HD] = -1.5 * (t + 1)
    k_hist, v_hist = kc.copy(), vc.copy()
    st, out = qo.decode_attention(p, x, 2, kc, vc)
    assert st == 0

    def decode_mat(packed, out_dim, in_dim):
        flat = np.arange(out_dim * in_dim)
        b = packed[flat // 2].astype(np.int32)
        nib = np.where(flat % 2 == 1, (b >> 4) & 0xF, b & 0xF)
        return np.where(nib >= 8, nib - 16, nib).astype(np.float32).reshape(out_dim, in_dim)

    norm = x * (1.0 / np.sqrt(np.mean(x * x) + 1e-6))
    q = decode_mat(qw, H, H) @ norm
    k = decode_mat(kw, KV, H) @ norm
    v = decode_mat(vw, KV, H) @ norm
    cos, sin = qo.decode_rope_table(3)
    for h in range(12):
        e, o = q[h * HD:h * HD + 64].copy(), q[h * HD + 64:(h + 1) * HD].copy()
        q[h * HD:h * HD + 64] = e * cos[2] - o * sin[2]
        q[h * HD + 64:(h + 1) * HD] = o * cos[2] + e * sin[2]
    for h in range(2):
        e, o = k[h * HD:h * HD + 64].copy(), k[h * HD + 64:(h + 1) * HD].copy()
        k[h * HD:h * HD + 64] = e * cos[2] - o * sin[2]
        k[h * HD + 64:(h + 1) * HD] = o * cos[2] + e * sin[2]
    k_all, v_all = k_hist.copy(), v_hist.copy()
    k_all[2 * KV:] = k
    v_all[2 * KV:] = v
    ctx = np.zeros(H, np.float32)
    for h in range(12):
        g = h // 6
        s = np.array([q[h * HD:(h + 1) * HD] @ k_all[t * KV + g * HD:t * KV + (g + 1) * HD] for t in range(3)]) / np.sqrt(HD)
        pr = np.exp(s - s.max())
        pr /= pr.sum()
        ctx[h * HD:(h + 1) * HD] = sum(pr[t] * v_all[t * KV + g * HD:t * KV + (g + 1) * HD] for t in range(3))
    ref_out = decode_mat(ow, H, H) @ ctx
    assert np.max(np.abs(out - ref_out)) < 1e-4
    assert np.max(np.abs(kc - k_all)) < 1e-4 and np.max(np.abs(vc - v_all)) < 1e-4


def test_decode_attention_smoke_kat():
    """verification/validate_decode_attention_smoke.py expected value on the oracle."""
    H, KV = qo.HIDDEN, qo.KV_WIDTH
    p = qo.LayerParams(4)
    for name, (o, i) in {"q_w": (H, H), "k_w": (KV, H), "v_w": (KV, H), "o_w": (H, H)}.items():
        w = np.zeros(o * i // 2, np.uint8)
        w[0] = 1
        p.tensors[name] = w
    p.tensors.update(q_s=np.ones(H, np.float32), k_s=np.ones(KV, np.float32), v_s=np.ones(KV, np.float32),
                     o_s=np.ones(H, np.float32), q_bias=np.zeros(H, np.float32), k_bias=np.zeros(KV, np.float32),
                     v_bias=np.zeros(KV, np.float32), input_layernorm=np.ones(H, np.float32))
    x = np.zeros(H, np.float32)
    x[0] = 1.0
    kc, vc = np.zeros(KV, np.float32), np.zeros(KV, np.float32)
    st, out = qo.decode_attention(p, x, 0, kc, vc)
    expected = 1.0 / np.sqrt(1.0 / H + 1e-6)
    assert st == 0 and np.isclose(kc[0], expected, atol=1e-5) and np.isclose(out[0], expected, atol=1e-5)
    assert np.count_nonzero(out[1:]) == 0


# ---- restatement cross-checks of the elementwise arithmetic (numpy float32 = IEEE single) ----------
F = np.float32


def np_approx_exp(v: F) -> F:
    if v <= F(-16.0):
        return F(0.0)
    steps, s = 0, F(v)
    while s < F(-1.0):
        s = F(s * F(0.5))
        steps += 1
    term, series = F(1.0), F(1.0)
    for d in range(1, 7):
        term = F(term * F(s / F(d)))
        series = F(series + term)
    for _ in range(steps):
        series = F(series * series)
    return series if series > F(0.0) else F(0.0)


def np_approx_sqrt(v: F) -> F:
    if v <= F(0.0):
        return F(0.0)
    g = v if v > F(1.0) else F(1.0)
    for _ in range(6):
        g = F(F(0.5) * F(g + F(v / g)))
    return g


def test_approx_exp_and_sqrt_bit_exact():
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.uniform(-20, 2, 2000), [-16.0, -15.999, -1.0, -0.999, 0.0, 1.0, 12.0, -12.0]])
    for v in vals.astype(np.float32):
        assert np.float32(qo.approx_exp(float(v))).tobytes() == np_approx_exp(v).tobytes(), v
    for v in np.concatenate([rng.uniform(0, 4, 1000), rng.uniform(0, 1e-3, 500), [0.0, 1.0, 8e-4]]).astype(np.float32):
        assert np.float32(qo.approx_sqrt(float(v))).tobytes() == np_approx_sqrt(v).tobytes(), v
    # above -1 there is no range reduction: the reference's SiLU of -12 uses approx_exp(12) = the degree-6
    # Taylor sum 7457.8, far from e^12 = 162754.8; kept, not fixed
    assert abs(qo.approx_exp(12.0) - 7457.8) < 0.01


def test_prefill_rope_table_bit_exact():
    cos, sin = qo.prefill_rope_table(70)
    step = F(0.8058421877614801)
    pi, two_pi, half_pi = F(3.14159265358979323846), F(6.28318530717958647692), F(1.57079632679489661923)
    for pos in (0, 1, 17, 69):
        inv = F(1.0)
        for pair in range(64):
            a = F(F(pos) * inv)
            while a > pi:
                a = F(a - two_pi)
            while a < -pi:
                a = F(a + two_pi)
            sign = F(1.0)
            if a > half_pi:
                a, sign = F(pi - a), F(-1.0)
            elif a < -half_pi:
                a, sign = F(-pi - a), F(-1.0)
            x2 = F(a * a)
            t = F(F(1.0) + F(x2 * F(F(-1.0 / 6.0) + F(x2 * F(F(1.0 / 120.0) + F(x2 * F(-1.0 / 5040.0)))))))
            s = F(a * t)
            c = F(sign * F(F(1.0) + F(x2 * F(F(-0.5) + F(x2 * F(F(1.0 / 24.0) + F(x2 * F(-1.0 / 720.0))))))))
            assert cos[pos, pair].tobytes() == c.tobytes() and sin[pos, pair].tobytes() == s.tobytes()
            inv = F(inv * step)


def test_quantizer_matches_reference_formula():
    w = qo.synth(3, 99, 256 * 1536, 0, 0.02)
    for wb in (4, 8):
        a = qo.quantize_rows(w, 256, 1536, wb)
        b = qo.quantize_rows_numpy(w.reshape(256, 1536), wb)
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    z = np.zeros(2 * 16, np.float32)
    codes, scales = qo.quantize_rows(z, 2, 16, 4)
    assert np.all(scales == 1.0) and np.count_nonzero(codes) == 0


def test_bf16_rounding_matches_reference_formula():
    rng = np.random.default_rng(1)
    x = rng.normal(0, 3, 10000).astype(np.float32)
    x[:4] = [1.0, 1.00390625, 1.0078125 + 2 ** -9, -2.5]
    got = qo.round_bf16(x)
    bits = x.copy().view(np.uint32)
    bits = (bits + np.uint32(0x7FFF) + ((bits >> 16) & 1)) & np.uint32(0xFFFF0000)
    assert np.array_equal(got.view(np.uint32), bits)


def test_synthetic_generator_statistics_and_determinism():
    a = qo.synth(5, 7, 200000, 0.0, 0.02)
    b = qo.synth(5, 7, 200000, 0.0, 0.02)
    c = qo.synth(6, 7, 1000, 0.0, 0.02)
    assert np.array_equal(a, b) and not np.array_equal(a[:1000], c)
    assert abs(float(a.mean())) < 2e-4 and abs(float(a.std()) - 0.02) < 2e-4
    assert float(np.abs(a).max()) <= 6 * 0.02 + 1e-6  # Irwin-Hall(12) support is +-6 sigma


def test_attention_scaling_constant(golden):
    assert np.float32(0.08838834764831845) == np.float32(1.0 / np.sqrt(128.0))
    assert np.float32(golden["attention_scaling_f32"]) == np.float32(0.08838834764831845)
