#!/usr/bin/env python3
"""Generate tests/golden/golden.json: digests and sample values of the reference's own host libraries
(built from the reference sources into oracle/_ref/ by `make -C oracle ref`) on seeded synthetic cases,
plus the reference test suite's sparse known-answer cases. Every digest is also checked against the C
restatement (oracle/libqwen_oracle.so) before it is written, so the fixture both pins the restatement and
records the reference's outputs for hosts where the reference cannot be built.

Run from the repository root:  python tests/golden/make_golden.py
Needs the reference sources (for oracle/_ref); takes about a minute.
"""
from __future__ import annotations

import hashlib
import json
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))
import qwen_full_model  # noqa: E402
import qwen_oracle as qo  # noqa: E402

OUT = Path(__file__).resolve().parent / "golden.json"


def digest(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def head(a: np.ndarray, n: int = 8) -> list[float]:
    return [float(v) for v in np.asarray(a, np.float32).reshape(-1)[:n]]


def kv_history(seed: int, past: int, size: int) -> tuple[np.ndarray, np.ndarray]:
    k = np.zeros(size, np.float32)
    v = np.zeros(size, np.float32)
    k[:past * qo.KV_WIDTH] = qo.synth(seed, qo.STREAM_ACT + 1, past * qo.KV_WIDTH)
    v[:past * qo.KV_WIDTH] = qo.synth(seed, qo.STREAM_ACT + 2, past * qo.KV_WIDTH)
    return k, v


def decode_cases(ref: qo.RefLibs) -> list[dict]:
    cases = []
    for seed, past in ((11, 128), (12, 5), (13, 0)):
        p = qo.synth_layer(seed, 0, 4)
        x = qo.synth(seed, qo.STREAM_ACT, qo.HIDDEN)
        kc, vc = kv_history(seed, past, (past + 1) * qo.KV_WIDTH)
        k2, v2 = kc.copy(), vc.copy()
        st, out = qo.decode_layer(p, x, past, kc, vc)
        out2 = np.zeros(qo.HIDDEN, np.float32)
        st2 = ref.decode.qwen_decode_layer_smoke_forward(
            x, past, p["input_layernorm"], p["post_attention_layernorm"], p["q_w"], p["k_w"], p["v_w"], p["o_w"],
            p["gate_w"], p["up_w"], p["down_w"], p["q_bias"], p["k_bias"], p["v_bias"], p["q_s"], p["k_s"], p["v_s"],
            p["o_s"], p["gate_s"], p["up_s"], p["down_s"], k2, v2, out2)
        assert st == st2 == 0
        assert np.array_equal(out, out2) and np.array_equal(kc, k2) and np.array_equal(vc, v2), "port != reference"
        row = slice(past * qo.KV_WIDTH, (past + 1) * qo.KV_WIDTH)
        cases.append(dict(kind="decode_layer", seed=seed, past=past, out_sha=digest(out2), kv_sha=digest(k2[row], v2[row]),
                          out_head=head(out2), k_head=head(k2[row]), v_head=head(v2[row])))
        # attention half alone
        k3, v3 = kv_history(seed, past, (past + 1) * qo.KV_WIDTH)
        a3 = np.zeros(qo.HIDDEN, np.float32)
        st3 = ref.decode.qwen_decode_attention_smoke_forward(
            x, past, p["input_layernorm"], p["q_w"], p["k_w"], p["v_w"], p["o_w"], p["q_bias"], p["k_bias"],
            p["v_bias"], p["q_s"], p["k_s"], p["v_s"], p["o_s"], k3, v3, a3)
        st4, a4 = qo.decode_attention(p, x, past, *kv_history(seed, past, (past + 1) * qo.KV_WIDTH))
        assert st3 == st4 == 0 and np.array_equal(a3, a4)
        cases.append(dict(kind="decode_attention", seed=seed, past=past, out_sha=digest(a3), out_head=head(a3)))
        # MLP half alone on the attention output
        m5 = np.zeros(qo.HIDDEN, np.float32)
        st5 = ref.decode.qwen_decode_mlp_smoke_forward(a3, p["post_attention_layernorm"], p["gate_w"], p["up_w"],
                                                       p["down_w"], p["gate_s"], p["up_s"], p["down_s"], m5)
        st6, m6 = qo.decode_mlp(p, a3)
        assert st5 == st6 == 0 and np.array_equal(m5, m6)
        cases.append(dict(kind="decode_mlp", seed=seed, past=past, out_sha=digest(m5), out_head=head(m5)))
    return cases


def prefill_cases(ref: qo.RefLibs, ref_cap: qo.RefLibs | None) -> list[dict]:
    cases = []
    for seed, S, lib in ((21, 16, ref), (22, 7, ref), (23, 1, ref), (24, 130, ref_cap)):
        if lib is None:
            continue
        p = qo.synth_layer(seed, 0, 4)
        x = qo.synth(seed, qo.STREAM_ACT, S * qo.HIDDEN)
        kc = np.zeros(S * qo.KV_WIDTH, np.float32)
        vc = kc.copy()
        k2, v2 = kc.copy(), kc.copy()
        st, out = qo.prefill_layer(p, x, S, kc, vc)
        out2 = np.zeros(S * qo.HIDDEN, np.float32)
        st2 = lib.prefill.qwen_prefill_layer_smoke_forward(
            x, S, *qo.tiles_tuple(), p["input_layernorm"], p["post_attention_layernorm"], p["q_w"], p["k_w"], p["v_w"],
            p["o_w"], p["gate_w"], p["up_w"], p["down_w"], p["q_bias"], p["k_bias"], p["v_bias"], p["q_s"], p["k_s"],
            p["v_s"], p["o_s"], p["gate_s"], p["up_s"], p["down_s"], k2, v2, out2)
        assert st == st2 == 0, (st, st2)
        assert np.array_equal(out, out2) and np.array_equal(kc, k2) and np.array_equal(vc, v2), "port != reference"
        cases.append(dict(kind="prefill_layer", seed=seed, seq_len=S, capacity=4096 if lib is ref_cap else 128,
                          out_sha=digest(out2), kv_sha=digest(k2, v2), out_head=head(out2), k_head=head(k2)))
    return cases


def full_model_case(seed: int = 31, S: int = 8, steps: int = 4, kind: str = "full_model_w4") -> dict:
    rng = np.random.default_rng(seed)
    prompt = rng.integers(0, qo.VOCAB, S).tolist()
    m_ref = qwen_full_model.OracleModel(seed, 4, use_reference_libs=True)
    m_port = qwen_full_model.OracleModel(seed, 4)
    toks_ref, toks_port, hid = [], [], []
    t_ref, t_port = m_ref.prefill(prompt), m_port.prefill(prompt)
    assert all(np.array_equal(a, b) for a, b in zip(m_ref.hidden_trace, m_port.hidden_trace))
    hid.append(digest(*m_ref.hidden_trace))
    toks_ref.append(t_ref)
    toks_port.append(t_port)
    for _ in range(steps):
        t_ref, t_port = m_ref.decode(toks_ref[-1]), m_port.decode(toks_port[-1])
        assert all(np.array_equal(a, b) for a, b in zip(m_ref.hidden_trace, m_port.hidden_trace))
        hid.append(digest(*m_ref.hidden_trace))
        toks_ref.append(t_ref)
        toks_port.append(t_port)
    assert toks_ref == toks_port
    return dict(kind=kind, seed=seed, prompt=prompt, tokens=toks_ref, hidden_sha=hid,
                final_hidden_head=head(m_ref.hidden_trace[-1]))


def main() -> None:
    t0 = time.time()
    ref = qo.RefLibs()
    ref_cap = qo.RefLibs(prefill_path=qo.REF_PREFILL_CAP4096_LIB) if qo.REF_PREFILL_CAP4096_LIB.exists() else None
    golden = {
        "about": "reference host-library outputs on seeded synthetic inputs (oracle/qwen_oracle.py generators); "
                 "sha256 over the raw little-endian float32 bytes",
        "attention_scaling_f32": float(np.float32(1.0 / np.sqrt(np.float64(128.0)))),
        "cases": decode_cases(ref) + prefill_cases(ref, ref_cap) + [
            full_model_case(),
            # a longer greedy run: 32-token prompt, 16 decode steps
            full_model_case(seed=37, S=32, steps=16, kind="full_model_w4_long"),
        ],
    }
    OUT.write_text(json.dumps(golden, indent=1) + "\n")
    print(f"wrote {OUT} ({len(golden['cases'])} cases) in {time.time() - t0:.1f}s")


if __name__ == "__main__":
    main()
