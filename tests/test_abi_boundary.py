"""CPU tests of the drop-in boundary: the libraries load, export every entry point include/*.h declares, and
return the reference's status codes on every argument error that is detected before any GPU work. No
test here launches a kernel."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

import qwen_oracle as qo

ROOT = Path(__file__).resolve().parents[1]
HEADERS = {
    "qwen_decode_host_wrapper.h": "LIB_DECODE",
    "qwen_prefill_host_wrapper.h": "LIB_PREFILL",
    "qwen_b200_engine.h": "LIB_CORE",
    "qwen_b200_runtime.h": "LIB_CORE",
    "qwen_b200_ops.h": "LIB_CORE",
}


def declared(header: Path) -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b((?:qwen)_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def host(built_libs):
    from work_llm_accelerator_b200 import host as h

    return h


def test_every_declared_symbol_is_exported(host):
    import work_llm_accelerator_b200.build as b

    for header, lib_attr in HEADERS.items():
        names = declared(ROOT / "include" / header)
        assert names, header
        lib_path = getattr(b, lib_attr)
        nm = subprocess.run(["nm", "-D", "--defined-only", str(lib_path)], capture_output=True, text=True, check=True)
        exported = set(re.findall(r"\bT (\w+)", nm.stdout))
        missing = [n for n in names if n not in exported]
        assert not missing, (header, missing)
        lib = ctypes.CDLL(str(lib_path))
        for n in names:
            assert getattr(lib, n)


def test_reference_symbols_all_present(host, ref_libs):
    """Every entry point of the reference's two libraries is exported by the drop-in library of the same
    name (the layer0 fp32 golden layers included)."""
    import work_llm_accelerator_b200.build as b

    for ref_lib, ours in ((qo.REF_DECODE_LIB, b.LIB_DECODE), (qo.REF_PREFILL_LIB, b.LIB_PREFILL)):
        ref_syms = set(re.findall(r"\bT (qwen_\w+_forward)\b",
                                  subprocess.run(["nm", "-D", "--defined-only", str(ref_lib)], capture_output=True,
                                                 text=True).stdout))
        our_syms = set(re.findall(r"\bT (qwen_\w+)\b",
                                  subprocess.run(["nm", "-D", "--defined-only", str(ours)], capture_output=True,
                                                 text=True).stdout))
        assert ref_syms and ref_syms <= our_syms, ref_syms - our_syms


def _zero_ddr():
    lay = qo.layer_layout(4)
    return np.zeros(lay["total"], np.uint8), np.zeros(lay["total"] // 4, np.float32)


def test_decode_status_codes_match_reference(host, ref_libs):
    dec = host.load_decode_lib()
    w, s = _zero_ddr()
    sram = qo.sram_ports()
    kv = np.zeros(4 * qo.KV_WIDTH, np.float32)
    act = np.zeros(2 * qo.HIDDEN, np.float32)
    cases = [(28, 0), (-1, 0), (0, -1), (27, -5)]
    for layer, past in cases:
        a = dec.qwen_decode_top_smoke_forward(layer, past, 0, qo.HIDDEN * 4, 0, 0, 0, 2 * qo.KV_WIDTH * 4, w, s, kv,
                                              act, *sram)
        b = ref_libs.decode.qwen_decode_top_smoke_forward(layer, past, 0, qo.HIDDEN * 4, 0, 0, 0, 2 * qo.KV_WIDTH * 4,
                                                          w, s, kv, act, *sram)
        assert a == b == 10
    # negative history on the separate-array entry points -> 1
    z = np.zeros(qo.HIDDEN, np.float32)
    assert dec.qwen_decode_stub_forward(z, -1, z) == ref_libs.decode.qwen_decode_stub_forward(z, -1, z) == 1


def test_decode_null_ports(host):
    """A null port is reported as 11 (qwen_decode_top_wrapper.cpp:34-38); ctypes passes None as NULL."""
    dec = host.load_decode_lib()
    fn = dec.qwen_decode_top_smoke_forward
    saved = fn.argtypes
    try:
        fn.argtypes = [ctypes.c_int, ctypes.c_int] + [ctypes.c_uint64] * 6 + [ctypes.c_void_p] * 9
        w, s = _zero_ddr()
        ptrs = [w.ctypes.data, s.ctypes.data, np.zeros(4, np.float32).ctypes.data, np.zeros(4, np.float32).ctypes.data,
                np.zeros(1, np.uint8).ctypes.data, np.zeros(1, np.float32).ctypes.data,
                np.zeros(1, np.int32).ctypes.data, np.zeros(1, np.float32).ctypes.data,
                np.zeros(1, np.float32).ctypes.data]
        for i in range(9):
            p = list(ptrs)
            p[i] = None
            assert fn(0, 0, 0, 0, 0, 0, 0, 0, *p) == 11
    finally:
        fn.argtypes = saved


def test_prefill_status_codes_match_reference(host, ref_libs):
    pre = host.load_prefill_lib()
    w, s = _zero_ddr()
    sram = qo.sram_ports()
    S = 4
    H4, KV4 = qo.HIDDEN * 4, qo.KV_WIDTH * 4
    cases = [
        # (layer, seq, tiles, in, out, k, v) -> expected
        (0, S, {"attention_query": 16}, 0, S * H4, 0, S * KV4, 20),
        (0, S, {"attention_key": 32}, 0, S * H4, 0, S * KV4, 20),
        (0, S, {"attention_head_dim": 64}, 0, S * H4, 0, S * KV4, 1),
        (0, S, {"attention_seq": 256}, 0, S * H4, 0, S * KV4, 2),
        (0, S, {"attention_query_heads_parallel": 13}, 0, S * H4, 0, S * KV4, 2),
        (0, S, {"attention_kv_heads_parallel": 3}, 0, S * H4, 0, S * KV4, 2),
        (0, S, {"mlp_seq": 0}, 0, S * H4, 0, S * KV4, 20),
        (28, S, {}, 0, S * H4, 0, S * KV4, 20),
        (0, 0, {}, 0, S * H4, 0, S * KV4, 20),
        (0, 129, {}, 0, S * H4, 0, S * KV4, 20),
        (0, 40000, {}, 0, S * H4, 0, S * KV4, 20),
        (0, S, {}, 2, S * H4, 0, S * KV4, 22),          # misaligned input
        (0, S, {}, 0, 100, 0, S * KV4, 22),             # output overlaps input
        (0, S, {}, 0, S * H4, 0, 100 * 4, 22),          # v overlaps k
        (0, S, {}, 0, 128 * 3 * H4, 0, S * KV4, 22),    # output outside the activation window
        (0, S, {}, 0, S * H4, 255 * KV4, 0, 22),        # k outside the KV window
    ]
    for layer, seq, tiles, a_in, a_out, k_base, v_base, expect in cases:
        got = []
        for lib in (pre, ref_libs.prefill):
            x = np.zeros(3 * S * qo.HIDDEN, np.float32)
            kv = np.zeros(2 * S * qo.KV_WIDTH, np.float32)
            got.append(lib.qwen_prefill_top_smoke_forward(layer, seq, *qo.tiles_tuple(tiles), a_in, a_out, 0, 0,
                                                          k_base, v_base, w, s, kv, x, *sram))
        assert got[0] == got[1] == expect, (tiles, layer, seq, got)


def test_prefill_smoke_entry_status_codes(host, ref_libs):
    pre = host.load_prefill_lib()
    S = 3
    p = {k: np.zeros(1 << 24, np.uint8) for k in ("w",)}
    f = lambda n: np.zeros(n, np.float32)  # noqa: E731
    bw = p["w"]
    for tiles, expect in (({"attention_query": 64}, 2), ({"attention_key": 0}, 1), ({"attention_seq": 129}, 2),
                          ({"attention_hidden_proj": 128}, 2)):
        got = []
        for lib in (pre, ref_libs.prefill):
            got.append(lib.qwen_prefill_attention_smoke_forward(
                f(S * qo.HIDDEN), S, *qo.tiles_tuple(tiles)[:8], f(qo.HIDDEN), bw, bw, bw, bw, f(qo.HIDDEN),
                f(qo.KV_WIDTH), f(qo.KV_WIDTH), f(qo.HIDDEN), f(qo.KV_WIDTH), f(qo.KV_WIDTH), f(qo.HIDDEN),
                f(S * qo.KV_WIDTH), f(S * qo.KV_WIDTH), f(S * qo.HIDDEN)))
        assert got[0] == got[1] == expect, (tiles, got)
    for m_seq, m_hidden, m_ff, expect in ((1, 512, 640, 1), (1, 256, 641, 1), (0, 256, 640, 1), (1, 0, 640, 1)):
        got = []
        for lib in (pre, ref_libs.prefill):
            got.append(lib.qwen_prefill_mlp_smoke_forward(f(S * qo.HIDDEN), S, m_seq, m_hidden, m_ff, f(qo.HIDDEN), bw,
                                                          bw, bw, f(qo.INTER), f(qo.INTER), f(qo.HIDDEN),
                                                          f(S * qo.HIDDEN)))
        assert got[0] == got[1] == expect
    # glue: non-default tiles -> 2 before any work
    z = f(S * qo.HIDDEN)
    args = [f(qo.HIDDEN), f(qo.HIDDEN)] + [bw] * 7 + [f(qo.INTER)] * 10 + [f(S * qo.KV_WIDTH), f(S * qo.KV_WIDTH), z]
    for lib in (pre, ref_libs.prefill):
        assert lib.qwen_prefill_glue_smoke_forward(z, S, *qo.tiles_tuple({"mlp_ff": 320}), *args) == 2


def test_capacity_setting(host):
    cap = host.prefill_seq_capacity()
    assert cap == 128 or cap > 0
    with pytest.raises(ValueError):
        host.set_prefill_seq_capacity(0)
    with pytest.raises(ValueError):
        host.set_prefill_seq_capacity(40000)
    host.set_prefill_seq_capacity(4096)
    assert host.prefill_seq_capacity() == 4096
    host.set_prefill_seq_capacity(cap)


def test_fails_loudly_without_a_device(host, gpu_available):
    """On a machine without a CUDA device the product returns status 31 with a message; it never computes
    on the CPU."""
    if gpu_available:
        pytest.skip("a CUDA device is present")
    dec = host.load_decode_lib()
    w, s = _zero_ddr()
    kv = np.zeros(4 * qo.KV_WIDTH, np.float32)
    act = np.zeros(2 * qo.HIDDEN, np.float32)
    st = dec.qwen_decode_top_smoke_forward(0, 1, 0, qo.HIDDEN * 4, 0, 0, 0, 2 * qo.KV_WIDTH * 4, w, s, kv, act,
                                           *qo.sram_ports())
    assert st == 31
    assert "no CUDA device" in host.last_error()
    assert np.count_nonzero(act[qo.HIDDEN:]) == 0
    with pytest.raises(host.EngineError):
        host.Engine(0, 8, 1, 128)
