"""ctypes bindings for the oracle: the C restatement (libqwen_oracle.so) and the reference's own host
libraries built from its sources (oracle/_ref/).

TEST INFRASTRUCTURE ONLY. Imported by tests/, __graft_entry__.smoke() and bench.py's CPU legs, as the
checker; the product package never imports this module.

The synthetic-parameter layout helpers here restate the reference's DDR layout
(hls/common/llm_memory_layout.h:55-128) independently of the product's own copy, so that a layout
mistake in the product cannot hide behind a shared helper.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_LIB = HERE / "libqwen_oracle.so"
REF_DIR = HERE / "_ref"
REF_DECODE_LIB = REF_DIR / "libqwen_decode_stub.so"
REF_PREFILL_LIB = REF_DIR / "libqwen_prefill_stub.so"
REF_PREFILL_CAP4096_LIB = REF_DIR / "libqwen_prefill_stub_cap4096.so"

HIDDEN = 1536
INTER = 8960
HEADS = 12
KV_HEADS = 2
HEAD_DIM = 128
KV_WIDTH = KV_HEADS * HEAD_DIM
LAYERS = 28
VOCAB = 151936
EPS = 1.0e-6
MAX_SEQ = 32768

# reference default prefill tiles (hls/common/qwen2_model_config.h:55-69, llm_layer_dispatch.h:50-61)
DEFAULT_TILES = dict(
    attention_seq=128, attention_query=32, attention_key=64, attention_hidden_proj=64, attention_kv_proj=64,
    attention_head_dim=128, attention_query_heads_parallel=2, attention_kv_heads_parallel=1,
    mlp_seq=128, mlp_hidden=256, mlp_ff=640,
)
TILE_ORDER = list(DEFAULT_TILES.keys())

_F = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_B = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_I = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_H = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_c = ctypes


def build_port() -> Path:
    """Build libqwen_oracle.so with oracle/Makefile if it is missing."""
    if not PORT_LIB.exists():
        subprocess.run(["make", "-s", "-C", str(HERE), "port"], check=True)
    return PORT_LIB


_port = None


def port() -> ctypes.CDLL:
    global _port
    if _port is None:
        lib = ctypes.CDLL(str(build_port()))
        lib.oracle_decode_attention.argtypes = [_c.c_int, _F, _c.c_int, _F, _B, _B, _B, _B, _F, _F, _F, _F, _F, _F, _F,
                                                _F, _F, _F]
        lib.oracle_decode_mlp.argtypes = [_c.c_int, _F, _F, _B, _B, _B, _F, _F, _F, _F]
        lib.oracle_prefill_attention.argtypes = [_c.c_int, _F, _c.c_int, _F, _B, _B, _B, _B, _F, _F, _F, _F, _F, _F,
                                                 _F, _F, _F, _F]
        lib.oracle_prefill_mlp.argtypes = [_c.c_int, _F, _c.c_int, _F, _B, _B, _B, _F, _F, _F, _F]
        for name in ("oracle_decode_attention", "oracle_decode_mlp", "oracle_prefill_attention", "oracle_prefill_mlp"):
            getattr(lib, name).restype = _c.c_int
        lib.oracle_expf_array.argtypes = [_F, _F, _c.c_uint64]
        lib.oracle_approx_exp.argtypes = [_c.c_float]
        lib.oracle_approx_exp.restype = _c.c_float
        lib.oracle_approx_sqrt.argtypes = [_c.c_float]
        lib.oracle_approx_sqrt.restype = _c.c_float
        lib.oracle_wrap_angle.argtypes = [_c.c_float]
        lib.oracle_wrap_angle.restype = _c.c_float
        lib.oracle_approx_sincos.argtypes = [_c.c_float, _c.POINTER(_c.c_float), _c.POINTER(_c.c_float)]
        lib.oracle_prefill_rope_cos_sin.argtypes = [_c.c_int, _F, _F]
        lib.oracle_decode_rope_cos_sin.argtypes = [_c.c_int, _F, _F]
        lib.oracle_decode_rmsnorm.argtypes = [_F, _F, _c.c_float, _F]
        lib.oracle_prefill_rmsnorm.argtypes = [_F, _F, _c.c_float, _F]
        lib.oracle_round_bf16.argtypes = [_F, _c.c_uint64]
        lib.oracle_quantize_rows.argtypes = [_F, _c.c_int, _c.c_int, _c.c_int, _B, _F]
        lib.oracle_synth_normal.argtypes = [_c.c_uint64, _c.c_uint64, _c.c_uint64, _c.c_float, _c.c_float]
        lib.oracle_synth_normal.restype = _c.c_float
        lib.oracle_synth_fill.argtypes = [_c.c_uint64, _c.c_uint64, _c.c_uint64, _c.c_float, _c.c_float, _F]
        lib.oracle_f32_to_f16.argtypes = [_c.c_float]
        lib.oracle_f32_to_f16.restype = _c.c_uint16
        lib.oracle_lm_head_argmax.argtypes = [_F, _F, _H, _c.c_int, _c.c_void_p]
        lib.oracle_lm_head_argmax.restype = _c.c_int
        lib.oracle_project.argtypes = [_F, _B, _c.c_int, _c.c_void_p, _F, _c.c_int, _c.c_int, _F]
        _port = lib
    return _port


# ---------------------------------------------------------------------------------------------------
# layout (restated from hls/common/llm_memory_layout.h:55-128; wbits=8 uses one byte per weight)
# ---------------------------------------------------------------------------------------------------
_WEIGHT_SHAPES = {
    "q": (HIDDEN, HIDDEN), "k": (KV_WIDTH, HIDDEN), "v": (KV_WIDTH, HIDDEN), "o": (HIDDEN, HIDDEN),
    "gate": (INTER, HIDDEN), "up": (INTER, HIDDEN), "down": (HIDDEN, INTER),
}


def weight_bytes(name: str, wbits: int) -> int:
    out_dim, in_dim = _WEIGHT_SHAPES[name]
    return out_dim * in_dim * wbits // 8


def layer_layout(wbits: int = 4) -> dict[str, int]:
    off = 0
    lay: dict[str, int] = {}

    def put(key: str, nbytes: int) -> None:
        nonlocal off
        lay[key] = off
        off += nbytes

    put("input_layernorm", HIDDEN * 4)
    for name in ("q", "k", "v", "o"):
        put(f"{name}_weight", weight_bytes(name, wbits))
    put("post_attention_layernorm", HIDDEN * 4)
    for name in ("gate", "up", "down"):
        put(f"{name}_weight", weight_bytes(name, wbits))
    put("q_bias", HIDDEN * 4)
    put("k_bias", KV_WIDTH * 4)
    put("v_bias", KV_WIDTH * 4)
    put("q_scale", HIDDEN * 4)
    put("k_scale", KV_WIDTH * 4)
    put("v_scale", KV_WIDTH * 4)
    put("o_scale", HIDDEN * 4)
    put("gate_scale", INTER * 4)
    put("up_scale", INTER * 4)
    put("down_scale", HIDDEN * 4)
    lay["total"] = off
    return lay


# ---------------------------------------------------------------------------------------------------
# synthetic parameters (deterministic generator shared with the device)
# ---------------------------------------------------------------------------------------------------
STREAM = {
    "input_layernorm": 0, "q": 1, "k": 2, "v": 3, "o": 4, "post_attention_layernorm": 5, "gate": 6, "up": 7,
    "down": 8, "q_bias": 9, "k_bias": 10, "v_bias": 11,
}
STREAM_EMBED = 1 << 20
STREAM_FINAL_NORM = (1 << 20) + 1
STREAM_ACT = 1 << 21  # + user index: activations / KV history


def layer_stream(layer: int, name: str) -> int:
    return layer * 32 + STREAM[name]


def synth(seed: int, stream: int, count: int, mean: float = 0.0, sigma: float = 1.0) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    port().oracle_synth_fill(seed, stream, count, mean, sigma, out)
    return out


def quantize_rows(w: np.ndarray, out_dim: int, in_dim: int, wbits: int) -> tuple[np.ndarray, np.ndarray]:
    w = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    nbytes = out_dim * in_dim * wbits // 8
    codes = np.zeros(nbytes, dtype=np.uint8)
    scales = np.zeros(out_dim, dtype=np.float32)
    port().oracle_quantize_rows(w, out_dim, in_dim, wbits, codes, scales)
    return codes, scales


def quantize_rows_numpy(matrix: np.ndarray, wbits: int) -> tuple[np.ndarray, np.ndarray]:
    """numpy statement of real_host_top_backend.py:31-41 (qmax 7 / nibbles), extended to int8 (qmax 127)."""
    qmax = 127.0 if wbits == 8 else 7.0
    lo, hi = (-128, 127) if wbits == 8 else (-8, 7)
    matrix = np.asarray(matrix, dtype=np.float32)
    max_abs = np.max(np.abs(matrix), axis=1)
    scales = np.where(max_abs > 0.0, max_abs / np.float32(qmax), np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint(matrix / scales[:, None]).astype(np.int32), lo, hi)
    if wbits == 8:
        return q.astype(np.int8).view(np.uint8).reshape(-1).copy(), scales
    nib = np.where(q < 0, q + 16, q).astype(np.uint8).reshape(-1)
    if nib.size % 2:
        nib = np.concatenate([nib, np.zeros(1, np.uint8)])
    return (nib[0::2] | (nib[1::2] << 4)).astype(np.uint8), scales


@dataclass
class LayerParams:
    """One decoder layer's quantized parameters, as separate arrays and as the reference DDR images."""

    wbits: int
    tensors: dict[str, np.ndarray] = field(default_factory=dict)

    def ddr(self) -> tuple[np.ndarray, np.ndarray]:
        lay = layer_layout(self.wbits)
        weight_ddr = np.zeros(lay["total"], dtype=np.uint8)
        scale_ddr = np.zeros((lay["total"] + 3) // 4, dtype=np.float32)
        for name in ("q", "k", "v", "o", "gate", "up", "down"):
            off = lay[f"{name}_weight"]
            w = self.tensors[f"{name}_w"]
            weight_ddr[off:off + w.size] = w
            so = lay[f"{name}_scale"] // 4
            s = self.tensors[f"{name}_s"]
            scale_ddr[so:so + s.size] = s
        for name in ("input_layernorm", "post_attention_layernorm", "q_bias", "k_bias", "v_bias"):
            so = lay[name] // 4
            v = self.tensors[name]
            scale_ddr[so:so + v.size] = v
        return weight_ddr, scale_ddr

    def __getitem__(self, key: str) -> np.ndarray:
        return self.tensors[key]


def synth_layer(seed: int, layer: int, wbits: int, weight_sigma: float = 0.02) -> LayerParams:
    """Seeded synthetic layer: weights N(0, sigma) quantized per output channel, biases N(0, 0.02),
    RMSNorm weights N(1, 0.02)."""
    p = LayerParams(wbits)
    for name, (out_dim, in_dim) in _WEIGHT_SHAPES.items():
        w = synth(seed, layer_stream(layer, name), out_dim * in_dim, 0.0, weight_sigma)
        p.tensors[f"{name}_w"], p.tensors[f"{name}_s"] = quantize_rows(w, out_dim, in_dim, wbits)
    for name in ("input_layernorm", "post_attention_layernorm"):
        p.tensors[name] = synth(seed, layer_stream(layer, name), HIDDEN, 1.0, 0.02)
    p.tensors["q_bias"] = synth(seed, layer_stream(layer, "q_bias"), HIDDEN, 0.0, 0.02)
    p.tensors["k_bias"] = synth(seed, layer_stream(layer, "k_bias"), KV_WIDTH, 0.0, 0.02)
    p.tensors["v_bias"] = synth(seed, layer_stream(layer, "v_bias"), KV_WIDTH, 0.0, 0.02)
    return p


def synth_embedding(seed: int) -> np.ndarray:
    """fp16 [VOCAB, HIDDEN] table N(0, 0.02), as uint16 bits."""
    vals = synth(seed, STREAM_EMBED, VOCAB * HIDDEN, 0.0, 0.02)
    return vals.astype(np.float16).view(np.uint16).reshape(VOCAB, HIDDEN)


def synth_final_norm(seed: int) -> np.ndarray:
    return synth(seed, STREAM_FINAL_NORM, HIDDEN, 1.0, 0.02)


# ---------------------------------------------------------------------------------------------------
# oracle calls (numpy in, numpy out)
# ---------------------------------------------------------------------------------------------------
def _f(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).reshape(-1)


def decode_attention(p: LayerParams, x: np.ndarray, past: int, k_cache: np.ndarray, v_cache: np.ndarray):
    """Returns (status, out); k_cache / v_cache (flat, >= (past+1)*256) are updated in place."""
    out = np.zeros(HIDDEN, np.float32)
    st = port().oracle_decode_attention(p.wbits, _f(x), past, p["input_layernorm"], p["q_w"], p["k_w"], p["v_w"],
                                        p["o_w"], p["q_bias"], p["k_bias"], p["v_bias"], p["q_s"], p["k_s"],
                                        p["v_s"], p["o_s"], k_cache, v_cache, out)
    return st, out


def decode_mlp(p: LayerParams, a: np.ndarray):
    out = np.zeros(HIDDEN, np.float32)
    st = port().oracle_decode_mlp(p.wbits, _f(a), p["post_attention_layernorm"], p["gate_w"], p["up_w"], p["down_w"],
                                  p["gate_s"], p["up_s"], p["down_s"], out)
    return st, out


def decode_layer(p: LayerParams, x: np.ndarray, past: int, k_cache: np.ndarray, v_cache: np.ndarray):
    st, a = decode_attention(p, x, past, k_cache, v_cache)
    if st:
        return st, None
    return decode_mlp(p, a)


def prefill_attention(p: LayerParams, x: np.ndarray, seq_len: int, k_cache: np.ndarray, v_cache: np.ndarray):
    out = np.zeros(seq_len * HIDDEN, np.float32)
    st = port().oracle_prefill_attention(p.wbits, _f(x), seq_len, p["input_layernorm"], p["q_w"], p["k_w"],
                                         p["v_w"], p["o_w"], p["q_bias"], p["k_bias"], p["v_bias"], p["q_s"],
                                         p["k_s"], p["v_s"], p["o_s"], k_cache, v_cache, out)
    return st, out


def prefill_mlp(p: LayerParams, a: np.ndarray, seq_len: int):
    out = np.zeros(seq_len * HIDDEN, np.float32)
    st = port().oracle_prefill_mlp(p.wbits, _f(a), seq_len, p["post_attention_layernorm"], p["gate_w"], p["up_w"],
                                   p["down_w"], p["gate_s"], p["up_s"], p["down_s"], out)
    return st, out


def prefill_layer(p: LayerParams, x: np.ndarray, seq_len: int, k_cache: np.ndarray, v_cache: np.ndarray):
    st, a = prefill_attention(p, x, seq_len, k_cache, v_cache)
    if st:
        return st, None
    return prefill_mlp(p, a, seq_len)


def round_bf16(x: np.ndarray) -> np.ndarray:
    y = np.ascontiguousarray(x, dtype=np.float32).copy()
    port().oracle_round_bf16(y.reshape(-1), y.size)
    return y


def host_expf(x: np.ndarray) -> np.ndarray:
    """expf of every element by this machine's C library (the reference host library's std::exp on floats)."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    port().oracle_expf_array(x, y, x.size)
    return y


def approx_exp(v: float) -> float:
    return port().oracle_approx_exp(v)


def approx_sqrt(v: float) -> float:
    return port().oracle_approx_sqrt(v)


def approx_sincos(a: float) -> tuple[float, float]:
    s, c = ctypes.c_float(), ctypes.c_float()
    port().oracle_approx_sincos(a, ctypes.byref(s), ctypes.byref(c))
    return s.value, c.value


def prefill_rope_table(positions: int) -> tuple[np.ndarray, np.ndarray]:
    cos = np.zeros((positions, HEAD_DIM // 2), np.float32)
    sin = np.zeros((positions, HEAD_DIM // 2), np.float32)
    for pos in range(positions):
        port().oracle_prefill_rope_cos_sin(pos, cos[pos], sin[pos])
    return cos, sin


def decode_rope_table(positions: int) -> tuple[np.ndarray, np.ndarray]:
    cos = np.zeros((positions, HEAD_DIM // 2), np.float32)
    sin = np.zeros((positions, HEAD_DIM // 2), np.float32)
    for pos in range(positions):
        port().oracle_decode_rope_cos_sin(pos, cos[pos], sin[pos])
    return cos, sin


def lm_head_argmax(hidden: np.ndarray, norm_w: np.ndarray, embed_u16: np.ndarray, want_logits: bool = False):
    logits = np.zeros(VOCAB, np.float32) if want_logits else None
    tok = port().oracle_lm_head_argmax(_f(hidden), _f(norm_w), np.ascontiguousarray(embed_u16).reshape(-1), VOCAB,
                                       logits.ctypes.data if want_logits else None)
    return (tok, logits) if want_logits else tok


# ---------------------------------------------------------------------------------------------------
# the reference's own host libraries (built from its sources by oracle/Makefile)
# ---------------------------------------------------------------------------------------------------
class RefLibs:
    """ctypes handles on the reference .so files with the argtypes the reference's callers use
    (verification/real_host_top_backend.py:78-136, verification/validate_*_smoke.py)."""

    def __init__(self, decode_path: Path = REF_DECODE_LIB, prefill_path: Path = REF_PREFILL_LIB):
        if not Path(decode_path).exists() or not Path(prefill_path).exists():
            raise FileNotFoundError("reference libraries not built (make -C oracle ref)")
        self.decode = ctypes.CDLL(str(decode_path))
        self.prefill = ctypes.CDLL(str(prefill_path))
        configure_abi(self.decode, self.prefill)


def configure_abi(decode: ctypes.CDLL | None, prefill: ctypes.CDLL | None) -> None:
    """Set argtypes/restype for every exported entry point of the reference C-ABI
    (hls/decode_only/qwen_decode_host_wrapper.h:9-113, hls/prefill_only/qwen_prefill_host_wrapper.h:9-215).
    Used for both the reference libraries and the product's drop-in libraries."""
    i, u64 = _c.c_int, _c.c_uint64
    if decode is not None:
        decode.qwen_decode_stub_forward.argtypes = [_F, i, _F]
        decode.qwen_decode_attention_smoke_forward.argtypes = [_F, i, _F, _B, _B, _B, _B, _F, _F, _F, _F, _F, _F, _F,
                                                               _F, _F, _F]
        decode.qwen_decode_mlp_smoke_forward.argtypes = [_F, _F, _B, _B, _B, _F, _F, _F, _F]
        decode.qwen_decode_top_smoke_forward.argtypes = [i, i, u64, u64, u64, u64, u64, u64, _B, _F, _F, _F, _B, _F,
                                                         _I, _F, _F]
        decode.qwen_decode_layer_smoke_forward.argtypes = [_F, i, _F, _F, _B, _B, _B, _B, _B, _B, _B, _F, _F, _F, _F,
                                                           _F, _F, _F, _F, _F, _F, _F, _F, _F]
        for n in ("qwen_decode_stub_forward", "qwen_decode_attention_smoke_forward", "qwen_decode_mlp_smoke_forward",
                  "qwen_decode_top_smoke_forward", "qwen_decode_layer_smoke_forward"):
            getattr(decode, n).restype = i
        if hasattr(decode, "qwen_decode_layer0_reference_forward"):
            # pointers as c_void_p: the biases may be null
            vp = _c.c_void_p
            decode.qwen_decode_layer0_reference_forward.argtypes = [vp, i] + [vp] * 18 + [_c.c_float, vp, vp, vp]
            decode.qwen_decode_layer0_reference_forward.restype = i
    if prefill is not None:
        t11 = [i] * 11
        prefill.qwen_prefill_stub_forward.argtypes = [_F, i] + t11 + [_F]
        prefill.qwen_prefill_attention_smoke_forward.argtypes = [_F, i] + [i] * 8 + [_F, _B, _B, _B, _B] + [_F] * 10
        prefill.qwen_prefill_mlp_smoke_forward.argtypes = [_F, i, i, i, i, _F, _B, _B, _B, _F, _F, _F, _F]
        prefill.qwen_prefill_layer_smoke_forward.argtypes = [_F, i] + t11 + [_F, _F] + [_B] * 7 + [_F] * 13
        prefill.qwen_prefill_glue_smoke_forward.argtypes = [_F, i] + t11 + [_F, _F] + [_B] * 7 + [_F] * 13
        prefill.qwen_prefill_top_smoke_forward.argtypes = [i, i] + t11 + [u64] * 6 + [_B, _F, _F, _F, _B, _F, _I, _F,
                                                                                       _F]
        for n in ("qwen_prefill_stub_forward", "qwen_prefill_attention_smoke_forward", "qwen_prefill_mlp_smoke_forward",
                  "qwen_prefill_layer_smoke_forward", "qwen_prefill_glue_smoke_forward",
                  "qwen_prefill_top_smoke_forward"):
            getattr(prefill, n).restype = i
        if hasattr(prefill, "qwen_prefill_layer0_reference_forward"):
            vp = _c.c_void_p
            prefill.qwen_prefill_layer0_reference_forward.argtypes = [vp, i] + [vp] * 16 + [_c.c_float, vp]
            prefill.qwen_prefill_layer0_reference_forward.restype = i
            prefill.qwen_prefill_layer0_reference_forward_with_cache.argtypes = ([vp, i] + [vp] * 16 +
                                                                                 [_c.c_float, vp, vp, vp])
            prefill.qwen_prefill_layer0_reference_forward_with_cache.restype = i


def sram_ports() -> tuple:
    """The five SRAM ports the reference's caller passes (1-element arrays; only null-checked),
    verification/real_host_top_backend.py:190-197."""
    return (np.zeros(1, np.uint8), np.zeros(1, np.float32), np.zeros(1, np.int32), np.zeros(1, np.float32),
            np.zeros(1, np.float32))


def tiles_tuple(tiles: dict | None = None) -> tuple:
    t = dict(DEFAULT_TILES)
    if tiles:
        t.update(tiles)
    return tuple(int(t[k]) for k in TILE_ORDER)


def reference_threads() -> int:
    return int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
