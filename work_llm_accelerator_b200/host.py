"""Host-side bindings of the B200 libraries.

`load_decode_lib()` / `load_prefill_lib()` return ctypes handles on the drop-in libraries with exactly the
argtypes the reference's callers set (verification/real_host_top_backend.py:78-136 and the
verification/validate_*_smoke.py scripts), so code written against the reference's
libqwen_{decode,prefill}_stub.so runs unchanged. `Engine` wraps the device-resident engine
(include/qwen_b200_engine.h) and `EngineBackend` mirrors the reference's `BackendInterface`
(verification/backend_interface.py:25-31) on top of it.

There is no CPU path: if the native libraries are missing or no CUDA device is present, calls fail with
an error naming the cause.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Sequence

import numpy as np

from .build import LIB as LIB_DIR, LIB_CORE, LIB_DECODE, LIB_PREFILL

HIDDEN = 1536
INTER = 8960
KV_WIDTH = 256
LAYERS = 28
VOCAB = 151936

STATUS_TEXT = {
    0: "ok", 1: "invalid argument", 2: "capacity exceeded", 10: "invalid decode descriptor", 11: "null decode port",
    20: "invalid prefill descriptor", 21: "null prefill port", 22: "invalid prefill memory window",
    30: "CUDA failure", 31: "no usable CUDA device",
}

_F = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_B = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_I32 = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_U16 = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")


class NativeLibraryMissing(RuntimeError):
    pass


def _open(path: Path) -> ctypes.CDLL:
    if not path.exists():
        raise NativeLibraryMissing(
            f"{path.name} is not built; run `python -m work_llm_accelerator_b200.build` (needs nvcc) first")
    return ctypes.CDLL(str(path))


_core: ctypes.CDLL | None = None


def core_lib() -> ctypes.CDLL:
    global _core
    if _core is None:
        lib = _open(LIB_CORE)
        lib.qwen_b200_last_error.restype = ctypes.c_char_p
        lib.qwen_b200_device_count.restype = ctypes.c_int
        lib.qwen_b200_prefill_seq_capacity.restype = ctypes.c_int
        lib.qwen_b200_set_prefill_seq_capacity.argtypes = [ctypes.c_int]
        lib.qwen_b200_set_prefill_seq_capacity.restype = ctypes.c_int
        _configure_engine(lib)
        lib.qwen_b200_decode_attention.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int, ctypes.c_void_p,
                                                                            ctypes.c_void_p]
        lib.qwen_b200_decode_attention.restype = ctypes.c_int
        lib.qwen_b200_w8_digit_products.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                                    ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        lib.qwen_b200_w8_digit_products.restype = ctypes.c_int
        lib.qwen_b200_w8_digit_planes.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                                  ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        lib.qwen_b200_w8_digit_planes.restype = ctypes.c_int
        lib.qwen_b200_prefill_attention.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int, ctypes.c_void_p,
                                                                             ctypes.c_int, ctypes.c_void_p]
        lib.qwen_b200_prefill_attention.restype = ctypes.c_int
        lib.qwen_b200_prefill_approx_exp.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong,
                                                     ctypes.c_void_p]
        lib.qwen_b200_prefill_approx_exp.restype = ctypes.c_int
        lib.qwen_b200_exact_expf.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p]
        lib.qwen_b200_exact_expf.restype = ctypes.c_int
        lib.qwen_b200_kernel_error.argtypes = [ctypes.c_int]
        lib.qwen_b200_kernel_error.restype = ctypes.c_uint
        _core = lib
    return _core


def last_error() -> str:
    return core_lib().qwen_b200_last_error().decode(errors="replace")


def configure_decode_abi(lib: ctypes.CDLL) -> ctypes.CDLL:
    i, u64 = ctypes.c_int, ctypes.c_uint64
    lib.qwen_decode_stub_forward.argtypes = [_F, i, _F]
    lib.qwen_decode_attention_smoke_forward.argtypes = [_F, i, _F, _B, _B, _B, _B] + [_F] * 10
    lib.qwen_decode_mlp_smoke_forward.argtypes = [_F, _F, _B, _B, _B, _F, _F, _F, _F]
    top = [i, i] + [u64] * 6 + [_B, _F, _F, _F, _B, _F, _I32, _F, _F]
    lib.qwen_decode_top_smoke_forward.argtypes = top
    layer = [_F, i, _F, _F] + [_B] * 7 + [_F] * 13
    lib.qwen_decode_layer_smoke_forward.argtypes = layer
    names = ["qwen_decode_stub_forward", "qwen_decode_attention_smoke_forward", "qwen_decode_mlp_smoke_forward",
             "qwen_decode_top_smoke_forward", "qwen_decode_layer_smoke_forward"]
    if hasattr(lib, "qwen_decode_top_smoke_forward_w8"):
        lib.qwen_decode_top_smoke_forward_w8.argtypes = top
        lib.qwen_decode_layer_smoke_forward_w8.argtypes = layer
        names += ["qwen_decode_top_smoke_forward_w8", "qwen_decode_layer_smoke_forward_w8"]
    # layer0 golden layer: every pointer as c_void_p (biases may be null), rms_eps as float
    vp = ctypes.c_void_p
    lib.qwen_decode_layer0_reference_forward.argtypes = [vp, i] + [vp] * 18 + [ctypes.c_float, vp, vp, vp]
    names.append("qwen_decode_layer0_reference_forward")
    for n in names:
        getattr(lib, n).restype = i
    return lib


def configure_prefill_abi(lib: ctypes.CDLL) -> ctypes.CDLL:
    i, u64 = ctypes.c_int, ctypes.c_uint64
    t11 = [i] * 11
    lib.qwen_prefill_stub_forward.argtypes = [_F, i] + t11 + [_F]
    lib.qwen_prefill_attention_smoke_forward.argtypes = [_F, i] + [i] * 8 + [_F, _B, _B, _B, _B] + [_F] * 10
    lib.qwen_prefill_mlp_smoke_forward.argtypes = [_F, i, i, i, i, _F, _B, _B, _B, _F, _F, _F, _F]
    layer = [_F, i] + t11 + [_F, _F] + [_B] * 7 + [_F] * 13
    lib.qwen_prefill_layer_smoke_forward.argtypes = layer
    lib.qwen_prefill_glue_smoke_forward.argtypes = layer
    top = [i, i] + t11 + [u64] * 6 + [_B, _F, _F, _F, _B, _F, _I32, _F, _F]
    lib.qwen_prefill_top_smoke_forward.argtypes = top
    names = ["qwen_prefill_stub_forward", "qwen_prefill_attention_smoke_forward", "qwen_prefill_mlp_smoke_forward",
             "qwen_prefill_layer_smoke_forward", "qwen_prefill_glue_smoke_forward", "qwen_prefill_top_smoke_forward"]
    if hasattr(lib, "qwen_prefill_top_smoke_forward_w8"):
        lib.qwen_prefill_top_smoke_forward_w8.argtypes = top
        lib.qwen_prefill_layer_smoke_forward_w8.argtypes = layer
        names += ["qwen_prefill_top_smoke_forward_w8", "qwen_prefill_layer_smoke_forward_w8"]
    vp = ctypes.c_void_p
    lib.qwen_prefill_layer0_reference_forward.argtypes = [vp, i] + [vp] * 16 + [ctypes.c_float, vp]
    lib.qwen_prefill_layer0_reference_forward_with_cache.argtypes = [vp, i] + [vp] * 16 + [ctypes.c_float, vp, vp, vp]
    names += ["qwen_prefill_layer0_reference_forward", "qwen_prefill_layer0_reference_forward_with_cache"]
    for n in names:
        getattr(lib, n).restype = i
    return lib


def load_decode_lib() -> ctypes.CDLL:
    core_lib()
    return configure_decode_abi(_open(LIB_DECODE))


def load_prefill_lib() -> ctypes.CDLL:
    core_lib()
    return configure_prefill_abi(_open(LIB_PREFILL))


def set_prefill_seq_capacity(capacity: int) -> None:
    st = core_lib().qwen_b200_set_prefill_seq_capacity(int(capacity))
    if st:
        raise ValueError(f"invalid prefill capacity {capacity}")


def prefill_seq_capacity() -> int:
    return core_lib().qwen_b200_prefill_seq_capacity()


# ---------------------------------------------------------------------------------------------------
# device-resident engine
# ---------------------------------------------------------------------------------------------------
def _configure_engine(lib: ctypes.CDLL) -> None:
    vp, i, u64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64
    lib.qwen_engine_create.argtypes = [i, i, i, i, ctypes.POINTER(vp)]
    lib.qwen_engine_destroy.argtypes = [vp]
    lib.qwen_engine_destroy.restype = None
    lib.qwen_engine_init_synthetic.argtypes = [vp, u64, ctypes.c_float]
    lib.qwen_engine_load_layer.argtypes = [vp, i, _B, _F]
    lib.qwen_engine_load_embedding.argtypes = [vp, _U16, _F]
    lib.qwen_engine_prefill.argtypes = [vp, i, _I32, i, _I32]
    lib.qwen_engine_prefill_chunk.argtypes = [vp, i, _I32, i, _I32]
    lib.qwen_engine_decode.argtypes = [vp, _I32, _I32, i, _I32]
    lib.qwen_engine_write_kv.argtypes = [vp, i, i, _F, _F, i]
    lib.qwen_engine_read_kv.argtypes = [vp, i, i, _F, _F, i]
    lib.qwen_engine_read_kv_hf.argtypes = [vp, i, i, _F, _F, i]
    lib.qwen_engine_write_kv_hf.argtypes = [vp, i, i, _F, _F, i]
    lib.qwen_engine_set_seq_len.argtypes = [vp, i, i]
    lib.qwen_engine_seq_len.argtypes = [vp, i]
    lib.qwen_engine_reset.argtypes = [vp, i]
    lib.qwen_engine_set_option.argtypes = [vp, ctypes.c_char_p, ctypes.c_longlong]
    lib.qwen_engine_read_hidden.argtypes = [vp, _F, ctypes.c_longlong]
    lib.qwen_engine_read_logits.argtypes = [vp, _F, ctypes.c_longlong]
    lib.qwen_engine_read_trace.argtypes = [vp, np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS"),
                                           ctypes.c_longlong, ctypes.POINTER(ctypes.c_int),
                                           ctypes.POINTER(ctypes.c_int)]
    lib.qwen_engine_bench_decode.argtypes = [vp, _I32, _I32, i, i, i, ctypes.POINTER(ctypes.c_float)]
    lib.qwen_engine_decode_device.argtypes = [vp, _I32, vp, i, vp]
    lib.qwen_engine_read_layer.argtypes = [vp, i, _B, _F]
    lib.qwen_engine_profile_kernels.argtypes = [vp, i, i, i, _F]
    lib.qwen_engine_profile_decode.argtypes = [vp, i, i, i, _F]
    lib.qwen_engine_profile_batched.argtypes = [vp, _I32, _I32, i, i, _F]
    lib.qwen_engine_stream.argtypes = [vp]
    lib.qwen_engine_stream.restype = vp
    lib.qwen_engine_kernels_per_decode_step.argtypes = [vp, i]
    lib.qwen_engine_nccl_unique_id.argtypes = [ctypes.c_char_p]
    lib.qwen_engine_nccl_init.argtypes = [vp, ctypes.c_char_p, i, i]
    lib.qwen_engine_gather_tokens.argtypes = [vp, vp, i, vp]
    lib.qwen_engine_gather_tokens_async.argtypes = [vp, vp, i, vp]
    lib.qwen_engine_gather_join.argtypes = [vp]
    for n in ("qwen_engine_create", "qwen_engine_init_synthetic", "qwen_engine_load_layer", "qwen_engine_load_embedding",
              "qwen_engine_prefill", "qwen_engine_decode", "qwen_engine_write_kv", "qwen_engine_read_kv",
              "qwen_engine_set_seq_len", "qwen_engine_seq_len", "qwen_engine_reset", "qwen_engine_set_option",
              "qwen_engine_read_hidden", "qwen_engine_read_logits", "qwen_engine_bench_decode",
              "qwen_engine_kernels_per_decode_step", "qwen_engine_decode_device", "qwen_engine_read_layer",
              "qwen_engine_profile_kernels", "qwen_engine_read_trace", "qwen_engine_profile_decode",
              "qwen_engine_profile_batched", "qwen_engine_nccl_unique_id", "qwen_engine_nccl_init",
              "qwen_engine_gather_tokens", "qwen_engine_gather_tokens_async", "qwen_engine_gather_join",
              "qwen_engine_read_kv_hf", "qwen_engine_write_kv_hf",
              "qwen_engine_prefill_chunk"):
        getattr(lib, n).restype = i


def _layer_total(wbits: int) -> int:
    """Bytes of one layer's DDR image (hls/common/llm_memory_layout.h:84-128; 1-byte weights for wbits 8)."""
    w = (2 * HIDDEN * HIDDEN + 2 * KV_WIDTH * HIDDEN + 3 * INTER * HIDDEN) * wbits // 8
    return w + 2 * HIDDEN * 4 + (HIDDEN + 2 * KV_WIDTH) * 4 + (3 * HIDDEN + 2 * KV_WIDTH + 2 * INTER) * 4


class EngineError(RuntimeError):
    pass


def _check(status: int, what: str) -> None:
    if status != 0:
        raise EngineError(f"{what} failed with status {status} ({STATUS_TEXT.get(status, '?')}): {last_error()}")


class Engine:
    """Device-resident 28-layer engine on one GPU (include/qwen_b200_engine.h)."""

    def __init__(self, device: int = 0, wbits: int = 8, max_seqs: int = 1, max_len: int = 4096):
        self.lib = core_lib()
        self.wbits = wbits
        self.max_seqs = max_seqs
        self.max_len = max_len
        h = ctypes.c_void_p()
        _check(self.lib.qwen_engine_create(device, wbits, max_seqs, max_len, ctypes.byref(h)), "qwen_engine_create")
        self.handle = h

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.qwen_engine_destroy(self.handle)
            self.handle = None

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    def init_synthetic(self, seed: int, weight_sigma: float = 0.02) -> None:
        _check(self.lib.qwen_engine_init_synthetic(self.handle, seed, weight_sigma), "init_synthetic")

    def load_layer(self, layer: int, weight_ddr: np.ndarray, scale_ddr: np.ndarray) -> None:
        _check(self.lib.qwen_engine_load_layer(self.handle, layer, np.ascontiguousarray(weight_ddr, np.uint8),
                                               np.ascontiguousarray(scale_ddr, np.float32)), "load_layer")

    def load_embedding(self, embed_u16: np.ndarray, final_norm: np.ndarray) -> None:
        _check(self.lib.qwen_engine_load_embedding(self.handle, np.ascontiguousarray(embed_u16, np.uint16).reshape(-1),
                                                   np.ascontiguousarray(final_norm, np.float32)), "load_embedding")

    def set_option(self, name: str, value: int) -> None:
        _check(self.lib.qwen_engine_set_option(self.handle, name.encode(), int(value)), f"set_option({name})")

    def prefill(self, slot: int, tokens: Sequence[int]) -> int:
        toks = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros(1, np.int32)
        _check(self.lib.qwen_engine_prefill(self.handle, slot, toks, toks.size, out), "prefill")
        return int(out[0])

    def prefill_chunk(self, slot: int, tokens: Sequence[int]) -> int:
        """Continue the slot's prompt with more tokens (chunked prefill); returns the greedy next token."""
        toks = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros(1, np.int32)
        _check(self.lib.qwen_engine_prefill_chunk(self.handle, slot, toks, toks.size, out), "prefill_chunk")
        return int(out[0])

    def decode(self, slots: Sequence[int], tokens: Sequence[int]) -> np.ndarray:
        s = np.ascontiguousarray(slots, np.int32)
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros(s.size, np.int32)
        _check(self.lib.qwen_engine_decode(self.handle, s, t, s.size, out), "decode")
        return out

    def write_kv(self, slot: int, layer: int, k: np.ndarray, v: np.ndarray) -> None:
        k = np.ascontiguousarray(k, np.float32).reshape(-1)
        v = np.ascontiguousarray(v, np.float32).reshape(-1)
        _check(self.lib.qwen_engine_write_kv(self.handle, slot, layer, k, v, k.size // KV_WIDTH), "write_kv")

    def read_kv(self, slot: int, layer: int, n_tokens: int) -> tuple[np.ndarray, np.ndarray]:
        k = np.zeros(n_tokens * KV_WIDTH, np.float32)
        v = np.zeros(n_tokens * KV_WIDTH, np.float32)
        _check(self.lib.qwen_engine_read_kv(self.handle, slot, layer, k, v, n_tokens), "read_kv")
        return k, v

    def read_kv_hf(self, slot: int, layer: int, n_tokens: int) -> tuple[np.ndarray, np.ndarray]:
        """K and V of one layer in the Hugging Face cache layout [2 kv heads][n_tokens][128] (head-major)."""
        k = np.zeros(KV_WIDTH * n_tokens, np.float32)
        v = np.zeros(KV_WIDTH * n_tokens, np.float32)
        _check(self.lib.qwen_engine_read_kv_hf(self.handle, slot, layer, k, v, n_tokens), "read_kv_hf")
        return k.reshape(2, n_tokens, 128), v.reshape(2, n_tokens, 128)

    def write_kv_hf(self, slot: int, layer: int, k: np.ndarray, v: np.ndarray) -> None:
        k = np.ascontiguousarray(k, np.float32).reshape(-1)
        v = np.ascontiguousarray(v, np.float32).reshape(-1)
        _check(self.lib.qwen_engine_write_kv_hf(self.handle, slot, layer, k, v, k.size // KV_WIDTH), "write_kv_hf")

    def set_seq_len(self, slot: int, n: int) -> None:
        _check(self.lib.qwen_engine_set_seq_len(self.handle, slot, n), "set_seq_len")

    def seq_len(self, slot: int) -> int:
        return self.lib.qwen_engine_seq_len(self.handle, slot)

    def reset(self, slot: int) -> None:
        _check(self.lib.qwen_engine_reset(self.handle, slot), "reset")

    def read_trace(self, ctas: int = 148) -> np.ndarray:
        """Timeline of the last persistent-kernel step: [ctas][28][slots] global-timer ns (option "trace")."""
        c, sl = ctypes.c_int(), ctypes.c_int()
        out = np.zeros(ctas * 28 * 64, np.uint64)  # up to 64 slots
        _check(self.lib.qwen_engine_read_trace(self.handle, out, out.size, ctypes.byref(c), ctypes.byref(sl)),
               "read_trace")
        return out[:c.value * 28 * sl.value].reshape(c.value, 28, sl.value)

    def read_hidden(self, rows: int) -> np.ndarray:
        out = np.zeros(LAYERS * rows * HIDDEN, np.float32)
        _check(self.lib.qwen_engine_read_hidden(self.handle, out, out.size), "read_hidden")
        return out.reshape(LAYERS, rows, HIDDEN)

    def read_logits(self, rows: int) -> np.ndarray:
        out = np.zeros(rows * VOCAB, np.float32)
        _check(self.lib.qwen_engine_read_logits(self.handle, out, out.size), "read_logits")
        return out.reshape(rows, VOCAB)

    def bench_decode(self, slots: Sequence[int], first_tokens: Sequence[int], steps: int, warmup: int) -> float:
        s = np.ascontiguousarray(slots, np.int32)
        t = np.ascontiguousarray(first_tokens, np.int32)
        ms = ctypes.c_float()
        _check(self.lib.qwen_engine_bench_decode(self.handle, s, t, s.size, steps, warmup, ctypes.byref(ms)),
               "bench_decode")
        return float(ms.value)

    def decode_device(self, slots: Sequence[int], d_tokens_ptr: int, d_next_ptr: int) -> None:
        s = np.ascontiguousarray(slots, np.int32)
        _check(self.lib.qwen_engine_decode_device(self.handle, s, ctypes.c_void_p(d_tokens_ptr), s.size,
                                                  ctypes.c_void_p(d_next_ptr)), "decode_device")

    def read_layer(self, layer: int) -> tuple[np.ndarray, np.ndarray]:
        total = _layer_total(self.wbits)
        w = np.zeros(total, np.uint8)
        s = np.zeros(total // 4, np.float32)
        _check(self.lib.qwen_engine_read_layer(self.handle, layer, w, s), "read_layer")
        return w, s

    def profile_kernels(self, n: int, past: int, iters: int = 56) -> dict[str, float]:
        out = np.zeros(6, np.float32)
        _check(self.lib.qwen_engine_profile_kernels(self.handle, n, past, iters, out), "profile_kernels")
        return dict(zip(("qkv", "attention", "o", "gate_up", "down", "lm_head"), map(float, out)))

    def profile_decode(self, slot: int, first_token: int, steps: int) -> dict[str, float]:
        """Mean device milliseconds per eager decode step of the layer part and of the LM head kernel."""
        out = np.zeros(2, np.float32)
        _check(self.lib.qwen_engine_profile_decode(self.handle, slot, first_token, steps, out), "profile_decode")
        return {"layers": float(out[0]), "lm_head": float(out[1])}

    def profile_batched(self, slots: Sequence[int], first_tokens: Sequence[int], steps: int) -> dict[str, float]:
        """Mean device milliseconds per batched decode step by kernel group."""
        s = np.ascontiguousarray(slots, np.int32)
        t = np.ascontiguousarray(first_tokens, np.int32)
        out = np.zeros(8, np.float32)
        _check(self.lib.qwen_engine_profile_batched(self.handle, s, t, s.size, steps, out), "profile_batched")
        names = ("rmsnorm", "digits", "qkv", "attention", "o", "gate_up", "down", "lm_head")
        return dict(zip(names, map(float, out)))

    def nccl_init(self, unique_id: bytes, nranks: int, rank: int) -> None:
        """Join the token-exchange communicator (include/qwen_b200_engine.h; blocks until all ranks joined)."""
        if len(unique_id) != 128:
            raise ValueError("an NCCL unique id is 128 bytes")
        _check(self.lib.qwen_engine_nccl_init(self.handle, unique_id, nranks, rank), "nccl_init")

    def gather_tokens(self, d_local_ptr: int, n: int, d_all_ptr: int) -> None:
        """Enqueue the all-gather of n int32 ids per rank on the engine's stream (device pointers)."""
        _check(self.lib.qwen_engine_gather_tokens(self.handle, d_local_ptr, n, d_all_ptr), "gather_tokens")

    def gather_tokens_async(self, d_local_ptr: int, n: int, d_all_ptr: int) -> None:
        """The same all-gather on a side stream, beside the engine's following steps (see the C header)."""
        _check(self.lib.qwen_engine_gather_tokens_async(self.handle, d_local_ptr, n, d_all_ptr), "gather_tokens_async")

    def gather_join(self) -> None:
        """Make the engine's stream wait for the last asynchronous gather."""
        _check(self.lib.qwen_engine_gather_join(self.handle), "gather_join")

    def stream(self) -> int:
        return int(self.lib.qwen_engine_stream(self.handle) or 0)

    def kernels_per_decode_step(self, n: int) -> int:
        return self.lib.qwen_engine_kernels_per_decode_step(self.handle, n)


# ---------------------------------------------------------------------------------------------------
# BackendInterface mirror (verification/backend_interface.py:13-31)
# ---------------------------------------------------------------------------------------------------
@dataclass
class PrefillResult:
    logits: Any
    cache: Any


@dataclass
class DecodeResult:
    logits: Any
    cache: Any


class EngineBackend:
    """prefill / decode_step over the device-resident engine, shaped like the reference's
    RealHostTopBackend (verification/real_host_top_backend.py:208-351): input ids in, logits and a cache
    handle out. The cache handle is the engine slot; KV stays in HBM. `hf_cache` exports it in the Hugging
    Face per-layer layout the reference returns ((k, v) per layer, each [1][2][seq][128])."""

    def __init__(self, engine: Engine, slot: int = 0):
        self.engine = engine
        self.slot = slot
        engine.set_option("logits", 1)

    def prefill(self, input_ids) -> PrefillResult:
        ids = np.asarray(input_ids, dtype=np.int64).reshape(-1)
        self.engine.reset(self.slot)
        self.engine.prefill(self.slot, ids.astype(np.int32))
        return PrefillResult(logits=self.engine.read_logits(1), cache=self.slot)

    def decode_step(self, input_ids, cache) -> DecodeResult:
        if cache is None:
            raise ValueError("decode_step requires a prefill cache.")
        ids = np.asarray(input_ids, dtype=np.int64).reshape(-1)
        self.engine.decode([cache], ids[-1:].astype(np.int32))
        return DecodeResult(logits=self.engine.read_logits(1), cache=cache)

    def hf_cache(self, cache) -> tuple:
        """The slot's KV cache as the reference's cache tuple: 28 x (k, v), each float32 [1][2][seq][128]."""
        n = self.engine.seq_len(cache)
        layers = []
        for layer in range(LAYERS):
            k, v = self.engine.read_kv_hf(cache, layer, n)
            layers.append((k[None], v[None]))
        return tuple(layers)


def decode_attention(q_ptr: int, k_ptr: int, v_ptr: int, seq_len: int, ctx_ptr: int, stream: int = 0) -> None:
    """Device-pointer decode attention (include/qwen_b200_ops.h): raw device addresses in, enqueued on
    `stream`."""
    st = core_lib().qwen_b200_decode_attention(q_ptr, k_ptr, v_ptr, seq_len, ctx_ptr, stream or None)
    if st != 0:
        raise EngineError(f"qwen_b200_decode_attention failed with status {st}: {last_error()}")


def w8_digit_products(codes_ptr: int, rows: int, k: int, x_ptr: int, n_tokens: int, acc_ptr: int, step_ptr: int,
                      stream: int = 0) -> None:
    """Integer core of the W8 tensor-core projections (include/qwen_b200_ops.h): acc[r][4d+t] = sum_i
    codes[r][i] * digit_d(x[t])[i] and the per-token steps, on device buffers."""
    st = core_lib().qwen_b200_w8_digit_products(codes_ptr, rows, k, x_ptr, n_tokens, acc_ptr, step_ptr,
                                                 stream or None)
    if st != 0:
        raise EngineError(f"qwen_b200_w8_digit_products failed with status {st}: {last_error()}")


def kernel_error(reset: bool = False) -> int:
    """Error flag of the streaming kernels on the current device (1 = a bounded pipeline wait gave up)."""
    return int(core_lib().qwen_b200_kernel_error(1 if reset else 0))


def prefill_attention(q_ptr: int, k_ptr: int, v_ptr: int, seq_len: int, ctx_ptr: int, mode: int = 0,
                      stream: int = 0) -> None:
    """Device-pointer causal prefill attention (include/qwen_b200_ops.h); mode 0 tensor cores, 1 CUDA cores."""
    st = core_lib().qwen_b200_prefill_attention(q_ptr, k_ptr, v_ptr, seq_len, ctx_ptr, mode, stream or None)
    if st != 0:
        raise EngineError(f"qwen_b200_prefill_attention failed with status {st}: {last_error()}")


def prefill_approx_exp(x_ptr: int, y_ptr: int, n: int, stream: int = 0) -> None:
    """y = the prefill softmax exponential of x, as the tensor-core attention evaluates it (device buffers)."""
    st = core_lib().qwen_b200_prefill_approx_exp(x_ptr, y_ptr, n, stream or None)
    if st != 0:
        raise EngineError(f"qwen_b200_prefill_approx_exp failed with status {st}: {last_error()}")


def nccl_unique_id() -> bytes:
    """A new 128-byte NCCL communicator id for Engine.nccl_init (made on one rank, passed to the others)."""
    buf = ctypes.create_string_buffer(128)
    _check(core_lib().qwen_engine_nccl_unique_id(buf), "nccl_unique_id")
    return buf.raw


def exact_expf(x_ptr: int, y_ptr: int, n: int, stream: int = 0) -> None:
    """y = expf(x) as the reference host library's C library computes it (device buffers; include/qwen_b200_ops.h)."""
    st = core_lib().qwen_b200_exact_expf(x_ptr, y_ptr, n, stream or None)
    if st != 0:
        raise EngineError(f"qwen_b200_exact_expf failed with status {st}: {last_error()}")


def w8_digit_planes(codes_ptr: int, rows: int, k: int, x_ptr: int, n_tokens: int, acc_ptr: int, step_ptr: int,
                    stream: int = 0) -> None:
    """Many-token integer core (include/qwen_b200_ops.h): acc[d][t][r] = sum_i codes[r][i] * digit_d(x[t])[i]."""
    st = core_lib().qwen_b200_w8_digit_planes(codes_ptr, rows, k, x_ptr, n_tokens, acc_ptr, step_ptr, stream or None)
    if st != 0:
        raise EngineError(f"qwen_b200_w8_digit_planes failed with status {st}: {last_error()}")
