"""B200-native quantized Qwen2.5-1.5B decoder-layer hot path.

Native libraries (built in-tree by `work_llm_accelerator_b200.build`):
  lib/libqwen_b200.so          sm_100a kernels, runtime, device-resident engine
  lib/libqwen_decode_stub.so   drop-in for the reference's decode host library
  lib/libqwen_prefill_stub.so  drop-in for the reference's prefill host library
"""
from .build import ALL_LIBS, LIB_CORE, LIB_DECODE, LIB_PREFILL  # noqa: F401
from .build import build as build_native  # noqa: F401

__all__ = ["build_native", "LIB_CORE", "LIB_DECODE", "LIB_PREFILL", "ALL_LIBS"]
