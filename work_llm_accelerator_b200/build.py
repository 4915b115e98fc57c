"""Build the native libraries in-tree (work_llm_accelerator_b200/lib/):

  libqwen_b200.so          all CUDA kernels (sm_100a), the runtime and the device-resident engine
  libqwen_decode_stub.so   drop-in C-ABI of the reference's decode library   (links libqwen_b200.so)
  libqwen_prefill_stub.so  drop-in C-ABI of the reference's prefill library  (links libqwen_b200.so)

nvcc cross-compiles for sm_100a without a GPU, so this runs on a CPU-only machine. The CUDA runtime
is linked statically into libqwen_b200.so, so the libraries need only the driver at run time.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "lib"
INCLUDE = PKG.parent / "include"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                     "-Xptxas", "-warn-spills"]
CU_SOURCES = ["decode_gemv.cu", "attention.cu", "prefill_simt.cu", "misc.cu", "runtime.cu", "engine.cu", "ops.cu", "ops_noalloc.cu", "qgemm.cu", "decode_stack.cu", "decode_bs1.cu", "tgemm.cu", "lmhead.cu", "attention_tc.cu", "exact.cu", "layer0_ref.cu"]
CXX = os.environ.get("QWEN_B200_CXX", "g++")

LIB_CORE = LIB / "libqwen_b200.so"
LIB_DECODE = LIB / "libqwen_decode_stub.so"
LIB_PREFILL = LIB / "libqwen_prefill_stub.so"
ALL_LIBS = (LIB_CORE, LIB_DECODE, LIB_PREFILL)


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + proc.stdout + proc.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} ... {cmd[-1]}")


def _newer(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return False
    t = target.stat().st_mtime
    return all(d.stat().st_mtime <= t for d in deps)


def build(force: bool = False, verbose: bool = False) -> list[Path]:
    LIB.mkdir(exist_ok=True)
    objdir = LIB / "obj"
    objdir.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))

    def compile_one(src: str) -> Path:
        s = CSRC / src
        o = objdir / (src + ".o")
        if force or not _newer(o, [s] + headers):
            if verbose:
                print("nvcc", src, flush=True)
            _run([NVCC, *NVCC_FLAGS, "-c", str(s), "-o", str(o)])
        return o

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, CU_SOURCES))
    if force or not _newer(LIB_CORE, objs):
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-Xlinker", "-soname=libqwen_b200.so", "-o", str(LIB_CORE),
              *map(str, objs), "-lpthread", "-ldl", "-lrt"])
    for abi_src, target in (("abi_decode.cpp", LIB_DECODE), ("abi_prefill.cpp", LIB_PREFILL)):
        s = CSRC / abi_src
        if force or not _newer(target, [s, LIB_CORE] + headers):
            _run([CXX, "-std=c++17", "-O2", "-fPIC", "-shared", str(s), "-o", str(target), f"-L{LIB}", "-Wl,--no-as-needed",
                  "-lqwen_b200", "-Wl,-rpath,$ORIGIN"])
    return list(ALL_LIBS)


if __name__ == "__main__":
    for p in build(force="--force" in sys.argv, verbose=True):
        print(p)
