import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the product's CUDA path")
    config.addinivalue_line("markers", "slow: takes more than a few seconds on the CPU")


def _has_gpu() -> bool:
    try:
        from work_llm_accelerator_b200 import host

        return host.core_lib().qwen_b200_device_count() > 0
    except Exception:
        return False


@pytest.fixture(scope="session")
def gpu_available() -> bool:
    return _has_gpu()


@pytest.fixture(scope="session")
def built_libs():
    """Build (or reuse) the product libraries and the oracle port."""
    from work_llm_accelerator_b200 import build as b

    b.build()
    import qwen_oracle as qo

    qo.build_port()
    return b


@pytest.fixture(scope="session")
def ref_libs():
    import qwen_oracle as qo

    if not (qo.REF_DECODE_LIB.exists() and qo.REF_PREFILL_LIB.exists()):
        pytest.skip("reference libraries not built here (make -C oracle ref needs the reference sources)")
    return qo.RefLibs()


@pytest.fixture(scope="session")
def golden():
    import json

    return json.loads((ROOT / "tests" / "golden" / "golden.json").read_text())
