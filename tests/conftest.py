import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def built_lib():
    from aethermind_b200 import build
    build.build()
    from aethermind_b200 import _lib
    return _lib.lib()


@pytest.fixture(scope="session")
def oracle_lib():
    import subprocess
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "oracle"], check=True)
    import oracle
    return oracle
