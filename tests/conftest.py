"""Shared test setup.

* registers the `gpu` marker (tests that need a B200; everything else runs on CPU);
* puts the backend package, the repo root (oracle/) and tests/golden on sys.path;
* builds the backend library and the oracle when missing;
* gives the session its own cubin cache directory;
* clears the backend's plan cache before every test, as the reference's
  suite clears its JIT cache (bafe/tests/conftest.py:25-30).
"""
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "bafe-basic-algibra-fusion-engine-_b200"
for p in (str(PKG), str(ROOT), str(ROOT / "tests" / "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)

if not (PKG / "lib" / "libbafe_cuda.so").exists():
    subprocess.run(["make", "-s", "-C", str(PKG), "lib"], check=True)
if not (ROOT / "oracle" / "_build" / "liboracle.so").exists():
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "all"], check=True)

os.environ.setdefault("BAFE_CACHE_DIR", tempfile.mkdtemp(prefix="bafe_test_cache_"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(autouse=True)
def _clear_plans():
    import bafe_b200
    bafe_b200.jit_clear()
    bafe_b200.set_option("gemm_precision", "auto")
    bafe_b200.set_option("host_panels", "auto")
    yield


@pytest.fixture(scope="session")
def cuda():
    if not gpu_available():
        pytest.fail("this test needs a CUDA device")
    import torch
    return torch
