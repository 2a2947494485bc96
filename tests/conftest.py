"""Test configuration: markers, import paths and the shared library build."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "pentanet-v1.0_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; parity tests through the C ABI")


def pytest_sessionstart(session):
    # The oracle and the library are built artefacts; build them if missing
    # (nvcc cross-compiles without a GPU).
    import subprocess
    if not os.path.exists(os.path.join(ROOT, "oracle", "libpenta_oracle.so")):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle")], check=True,
                       stdout=subprocess.DEVNULL)
    import build as pkg_build  # pentanet-v1.0_b200/build.py
    if not os.path.exists(pkg_build.OUT):
        pkg_build.build()


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"GPU tests need an sm_100 device, got sm_{major}{minor}"
    return torch.device("cuda", 0)
