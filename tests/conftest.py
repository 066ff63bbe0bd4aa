"""Test configuration: the `gpu` marker, builds of the library and the oracle."""
import os
import subprocess
import sys
import pathlib

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _make(dirpath):
    subprocess.run(["make", "-s", "-C", str(dirpath)], check=True)


@pytest.fixture(scope="session", autouse=True)
def built_libraries():
    """Builds liboracle.so (g++) and libnerf_b200.so (nvcc) when absent or stale."""
    _make(ROOT / "oracle")
    if not os.environ.get("NERF_B200_SKIP_BUILD"):
        _make(ROOT / "nerf_b200" / "csrc")
    yield


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    return torch
