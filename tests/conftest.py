"""Shared test setup: paths, the `gpu` marker, and on-demand builds.

The CUDA library (nvcc cross-compiles for sm_100a without a GPU) and the CPU
oracle are built in-tree when missing, so a fresh checkout can run the suite.
"""
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def _ensure_built() -> None:
    if not (ROOT / "graphzero_b200" / "libgraphzero_b200.so").exists():
        subprocess.run([sys.executable, str(ROOT / "graphzero_b200" / "build.py")], check=True)
    if not (ROOT / "oracle" / "_build" / "liboracle.so").exists():
        subprocess.run(["make", "-s", "-C", str(ROOT / "oracle")], check=True)


_ensure_built()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
