"""Test configuration: the `gpu` marker, import paths, and shared fixtures.

`-m "not gpu"` runs here (no GPU): the oracle against golden vectors, host
logic, gloo multi-process tests, and that libltxb.so loads and exports every
symbol include/ltxb.h declares. `-m gpu` needs a B200 and calls the CUDA
kernels through the C ABI, checking them against the oracle.
"""

import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "ltx-zml_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a); runs the kernels through the C ABI")


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu-marked test run without a CUDA device")
    return torch.device("cuda:0")
