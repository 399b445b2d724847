"""Test configuration: import paths and the `gpu` marker.

`-m "not gpu"` tests run anywhere (oracle vs golden fixtures, host logic, C-ABI
loading).  `-m gpu` tests call the sm_100a kernels through the C ABI and
compare with the oracle; they are skipped only when no CUDA device exists.
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "comfyui-zimage-triton_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
