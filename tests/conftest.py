"""pytest configuration: the `gpu` marker and shared fixtures.

`-m "not gpu"` runs everywhere (oracle vs golden fixtures, host logic, C-ABI
loading and argument validation).  `-m gpu` needs an sm_100 GPU and calls the
CUDA library through its C ABI.
"""
import importlib
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


@pytest.fixture(scope="session")
def bs():
    """The product package (directory name starts with a digit)."""
    return importlib.import_module("355_1_trans_b200")


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"needs sm_100, found sm_{major}{minor}")
    return torch.device("cuda:0")
