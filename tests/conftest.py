"""pytest configuration: the `gpu` marker and shared fixtures.

`-m "not gpu"` runs everywhere (oracle vs golden fixtures, host logic, C-ABI
loading and argument validation).  `-m gpu` needs an sm_100 GPU and calls the
CUDA library through its C ABI.
"""
import importlib
import json
import os
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


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """Per parity check: how many elements passed only through the
    fp32-accumulation floor (1e-6 * sum|term|) of the tolerance.  Written as
    JSON to $BSG_PARITY_REPORT when that is set."""
    from helpers import PARITY_LOG
    if not PARITY_LOG:
        return
    total = sum(n for _, _, n, _, _ in PARITY_LOG)
    floor = sum(f for _, f, _, _, _ in PARITY_LOG)
    tr = terminalreporter
    tr.section("parity: elements passing only through the fp32-accumulation floor")
    tr.write_line(f"{len(PARITY_LOG)} checks, {total} elements, {floor} pass only through the floor "
                  f"({floor / max(total, 1):.2e})")
    for what, f, n, max_rel, cd in PARITY_LOG:
        if f:
            tr.write_line(f"  {what}: {f} of {n}")
    path = os.environ.get("BSG_PARITY_REPORT")
    if path:
        Path(path).write_text(json.dumps(
            [{"check": w, "floor_only": f, "elements": n, "max_rel": r, "calc_diff": c}
             for w, f, n, r, c in PARITY_LOG], indent=1))
