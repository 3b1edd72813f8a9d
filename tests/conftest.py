"""Shared test setup.

Markers:
  gpu  -- needs a CUDA device (B200); run with `pytest -m gpu`.
The CPU suite (`-m "not gpu"`) checks the oracle against the reference's golden
vectors and its compiled host code, the host logic, and that the C-ABI library
loads and exports every declared symbol.
"""
from __future__ import annotations

import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
PKG = ROOT / "blackwell-kernel-sm_120_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import bindings
    return bindings


@pytest.fixture(scope="session")
def ref_lib():
    from oracle import bindings
    if not bindings.ref_available():
        pytest.skip("oracle/_ref not built (needs the reference sources)")
    return bindings
