"""Test set-up: import paths, the `gpu` marker, shared fixtures.

`-m "not gpu"` runs on any host (oracle vs golden vectors, host logic, library exports).
`-m gpu` needs a B200 and runs the parity tests through the C ABI.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PACKAGE = ROOT / "attention-rank_b200"
for path in (str(PACKAGE), str(ROOT)):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (parity tests through the C ABI)")
    config.addinivalue_line("markers", "slow: long-running (full 7B-architecture parity)")


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
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def reference_lib():
    """The reference's own implementation compiled by oracle/Makefile (None when not built)."""
    from oracle import reference
    return reference.load_or_none()
