"""Shared test set-up: import paths, the `gpu` marker, and fixtures.

`-m "not gpu"` runs the oracle against the reference's known answers, the host logic and
the C ABI's exports on CPU; `-m gpu` runs the parity tests proper (CUDA path vs oracle)
on a B200.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for sub in ("splatting-rs_b200", "oracle", "tests"):
    p = str(ROOT / sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def oracle_module():
    import oracle

    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def ctx():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("the gpu tests need a CUDA device")
    import splat_b200 as sb

    return sb.Context(0)
