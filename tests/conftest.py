"""Shared pytest setup.

``-m gpu`` tests need a B200 and the in-tree ``libtk_b200.so``; everything
else runs on the CPU. The product modules live in ``transformer-kernel_b200/``
(a directory, like the reference's ``src/``), which is put on ``sys.path``
here the same way the reference's tests put ``src/`` there.
"""

from __future__ import annotations

import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
PKG = ROOT / "transformer-kernel_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 and the built libtk_b200.so")
    config.addinivalue_line("markers", "slow: long CPU-oracle cases")


@pytest.fixture(scope="session")
def golden():
    import torch

    return torch.load(ROOT / "tests" / "golden" / "golden.pt", weights_only=False)


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu-marked test run without a visible CUDA device")
    return torch.device("cuda:0")
