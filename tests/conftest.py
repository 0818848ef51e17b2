"""Shared test setup.

Markers:
  gpu -- needs a B200 and the built libodi_cuda.so; run with `-m gpu`.
Everything unmarked runs on a CPU-only host.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device and libodi_cuda.so")


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN))


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle

    oracle.lib()  # builds liboracle.so if missing
    return oracle


@pytest.fixture(scope="session")
def cuda_lib():
    """The product library on a GPU host; fails loudly if it or the GPU is missing."""
    import torch

    import odiengine_b200 as ob

    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    ob.init(0)
    torch.cuda.set_device(0)
    return ob
