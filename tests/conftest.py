import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import cpq_oracle

    cpq_oracle.build()
    return cpq_oracle


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for a test marked gpu")
    from codpiece_b200 import build, mul_mat

    build.build()
    mul_mat.init(0)
    return torch


def rel_err(y, ref):
    """max|y - ref| / max(|ref|, eps): the parity metric (tolerance 1e-3)."""
    import numpy as np

    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


TOL = 1e-3  # max relative error vs the CPU oracle (accumulation order differs)
