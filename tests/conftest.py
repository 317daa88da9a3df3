"""Shared fixtures.  GPU tests carry @pytest.mark.gpu and call the CUDA path through
libvbq.so; CPU tests check the oracle, the host logic and the C-ABI surface."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"

def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU (runs the sm_100a kernels)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import load_oracle
    return load_oracle()


@pytest.fixture(scope="session")
def reflib():
    from oracle import load_ref
    r = load_ref()
    if r is None:
        pytest.skip("compiled reference (oracle/_ref) not available")
    return r


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    from vibeblade_b200 import _lib
    _lib.load()  # fail loudly if the sm_100a library is missing
    return torch.device("cuda:0")


def max_rel(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.abs(b).max()
    return float(np.abs(a - b).max() / (den if den > 0 else 1.0))


def bits_equal(a, b) -> bool:
    """Bit-exact float32 comparison; NaNs compare equal to NaNs (GPU and x86 produce
    different NaN payloads, e.g. 0*inf)."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    if a.shape != b.shape:
        return False
    na, nb = np.isnan(a), np.isnan(b)
    if not np.array_equal(na, nb):
        return False
    return bool(np.array_equal(a.view(np.uint32)[~na], b.view(np.uint32)[~nb]))
