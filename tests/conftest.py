"""Test set-up: import paths, the `gpu` marker, shared helpers.

`-m "not gpu"` runs here without a GPU (oracle vs golden vectors, host logic,
the C ABI's exports and argument checks); `-m gpu` runs the CUDA parity tests
on a B200 through the C ABI.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "grpc-unlimited-ocr_b200")
for p in (PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the sm_100a kernels")


def max_rel(got, want) -> float:
    """max |got - want| / max |want|, the reference's test metric (tests/cuda_ops_test.cpp:47-54)."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    scale = max(1e-9, float(np.abs(want).max()) if want.size else 0.0)
    return float(np.abs(got - want).max() / scale) if want.size else 0.0


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
