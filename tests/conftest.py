"""Shared test configuration.

Markers: `gpu` tests need a CUDA device (B200) and call the C ABI; everything
else runs on CPU.  Tolerances are the ones the parity bar states:
  * RTOL_EXACT  1e-5  fp32 elementwise, reduction and Adam paths
  * RTOL_TC     2e-3  per gradient tensor where TF32 tensor cores replace the
                      reference's fp32 FMA products
Relative error of a tensor = max|a - b| / max|b| (rel_err); for whole
training steps on TF32 tensor cores the normwise error ||a - b||_2 / ||b||_2
(norm_err) is used, the usual measure of a computed tensor's accuracy.
"""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

RTOL_EXACT = 1e-5
RTOL_TC = 2e-3


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); calls the sm_100a kernels")


def rel_err(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    denom = max(np.max(np.abs(b)) if b.size else 0.0, 1e-30)
    return float(np.max(np.abs(a - b)) / denom) if a.size else 0.0


def norm_err(a, b):
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture
def rng():
    return np.random.default_rng(1234)


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
