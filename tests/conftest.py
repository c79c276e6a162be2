"""Test configuration: registers the `gpu` marker and shared fixtures.

`-m "not gpu"` runs the CPU suite (oracle vs golden vectors, host logic,
C-ABI exports, gloo multi-rank logic); `-m gpu` runs the parity tests
proper on a B200 through the C ABI.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200); runs through libfeml_b200.so")


def tol_ok(got, want, atol=1e-3, rtol=1e-4):
    """The path's tolerance: |got - want| <= 1e-3 + 1e-4 * |want| elementwise."""
    import numpy as np
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    err = np.abs(got - want) - (atol + rtol * np.abs(want))
    return bool(np.all(err <= 0)), float(np.max(np.abs(got - want))) if got.size else 0.0


@pytest.fixture(scope="session")
def b200():
    """One shared B200 backend for the GPU tests (the reference's CUDA tests
    share one backend the same way, feml-cuda/tests/cuda_integration.rs:14-24).
    No skip: on a GPU run a missing device is a failure."""
    import feml_b200 as F
    be = F.B200Backend.open(0)
    yield be
    be.close()
