"""Test configuration: the `gpu` marker and shared fixtures.

`-m "not gpu"` runs the oracle known-answer tests, host-side logic and the
C-ABI symbol checks on CPU; `-m gpu` runs the parity tests through the C ABI
on a B200.
"""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built library")


# Parity tolerance for floating-point outputs: elementwise
# |gpu - ref| <= ATOL + RTOL * |ref|.
RTOL = 1e-2
ATOL = 1e-3


def assert_close(actual, expected, rtol=RTOL, atol=ATOL, what="output"):
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    assert actual.shape == expected.shape, f"{what}: shape {actual.shape} != {expected.shape}"
    err = np.abs(actual - expected)
    bound = atol + rtol * np.abs(expected)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(
            f"{what}: {int(bad.sum())}/{bad.size} elements outside {rtol} rel / {atol} abs; "
            f"worst at {i}: {actual[i]} vs {expected[i]}")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.lib()
    return O


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.skip("needs an sm_100 device")
    return torch
