import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def quant_golden():
    return dict(np.load(os.path.join(GOLDEN, "quant_golden.npz")))


@pytest.fixture(scope="session")
def cache_golden():
    return dict(np.load(os.path.join(GOLDEN, "cache_golden.npz")))


def golden_to_f32(arr, dtype):
    """Fixture arrays -> float32 values (bf16 is stored as raw uint16 bits)."""
    from oracle.quant_ref import bf16_bits_to_f32
    if dtype == "bf16" and arr.dtype == np.uint16:
        return bf16_bits_to_f32(arr)
    return np.asarray(arr, dtype=np.float32)
