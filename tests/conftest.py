"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; everything else runs on CPU.

Parity tolerance for fp32 outputs: max-abs-rel
    max|gpu - ref| / max|ref| <= 1e-3
Quantized bytes, decoded floats and int32 block dots must match exactly.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

TOL = 1e-3
GOLDEN = os.path.join(ROOT, "tests", "golden", "golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and libpxq.so")


def max_abs_rel(got, ref) -> float:
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    scale = max(float(np.abs(ref).max()), 1e-30)
    return float(np.abs(got - ref).max()) / scale


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN))


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle, oracle_available

    if not oracle_available():
        pytest.fail("oracle/_build/libpxq_oracle.so missing: run __graft_entry__.build()")
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference, reference_available

    if not reference_available():
        pytest.skip("reference build oracle/_ref/libpixref.so not present")
    return Reference()


@pytest.fixture(scope="session")
def pxq():
    import torch

    from pixelina_b200 import pxq as _pxq

    assert torch.cuda.is_available(), "GPU test needs CUDA"
    _pxq.init(0)
    return _pxq
