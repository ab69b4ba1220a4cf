"""Test configuration: the `gpu` marker, and shared fixture loading.

CPU tests (-m "not gpu") check the oracle against the reference's golden vectors, the host
packing, and that the C-ABI library loads and exports its symbols.  GPU tests (-m gpu) are the
parity tests proper: they call libtrixium_b200.so through the C ABI and compare with the oracle.
"""
import glob
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        have_gpu = torch.cuda.is_available()
    except Exception:
        have_gpu = False
    if not have_gpu:
        skip = pytest.mark.skip(reason="no CUDA device in this container")
        for it in items:
            if "gpu" in it.keywords:
                it.add_marker(skip)


def golden_matvec_files():
    return sorted(glob.glob(os.path.join(GOLDEN, "matvec_*.npz")))


def load(path):
    return dict(np.load(path))


def fp_rel_err(got, ref):
    """Relative error with the denominator floored at 1% of the reference's RMS, so elements
    that cancel to ~0 do not dominate (the fp-mode tolerance is 1e-3 of this)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    if ref.size == 0:
        return 0.0
    floor = max(1e-2 * float(np.sqrt(np.mean(ref * ref))), 1e-30)
    return float(np.max(np.abs(got - ref) / np.maximum(np.abs(ref), floor)))
