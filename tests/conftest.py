import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")

# Parity bar against the fp32 oracle for bf16 inputs with fp32 accumulation.
MAX_ABS_TOL = 2e-2
MEAN_ABS_TOL = 2e-3


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        have_gpu = torch.cuda.is_available()
    except Exception:
        have_gpu = False
    if have_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def err_stats(out, ref):
    import numpy as np
    d = np.abs(np.asarray(out, dtype=np.float64) - np.asarray(ref, dtype=np.float64))
    return float(d.max()), float(d.mean())


def assert_close(out, ref, max_tol=MAX_ABS_TOL, mean_tol=MEAN_ABS_TOL, what=""):
    import numpy as np
    out = np.asarray(out, dtype=np.float64)
    assert np.isfinite(out).all(), f"{what}: non-finite values in output"
    mx, mean = err_stats(out, ref)
    assert mx <= max_tol and mean <= mean_tol, \
        f"{what}: max abs err {mx:.3e} (tol {max_tol}), mean abs err {mean:.3e} (tol {mean_tol})"
