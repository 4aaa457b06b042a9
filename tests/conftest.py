import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA GPU in this environment")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def close(out, exp, tol=2e-3, cos_min=0.99999):
    """The reference's kernel gate (``scripts/verify-kernels.mjs:104``):
    ``max|d| < 2e-3`` and cosine similarity ``> 0.99999``."""
    import numpy as np
    out = np.asarray(out, np.float64).ravel()
    exp = np.asarray(exp, np.float64).ravel()
    mad = float(np.abs(out - exp).max()) if out.size else 0.0
    cos = float(out @ exp / (np.linalg.norm(out) * np.linalg.norm(exp) + 1e-9)) if out.size else 1.0
    return mad < tol and cos > cos_min, mad, cos
