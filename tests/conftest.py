import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"

# Parity bar for the fused kernel (fp16 inputs, fp32 accumulation), from the
# north-star specification: max-abs error 2e-2 and relative L2 error 1e-3
# against the reference's CPU ground truth on identical inputs.
MAX_ABS_TOL = 2e-2
REL_L2_TOL = 1e-3


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def lib():
    """libfused3s.so, built in-tree if it is missing or stale."""
    from fused3s_b200 import build, _lib
    build.build()
    return _lib.load()


@pytest.fixture(scope="session")
def golden_graphs():
    z = np.load(GOLDEN / "graphs.npz")
    cases = sorted({k.split("/")[0] for k in z.files})
    return {c: {k.split("/")[1]: z[k] for k in z.files if k.startswith(c + "/")} for c in cases}


@pytest.fixture(scope="session")
def golden_attention():
    z = np.load(GOLDEN / "attention.npz")
    cases = sorted({k.split("/")[0] for k in z.files})
    return {c: {k.split("/")[1]: z[k] for k in z.files if k.startswith(c + "/")} for c in cases}
