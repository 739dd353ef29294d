import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100) device")
    config.addinivalue_line("markers", "slow: full-size problems (seconds to minutes)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_cuda = torch.cuda.is_available()
    except Exception:
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def lib():
    """The in-tree C ABI library (built here if missing or stale)."""
    from cutedsl_pingpong_gemm_b200 import _build, _lib
    _build.build()
    return _lib.load()


@pytest.fixture(scope="session")
def golden_fdm():
    with open(os.path.join(GOLDEN, "fast_divmod.json")) as f:
        return json.load(f)["cases"]


@pytest.fixture(scope="session")
def golden_maps():
    with open(os.path.join(GOLDEN, "tile_maps.json")) as f:
        index = json.load(f)
    arrays = np.load(os.path.join(GOLDEN, "tile_maps.npz"))
    return index, {k: arrays[k].astype(np.int32) for k in arrays.files}
