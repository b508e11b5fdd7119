"""Shared test configuration: the `gpu` marker and common helpers."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and libhiggs_cuda.so")


def pytest_collection_modifyitems(config, items):
    # A gpu-marked test on a machine without CUDA is skipped with the reason;
    # the driver selects them with -m gpu only on the GPU box.
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
def golden():
    return dict(np.load(os.path.join(GOLDEN, "oracle_vectors.npz")))


@pytest.fixture(scope="session")
def kat():
    import json
    with open(os.path.join(GOLDEN, "reference_kat.json")) as f:
        return json.load(f)
