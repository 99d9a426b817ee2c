"""Test configuration: the `gpu` marker and shared fixtures.

`-m "not gpu"` runs the CPU suite (oracle vs golden vectors, the C ABI's
exports, host logic, gloo multi-rank tests); `-m gpu` runs the parity tests on
a B200 through the C ABI.
"""

import json
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN_DIR = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: long-running case")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def golden_cases():
    with open(os.path.join(GOLDEN_DIR, "golden_index.json")) as f:
        return json.load(f)


def load_golden(name):
    return np.load(os.path.join(GOLDEN_DIR, f"golden_{name}.npz"))


@pytest.fixture(scope="session")
def tt():
    import torch_transformer_benchmark as T
    return T


@pytest.fixture(scope="session")
def pkg(tt):
    return tt._pkg
