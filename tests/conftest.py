"""Shared pytest setup: the `gpu` marker, repo imports and golden-fixture access."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import submission  # noqa: E402  registers the package as nvfp4_group_gemm_b200

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def gpu_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if gpu_available():
        return
    skip = pytest.mark.skip(reason="no sm_100 GPU in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def pkg():
    return submission.load_package()


@pytest.fixture(scope="session")
def golden_inputs():
    return np.load(os.path.join(GOLDEN_DIR, "golden_inputs.npz"))


@pytest.fixture(scope="session")
def golden_outputs():
    path = os.path.join(GOLDEN_DIR, "golden_outputs.npz")
    if not os.path.exists(path):
        pytest.skip("golden_outputs.npz (reference arithmetic run on a B200) not generated yet")
    return np.load(path)


def golden_case_names(data) -> list:
    return sorted({k.split("/")[0] for k in data.files})
