"""Shared pytest configuration: markers, import paths and golden fixtures."""

from __future__ import annotations

import json
import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
for path in (ROOT, ROOT / "oracle", GOLDEN):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built extension")
    config.addinivalue_line("markers", "slow: multi-second CPU test")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA GPU in this process")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden_table():
    return json.loads((GOLDEN / "golden.json").read_text())


@pytest.fixture(scope="session")
def golden_arrays():
    with np.load(GOLDEN / "golden_small.npz") as data:
        return {key: data[key] for key in data.files}


@pytest.fixture(scope="session")
def golden_cases():
    import cases

    return cases.all_cases()


@pytest.fixture(autouse=True)
def no_kernel_side_error(request):
    """Every GPU test ends with the library's device status word at zero:
    a bounded wait that gave up (which leaves its outputs unwritten) fails
    the test even where the output buffer happened to hold the right values."""
    yield
    if "gpu" not in request.keywords:
        return
    import torch

    if not torch.cuda.is_available():
        return
    from se12_b200 import _lib

    if _lib.LIBRARY_PATH.exists() and _lib.is_loaded():
        from se12_b200.device import device_status

        torch.cuda.synchronize()
        status = device_status()
        assert status == 0, f"kernel-side error status {status:#x}"
