"""Shared pytest setup: the ``gpu`` marker, repo-root imports, and device helpers."""

from __future__ import annotations

import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

os.environ.setdefault("HF_HUB_OFFLINE", "1")
os.environ.setdefault("TRANSFORMERS_OFFLINE", "1")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU and the native library")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def cuda():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    from latefuse_b200 import _native

    dev = torch.device("cuda", 0)
    assert _native.lib().lf_device_supported(0) == 1, "not an sm_100 device"
    return dev
