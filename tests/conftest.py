"""Shared pytest setup: the ``gpu`` marker, the ``mes_b200`` package import and helpers."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import __graft_entry__  # noqa: E402

# A fresh checkout has no library yet: build it once (nvcc cross-compiles without a GPU).
if not os.path.exists(os.path.join(__graft_entry__.PKG_DIR, "lib", "libmes_b200.so")):
    __graft_entry__.build()
__graft_entry__.load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
