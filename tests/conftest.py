import os
import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
PKG = ROOT / "onionop.jl_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    # GPU tests are skipped (not failed) when no GPU is visible, so the CPU
    # suite (-m "not gpu") and an unfiltered run both work here.
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA GPU visible")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
