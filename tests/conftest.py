"""pytest configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a B200 (sm_100a) and the built libtttj_b200.so; the rest run
on the CPU.  Importing optimized_transformer registers the package directory
tttj-2026_b200/ as the importable package `tttj_2026_b200`.
"""
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

import optimized_transformer  # noqa: E402,F401  (registers tttj_2026_b200)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU and the built C library")
    config.addinivalue_line("markers", "slow: long-running full-size case")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
