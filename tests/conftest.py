"""Test configuration.

Markers: `gpu` tests need a CUDA device (run on the B200 box with
`pytest -m gpu`); everything else runs on a CPU-only machine
(`pytest -m "not gpu"`).  Paths: the repo root (oracle/, bench.py) and the
package root sparse-offload-infer_b200/ (soinfer) are put on sys.path, the
way the reference's root conftest exposes python/soinfer.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "sparse-offload-infer_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a); run with -m gpu on a B200")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
