"""pytest configuration: the ``gpu`` marker and import paths.

Tests marked ``gpu`` need a CUDA device (a B200); everything else runs on the
CPU.  The drop-in modules are flat (``import flash_attention_prefill``), like
the reference's ``attention/`` folder, so that folder goes on ``sys.path``.
"""

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "triton-ascend-kernels_b200")
for p in (REPO, os.path.join(PKG, "attention"), os.path.join(REPO, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
