"""Shared pytest setup: the `gpu` marker, import paths, and helpers.

GPU tests (``-m gpu``) call the CUDA library through the C-ABI; everything
else runs on CPU (oracle vs golden vectors, host logic, symbol exports, gloo
ranks)."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(ROOT, "hierarchical-block-attention_b200")
for p in (ROOT, PKG_ROOT, os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 and the built CUDA library")


def _cuda_ok():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_ok():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)
