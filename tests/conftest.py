"""Shared pytest configuration.

* ``gpu`` marker: tests that need a B200 (run with ``-m gpu``); they are skipped
  automatically when no CUDA device is visible.
* Puts the drop-in package (``flash-eq_b200/``) and the test-only oracle on
  ``sys.path``.
"""
from __future__ import annotations

import os
import sys

import pytest
import torch

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
PKG = os.path.join(ROOT, "flash-eq_b200")
ORACLE = os.path.join(ROOT, "oracle")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (PKG, ORACLE, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device; run with -m gpu")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device visible")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def golden(name: str):
    return torch.load(os.path.join(GOLDEN, name), weights_only=False)


@pytest.fixture
def cuda_device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device visible")
    return torch.device("cuda")


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double().cpu()
    b = b.double().cpu()
    den = b.norm().item()
    return (a - b).norm().item() / (den if den > 0 else 1.0)


def check_equivariance(out1, out2, rtol=1e-4, msg="equivariance"):
    """Max-abs relative difference, as the reference's tests/helpers.py:109-124."""
    rel = (out1 - out2).abs().max().item() / (out1.abs().max().item() + 1e-8)
    assert rel < rtol, f"{msg}: rel_diff={rel:.2e} (threshold={rtol:.0e})"
