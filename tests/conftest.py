"""Shared pytest configuration.

* Puts the repository root (``oracle``), ``dl-inference_b200/python``
  (``dli``, ``dli_sm100``, ``dli_export``) on ``sys.path``.
* Registers the ``gpu`` marker. GPU tests run through the CUDA kernels of
  ``libdli_sm100.so`` and are skipped only when no CUDA device exists; on a GPU
  host a missing library is an error, never a silent fallback.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "dl-inference_b200"
for p in (ROOT, PKG / "python"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built kernels")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_cuda = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
