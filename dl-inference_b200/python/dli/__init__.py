"""Python surface of the dli runtime with the sm_100a operator plugin.

Same names as the reference package (python/dli/__init__.py:5 of
yncxcw/dl-inference): ``dli.Engine``, ``dli.Graph``, ``dli.load_weights``.
``dli.PLUGIN_PATH`` is the in-tree operator plugin to pass to
``Engine.load_library``.
"""
from __future__ import annotations

from pathlib import Path

import torch as _torch  # noqa: F401  (loads libtorch before the native module)

from ._dli_native import Engine, Graph, load_weights

PLUGIN_PATH = str(Path(__file__).resolve().parents[2] / "lib" / "libdli_sm100_ops.so")

__all__ = ["Engine", "Graph", "load_weights", "PLUGIN_PATH"]
