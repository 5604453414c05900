"""Python surface of the dli runtime with the sm_100a operator plugin.

Same names as the reference package (python/dli/__init__.py:5 of
yncxcw/dl-inference): ``dli.Engine``, ``dli.Graph``, ``dli.load_weights``.
``dli.PLUGIN_PATH`` is the in-tree operator plugin to pass to
``Engine.load_library``. ``dli.ProfileSession`` times every graph node of the
runs it is passed to (``engine.run(graph, inputs, profile=session)``) and
writes ``dli.profile.v1`` JSON; ``python -m dli.profile`` analyses it.
"""
from __future__ import annotations

from pathlib import Path

import torch as _torch  # noqa: F401  (loads libtorch before the native module)

from ._dli_native import Engine, Graph, ProfileSession, load_weights

PLUGIN_PATH = str(Path(__file__).resolve().parents[2] / "lib" / "libdli_sm100_ops.so")

__all__ = ["Engine", "Graph", "ProfileSession", "load_weights", "PLUGIN_PATH"]
