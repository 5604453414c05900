"""CPU checks of the C ABI boundary: the kernel library loads without a GPU and
exports every entry point declared in include/dli_sm100.h, and the Python
binding declares a signature for each of them."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import dli_sm100

HEADER = Path(__file__).resolve().parents[1] / "include" / "dli_sm100.h"


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"\b(dli_sm100_\w+)\s*\(", text))


def test_header_declares_the_operator_entry_points():
    names = declared_functions()
    for op in ("linear", "matmul", "conv2d", "rms_norm", "rotary_embedding", "attention", "embedding",
               "add", "mul", "silu", "relu", "softmax", "max_pool2d", "batch_norm2d", "transpose2d"):
        assert f"dli_sm100_{op}" in names, op


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(dli_sm100.LIB_PATH))
    missing = [n for n in sorted(declared_functions()) if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_the_header():
    assert declared_functions() == set(dli_sm100.SIGNATURES)


def test_abi_version_and_queries_without_gpu():
    lib = dli_sm100.lib()
    assert lib.dli_sm100_abi_version() == 1
    assert lib.dli_sm100_last_error() == b""
    # workspace queries are pure host arithmetic
    assert lib.dli_sm100_linear_workspace_size(64, 1024, 4096, 0) == 0  # fp32: no scratch
    assert lib.dli_sm100_attention_workspace_size(1, 4, 4, 8, 8, 7, 2) == 0  # head_dim 7: fallback
