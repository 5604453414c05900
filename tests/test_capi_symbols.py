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


def test_tp_exchange_buffer_size_is_host_arithmetic():
    """Exchange buffer bytes: a 4096-aligned header of per-row epochs (all-reduce and
    argmax), then 2 slots x tp x max_rows rows of 8-byte words carrying 4 payload
    bytes each, then 2 slots x tp x max_rows argmax candidates of two words."""
    lib = dli_sm100.lib()
    tp, rows, elems = 2, 64, 3584
    header = 4096  # 2 * 64 * 4 bytes of epochs, rounded up to 4096
    words = 2 * tp * rows * (elems * 2 // 4) * 8
    argmax = 2 * tp * rows * 2 * 8
    assert lib.dli_sm100_tp_exchange_bytes(tp, rows, elems, 2) == header + words + argmax
    assert lib.dli_sm100_tp_exchange_bytes(4, 256, 8192, 0) == 4096 + 2 * 4 * 256 * 8192 * 8 + 2 * 4 * 256 * 16
    assert lib.dli_sm100_tp_exchange_bytes(9, 64, 3584, 2) == 0  # more than 8 ranks
    assert lib.dli_sm100_tp_exchange_bytes(2, 64, 3584, 1) == 0  # int64 is not an exchange dtype
