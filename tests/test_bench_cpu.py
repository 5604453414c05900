"""CPU tests of bench.py's host-side baselines (the reference's CPU path, PyTorch
eager): both report a positive rate in the bench's units, the cores they used
and a sample description, on a tiny Qwen2 shape so the test takes seconds."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
from dli_export.qwen2 import Qwen2Shape  # noqa: E402

TINY = Qwen2Shape(hidden=64, layers=3, q_heads=4, kv_heads=2, head_dim=16, intermediate=128, vocab=256)


def test_cpu_prefill_reports_tokens_per_second():
    r = bench.cpu_prefill(TINY, prompt=48, seconds=0.05)
    assert r["unit"] == "tok/s (prefill)" and r["kind"] == "reference"
    assert r["value"] > 0 and r["cores"] >= 1
    # one sequence of 48 tokens through 3 layers: the rate is the tokens over the scaled time
    assert r["value"] == pytest.approx(48 / (r["ms_per_sequence"] / 1e3))
    assert "48-token sequence" in r["sample"] and "x3 layers" in r["sample"]


def test_cpu_decode_baseline_reports_tokens_per_second():
    r = bench.cpu_baseline(TINY, batch=2, prompt=16, seconds=0.05)
    assert r["unit"] == "tok/s (decode)" and r["kind"] == "reference"
    assert r["value"] > 0 and r["cores"] >= 1
    assert r["value"] == pytest.approx(2 / (r["ms_per_step"] / 1e3))
