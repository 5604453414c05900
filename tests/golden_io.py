"""Reader for the golden fixtures written by tests/golden/make_golden.py."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"

OPS = ("linear", "matmul", "rms_norm", "rotary_embedding", "attention", "embedding", "add", "mul",
       "silu", "relu", "softmax", "max_pool2d", "batch_norm2d", "transpose", "conv2d", "reshape")


def load_cases(op: str) -> list[dict]:
    data = np.load(GOLDEN / f"{op}.npz")
    cases = []
    for i in range(int(data["count"])):
        prefix = f"c{i}/"
        case = {"inputs": {}, "outputs": {}, "expected": {},
                "attrs": json.loads(bytes(data[f"{prefix}attrs"]).decode())}
        for key in data.files:
            if not key.startswith(prefix) or key == f"{prefix}attrs":
                continue
            _, kind, name = key.split("/", 2)
            {"in": case["inputs"], "out": case["outputs"], "expected": case["expected"]}[kind][name] = data[key]
        cases.append(case)
    return cases


def all_cases():
    for op in OPS:
        for i, case in enumerate(load_cases(op)):
            yield op, i, case
