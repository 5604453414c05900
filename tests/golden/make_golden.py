"""Regenerates the golden fixtures in tests/golden/*.npz from the reference itself.

Run where a checkout of the reference exists, naming its root:

    python tests/golden/make_golden.py <dl-inference checkout>
    DLI_REFERENCE_ROOT=<dl-inference checkout> python tests/golden/make_golden.py

For every dli.graph.v1 operator this script executes the reference's own Triton
kernel (python/dli_ops/aot/<op>/kernel.py) on CPU through the Triton
interpreter (TRITON_INTERPRET=1), launched with the grid, block constants and
argument order of the reference launcher (python/dli_ops/aot/<op>/template.cc,
tools/build_triton_aot_ops.py:119-328). Cases come from two sources:

* the literal vectors of the reference operator tests
  (tests/operators/test_*.py), captured by executing those test modules with a
  stand-in for their ``operator_test_support`` helper; the tests' own expected
  tensors are stored next to the kernel outputs;
* seeded random cases at small shapes (including ragged sizes and every
  attribute the launchers read).

Each fixture stores, per case ``c<i>``: ``c<i>/in/<name>`` arrays,
``c<i>/out/<name>`` reference-kernel outputs, optional ``c<i>/expected/<name>``
(from the reference test), and ``c<i>/attrs`` (JSON bytes). The reference is not
needed at test time: only the .npz files are read.
"""
from __future__ import annotations

import importlib.util
import json
import math
import os
import sys
import types
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

REF_ARG = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DLI_REFERENCE_ROOT", "")
REF = Path(REF_ARG)
AOT = REF / "python" / "dli_ops" / "aot"
OUT = Path(__file__).resolve().parent


def _kernel(op: str, name: str):
    spec = importlib.util.spec_from_file_location(f"ref_{op}", AOT / op / "kernel.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return getattr(mod, name)


def _cdiv(a: int, b: int) -> int:
    return (a + b - 1) // b


def _pow2(x: int) -> int:
    p = 1
    while p < x:
        p *= 2
    return p


# ---- launchers: argument order and grids of the reference template.cc files ----

def run_linear(inputs, attrs):  # linear/template.cc:17-33
    x, w = inputs["x"], inputs["weight"]
    b = inputs.get("bias")
    m = int(np.prod(x.shape[:-1]))
    n, k = w.shape
    out = torch.empty(*x.shape[:-1], n)
    _kernel("linear", "linear_kernel")[(_cdiv(m, 16), _cdiv(n, 16))](
        x, w, b if b is not None else out, out, m, n, k=k, has_bias=b is not None,
        BLOCK_M=16, BLOCK_N=16, BLOCK_K=32)
    return {"output": out}


def run_matmul(inputs, attrs):  # matmul/template.cc:17-29
    a, b = inputs["a"], inputs["b"]
    m, k = a.shape
    n = b.shape[1]
    out = torch.empty(m, n)
    _kernel("matmul", "matmul_kernel")[(_cdiv(m, 16), _cdiv(n, 16))](
        a, b, out, m, n, k=k, BLOCK_M=16, BLOCK_N=16, BLOCK_K=32)
    return {"output": out}


def run_rms_norm(inputs, attrs):  # rms_norm/template.cc:15-27
    x, w = inputs["x"], inputs["weight"]
    hidden = x.shape[-1]
    rows = x.numel() // hidden
    eps = float(attrs.get("eps", 1e-6))
    out = torch.empty_like(x)
    _kernel("rms_norm", "rms_norm_kernel")[(rows,)](
        x, w, out, rows, eps, hidden=hidden, BLOCK_D=max(16, _pow2(hidden)))
    return {"output": out}


def run_rotary(inputs, attrs):  # rotary/template.cc:4-26
    q, k, cos, sin = inputs["q"], inputs["k"], inputs["cos"], inputs["sin"]
    out_q, out_k = q.clone(), k.clone()
    head_dim, seq, pairs = q.shape[3], q.shape[2], cos.shape[1]
    total = int(np.prod(q.shape[:-1])) * pairs
    start = int(attrs.get("start_pos", 0))
    _kernel("rotary", "rotary_kernel")[(_cdiv(total, 128),)](
        q, k, cos, sin, out_q, out_k, total, start, head_dim=head_dim, seq=seq,
        rotary_pairs=pairs, BLOCK=128)
    return {"out_q": out_q, "out_k": out_k}


def run_attention(inputs, attrs):  # attention/template.cc:26-47, scale from build_triton_aot_ops.py:283
    q, k, v = inputs["q"], inputs["k"], inputs["v"]
    b, h, sq, d = q.shape
    sk = k.shape[2]
    out = torch.empty_like(q)
    causal = bool(attrs.get("causal", False))
    _kernel("attention", "attention_kernel")[(b * h, _cdiv(sq, 16))](
        q, k, v, out, seq_q=sq, seq_k=sk, head_dim=d, causal=causal, scale=1.0 / (d ** 0.5),
        BLOCK_M=16, BLOCK_N=32, BLOCK_D=max(16, _pow2(d)))
    return {"output": out}


def run_embedding(inputs, attrs):  # embedding/template.cc:15-29
    ids, table = inputs["ids"], inputs["table"]
    hidden = table.shape[1]
    total = ids.numel()
    out = torch.empty(*ids.shape, hidden)
    _kernel("embedding", "embedding_kernel")[(_cdiv(total, 16), _cdiv(hidden, 32))](
        ids, table, out, total, hidden=hidden, BLOCK_T=16, BLOCK_D=max(16, _pow2(hidden)))
    return {"output": out}


def _binary(op):
    def run(inputs, attrs):  # add/template.cc, mul/template.cc
        names = list(inputs)
        a, b = inputs[names[0]], inputs[names[1]]
        out = torch.empty_like(a)
        total, width = a.numel(), b.numel()
        _kernel(op, f"{op}_kernel")[(_cdiv(total, 256),)](a, b, out, total, width, BLOCK=256)
        return {"output": out}
    return run


def _unary(op):
    def run(inputs, attrs):  # silu/template.cc, relu/template.cc
        x = inputs["x"]
        out = torch.empty_like(x)
        total = x.numel()
        _kernel(op, f"{op}_kernel")[(_cdiv(total, 256),)](x, out, total, BLOCK=256)
        return {"output": out}
    return run


def run_softmax(inputs, attrs):  # softmax/template.cc:23-35
    x = inputs["x"]
    width = x.shape[-1]
    rows = x.numel() // width
    out = torch.empty_like(x)
    _kernel("softmax", "softmax_kernel")[(rows,)](x, out, rows, width, BLOCK=max(8, _pow2(width)))
    return {"output": out}


def run_max_pool2d(inputs, attrs):  # max_pool2d/template.cc:8-27
    x = inputs["x"]
    ks = attrs.get("kernel_size", [2, 2])
    st = attrs.get("stride", ks)
    pad = attrs.get("padding", [0, 0])
    n, c, h, w = x.shape
    oh = (h + 2 * pad[0] - ks[0]) // st[0] + 1
    ow = (w + 2 * pad[1] - ks[1]) // st[1] + 1
    total = n * c * oh * ow
    out = torch.empty(n, c, oh, ow)
    _kernel("max_pool2d", "max_pool2d_kernel")[(_cdiv(total, 128),)](
        x, out, total, n, c, h, w, oh, ow, st[0], st[1], pad[0], pad[1], k_h=ks[0], k_w=ks[1],
        BLOCK=128)
    return {"output": out}


def run_batch_norm2d(inputs, attrs):  # batch_norm2d/template.cc:8-31
    x = inputs["x"]
    total, channels = x.numel(), x.shape[1]
    spatial = x.shape[2] * x.shape[3]
    eps = float(attrs.get("eps", 1e-5))
    out = torch.empty_like(x)
    _kernel("batch_norm2d", "batch_norm2d_kernel")[(_cdiv(total, 256),)](
        x, inputs["weight"], inputs["bias"], inputs["running_mean"], inputs["running_var"], out,
        total, channels, spatial, eps, BLOCK=256)
    return {"output": out}


def run_transpose(inputs, attrs):  # transpose/template.cc:9-17
    x = inputs["x"]
    rows, cols = x.shape
    out = torch.empty(cols, rows)
    _kernel("transpose", "transpose2d_kernel")[(_cdiv(rows, 16), _cdiv(cols, 16))](
        x, out, rows, cols, BLOCK_M=16, BLOCK_N=16)
    return {"output": out}


def run_conv2d(inputs, attrs):  # conv2d/template.cc:8-35
    x, w = inputs["x"], inputs["weight"]
    b = inputs.get("bias")
    st = attrs.get("stride", [1, 1])
    pad = attrs.get("padding", [0, 0])
    n, _, h, wd = x.shape
    oc, ic, kh, kw = w.shape
    oh = (h + 2 * pad[0] - kh) // st[0] + 1
    ow = (wd + 2 * pad[1] - kw) // st[1] + 1
    total = n * oc * oh * ow
    out = torch.empty(n, oc, oh, ow)
    _kernel("conv2d", "conv2d_kernel")[(_cdiv(total, 128),)](
        x, w, b if b is not None else out, out, total, n, h, wd, oc, oh, ow, st[0], st[1], pad[0],
        pad[1], in_c=ic, k_h=kh, k_w=kw, has_bias=b is not None, BLOCK=128)
    return {"output": out}


def run_reshape(inputs, attrs):  # reshape/template.cc:1-11 (a view; no kernel)
    x = inputs["x"]
    return {"output": x.reshape(attrs["shape"]).clone()}


RUNNERS = {
    "linear": run_linear, "matmul": run_matmul, "rms_norm": run_rms_norm,
    "rotary_embedding": run_rotary, "attention": run_attention, "embedding": run_embedding,
    "add": _binary("add"), "mul": _binary("mul"), "silu": _unary("silu"), "relu": _unary("relu"),
    "softmax": run_softmax, "max_pool2d": run_max_pool2d, "batch_norm2d": run_batch_norm2d,
    "transpose": run_transpose, "conv2d": run_conv2d, "reshape": run_reshape,
}

CASES: dict[str, list[dict]] = {op: [] for op in RUNNERS}


def record(op, inputs, attrs, outputs, expected=None):
    CASES[op].append({"inputs": inputs, "attrs": attrs or {}, "outputs": outputs,
                      "expected": expected or {}})


# ---- capture the reference operator tests -----------------------------------------

def capture_reference_tests() -> None:
    support = types.ModuleType("operator_test_support")
    support.CUDA_AVAILABLE = True
    state: dict = {}

    def run_operator(op_type, inputs, outputs=None, attrs=None):
        res = RUNNERS[op_type]({k: v.clone() for k, v in inputs.items()}, attrs or {})
        names = outputs or ["output"]
        res = {n: res[n] if n in res else list(res.values())[i] for i, n in enumerate(names)}
        state["last"] = (op_type, {k: v.clone() for k, v in inputs.items()}, attrs or {}, res)
        state["expected"] = {}
        return res

    def assert_close(test, actual, expected):
        op_type, inputs, attrs, res = state["last"]
        for name, value in res.items():
            if value is actual:
                state["expected"][name] = expected.detach().clone()
        torch.testing.assert_close(actual, expected.cpu(), rtol=1e-3, atol=1e-3)

    support.run_operator = run_operator
    support.assert_close = assert_close
    sys.modules["operator_test_support"] = support
    import unittest

    for path in sorted((REF / "tests" / "operators").glob("test_*.py")):
        spec = importlib.util.spec_from_file_location(path.stem, path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        suite = unittest.defaultTestLoader.loadTestsFromModule(mod)
        for test in _flatten(suite):
            state.clear()
            result = unittest.TestResult()
            test.run(result)
            if result.errors or result.failures:
                raise RuntimeError(f"reference test {test.id()} failed under the interpreter: "
                                   f"{result.errors or result.failures}")
            op_type, inputs, attrs, res = state["last"]
            record(op_type, inputs, attrs, res, dict(state.get("expected", {})))


def _flatten(suite):
    for item in suite:
        if hasattr(item, "__iter__"):
            yield from _flatten(item)
        else:
            yield item


# ---- seeded random cases --------------------------------------------------------

def random_cases() -> None:
    g = torch.Generator().manual_seed(1234)

    def rn(*shape, scale=1.0):
        return torch.randn(*shape, generator=g) * scale

    def add_case(op, inputs, attrs=None):
        res = RUNNERS[op]({k: v.clone() for k, v in inputs.items()}, attrs or {})
        record(op, inputs, attrs, res)

    for m, k, n, bias in ((5, 64, 7, True), (3, 96, 33, False), (17, 130, 19, True), (1, 8, 3, True)):
        inp = {"x": rn(m, k), "weight": rn(n, k, scale=0.1)}
        if bias:
            inp["bias"] = rn(n, scale=0.1)
        add_case("linear", inp)
    add_case("linear", {"x": rn(2, 3, 40), "weight": rn(9, 40, scale=0.1), "bias": rn(9)})
    for m, k, n in ((5, 20, 7), (16, 64, 16), (33, 17, 3)):
        add_case("matmul", {"a": rn(m, k), "b": rn(k, n)})
    for rows, hidden in ((3, 37), (4, 128), (2, 896)):
        add_case("rms_norm", {"x": rn(rows, hidden), "weight": rn(hidden)}, {"eps": 1e-6})
    add_case("rms_norm", {"x": rn(2, 3, 8), "weight": rn(8)}, {"eps": 1e-5})
    for b, h, s, d, pairs, start in ((2, 3, 4, 8, 4, 2), (1, 2, 3, 6, 2, 0), (1, 1, 5, 128, 64, 7)):
        rows = start + s + 1
        ang = rn(rows, pairs)
        add_case("rotary_embedding", {"q": rn(b, h, s, d), "k": rn(b, h, s, d),
                                      "cos": torch.cos(ang), "sin": torch.sin(ang)},
                 {"start_pos": start})
    for b, h, sq, sk, d, causal in ((2, 2, 5, 5, 8, True), (2, 2, 5, 5, 8, False),
                                    (1, 3, 1, 7, 16, True), (1, 1, 3, 9, 4, True),
                                    (1, 2, 17, 40, 64, True), (1, 1, 33, 33, 128, True)):
        add_case("attention", {"q": rn(b, h, sq, d), "k": rn(b, h, sk, d), "v": rn(b, h, sk, d)},
                 {"causal": causal})
    ids = torch.randint(0, 11, (3, 4), generator=g, dtype=torch.int64)
    add_case("embedding", {"ids": ids, "table": rn(11, 6)})
    add_case("embedding", {"ids": torch.randint(0, 50, (7,), generator=g, dtype=torch.int64),
                           "table": rn(50, 128)})
    for op in ("add", "mul"):
        add_case(op, {"x": rn(4, 5), "b": rn(5)})
        add_case(op, {"x": rn(3, 8), "b": rn(2)})
        add_case(op, {"x": rn(6, 16), "b": rn(6, 16)})
    for op in ("silu", "relu"):
        add_case(op, {"x": rn(7, 9, scale=4.0)})
    add_case("softmax", {"x": rn(3, 5)})
    add_case("softmax", {"x": rn(2, 40, scale=3.0)})
    add_case("max_pool2d", {"x": rn(2, 3, 7, 9)}, {"kernel_size": [2, 2], "stride": [2, 2],
                                                   "padding": [0, 0]})
    add_case("max_pool2d", {"x": rn(1, 2, 6, 6)}, {"kernel_size": [3, 3], "stride": [1, 1],
                                                   "padding": [1, 1]})
    add_case("batch_norm2d", {"x": rn(2, 3, 4, 5), "weight": rn(3), "bias": rn(3),
                              "running_mean": rn(3), "running_var": rn(3).abs() + 0.5},
             {"eps": 1e-5})
    add_case("transpose", {"x": rn(5, 7)}, {"perm": [1, 0]})
    add_case("transpose", {"x": rn(16, 33)}, {"perm": [1, 0]})
    add_case("conv2d", {"x": rn(2, 3, 6, 7), "weight": rn(4, 3, 3, 3, scale=0.3), "bias": rn(4)},
             {"stride": [1, 1], "padding": [1, 1]})
    add_case("conv2d", {"x": rn(1, 2, 8, 8), "weight": rn(3, 2, 2, 2)},
             {"stride": [2, 2], "padding": [0, 0]})
    add_case("conv2d", {"x": rn(1, 16, 5, 5), "weight": rn(8, 16, 3, 3, scale=0.2), "bias": rn(8)},
             {"stride": [1, 1], "padding": [1, 1]})
    add_case("reshape", {"x": rn(2, 3, 4)}, {"shape": [4, -1]})


def save() -> None:
    for op, cases in CASES.items():
        arrays = {}
        for i, case in enumerate(cases):
            for name, t in case["inputs"].items():
                arrays[f"c{i}/in/{name}"] = t.numpy()
            for name, t in case["outputs"].items():
                arrays[f"c{i}/out/{name}"] = t.numpy()
            for name, t in case["expected"].items():
                arrays[f"c{i}/expected/{name}"] = t.numpy()
            arrays[f"c{i}/attrs"] = np.frombuffer(json.dumps(case["attrs"]).encode(), dtype=np.uint8)
        arrays["count"] = np.array(len(cases))
        np.savez_compressed(OUT / f"{op}.npz", **arrays)
        print(f"{op}: {len(cases)} cases")


def main() -> int:
    if not REF_ARG or not AOT.exists():
        print(f"reference checkout not found at {REF_ARG!r}: pass its root as the first argument "
              "or in DLI_REFERENCE_ROOT", file=sys.stderr)
        return 1
    capture_reference_tests()
    random_cases()
    save()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
