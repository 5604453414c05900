"""The reference's own GPU kernels next to this repository's, on the same inputs.

oracle/ref_triton.py compiles the reference's Triton kernel sources
(python/dli_ops/aot/<op>/kernel.py) for sm_100a into oracle/_ref/triton/.
These tests launch those cubins through the CUDA driver the way the reference
launcher does (python/dli_ops/aot/<op>/template.cc: the same argument order and
grids, 128 threads), with the launch details a Triton 3.6 kernel needs that
the reference launcher predates (two trailing scratch pointers, and the
dynamic shared-memory limit raised above 48 KB where the kernel asks for more).

Each case checks parity in both directions against the float64 oracle: this
repository's kernel within its own tolerance, the reference kernel within a
TF32 tolerance (its fp32 tl.dot runs as TF32), and times both with CUDA events
over 20 launches captured in a CUDA graph (after 3 warm-up launches), so host
launch costs are excluded on both sides. The timings go to $DLI_REF_TIMING.
Skipped when the cubins were not built (no reference checkout at build time).
"""
from __future__ import annotations

import ctypes
import json
import math
import os
from pathlib import Path

import numpy as np
import pytest
import torch

import dli_sm100 as C
from oracle import ops as O

REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "triton"

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not (REF / "linear_k1024_b1.cubin").exists(),
                                 reason="reference Triton kernels not built (oracle/ref_triton.py)")]

TF32_TOL = 5e-3  # relative Frobenius error of a TF32 contraction of K <= 18944 N(0,1) x N(0,0.02) terms
CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES = 8


class RefKernel:
    """One compiled reference kernel, launched with cuLaunchKernel."""

    _cuda = None

    def __init__(self, spec_id: str):
        if RefKernel._cuda is None:
            RefKernel._cuda = ctypes.CDLL("libcuda.so.1")
        cu = RefKernel._cuda
        self.info = json.loads((REF / f"{spec_id}.json").read_text())
        assert self.info["global_scratch_size"] == 0 and self.info["profile_scratch_size"] == 0
        torch.cuda.synchronize()  # the primary context is current on this thread
        self._image = (REF / f"{spec_id}.cubin").read_bytes()
        self.module = ctypes.c_void_p()
        self._check(cu.cuModuleLoadData(ctypes.byref(self.module), ctypes.c_char_p(self._image)), "load")
        self.fn = ctypes.c_void_p()
        self._check(cu.cuModuleGetFunction(ctypes.byref(self.fn), self.module,
                                           self.info["symbol"].encode()), "function")
        if self.info["shared"] > 49152:
            self._check(cu.cuFuncSetAttribute(self.fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                              ctypes.c_int(self.info["shared"])), "shared limit")

    @staticmethod
    def _check(res: int, what: str) -> None:
        assert res == 0, f"CUDA driver call ({what}) returned {res}"

    def __call__(self, grid, **args) -> None:
        holders = []
        for p in self.info["params"]:
            name, kind = p.split(":")
            if name in ("global_scratch", "profile_scratch"):
                holders.append(ctypes.c_void_p(0))
            elif kind.startswith("*"):
                t = args[name]
                assert t.is_cuda and t.is_contiguous() and t.dtype == torch.float32, name
                holders.append(ctypes.c_void_p(t.data_ptr()))
            else:
                assert kind == "i32", kind
                holders.append(ctypes.c_int32(int(args[name])))
        params = (ctypes.c_void_p * len(holders))(*[ctypes.cast(ctypes.pointer(h), ctypes.c_void_p) for h in holders])
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        gx, gy, gz = grid
        self._check(RefKernel._cuda.cuLaunchKernel(self.fn, gx, gy, gz, 32 * self.info["num_warps"], 1, 1,
                                                   self.info["shared"], stream, params, None), "launch")


def _time(fn, reps=20) -> float:
    """Device time per launch: `reps` launches captured in one CUDA graph and
    replayed, so neither side's host launch cost (ctypes, tensor-map encoding)
    shows up in the figure."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(reps):
            fn()
    graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    graph.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def _rel(got, ref) -> float:
    got = got.double().cpu().numpy() if isinstance(got, torch.Tensor) else got
    return float(np.linalg.norm(got - ref) / np.linalg.norm(ref))


def _report(case: str, **fields) -> None:
    line = json.dumps({"case": case, **fields})
    print(line)
    path = os.environ.get("DLI_REF_TIMING")
    if path:
        with open(path, "a") as f:
            f.write(line + "\n")


@pytest.mark.parametrize("spec,m,n,k,bias", [
    ("linear_k1024_b1", 64, 4096, 1024, True),     # the single-linear workload
    ("linear_k4096_b1", 64, 4096, 4096, True),     # the CNN's fully-connected layers
    ("linear_k3584_b0", 32, 4608, 3584, False),    # 7B decode qkv projection
    ("linear_k18944_b0", 32, 3584, 18944, False),  # 7B decode down projection
])
def test_linear_against_reference_kernel(spec, m, n, k, bias):
    kern = RefKernel(spec)
    assert kern.info["constexprs"]["k"] == k
    g = torch.Generator(device="cuda").manual_seed(k + n)
    x = torch.randn(m, k, device="cuda", generator=g)
    w = torch.randn(n, k, device="cuda", generator=g) * 0.02
    b = torch.randn(n, device="cuda", generator=g) * 0.02 if bias else None
    y_ref = torch.empty(m, n, device="cuda")
    # reference launcher: grid (ceil(M/16), ceil(N/16)); no bias passes the output pointer
    launch = lambda: kern((math.ceil(m / 16), math.ceil(n / 16), 1), x=x, weight=w,  # noqa: E731
                          bias=b if bias else y_ref, out=y_ref, m=m, n=n)
    launch()
    ours = C.linear(x, w, b)
    torch.cuda.synchronize()
    oracle = O.linear(x.double().cpu().numpy(), w.double().cpu().numpy(),
                      b.double().cpu().numpy() if bias else None)
    assert _rel(ours, oracle) <= 1e-4
    assert _rel(y_ref, oracle) <= TF32_TOL
    t_ref = _time(launch)
    t_ours = _time(lambda: C.linear(x, w, b))
    xb, wb = x.bfloat16(), w.bfloat16()
    t_bf16 = _time(lambda: C.linear(xb, wb, b.bfloat16() if bias else None))
    _report(f"linear {m}x{n}x{k} fp32", reference_ms=t_ref, ours_ms=t_ours, ours_bf16_ms=t_bf16,
            reference_rel_err=_rel(y_ref, oracle), ours_rel_err=_rel(ours, oracle),
            speedup=t_ref / t_ours)


def test_conv1_against_reference_kernel():
    kern = RefKernel("conv_c3_k3x3_b1")
    n, c, h, wd, oc = 64, 3, 32, 32, 64
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(n, c, h, wd, device="cuda", generator=g)
    w = torch.randn(oc, c, 3, 3, device="cuda", generator=g) * 0.02
    b = torch.randn(oc, device="cuda", generator=g) * 0.02
    y_ref = torch.empty(n, oc, h, wd, device="cuda")
    total = n * oc * h * wd
    launch = lambda: kern((math.ceil(total / 128), 1, 1), x=x, w=w, bias=b, out=y_ref, total=total,  # noqa: E731
                          n_dim=n, h_dim=h, w_dim=wd, out_c=oc, out_h=h, out_w=wd, stride_h=1, stride_w=1,
                          pad_h=1, pad_w=1)
    launch()
    ours = C.conv2d(x, w, b, (1, 1), (1, 1))
    torch.cuda.synchronize()
    oracle = torch.nn.functional.conv2d(x.double().cpu(), w.double().cpu(), b.double().cpu(), padding=1).numpy()
    assert _rel(ours, oracle) <= 1e-4
    assert _rel(y_ref, oracle) <= 1e-4  # direct FMA convolution: fp32 exact
    t_ref = _time(launch)
    t_ours = _time(lambda: C.conv2d(x, w, b, (1, 1), (1, 1)))
    xh, wh, bh = x.half(), w.half(), b.half()
    t_f16 = _time(lambda: C.conv2d(xh, wh, bh, (1, 1), (1, 1)))
    _report("conv1 64x3x32x32 -> 64 k3 fp32", reference_ms=t_ref, ours_ms=t_ours, ours_f16_ms=t_f16,
            reference_rel_err=_rel(y_ref, oracle), ours_rel_err=_rel(ours, oracle), speedup=t_ref / t_ours)


@pytest.mark.parametrize("spec,bh,sq,sk", [
    ("attention_q1_k512_d128_c1", 1, 1, 512),
    ("attention_q1_k2048_d128_c1", 1, 1, 2048),
    ("attention_q1_k2048_d128_c1", 896, 1, 2048),   # 32 sequences x 28 heads, one decode token
    ("attention_q128_k128_d128_c1", 896, 128, 128),
])
def test_attention_against_reference_kernel(spec, bh, sq, sk):
    kern = RefKernel(spec)
    assert kern.info["constexprs"]["seq_q"] == sq and kern.info["constexprs"]["seq_k"] == sk
    d = 128
    g = torch.Generator(device="cuda").manual_seed(bh + sk)
    q = torch.randn(1, bh, sq, d, device="cuda", generator=g)
    k = torch.randn(1, bh, sk, d, device="cuda", generator=g)
    v = torch.randn(1, bh, sk, d, device="cuda", generator=g)
    o_ref = torch.empty_like(q)
    launch = lambda: kern((bh, math.ceil(sq / 16), 1), q=q, k=k, v=v, out=o_ref)  # noqa: E731
    launch()
    ours = C.attention(q, k, v, causal=True)
    torch.cuda.synchronize()
    oracle = O.attention(q.double().cpu().numpy(), k.double().cpu().numpy(), v.double().cpu().numpy(), True)
    assert _rel(ours, oracle) <= 1e-4
    assert _rel(o_ref, oracle) <= TF32_TOL
    t_ref = _time(launch)
    t_ours = _time(lambda: C.attention(q, k, v, causal=True))
    qb, kb, vb = q.bfloat16(), k.bfloat16(), v.bfloat16()
    t_bf16 = _time(lambda: C.attention(qb, kb, vb, causal=True))
    _report(f"attention bh{bh} q{sq} k{sk} d128 fp32", reference_ms=t_ref, ours_ms=t_ours, ours_bf16_ms=t_bf16,
            reference_rel_err=_rel(o_ref, oracle), ours_rel_err=_rel(ours, oracle), speedup=t_ref / t_ours)
