"""GPU parity of every C-ABI entry point of libdli_sm100.so against the oracle.

Tolerances (written per dtype, checked as a relative Frobenius error plus an
elementwise bound):
  float32  rel <= 1e-4   (north-star fp32 bound; the kernels accumulate in fp32)
  bfloat16 rel <= 1.5e-2 (inputs are rounded to bf16 first, the oracle runs on
                          the rounded values in fp32/fp64; the bound covers bf16
                          output rounding and bf16 P in attention)
  float16  rel <= 5e-3
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from golden_io import all_cases
from op_cases import capi_outputs, oracle_outputs
from oracle import ops as O

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 1.5e-2, torch.float16: 5e-3}


def rel_err(got, ref) -> float:
    got = torch.as_tensor(got).double().cpu()
    ref = torch.as_tensor(ref).double().cpu()
    den = ref.norm().item()
    return (got - ref).norm().item() / (den if den > 0 else 1.0)


def assert_close(got, ref, dtype, what=""):
    got = torch.as_tensor(got).double().cpu()
    ref = torch.as_tensor(ref).double().cpu()
    assert got.shape == ref.shape, f"{what}: shape {tuple(got.shape)} vs {tuple(ref.shape)}"
    tol = TOL[dtype]
    err = rel_err(got, ref)
    assert err <= tol, f"{what}: relative error {err:.3e} > {tol:.1e}"
    scale = max(ref.abs().max().item(), 1e-6)
    bad = (got - ref).abs() > (8 * tol * scale + 8 * tol * ref.abs())
    assert not bad.any(), f"{what}: {int(bad.sum())} elements out of the elementwise bound"


def rounded(a: np.ndarray, dtype) -> np.ndarray:
    """Rounds float inputs through `dtype` so the oracle sees what the kernel sees."""
    if a.dtype.kind != "f":
        return a
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).double().numpy()


CASES = list(all_cases())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16],
                         ids=["f32", "bf16", "f16"])
@pytest.mark.parametrize("op,idx,case", CASES, ids=[f"{op}-{i}" for op, i, _ in CASES])
def test_golden_case_through_capi(op, idx, case, dtype):
    inp = case["inputs"]
    if op == "rotary_embedding":
        # cos/sin tables stay fp32 in every dtype (reference tables are fp32, export.py:228-247)
        rinp = {k: (v if k in ("cos", "sin") else rounded(v, dtype)) for k, v in inp.items()}
    else:
        rinp = {k: rounded(v, dtype) for k, v in inp.items()}
    want = oracle_outputs(op, rinp, case["attrs"])
    got = capi_outputs(op, inp, case["attrs"], dtype)
    torch.cuda.synchronize()
    for name, ref in want.items():
        assert_close(got[name].float(), ref, dtype, f"{op}[{idx}].{name}")
    if dtype == torch.float32:
        # the reference kernel's own output (golden) as well, where its math is sound
        bad_ref = op == "attention" and not case["attrs"].get("causal", False) and \
            inp["k"].shape[2] % 32 != 0
        if not bad_ref:
            for name, ref in case["outputs"].items():
                assert_close(got[name].float(), ref, dtype, f"{op}[{idx}].{name} vs reference kernel")


# ---- contractions at model scale ------------------------------------------------------

LINEAR_SHAPES = [  # (M, N, K)
    (1, 896, 896), (8, 1152, 896), (8, 9728, 896), (8, 896, 4864), (32, 4608, 3584),
    (32, 3584, 18944), (64, 3696, 8192), (100, 200, 96), (128, 896, 896), (129, 1152, 896),
    (512, 4864, 896), (2048, 3584, 3584), (300, 37888 // 8, 3584), (7, 152064 // 16, 896),
    # tensor-parallel decode shards (7B at TP 2/4, 72B at TP 8): few tiles, so K is split
    # over clusters of 2..8 CTAs, including sizes that do not divide the 128-row tile
    (32, 3584, 3584), (32, 2304, 3584), (32, 3584, 1792), (32, 9472, 3584), (32, 3584, 896),
    (32, 1152, 3584), (16, 3584, 4736), (64, 1280, 8192), (64, 8192, 1024), (32, 640, 3584),
]


GLU_SHAPES = [  # (M, intermediate, K): decode (swap-AB, split-K clusters) and prefill tiles
    (1, 4864, 896), (8, 4864, 896), (32, 18944, 3584), (32, 9472, 3584), (32, 4736, 3584),
    (64, 3696, 8192), (128, 100, 64), (7, 96, 64), (129, 4864, 896), (512, 2368, 896), (2048, 1000, 512),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("m,inter,k", GLU_SHAPES)
def test_linear_silu_mul_matches_unfused(m, inter, k, dtype):
    """The fused gate/up GEMM + SwiGLU epilogue against an fp32 reference, and
    against linear -> silu_mul through the library: the fused form rounds once
    (from the fp32 accumulators) where the unfused graph rounds four times, so
    it must be at least as close to the fp32 reference."""
    import dli_sm100 as C
    from dli_export.qwen2 import glu_blocked

    g = torch.Generator(device="cuda").manual_seed(m + inter + k)
    x = torch.randn(m, k, device="cuda", generator=g).to(dtype)
    wg = (torch.randn(inter, k, device="cuda", generator=g) * 0.03).to(dtype)
    wu = (torch.randn(inter, k, device="cuda", generator=g) * 0.03).to(dtype)
    y = C.linear_silu_mul(x, glu_blocked(wg, wu), inter)
    y2 = C.linear_silu_mul(x, glu_blocked(wg, wu), inter)
    C.check_device_error()
    unfused = C.silu_mul(C.linear(x, torch.cat([wg, wu])))
    assert torch.equal(y, y2)
    gate, up = x.float() @ wg.float().T, x.float() @ wu.float().T
    ref = torch.nn.functional.silu(gate) * up
    assert_close(y.float(), ref, dtype, f"linear_silu_mul {m}x{inter}x{k}")
    assert rel_err(y.float(), ref) <= rel_err(unfused.float(), ref) * 1.02 + 1e-6


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("m,n,k", LINEAR_SHAPES)
def test_linear_tcgen05_model_shapes(m, n, k, dtype):
    import dli_sm100 as C

    g = torch.Generator(device="cuda").manual_seed(m * 7 + n + k)
    x = torch.randn(m, k, device="cuda", generator=g).to(dtype)
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.02).to(dtype)
    b = (torch.randn(n, device="cuda", generator=g) * 0.02).to(dtype)
    y = C.linear(x, w, b)
    y2 = C.linear(x, w, b)  # second call: same bits (deterministic split-K reduction)
    C.check_device_error()
    ref = x.float() @ w.float().T + b.float()
    assert_close(y.float(), ref, dtype, f"linear {m}x{n}x{k}")
    assert torch.equal(y, y2)


@pytest.mark.parametrize("m,n,k", [(32, 4608, 3584), (32, 3584, 3584), (32, 3584, 18944), (8, 1152, 896),
                                   (32, 152064, 3584), (64, 1280, 8192), (3, 700, 136), (40, 1000, 1024)])
def test_linear_stream_k_reuses_workspace(m, n, k):
    """Decode-sized linears whose tiles do not fill whole waves run stream-K:
    partial tiles through the caller's workspace, summed by the last contributor
    in CTA order. Three calls on one workspace must agree bit for bit (the
    per-tile counters return to zero after each call), match the no-workspace
    cluster path within bf16 tolerance, and match an fp32 reference; the LM-head
    shape also with float32 output."""
    import dli_sm100 as C

    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(n, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    L = C.lib()
    need = L.dli_sm100_linear_workspace_size(m, n, k, C.DTYPE_CODES[torch.bfloat16])
    ws = torch.zeros(max(need, 16), dtype=torch.uint8, device="cuda")
    outs = []
    for _ in range(3):
        y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
        C.check(L.dli_sm100_linear(C._ptr(x), C._ptr(w), C._ptr(b), C._ptr(y), m, n, k, C.DTYPE_CODES[torch.bfloat16],
                                   C._ptr(ws), need, C._stream()), "linear")
        outs.append(y)
    y_cluster = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    C.check(L.dli_sm100_linear(C._ptr(x), C._ptr(w), C._ptr(b), C._ptr(y_cluster), m, n, k,
                               C.DTYPE_CODES[torch.bfloat16], None, 0, C._stream()), "linear")
    C.check_device_error()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    ref = torch.nn.functional.linear(x.float(), w.float(), b.float())
    assert_close(outs[0].float(), ref, torch.bfloat16, f"stream-K linear {m}x{n}x{k}")
    assert_close(y_cluster.float(), ref, torch.bfloat16, f"cluster linear {m}x{n}x{k}")
    if need:
        counters = ws[need - ((n + 127) // 128 * 4 + 255) // 256 * 256:need]  # may include padding: all zero
        assert int(counters.count_nonzero()) == 0
    if n == 152064:
        y32 = C.linear_ex(x, w, b, out_dtype=torch.float32)
        y32b = C.linear_ex(x, w, b, out_dtype=torch.float32)
        assert torch.equal(y32, y32b)
        assert_close(y32, ref, torch.float16, "LM head fp32 logits")  # fp32 output: tighter than bf16


def test_linear_fp32_config1():
    """The single-linear workload: x[64,1024] . W[4096,1024]^T + b in fp32, rel-err <= 1e-4."""
    import dli_sm100 as C

    g = torch.Generator().manual_seed(0)
    x = torch.randn(64, 1024, generator=g)
    w = torch.randn(4096, 1024, generator=g) * 0.02
    b = torch.randn(4096, generator=g) * 0.02
    y = C.linear(x.cuda(), w.cuda(), b.cuda())
    ref = O.linear(x.numpy(), w.numpy(), b.numpy())
    assert rel_err(y, ref) <= 1e-4
    assert np.abs(y.cpu().double().numpy() - ref).max() <= 1e-4 * np.abs(ref).max()


@pytest.mark.parametrize("m,n,k", [(64, 4096, 1024), (32, 4608, 3584), (32, 3584, 18944), (1, 10, 4096),
                                   (70, 130, 52), (4096, 256, 64), (3, 7, 5), (129, 1000, 260)])
def test_linear_fp32_split_k_shapes(m, n, k):
    """Exact-fp32 linear at decode-sized, ragged and odd-K shapes (the cluster
    split-K FFMA kernel, or the scalar kernel where K is not a multiple of 4)."""
    import dli_sm100 as C

    g = torch.Generator(device="cuda").manual_seed(m * 7 + n + k)
    x = torch.randn(m, k, device="cuda", generator=g)
    w = torch.randn(n, k, device="cuda", generator=g) * 0.02
    b = torch.randn(n, device="cuda", generator=g) * 0.02
    y = C.linear(x, w, b)
    y2 = C.linear(x, w, b)
    ref = torch.nn.functional.linear(x.double(), w.double(), b.double())
    assert_close(y, ref, torch.float32, f"linear fp32 {m}x{n}x{k}")
    assert torch.equal(y, y2)  # deterministic split-K reduction


@pytest.mark.parametrize("m,n,k", [(64, 4096, 1024), (1, 4096, 4096), (128, 512, 2048), (600, 384, 1000)])
def test_linear_fp32_tcgen05_split_accuracy(m, n, k):
    """fp32 on tcgen05 through the three-term bf16 split (six bf16 products per
    K step): the dropped terms sit near 2^-26 of each product, so the error is
    that of an fp32 FFMA GEMM (3-9e-7 at these shapes), bound 2e-6 here, far
    inside the 1e-4 fp32 tolerance; NaN inputs propagate."""
    import dli_sm100 as C

    g = torch.Generator(device="cuda").manual_seed(11 * m + n + k)
    x = torch.randn(m, k, device="cuda", generator=g)
    w = torch.randn(n, k, device="cuda", generator=g) * 0.02
    b = torch.randn(n, device="cuda", generator=g) * 0.02
    ref = torch.nn.functional.linear(x.double(), w.double(), b.double())
    err = rel_err(C.linear(x, w, b).double().cpu(), ref.cpu())
    assert err <= 2e-6, f"fp32 split GEMM {m}x{n}x{k}: relative error {err:.2e}"
    x[0, k // 2] = float("nan")
    y = C.linear(x, w, b)
    assert torch.isnan(y[0]).all() and torch.isfinite(y[1:]).all()


@pytest.mark.parametrize("m,n,k", [(70, 132, 52), (64, 4096, 1024), (33, 257, 4000), (5, 12, 3), (16, 512, 8192)])
def test_matmul_fp32_shapes(m, n, k):
    import dli_sm100 as C

    g = torch.Generator(device="cuda").manual_seed(m + n * 3 + k)
    a = torch.randn(m, k, device="cuda", generator=g)
    b = torch.randn(k, n, device="cuda", generator=g) * 0.05
    assert_close(C.matmul(a, b), a.double() @ b.double(), torch.float32, f"matmul fp32 {m}x{n}x{k}")


def test_matmul_bf16_and_f32():
    import dli_sm100 as C

    g = torch.Generator(device="cuda").manual_seed(3)
    for dtype in (torch.float32, torch.bfloat16):
        a = torch.randn(70, 130, device="cuda", generator=g).to(dtype)
        b = torch.randn(130, 50, device="cuda", generator=g).to(dtype)
        assert_close(C.matmul(a, b).float(), a.float() @ b.float(), dtype, f"matmul {dtype}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", [
    (1, 4096, 1024),      # one row: tile width 64 + cluster split-K
    (16, 24, 64),         # N < 64: one 64-wide tile, columns masked
    (64, 4096, 1024),     # the single-linear workload as a matmul
    (300, 1000, 520),     # ragged M, N not a multiple of 64, K not a multiple of 64
    (512, 3584, 3584),    # 7B-width square-ish: tile width 256
    (4096, 2048, 1024),   # many tiles: persistent double-buffered kernel
])
def test_matmul_tcgen05_shapes(m, n, k, dtype):
    """bf16/f16 matmul with B [K, N] row-major (MN-major on the tensor core)
    against an fp64 product of the same rounded inputs."""
    import dli_sm100 as C

    g = torch.Generator(device="cuda").manual_seed(m + 5 * n + 7 * k)
    a = torch.randn(m, k, device="cuda", generator=g).to(dtype)
    b = (torch.randn(k, n, device="cuda", generator=g) * 0.05).to(dtype)
    y = C.matmul(a, b)
    assert y.dtype == dtype
    assert_close(y.float(), a.double() @ b.double(), dtype, f"matmul {dtype} {m}x{n}x{k}")
    assert torch.equal(y, C.matmul(a, b))  # deterministic (cluster split-K reduces in rank order)


ALEXNET_CONVS = [  # (C, H, OC) at k3 s1 p1
    (3, 32, 64), (64, 16, 192), (192, 8, 384), (384, 8, 256), (256, 8, 256)]


@pytest.mark.parametrize("n,c,h,w,oc,stride,pad", [(2, 3, 32, 32, 64, 1, 1), (1, 5, 17, 23, 20, 2, 1),
                                                    (3, 9, 15, 15, 17, 1, 0), (1, 64, 16, 16, 192, 2, 2)])
def test_conv2d_fp32_3x3_tiled(n, c, h, w, oc, stride, pad):
    """The tiled fp32 3x3 kernel at ragged sizes, both strides, channel counts
    not multiples of its 8/16 blocks: rel-err <= 1e-4 against float64."""
    import dli_sm100 as C

    g = torch.Generator(device="cuda").manual_seed(n + c + h + oc)
    x = torch.randn(n, c, h, w, device="cuda", generator=g)
    wt = torch.randn(oc, c, 3, 3, device="cuda", generator=g) * 0.05
    b = torch.randn(oc, device="cuda", generator=g) * 0.05
    y = C.conv2d(x, wt, b, (stride, stride), (pad, pad))
    ref = torch.nn.functional.conv2d(x.double(), wt.double(), b.double(), stride=stride, padding=pad)
    assert_close(y, ref, torch.float32, f"conv fp32 {c}->{oc} s{stride} p{pad}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32], ids=["f16", "bf16", "f32"])
@pytest.mark.parametrize("c,h,oc", ALEXNET_CONVS)
def test_conv2d_alexnet_shapes(c, h, oc, dtype):
    import dli_sm100 as C

    g = torch.Generator().manual_seed(c + h + oc)
    x = torch.randn(2, c, h, h, generator=g)
    w = torch.randn(oc, c, 3, 3, generator=g) * 0.02
    b = torch.randn(oc, generator=g) * 0.02
    xd, wd, bd = (t.to(dtype) for t in (x, w, b))
    y = C.conv2d(xd.cuda(), wd.cuda(), bd.cuda(), (1, 1), (1, 1))
    ref = torch.nn.functional.conv2d(xd.double(), wd.double(), bd.double(), padding=1)
    assert_close(y.float(), ref, dtype, f"conv {c}->{oc} @{h}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("n,c,h,w,oc,kh,kw,stride,pad", [
    (4, 64, 20, 20, 96, 1, 1, (1, 1), (0, 0)),     # 1x1: the gather is a plain copy
    (2, 16, 33, 31, 40, 5, 5, (1, 1), (2, 2)),     # 5x5, odd sizes, K = 400 (two k blocks, zero tail)
    (2, 3, 64, 64, 64, 7, 7, (2, 2), (3, 3)),      # 7x7 stride 2 stem, K = 147 (weight repacked to 152)
    (8, 128, 14, 14, 256, 3, 3, (2, 2), (0, 0)),   # stride 2, no padding, split-K plan
    (1, 32, 9, 40, 48, 3, 1, (1, 2), (1, 0)),      # non-square kernel and strides
])
def test_conv2d_implicit_gemm_shapes(n, c, h, w, oc, kh, kw, stride, pad, dtype):
    """bf16/f16 conv2d on the implicit-GEMM tcgen05 kernel (patches gathered into
    shared memory: kernel sizes, strides, padding, K tails and repacked weights)
    against an fp64 convolution of the same rounded inputs."""
    import dli_sm100 as C

    g = torch.Generator().manual_seed(n + c + h + oc + kh)
    x = torch.randn(n, c, h, w, generator=g).to(dtype)
    wt = (torch.randn(oc, c, kh, kw, generator=g) * 0.05).to(dtype)
    b = (torch.randn(oc, generator=g) * 0.05).to(dtype)
    y = C.conv2d(x.cuda(), wt.cuda(), b.cuda(), stride, pad)
    C.check_device_error()
    ref = torch.nn.functional.conv2d(x.double(), wt.double(), b.double(), stride=stride, padding=pad)
    assert_close(y.float(), ref, dtype, f"conv {c}->{oc} k{kh}x{kw} s{stride} p{pad}")


# ---- attention ----------------------------------------------------------------------

@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("b,hq,hkv,sq,sk,d,causal", [
    (2, 14, 2, 300, 300, 64, True), (1, 28, 4, 512, 512, 128, True), (1, 2, 2, 65, 130, 128, False),
    (1, 8, 1, 5, 77, 128, True), (2, 7, 1, 1, 513, 64, True), (1, 4, 4, 100, 100, 128, False)])
def test_attention_dense(b, hq, hkv, sq, sk, d, causal, dtype):
    import dli_sm100 as C

    g = torch.Generator(device="cuda").manual_seed(sq + sk + d)
    q = torch.randn(b, hq, sq, d, device="cuda", generator=g).to(dtype)
    k = torch.randn(b, hkv, sk, d, device="cuda", generator=g).to(dtype)
    v = torch.randn(b, hkv, sk, d, device="cuda", generator=g).to(dtype)
    out = C.attention(q, k, v, causal=causal)
    ref = torch.from_numpy(O.attention(q.double().cpu().numpy(), k.double().cpu().numpy(),
                                       v.double().cpu().numpy(), causal))
    assert_close(out.float(), ref, dtype, "attention")


@pytest.mark.parametrize("b,hq,hkv,sq,sk,d,causal", [
    (1, 1, 1, 1, 2048, 128, True), (1, 1, 1, 1, 517, 64, True), (2, 4, 4, 128, 128, 128, True),
    (1, 6, 2, 77, 300, 64, False), (3, 8, 1, 33, 33, 128, True), (2, 2, 2, 5, 1000, 128, True),
    (1, 4, 2, 200, 260, 128, True), (2, 3, 1, 150, 150, 64, True)])
def test_attention_fp32_tiles(b, hq, hkv, sq, sk, d, causal):
    """The fp32 attention kernel (64-row tiles, split-KV merged in a cluster for
    decode-sized rows) at the reference's dtype: rel-err <= 1e-4 against the oracle."""
    import dli_sm100 as C

    g = torch.Generator(device="cuda").manual_seed(sq * 5 + sk + d)
    q = torch.randn(b, hq, sq, d, device="cuda", generator=g)
    k = torch.randn(b, hkv, sk, d, device="cuda", generator=g)
    v = torch.randn(b, hkv, sk, d, device="cuda", generator=g)
    out = C.attention(q, k, v, causal=causal)
    ref = torch.from_numpy(O.attention(q.double().cpu().numpy(), k.double().cpu().numpy(),
                                       v.double().cpu().numpy(), causal))
    assert_close(out, ref, torch.float32, "attention fp32")


def test_attention_kvcache_fp32_positions():
    import dli_sm100 as C

    b, s, hq, hkv, d, cap = 3, 3, 4, 2, 128, 700
    positions = [0, 250, 696]
    g = torch.Generator(device="cuda").manual_seed(8)
    q = torch.randn(b, s, hq, d, device="cuda", generator=g)
    ck = torch.randn(b, hkv, cap, d, device="cuda", generator=g)
    cv = torch.randn(b, hkv, cap, d, device="cuda", generator=g)
    for i, p in enumerate(positions):  # stale rows past each sequence must not reach the output
        ck[i, :, p + s:] = float("nan")
        cv[i, :, p + s:] = float("nan")
    out = C.attention_kvcache(q, ck, cv, torch.tensor(positions, device="cuda"))
    assert torch.isfinite(out).all()
    assert_close(out, _cache_reference(q, ck, cv, positions), torch.float32, "attention_kvcache fp32")


def _cache_reference(q_bshd, ck, cv, positions):
    """Oracle over a cache: sequence b sees keys [0, positions[b] + S) bottom-right causal."""
    outs = []
    b, s, hq, d = q_bshd.shape
    for i in range(b):
        n = int(positions[i]) + s
        q = q_bshd[i:i + 1].permute(0, 2, 1, 3).double().cpu().numpy()
        k = ck[i:i + 1, :, :n].double().cpu().numpy()
        v = cv[i:i + 1, :, :n].double().cpu().numpy()
        outs.append(torch.from_numpy(O.attention(q, k, v, causal=True)).permute(0, 2, 1, 3))
    return torch.cat(outs, 0)


_RAG32 = [(i * 997) % 2559 for i in range(32)]  # ragged cache positions, 0 and near-capacity included


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("b,s,hq,hkv,d,cap,positions", [
    (4, 1, 28, 4, 128, 2560, [100, 513, 2000, 0]),
    (8, 1, 14, 2, 64, 768, [512, 600, 700, 767 - 1, 3, 64, 65, 128]),
    (2, 3, 64, 8, 128, 1024, [10, 500]),
    (2, 77, 14, 2, 64, 512, [0, 40]),
    # one token, <= 8 query rows per KV head: the cluster-merged decode kernel at the
    # 7B shape and its TP 2 / TP 4 shards, the 72B group of 8, a group of 6, 2 tokens x 4
    (32, 1, 28, 4, 128, 2560, _RAG32), (32, 1, 14, 2, 128, 2560, _RAG32), (32, 1, 7, 1, 128, 2560, _RAG32),
    (16, 1, 64, 8, 128, 4608, [(i * 1237) % 4607 for i in range(16)]), (3, 1, 12, 2, 64, 256, [0, 1, 254]),
    (4, 2, 16, 4, 128, 512, [0, 63, 64, 509]), (1, 1, 8, 1, 128, 64, [0]),
])
def test_attention_kvcache(b, s, hq, hkv, d, cap, positions, dtype):
    import dli_sm100 as C

    g = torch.Generator(device="cuda").manual_seed(b * s + cap)
    q = torch.randn(b, s, hq, d, device="cuda", generator=g).to(dtype)
    ck = torch.randn(b, hkv, cap, d, device="cuda", generator=g).to(dtype)
    cv = torch.randn(b, hkv, cap, d, device="cuda", generator=g).to(dtype)
    pos = torch.tensor(positions, dtype=torch.int64, device="cuda")
    out = C.attention_kvcache(q, ck, cv, pos)
    ref = _cache_reference(q, ck, cv, positions)
    assert_close(out.float(), ref, dtype, "attention_kvcache")


_DECODE_CHILD = r"""
import sys, torch
import dli_sm100 as C
cases = [(32, 1, 28, 4, 128, 2560, [(i * 997) % 2559 for i in range(32)]),
         (32, 1, 7, 1, 128, 2560, [(i * 997) % 2559 for i in range(32)]),
         (16, 1, 64, 8, 128, 4608, [(i * 1237) % 4607 for i in range(16)]),
         (3, 1, 12, 2, 64, 256, [0, 1, 254]), (4, 2, 16, 4, 128, 512, [0, 63, 64, 509]),
         (2, 1, 8, 1, 128, 200, [130, 5])]  # capacity not a multiple of the 64-key block
outs = []
for dtype in (torch.bfloat16, torch.float16):
    for (b, s, hq, hkv, d, cap, positions) in cases:
        g = torch.Generator(device="cuda").manual_seed(b * s + cap)
        q = torch.randn(b, s, hq, d, device="cuda", generator=g).to(dtype)
        ck = torch.randn(b, hkv, cap, d, device="cuda", generator=g).to(dtype)
        cv = torch.randn(b, hkv, cap, d, device="cuda", generator=g).to(dtype)
        for i, p in enumerate(positions):  # rows past each sequence: NaN
            ck[i, :, p + s:] = float("nan")
            cv[i, :, p + s:] = float("nan")
        out = C.attention_kvcache(q, ck, cv, torch.tensor(positions, dtype=torch.int64, device="cuda"))
        assert torch.isfinite(out.float()).all()
        outs.append(out.cpu())
C.check_device_error()
torch.save(outs, sys.argv[1])
print("decode child ok")
"""


def test_decode_cluster_tma_matches_cp_async(tmp_path):
    """The cluster decode kernel with K/V by TMA and mbarrier stages
    (DLI_SM100_ATTN_DECODE_TMA=1) against the cp.async form (=0, the default):
    the same arithmetic in the same order, so the outputs are bit-identical,
    with NaN in every cache row past a sequence (the TMA copy is not clipped to
    the sequence; the kernel zeroes those V rows). Knobs are read once per
    process, so each form runs in a child."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    import dli_sm100 as C

    here = Path(__file__).resolve().parent
    res = {}
    for tma in ("1", "0"):
        env = dict(os.environ, DLI_SM100_ATTN_DECODE_TMA=tma)
        env["PYTHONPATH"] = os.pathsep.join([str(here), str(here.parent), str(Path(C.__file__).resolve().parents[1]),
                                             env.get("PYTHONPATH", "")])
        out = tmp_path / f"tma{tma}.pt"
        r = subprocess.run([sys.executable, "-c", _DECODE_CHILD, str(out)], env=env, capture_output=True, text=True,
                           timeout=600)
        assert r.returncode == 0 and "decode child ok" in r.stdout, (r.stdout[-2000:], r.stderr[-3000:])
        res[tma] = torch.load(out)
    for a, b in zip(res["1"], res["0"]):
        assert torch.equal(a, b)


def test_qkv_rotary_cache_matches_oracle():
    import dli_sm100 as C

    b, s, hq, hkv, d, cap = 2, 5, 4, 2, 64, 32
    g = torch.Generator().manual_seed(11)
    qkv = torch.randn(b * s, (hq + 2 * hkv) * d, generator=g).to(torch.bfloat16)
    ang = torch.randn(64, d // 2, generator=g)
    cos, sin = torch.cos(ang), torch.sin(ang)
    positions = torch.tensor([3, 20])
    ck = torch.zeros(b, hkv, cap, d, dtype=torch.bfloat16, device="cuda")
    cv = torch.zeros_like(ck)
    qo = C.qkv_rotary_cache(qkv.cuda(), cos.cuda(), sin.cuda(), positions.cuda(), ck, cv, b, s, hq,
                            hkv, d)
    x = qkv.double().view(b, s, hq + 2 * hkv, d)
    q = x[:, :, :hq].permute(0, 2, 1, 3).numpy()
    k = x[:, :, hq:hq + hkv].permute(0, 2, 1, 3).numpy()
    v = x[:, :, hq + hkv:].permute(0, 2, 1, 3).numpy()
    rq, rk = O.rotary(q, k, cos.numpy(), sin.numpy(), positions=positions.numpy())
    assert_close(qo.float(), torch.from_numpy(rq).permute(0, 2, 1, 3), torch.bfloat16, "q_out")
    for i in range(b):
        p = int(positions[i])
        assert_close(ck[i, :, p:p + s].float(), rk[i], torch.bfloat16, "cache k")
        assert_close(cv[i, :, p:p + s].float(), v[i], torch.bfloat16, "cache v")
    # rows outside [p, p+s) stay untouched
    assert ck[0, :, :3].abs().sum().item() == 0 and ck[0, :, 8:].abs().sum().item() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("b,s,hq,hkv,d,k,pairs", [
    (32, 1, 28, 4, 128, 3584, 64),   # 7B decode
    (32, 1, 7, 1, 128, 3584, 64),    # 7B decode, TP 4 shard
    (8, 1, 14, 2, 64, 896, 32),      # 0.5B decode (a 128-row tile spans two heads)
    (64, 1, 8, 1, 128, 8192, 64),    # 72B decode, TP 8 shard
    (16, 2, 28, 4, 128, 3584, 48),   # two tokens per sequence, partial rotary (48 of 64 pairs)
])
def test_linear_qkv_rotary_cache_matches_two_step(b, s, hq, hkv, d, k, pairs, dtype):
    """The q|k|v projection with rotary + cache write in its GEMM epilogue against
    linear followed by qkv_rotary_cache: q, and the cache rows of every
    token, bit-identical; every other cache row untouched."""
    import dli_sm100 as C

    cap = 96
    g = torch.Generator(device="cuda").manual_seed(b + s + hq + k)
    x = torch.randn(b * s, k, device="cuda", generator=g).to(dtype)
    w = (torch.randn((hq + 2 * hkv) * d, k, device="cuda", generator=g) * 0.02).to(dtype)
    bias = (torch.randn((hq + 2 * hkv) * d, device="cuda", generator=g) * 0.02).to(dtype)
    ang = torch.randn(cap, pairs, device="cuda", generator=g)
    cos, sin = torch.cos(ang).contiguous(), torch.sin(ang).contiguous()
    positions = torch.randint(0, cap - s + 1, (b,), device="cuda", generator=g)
    fill = torch.randn(b, hkv, cap, d, device="cuda", generator=g).to(dtype)
    ck1, cv1, ck2, cv2 = fill.clone(), (fill * 2).clone(), fill.clone(), (fill * 2).clone()
    q1 = C.linear_qkv_rotary_cache(x, w, bias, cos, sin, positions, ck1, cv1, b, s, hq, hkv, d)
    assert q1 is not None, "decode shape expected on the fused path"
    qkv = C.linear(x, w, bias)
    q2 = C.qkv_rotary_cache(qkv, cos, sin, positions, ck2, cv2, b, s, hq, hkv, d)
    C.check_device_error()
    assert torch.equal(q1, q2)
    assert torch.equal(ck1, ck2) and torch.equal(cv1, cv2)
    assert not torch.equal(ck1, fill)  # the token rows were written


def test_linear_qkv_rotary_cache_declines_prefill():
    import dli_sm100 as C

    b, s, hq, hkv, d, k, cap = 2, 300, 4, 2, 64, 256, 512
    x = torch.randn(b * s, k, device="cuda").bfloat16()
    w = (torch.randn((hq + 2 * hkv) * d, k, device="cuda") * 0.02).bfloat16()
    bias = torch.zeros((hq + 2 * hkv) * d, device="cuda").bfloat16()
    cos = torch.ones(cap, d // 2, device="cuda")
    ck = torch.zeros(b, hkv, cap, d, device="cuda").bfloat16()
    assert C.linear_qkv_rotary_cache(x, w, bias, cos, cos, torch.zeros(b, dtype=torch.int64, device="cuda"),
                                     ck, ck.clone(), b, s, hq, hkv, d) is None


def test_kv_append_is_a_sequence_concat():
    import dli_sm100 as C

    g = torch.Generator().manual_seed(5)
    old = torch.randn(2, 3, 4, 8, generator=g)
    new = torch.randn(2, 3, 2, 8, generator=g)
    ck = torch.zeros(2, 3, 10, 8, device="cuda")
    cv = torch.zeros_like(ck)
    C.kv_append(ck, cv, old.cuda(), (old * 2).cuda(), 0)
    C.kv_append(ck, cv, new.cuda(), (new * 2).cuda(), 4)
    torch.testing.assert_close(ck[:, :, :6].cpu(), torch.cat([old, new], 2), rtol=0, atol=0)
    torch.testing.assert_close(cv[:, :, :6].cpu(), torch.cat([old, new], 2) * 2, rtol=0, atol=0)
    with pytest.raises(ValueError):
        C.kv_append(ck, cv, new.cuda(), new.cuda(), 9)


# ---- norms / elementwise --------------------------------------------------------------

@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
@pytest.mark.parametrize("rows,hidden", [(8, 896), (32, 3584), (64, 8192), (5, 100)])
def test_rms_norm_and_fused_residual(rows, hidden, dtype):
    import dli_sm100 as C

    g = torch.Generator(device="cuda").manual_seed(rows + hidden)
    r = torch.randn(rows, hidden, device="cuda", generator=g).to(dtype)
    dlt = torch.randn(rows, hidden, device="cuda", generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(hidden, device="cuda", generator=g)).to(dtype)
    assert_close(C.rms_norm(r, w).float(), O.rms_norm(r.double().cpu().numpy(), w.double().cpu().numpy()),
                 dtype, "rms_norm")
    normed, resid = C.add_rms_norm(r, dlt, w)
    ref_n, ref_r = O.add_rms_norm(r.double().cpu().numpy(), dlt.double().cpu().numpy(),
                                  w.double().cpu().numpy())
    assert_close(resid.float(), ref_r, dtype, "residual")
    assert_close(normed.float(), ref_n, dtype, "normed")
    # in-place residual update (residual_out aliases residual)
    r2 = r.clone()
    normed2, _ = C.add_rms_norm(r2, dlt, w, residual_out=r2)
    assert torch.equal(normed2, normed) and torch.equal(r2, resid)


def test_add_rms_norm_fp32_residual():
    """Residual stream in float32 around bf16 tensors: residual_out = residual +
    delta exactly in fp32; normed (bf16) against the float64 oracle. Rows of
    <= 8192 (multiples of 8) run the register-resident kernel, the others the
    two-pass one."""
    import dli_sm100 as C

    g = torch.Generator(device="cuda").manual_seed(9)
    for rows, hidden in ((5, 896), (33, 3584), (3, 100), (2, 8192), (2, 8200)):
        r = torch.randn(rows, hidden, device="cuda", generator=g) * 3
        dlt = torch.randn(rows, hidden, device="cuda", generator=g).to(torch.bfloat16)
        w = (1 + 0.1 * torch.randn(hidden, device="cuda", generator=g)).to(torch.bfloat16)
        normed, resid = C.add_rms_norm(r, dlt, w)
        assert resid.dtype == torch.float32 and normed.dtype == torch.bfloat16
        assert torch.equal(resid, r + dlt.float())
        ref_n, _ = O.add_rms_norm(r.double().cpu().numpy(), dlt.double().cpu().numpy(), w.double().cpu().numpy())
        assert_close(normed.float(), ref_n, torch.bfloat16, "add_rms_norm fp32 residual")
        r2 = r.clone()
        normed2, _ = C.add_rms_norm(r2, dlt, w, residual_out=r2)  # in place
        assert torch.equal(normed2, normed) and torch.equal(r2, resid)


@pytest.mark.parametrize("rows,width,dtype", [(32, 152064, torch.float32), (3, 50001, torch.bfloat16),
                                              (37, 16384, torch.float32), (40, 20000, torch.float32)])
def test_argmax_long_rows(rows, width, dtype):
    """Greedy-decoding argmax over a vocabulary: few long rows split over a
    cluster of CTAs per row (the first three shapes; 40 rows take the one-CTA
    form), against torch.argmax, with the row maximum planted twice (the lowest
    index wins) on both sides of a chunk boundary and at the last column."""
    import dli_sm100 as C

    g = torch.Generator(device="cuda").manual_seed(rows + width)
    x = torch.randn(rows, width, device="cuda", generator=g).to(dtype)
    chunk = -(-(-(-width // 8)) // 8) * 8
    x[0, chunk - 1] = 100.0
    x[0, chunk + 5] = 100.0
    x[1, width - 1] = 50.0
    x[2, 3] = 7.0
    x[2, width - 2] = 7.0
    assert torch.equal(C.argmax(x), torch.argmax(x.float(), -1))


def test_silu_mul_embedding_argmax_select_cast():
    import dli_sm100 as C

    g = torch.Generator(device="cuda").manual_seed(9)
    gu = torch.randn(6, 2 * 4864, device="cuda", generator=g).to(torch.bfloat16)
    assert_close(C.silu_mul(gu).float(), O.silu_mul(gu.double().cpu().numpy()), torch.bfloat16, "silu_mul")
    table = torch.randn(1000, 896, device="cuda", generator=g).to(torch.bfloat16)
    ids = torch.randint(0, 1000, (3, 7), device="cuda", generator=g)
    assert torch.equal(C.embedding(ids, table), table[ids])
    assert torch.equal(C.embedding(ids.int(), table), table[ids])
    logits = torch.randn(5, 152064, device="cuda", generator=g).to(torch.bfloat16)
    logits[2, 17] = 100.0
    logits[2, 18] = 100.0  # tie -> lowest index
    am = C.argmax(logits)
    assert am[2].item() == 17
    assert torch.equal(am, torch.from_numpy(O.argmax(logits.float().cpu().numpy())).cuda())
    x = torch.randn(4, 9, 33, device="cuda", generator=g)
    assert torch.equal(C.select_token(x, 8), x[:, 8])
    assert torch.equal(C.cast(x, torch.bfloat16), x.to(torch.bfloat16))
    assert torch.equal(C.cast(x.half(), torch.float32), x.half().float())


def test_device_error_word_reports_bad_embedding_id_and_clears():
    import dli_sm100 as C

    table = torch.randn(10, 8, device="cuda")
    ids = torch.tensor([1, 12, 3], device="cuda")
    out = C.embedding(ids, table)
    with pytest.raises(RuntimeError, match="embedding id"):
        C.check_device_error()
    assert out[1].abs().sum().item() == 0
    C.check_device_error()  # cleared


def test_invalid_arguments_raise_value_error():
    import dli_sm100 as C

    x = torch.randn(4, 8, device="cuda")
    w = torch.randn(3, 8, device="cuda")
    with pytest.raises(ValueError):
        C.check(C.lib().dli_sm100_linear(C._ptr(x), C._ptr(w), None, C._ptr(x), 4, -1, 8, 0, None, 0,
                                         C._stream()))
    with pytest.raises(ValueError):
        C.attention(torch.randn(1, 3, 2, 8, device="cuda"), torch.randn(1, 2, 2, 8, device="cuda"),
                    torch.randn(1, 2, 2, 8, device="cuda"))
    assert math.isfinite(1.0)
