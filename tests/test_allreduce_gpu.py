"""GPU tests of dli_sm100_allreduce_add_rms_norm, the tensor-parallel
all-reduce fused with the residual add and RMSNorm, on ONE device: every rank
of the group runs in one cooperative launch (ranks_in_launch = tp) over
exchange buffers that all live on this device, so the push / flag / bounded
wait protocol runs exactly as across GPUs, without two launches waiting on
each other.

Expected values: the rank-ordered fp32 sum of the partials rounded to the
dtype (what an all_reduce returns), fed to dli_sm100_add_rms_norm. The fused
kernel's residual output must match that bit for bit; its normed output may
differ by one rounding step (the sum of squares is reduced over a different
thread layout), so it is held to 1e-2 relative + absolute elementwise. Every
rank must hold the same bits. The float64 oracle (oracle/ops.py add_rms_norm
over the summed partials) bounds both at bf16 tolerance.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import dli_sm100 as C
from oracle import ops as O

pytestmark = pytest.mark.gpu


def _expected(residual, delta, w, eps):
    acc = delta[0].float()
    for k in range(1, delta.shape[0]):
        acc = acc + delta[k].float()
    summed = acc.to(delta.dtype)
    return C.add_rms_norm(residual[0], summed, w, eps)


def _case(tp, rows, hidden, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    residual = torch.randn(rows, hidden, device="cuda", generator=g).to(dtype)
    residual = residual.unsqueeze(0).expand(tp, rows, hidden).contiguous()  # replicated on every rank
    delta = (torch.randn(tp, rows, hidden, device="cuda", generator=g) * 0.5).to(dtype)
    w = (1 + 0.1 * torch.randn(hidden, device="cuda", generator=g)).to(dtype)
    return residual, delta, w


@pytest.mark.parametrize("tp", [2, 4, 8])
@pytest.mark.parametrize("rows,hidden", [(1, 896), (32, 3584), (64, 8192), (7, 1024)])
def test_fused_allreduce_matches_sum_then_add_rms_norm(tp, rows, hidden):
    # all ranks' CTAs (rows x tp) must be resident in one launch on this device
    rows = min(rows, 256 // tp)
    group = C.ExchangeGroup(tp, max_rows=64, row_elems=8192, dtype=torch.bfloat16)
    for seed in range(3):  # consecutive calls: epochs advance, slots alternate
        residual, delta, w = _case(tp, rows, hidden, torch.bfloat16, seed)
        normed, res_out = group.allreduce_add_rms_norm(residual, delta, w, eps=1e-6)
        ref_n, ref_r = _expected(residual, delta, w, 1e-6)
        torch.cuda.synchronize()
        for k in range(tp):
            assert torch.equal(res_out[k], ref_r), (seed, k)
            assert torch.equal(normed[k], normed[0]), (seed, k)
        torch.testing.assert_close(normed[0].float(), ref_n.float(), rtol=1e-2, atol=1e-2)
    # float64 oracle on the last case
    d64 = delta.double().cpu().numpy().sum(0)
    on, orr = O.add_rms_norm(residual[0].double().cpu().numpy(), d64, w.double().cpu().numpy(), 1e-6)
    rel = np.linalg.norm(normed[0].double().cpu().numpy() - on) / np.linalg.norm(on)
    assert rel < 1.5e-2, rel
    C.check_device_error()


@pytest.mark.parametrize("tp", [2, 4])
def test_fp32_residual_stream(tp):
    """bf16 partials around a float32 residual (the exported graphs' residual
    stream): residual_out = residual + bf16(sum of partials) in fp32, bit for bit
    as dli_sm100_add_rms_norm_ex computes it, identical on every rank."""
    rows, hidden = 32, 3584
    group = C.ExchangeGroup(tp, max_rows=64, row_elems=4096, dtype=torch.bfloat16)
    for seed in range(2):
        residual, delta, w = _case(tp, rows, hidden, torch.bfloat16, 20 + seed)
        # an fp32 residual (below bf16 resolution), replicated on every rank
        noise = 1e-3 * torch.randn(rows, hidden, device="cuda")
        residual = (residual[0].float() + noise).unsqueeze(0).expand(tp, rows, hidden).contiguous()
        normed, res_out = group.allreduce_add_rms_norm(residual, delta, w, eps=1e-6)
        ref_n, ref_r = _expected(residual, delta, w, 1e-6)
        torch.cuda.synchronize()
        assert res_out.dtype == torch.float32 and normed.dtype == torch.bfloat16
        for k in range(tp):
            assert torch.equal(res_out[k], ref_r), (seed, k)
            assert torch.equal(normed[k], normed[0]), (seed, k)
        torch.testing.assert_close(normed[0].float(), ref_n.float(), rtol=1e-2, atol=1e-2)
    C.check_device_error()


def test_fp32_and_changing_row_counts():
    tp = 4
    group = C.ExchangeGroup(tp, max_rows=128, row_elems=4096, dtype=torch.float32)
    for seed, rows in enumerate([128, 3, 64, 128, 1]):
        residual, delta, w = _case(tp, rows, 4096, torch.float32, 10 + seed)
        normed, res_out = group.allreduce_add_rms_norm(residual, delta, w, eps=1e-5)
        ref_n, ref_r = _expected(residual, delta, w, 1e-5)
        torch.cuda.synchronize()
        for k in range(tp):
            assert torch.equal(res_out[k], ref_r), (rows, k)
            assert torch.equal(normed[k], normed[0]), (rows, k)
        torch.testing.assert_close(normed[0], ref_n, rtol=1e-5, atol=1e-5)
    C.check_device_error()


def test_missing_peer_times_out_with_an_error_status():
    """Only rank 0 of a two-rank group is launched: its wait for rank 1's rows
    (a flag nothing sets) must run out after the stated limit and report through
    the device error word; the context stays usable."""
    group = C.ExchangeGroup(2, max_rows=8, row_elems=1024, dtype=torch.bfloat16)
    residual, delta, w = _case(2, 4, 1024, torch.bfloat16, 0)
    group.allreduce_add_rms_norm(residual, delta, w, timeout_ns=50_000_000, ranks=1)
    with pytest.raises(RuntimeError, match="exchange"):
        C.check_device_error()
    # the device still works and the error word was cleared
    x = torch.ones(4, 1024, device="cuda", dtype=torch.bfloat16)
    C.rms_norm(x, torch.ones(1024, device="cuda", dtype=torch.bfloat16))
    C.check_device_error()


def test_rejects_shapes_beyond_the_exchange_buffer():
    group = C.ExchangeGroup(2, max_rows=8, row_elems=1024, dtype=torch.bfloat16)
    residual, delta, w = _case(2, 16, 1024, torch.bfloat16, 0)
    with pytest.raises(RuntimeError, match="exceed"):
        group.allreduce_add_rms_norm(residual, delta, w)


@pytest.mark.parametrize("tp", [2, 4, 8])
@pytest.mark.parametrize("rows,width", [(32, 152064 // 4), (8, 151936 // 8), (1, 1000), (64, 4096)])
def test_vocab_parallel_argmax_matches_argmax_over_the_whole_row(tp, rows, width):
    """dli_sm100_allgather_argmax over a vocabulary split into tp slices equals
    dli_sm100_argmax over the concatenated row, on every rank, on consecutive
    calls (epochs advance) that also alternate with all-reduce calls on the same
    buffers; planted ties across slices must go to the lowest id."""
    rows = min(rows, 256 // tp)
    group = C.ExchangeGroup(tp, max_rows=64, row_elems=4096, dtype=torch.bfloat16)
    g = torch.Generator(device="cuda").manual_seed(tp * 1000 + rows)
    for step in range(3):
        logits = torch.randn(tp, rows, width, device="cuda", generator=g).to(torch.bfloat16)
        if rows > 1:  # the same maximum in the last slice and the first: the first slice's id wins
            logits[:, 1, :] = -1.0
            logits[tp - 1, 1, 5] = 7.0
            logits[0, 1, 3] = 7.0
        got = group.allgather_argmax(logits)
        full = logits.permute(1, 0, 2).reshape(rows, tp * width).contiguous()
        ref = C.argmax(full)
        torch.cuda.synchronize()
        for k in range(tp):
            assert torch.equal(got[k], ref), (step, k)
        if rows > 1:
            assert int(got[0, 1]) == 3
        # an all-reduce on the same buffers between the argmax calls
        residual, delta, w = _case(tp, min(rows, 4), 1024, torch.bfloat16, step)
        group.allreduce_add_rms_norm(residual, delta, w)
    C.check_device_error()


def test_vocab_parallel_argmax_missing_peer_times_out():
    group = C.ExchangeGroup(2, max_rows=8, row_elems=1024, dtype=torch.bfloat16)
    logits = torch.randn(2, 4, 512, device="cuda").to(torch.bfloat16)
    group.allgather_argmax(logits, timeout_ns=50_000_000, ranks=1)
    with pytest.raises(RuntimeError, match="exchange"):
        C.check_device_error()


@pytest.mark.parametrize("tp,rows,n,k", [
    (2, 32, 3584, 1792),    # 7B o_proj at TP 2, the benchmark's 32 sequences
    (4, 16, 3584, 4736),    # 7B down_proj at TP 4, 16 sequences per data-parallel group
    (8, 16, 8192, 1024),    # 72B o_proj at TP 8
    (4, 7, 3584, 896),      # ragged row count
])
@pytest.mark.parametrize("res32", [True, False], ids=["res32", "res16"])
def test_gemm_pushed_exchange_matches_two_kernel_path(tp, rows, n, k, res32):
    """A row-split projection whose GEMM pushes its partial rows straight into
    the exchange buffers from its split-K epilogue
    (dli_sm100_linear_exchange_push), then the sum + residual add + RMSNorm
    (dli_sm100_exchange_add_rms_norm_ex), against linear + the fused all-reduce
    of the partial outputs: bit-identical on every rank, over consecutive calls
    (epochs advance, slots alternate)."""
    dtype = torch.bfloat16
    fused = C.ExchangeGroup(tp, max_rows=64, row_elems=8192, dtype=dtype)
    plain = C.ExchangeGroup(tp, max_rows=64, row_elems=8192, dtype=dtype)
    g = torch.Generator(device="cuda").manual_seed(tp * 7 + rows + n + k)
    w = (torch.randn(tp, n, k, device="cuda", generator=g) * 0.02).to(dtype)
    norm_w = (1 + 0.1 * torch.randn(n, device="cuda", generator=g)).to(dtype)
    for step in range(3):
        x = torch.randn(tp, rows, k, device="cuda", generator=g).to(dtype)
        res = torch.randn(rows, n, device="cuda", generator=g).to(torch.float32 if res32 else dtype)
        res = res.unsqueeze(0).expand(tp, rows, n).contiguous()
        got = fused.linear_allreduce_add_rms_norm(x, w, res, norm_w, eps=1e-6)
        assert got is not None, "shape expected on the fused path"
        delta = torch.stack([C.linear(x[r], w[r]) for r in range(tp)])
        ref_n, ref_r = plain.allreduce_add_rms_norm(res, delta, norm_w, eps=1e-6)
        C.check_device_error()
        assert torch.equal(got[0], ref_n), step
        assert torch.equal(got[1], ref_r), step


def test_gemm_pushed_exchange_declines_prefill_rows():
    """More than 128 rows (prefill) is outside the fused path: UNSUPPORTED, nothing launched."""
    group = C.ExchangeGroup(2, max_rows=512, row_elems=3584, dtype=torch.bfloat16)
    x = torch.randn(2, 300, 1792, device="cuda").bfloat16()
    w = (torch.randn(2, 3584, 1792, device="cuda") * 0.02).bfloat16()
    res = torch.randn(2, 300, 3584, device="cuda")
    assert group.linear_allreduce_add_rms_norm(x, w, res, torch.ones(3584, device="cuda").bfloat16()) is None
