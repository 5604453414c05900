"""GPU test of dli_sm100_attention_kvcache_noalloc, the KV-cache attention entry
point for callers that cannot allocate device memory (a fixed memory budget, an
allocator owned by another runtime, or a hot path that must not lock the
allocator). It takes its split-KV scratch from a fixed array inside the library
instead of a caller workspace.

Checked through the C ABI against dli_sm100_attention_kvcache (the entry point
with a caller workspace) on two calls in a row with different inputs, so
leftovers of the first call in the shared array cannot leak into the second,
and against the CPU oracle (float64) at the same shape, with ragged cache
positions, some so short that most key splits of their sequence are empty.
The case decodes two tokens per sequence at the 7B head shape: 2 x 7 query
rows per KV head take the split-KV kernel whose partials need scratch (single
tokens take the cluster kernel, which needs none);
bf16 tolerance as in test_ops_gpu.py (relative Frobenius error <= 1.5e-2; the two
calls run the same kernels, so in practice they agree exactly). The file name
sorts last so a run that stops at the first failure has run everything else.
"""
from __future__ import annotations

import pytest
import torch

import dli_sm100 as C
from oracle import ops as O

pytestmark = pytest.mark.gpu

TOL = 1.5e-2


def _noalloc(q, ck, cv, pos):
    b, s, hq, d = q.shape
    hkv, cap = ck.shape[1], ck.shape[2]
    out = torch.empty_like(q)
    st = C.lib().dli_sm100_attention_kvcache_noalloc(C._ptr(q), C._ptr(ck), C._ptr(cv), C._ptr(pos),
                                                     C._ptr(out), b, s, hq, hkv, cap, d, 0.0, C._dt(q),
                                                     C._stream())
    C.check(st, "attention_kvcache_noalloc")
    return out


def _case(seed, b=32, hq=28, hkv=4, d=128, cap=2560, seq=2):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(b, seq, hq, d, device="cuda", generator=g).to(torch.bfloat16)
    ck = torch.randn(b, hkv, cap, d, device="cuda", generator=g).to(torch.bfloat16)
    cv = torch.randn(b, hkv, cap, d, device="cuda", generator=g).to(torch.bfloat16)
    pos = torch.randint(1, cap - seq, (b,), device="cuda", generator=g)
    return q, ck, cv, pos


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    # the 7B head shape, two tokens: split-KV partials live in the fixed scratch array
    need = C.lib().dli_sm100_attention_kvcache_workspace_size(32, 2, 28, 4, 2560, 128, 2)
    assert 0 < need <= C.lib().dli_sm100_attention_kvcache_noalloc_max_scratch()
    for seed in (1, 2):
        q, ck, cv, pos = _case(seed)
        got = _noalloc(q, ck, cv, pos)
        ref = C.attention_kvcache(q, ck, cv, pos)
        torch.cuda.synchronize()
        err = ((got.float() - ref.float()).norm() / ref.float().norm()).item()
        assert err <= TOL, (seed, err)
    C.check_device_error()


def _oracle(q, ck, cv, positions):
    """float64 oracle over the cache: sequence b sees keys [0, positions[b] + S), bottom-right causal."""
    b, s = q.shape[:2]
    outs = []
    for i in range(b):
        n = int(positions[i]) + s
        qi = q[i:i + 1].permute(0, 2, 1, 3).double().cpu().numpy()
        outs.append(torch.from_numpy(O.attention(qi, ck[i:i + 1, :, :n].double().cpu().numpy(),
                                                 cv[i:i + 1, :, :n].double().cpu().numpy(),
                                                 causal=True)).permute(0, 2, 1, 3))
    return torch.cat(outs, 0)


def test_noalloc_matches_oracle_with_empty_splits():
    short = [0, 1, 3, 7, 15, 63, 64, 65, 127, 200]
    for seed, positions in ((3, short + [(i * 997) % 2557 for i in range(22)]),
                            (4, [(i * 1231) % 2557 for i in range(22)] + short[::-1])):
        q, ck, cv, _ = _case(seed)
        pos = torch.tensor(positions, device="cuda", dtype=torch.int64)
        got = _noalloc(q, ck, cv, pos)
        torch.cuda.synchronize()
        ref = _oracle(q, ck, cv, positions)
        err = ((got.double().cpu() - ref).norm() / ref.norm()).item()
        assert err <= TOL, (seed, err)
        rows = (got.double().cpu() - ref).flatten(2).norm(dim=-1) / ref.flatten(2).norm(dim=-1)
        assert rows.max().item() <= 3 * TOL, (seed, rows.max().item())
    C.check_device_error()


_REJECT = r"""
import sys, torch
import dli_sm100 as C
b, hq, hkv, d, cap = 32, 28, 4, 128, 2560
need = C.lib().dli_sm100_attention_kvcache_workspace_size(b, 2, hq, hkv, cap, d, 2)
assert need > C.lib().dli_sm100_attention_kvcache_noalloc_max_scratch(), need
q = torch.zeros(16, device="cuda", dtype=torch.bfloat16)  # never read: the call is rejected first
st = C.lib().dli_sm100_attention_kvcache_noalloc(C._ptr(q), C._ptr(q), C._ptr(q), C._ptr(q), C._ptr(q),
                                                 b, 2, hq, hkv, cap, d, 0.0, 2, C._stream())
assert st == C.DLI_ERR_WORKSPACE, st
assert "scratch" in C.last_error(), C.last_error()
print("rejected")
"""


def test_noalloc_rejects_shapes_beyond_its_scratch():
    """With the default launch shapes no decode plan needs more than the fixed
    array; a tuning knob that asks for 8x more split-KV CTAs does, and the call
    must then fail cleanly (knobs are read once per process: run in a child)."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    env = dict(os.environ, DLI_SM100_ATTN_WAVES="8")
    env["PYTHONPATH"] = os.pathsep.join([str(Path(C.__file__).resolve().parents[1]),
                                         env.get("PYTHONPATH", "")])
    res = subprocess.run([sys.executable, "-c", _REJECT], env=env, capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0 and "rejected" in res.stdout, res.stderr[-2000:]
