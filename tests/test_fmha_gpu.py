"""GPU parity of the tcgen05 prefill attention kernel (k_fmha.cu): S = Q K^T and
O in tensor memory, K/V tiles by TMA, P written back over S in tensor memory
(default) or through a shared-memory tile (DLI_SM100_ATTN_FMHA_P=0).

Every bf16/f16 prefill with head_dim 64/128 and TMA-compatible strides runs it
(dense `attention` and `attention_kvcache` with several query rows per KV head).
Checked against the float64 oracle at small shapes and against a plain PyTorch
fp32 reference on the GPU at the model shapes (7B: 28/4 heads, D 128; 0.5B:
14/2 heads, D 64), with the bf16/f16 tolerances of test_ops_gpu.py. Cases cover
sequence lengths that are not multiples of the 128-row tile, chunked prefill
(cache positions > 0, bottom-right causal), non-causal attention with fewer
queries than keys, and cache rows past each sequence filled with NaN (they
must not reach the output). A child process with DLI_SM100_ATTN_FMHA=2 proves
the cases ran on this kernel and not on the mma.sync fallback.
"""
from __future__ import annotations

import math
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

import dli_sm100 as C
from oracle import ops as O
from test_ops_gpu import assert_close

pytestmark = pytest.mark.gpu


def torch_cache_attention(q, ck, cv, positions, causal=True):
    """fp32 reference: q [B,S,Hq,D], cache [B,Hkv,cap,D]; sequence b sees keys
    [0, positions[b] + S), bottom-right causal."""
    b, s, hq, d = q.shape
    hkv = ck.shape[1]
    out = torch.empty(b, s, hq, d, dtype=torch.float32, device=q.device)
    for i in range(b):
        n = int(positions[i]) + s
        qi = q[i].float().permute(1, 0, 2)                          # [Hq,S,D]
        ki = ck[i, :, :n].float().repeat_interleave(hq // hkv, 0)   # [Hq,n,D]
        vi = cv[i, :, :n].float().repeat_interleave(hq // hkv, 0)
        sc = qi @ ki.transpose(1, 2) / math.sqrt(d)
        if causal:
            rows = torch.arange(s, device=q.device)[:, None]
            cols = torch.arange(n, device=q.device)[None, :]
            sc = sc.masked_fill(cols > rows + (n - s), float("-inf"))
        out[i] = (torch.softmax(sc, -1) @ vi).permute(1, 0, 2)
    return out


def _cache_case(b, s, hq, hkv, d, cap, positions, dtype, seed, nan_tail=False):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(b, s, hq, d, device="cuda", generator=g).to(dtype)
    ck = torch.randn(b, hkv, cap, d, device="cuda", generator=g).to(dtype)
    cv = torch.randn(b, hkv, cap, d, device="cuda", generator=g).to(dtype)
    if nan_tail:
        for i, p in enumerate(positions):
            ck[i, :, p + s:] = float("nan")
            cv[i, :, p + s:] = float("nan")
    pos = torch.tensor(positions, dtype=torch.int64, device="cuda")
    return q, ck, cv, pos


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("b,s,hq,hkv,d,cap,positions", [
    (2, 129, 8, 2, 128, 512, [0, 200]),        # one row past a tile, chunked second sequence
    (1, 127, 4, 4, 64, 256, [0]),              # one row short of a tile, MHA
    (3, 40, 7, 1, 128, 400, [0, 1, 300]),      # group of 7 (7B TP 4 shard), short prompt
])
def test_fmha_kvcache_small_against_oracle(b, s, hq, hkv, d, cap, positions, dtype):
    q, ck, cv, pos = _cache_case(b, s, hq, hkv, d, cap, positions, dtype, seed=b * s + d)
    out = C.attention_kvcache(q, ck, cv, pos)
    ref = []
    for i in range(b):
        n = positions[i] + s
        qi = q[i:i + 1].permute(0, 2, 1, 3).double().cpu().numpy()
        ref.append(torch.from_numpy(O.attention(qi, ck[i:i + 1, :, :n].double().cpu().numpy(),
                                                cv[i:i + 1, :, :n].double().cpu().numpy(),
                                                causal=True)).permute(0, 2, 1, 3))
    assert_close(out.float(), torch.cat(ref, 0), dtype, "fmha kvcache")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("b,s,hq,hkv,d,cap,positions,nan_tail", [
    (2, 2048, 28, 4, 128, 2560, [0, 0], False),          # 7B prefill rows, the bench's layout
    (8, 512, 14, 2, 64, 768, [0] * 8, False),            # 0.5B prefill (config workload)
    (4, 1000, 28, 4, 128, 2048, [0, 17, 500, 1048], True),  # ragged chunks, NaN past each sequence
    (2, 300, 64, 8, 128, 640, [0, 333], True),           # 72B head layout (group 8)
])
def test_fmha_kvcache_model_shapes(b, s, hq, hkv, d, cap, positions, nan_tail, dtype):
    q, ck, cv, pos = _cache_case(b, s, hq, hkv, d, cap, positions, dtype, seed=s + hq, nan_tail=nan_tail)
    out = C.attention_kvcache(q, ck, cv, pos)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    ck2, cv2 = torch.nan_to_num(ck), torch.nan_to_num(cv)  # the reference only reads visible rows
    ref = torch_cache_attention(q, ck2, cv2, positions)
    assert_close(out.float(), ref, dtype, "fmha kvcache (model shape)")
    C.check_device_error()


def test_fmha_repeated_launches_are_bit_identical():
    """The kernel is deterministic (fixed MMA and reduction order), so repeated
    launches on the same inputs must return the same bits. A synchronisation
    race between the tensor pipe and the softmax warps shows up here as a
    launch that differs: the epilogue once read O before the last two P V
    products had landed, which made the model-shape test fail now and then."""
    q, ck, cv, pos = _cache_case(2, 2048, 28, 4, 128, 2560, [0, 0], torch.bfloat16, seed=2076)
    first = C.attention_kvcache(q, ck, cv, pos)
    torch.cuda.synchronize()
    ref = torch_cache_attention(q, ck, cv, [0, 0])
    assert_close(first.float(), ref, torch.bfloat16, "fmha first launch")
    bad = 0
    for _ in range(200):
        out = C.attention_kvcache(q, ck, cv, pos)
        bad += int(not torch.equal(out, first))
    torch.cuda.synchronize()
    C.check_device_error()
    assert bad == 0, f"{bad} of 200 launches differ from the first"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("b,hq,hkv,sq,sk,d,causal", [
    (2, 8, 2, 200, 700, 128, False), (1, 4, 1, 256, 256, 64, True), (2, 6, 3, 333, 1000, 64, True)])
def test_fmha_dense(b, hq, hkv, sq, sk, d, causal, dtype):
    g = torch.Generator(device="cuda").manual_seed(sq * 3 + sk)
    q = torch.randn(b, hq, sq, d, device="cuda", generator=g).to(dtype)
    k = torch.randn(b, hkv, sk, d, device="cuda", generator=g).to(dtype)
    v = torch.randn(b, hkv, sk, d, device="cuda", generator=g).to(dtype)
    out = C.attention(q, k, v, causal=causal)
    ref = torch_cache_attention(q.permute(0, 2, 1, 3), k, v, [sk - sq] * b, causal=causal)
    assert_close(out.float(), ref.permute(0, 2, 1, 3), dtype, "fmha dense")


_STRICT = r"""
import math, torch
import dli_sm100 as C
from test_fmha_gpu import torch_cache_attention, _cache_case
from test_ops_gpu import assert_close
for (b, s, hq, hkv, d, cap, pos) in [(2, 2048, 28, 4, 128, 2560, [0, 0]), (8, 512, 14, 2, 64, 768, [0] * 8),
                                     (2, 129, 8, 2, 128, 512, [0, 200])]:
    q, ck, cv, p = _cache_case(b, s, hq, hkv, d, cap, pos, torch.bfloat16, seed=1)
    out = C.attention_kvcache(q, ck, cv, p)
    assert_close(out.float(), torch_cache_attention(q, ck, cv, pos), torch.bfloat16, "strict")
g = torch.Generator(device="cuda").manual_seed(5)
q, k, v = (torch.randn(2, 6, n, 128, device="cuda", generator=g).bfloat16() for n in (200, 700, 700))
ref = torch_cache_attention(q.permute(0, 2, 1, 3), k, v, [500, 500], causal=False)
assert_close(C.attention(q, k, v, causal=False).float(), ref.permute(0, 2, 1, 3), torch.bfloat16, "strict dense")
C.check_device_error()
print("fmha strict ok")
"""


@pytest.mark.parametrize("block_keys,p_tmem", [("128", "1"), ("64", "1"), ("128", "0"), ("64", "0")],
                         ids=["bn128-ptmem", "bn64-ptmem", "bn128-psmem", "bn64-psmem"])
def test_prefill_runs_on_tcgen05_kernel(block_keys, p_tmem):
    """DLI_SM100_ATTN_FMHA=2 turns a fallback to the mma.sync kernel into an
    error, so these shapes provably ran on the tcgen05 kernel, with 128-key
    blocks (one CTA per SM) and with 64-key blocks (two CTAs per SM), P in
    tensor memory and in shared memory; knobs are read once per process, so
    each runs in a child."""
    env = dict(os.environ, DLI_SM100_ATTN_FMHA="2", DLI_SM100_ATTN_FMHA_BN=block_keys,
               DLI_SM100_ATTN_FMHA_P=p_tmem)
    here = Path(__file__).resolve().parent
    env["PYTHONPATH"] = os.pathsep.join([str(here), str(here.parent), str(Path(C.__file__).resolve().parents[1]),
                                         env.get("PYTHONPATH", "")])
    res = subprocess.run([sys.executable, "-c", _STRICT], env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0 and "fmha strict ok" in res.stdout, (res.stdout[-2000:], res.stderr[-3000:])


@pytest.mark.parametrize("b,s,hq,hkv,d,cap,positions", [
    (4, 1, 8, 8, 128, 2048, [2047, 100, 0, 1500]),   # MHA decode, ragged contexts (one of 1 key)
    (3, 1, 28, 4, 128, 700, [699, 64, 333]),         # 7B heads: 7 query rows per KV head
    (2, 1, 64, 8, 128, 300, [299, 31]),              # 72B group: 8 rows
    (2, 2, 14, 2, 64, 600, [500, 5]),                # two tokens at group 7: 14 rows -> the tile kernel
    (1, 4, 2, 1, 64, 4096, [4000]),                  # 8 rows from 4 positions x group 2, long context
    (96, 1, 1, 1, 128, 256, list(range(0, 192, 2))),  # many heads, a few keys each
])
def test_f32_decode_attention_against_fp32_reference(b, s, hq, hkv, d, cap, positions):
    """fp32 attention over the KV cache with few query rows per KV head (the
    decode kernel: one warp per key range, merged across warps and a cluster),
    against a PyTorch fp32 reference at the fp32 tolerance. Cache rows past each
    sequence hold NaN and must not reach the output."""
    q, ck, cv, pos = _cache_case(b, s, hq, hkv, d, cap, positions, torch.float32, seed=b + s + hq, nan_tail=True)
    out = C.attention_kvcache(q, ck, cv, pos)
    C.check_device_error()
    assert torch.isfinite(out).all()
    assert_close(out, torch_cache_attention(q, ck, cv, positions), torch.float32, "fp32 decode attention")
    assert torch.equal(out, C.attention_kvcache(q, ck, cv, pos))  # deterministic merge
