"""Single-kernel cases of the Qwen2 hot path, for timing and for profilers.

    python -m dli_sm100.profile_cases <case> [--reps N]

Each case builds its inputs once (every case's operands exceed the 126 MB L2,
or it states otherwise), runs 3 warm-up launches and N timed launches through the
C ABI, and prints one JSON line with the mean launch time (CUDA events) and the
algorithmic bytes / FLOPs of one launch. Cases use the Qwen2-7B decode/prefill
shapes of the benchmark (batch 32, 2048-token prompts). The attention prefill
cases are tensor-bound; their operands may fit in L2.
"""
from __future__ import annotations

import argparse
import json

import torch

import dli_sm100 as C

BF = torch.bfloat16


def _gemm(m, n, k):
    x = torch.randn(m, k, device="cuda").to(BF)
    w = (torch.randn(n, k, device="cuda") * 0.02).to(BF)
    return (lambda: C.linear(x, w)), 2 * (n * k + m * (n + k)), 2.0 * m * n * k


def _gemm_f32(m, n, k):
    x = torch.randn(m, k, device="cuda")
    w = torch.randn(n, k, device="cuda") * 0.02
    b = torch.randn(n, device="cuda") * 0.02
    return (lambda: C.linear(x, w, b)), 4 * (n * k + m * (n + k) + n), 2.0 * m * n * k


def _glu(m, inter, k):
    from dli_export.qwen2 import glu_blocked

    x = torch.randn(m, k, device="cuda").to(BF)
    w = glu_blocked((torch.randn(inter, k, device="cuda") * 0.02).to(BF),
                    (torch.randn(inter, k, device="cuda") * 0.02).to(BF))
    return (lambda: C.linear_silu_mul(x, w, inter)), 2 * (2 * inter * k + m * (inter + k)), 4.0 * m * inter * k


def _attn_decode(b=32, hq=28, hkv=4, d=128, cap=2560, ctx=2304):
    q = torch.randn(b, 1, hq, d, device="cuda").to(BF)
    ck = torch.randn(b, hkv, cap, d, device="cuda").to(BF)
    cv = torch.randn(b, hkv, cap, d, device="cuda").to(BF)
    pos = torch.full((b,), ctx - 1, dtype=torch.int64, device="cuda")
    kv_bytes = 2 * b * hkv * ctx * d * 2
    return (lambda: C.attention_kvcache(q, ck, cv, pos)), kv_bytes + 2 * b * hq * d * 2, \
        4.0 * b * hq * ctx * d


def _attn_prefill(b=2, hq=28, hkv=4, d=128, s=2048):
    q = torch.randn(b, s, hq, d, device="cuda").to(BF)
    ck = torch.randn(b, hkv, s, d, device="cuda").to(BF)
    cv = torch.randn(b, hkv, s, d, device="cuda").to(BF)
    pos = torch.zeros(b, dtype=torch.int64, device="cuda")
    flops = 2.0 * b * hq * d * s * (s + 1)  # causal QK^T + PV
    return (lambda: C.attention_kvcache(q, ck, cv, pos)), 2 * b * s * d * 2 * (hq + 2 * hkv), flops


def _attn_f32(bh=896, sq=128, sk=128, d=128):
    # the reference attention kernel's shapes in its own dtype (fp32, bottom-right causal)
    q = torch.randn(1, bh, sq, d, device="cuda")
    k = torch.randn(1, bh, sk, d, device="cuda")
    v = torch.randn(1, bh, sk, d, device="cuda")
    visible = sq * (sk - sq) + sq * (sq + 1) // 2  # keys seen, summed over the query rows
    return (lambda: C.attention(q, k, v, causal=True)), 4 * bh * d * (2 * sq + 2 * sk), 4.0 * bh * d * visible


CASES = {
    "gemm_decode_gate_up": lambda: _gemm(32, 37888, 3584),
    "gemm_decode_qkv": lambda: _gemm(32, 4608, 3584),   # 33 MB of weights: fits L2
    "gemm_decode_o": lambda: _gemm(32, 3584, 3584),     # 26 MB: fits L2
    "gemm_decode_down": lambda: _gemm(32, 3584, 18944),
    "gemm_decode_lm_head": lambda: _gemm(32, 152064, 3584),
    "gemm_prefill_gate_up": lambda: _gemm(8192, 37888, 3584),
    "gemm_prefill_o": lambda: _gemm(8192, 3584, 3584),
    "gemm_f32_linear": lambda: _gemm_f32(64, 4096, 1024),       # config 1 (16 MB weights: fits L2)
    "gemm_f32_decode_qkv": lambda: _gemm_f32(32, 4608, 3584),   # fp32 7B qkv shape (66 MB: fits L2)
    "glu_decode_gate_up": lambda: _glu(32, 18944, 3584),
    "glu_prefill_gate_up": lambda: _glu(8192, 18944, 3584),
    "attn_decode": _attn_decode,
    "attn_decode_tp4": lambda: _attn_decode(hq=7, hkv=1),
    "attn_prefill": _attn_prefill,
    "attn_prefill_b32": lambda: _attn_prefill(b=32, s=2048),          # the benchmark's prefill launch
    "attn_prefill_0_5b": lambda: _attn_prefill(b=8, hq=14, hkv=2, d=64, s=512),
    "attn_f32_tiles": _attn_f32,
    "attn_f32_decode": lambda: _attn_f32(sq=1, sk=2048),   # one query row per head: HBM-bound
}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--reps", type=int, default=10)
    args = ap.parse_args()
    fn, nbytes, flops = CASES[args.case]()
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    C.check_device_error()
    ms = a.elapsed_time(b) / args.reps
    print(json.dumps({"case": args.case, "ms": ms, "bytes": nbytes, "flops": flops,
                      "GB/s": nbytes / ms / 1e6, "TFLOP/s": flops / ms / 1e9}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
