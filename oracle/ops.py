"""CPU oracle for the dli.graph.v1 operators — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy (float64 arithmetic unless noted), what each
reference operator computes, following the reference kernels line by line
(paths relative to the yncxcw/dl-inference project root). It is the checker
for the CUDA kernels of ``libdli_sm100.so``: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it.
The product path never calls it.

Pinning: ``tests/test_oracle_golden.py`` checks every function here against
``tests/golden/*.npz`` — outputs of the reference's own Triton kernels
(``python/dli_ops/aot/<op>/kernel.py``) executed by the Triton CPU interpreter
with the launch grids of the reference ``template.cc`` files, plus the literal
vectors of the reference operator tests (``tests/operators/test_*.py``).
``tests/golden/make_golden.py`` regenerates them.
"""
from __future__ import annotations

import math

import numpy as np


def _f(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float64)


def linear(x, w, b=None) -> np.ndarray:
    """y = x . w^T (+ b) over the last dim of x.

    python/dli_ops/aot/linear/kernel.py:24-44 (acc += dot(x_tile, w_tile^T); bias
    added once, kernel.py:39-40); M = product of leading dims
    (python/dli_ops/aot/linear/template.cc:23).
    """
    x = _f(x)
    y = x.reshape(-1, x.shape[-1]) @ _f(w).T
    if b is not None:
        y = y + _f(b)[None, :]
    return y.reshape(*x.shape[:-1], _f(w).shape[0])


def matmul(a, b) -> np.ndarray:
    """out = a . b, 2-D (python/dli_ops/aot/matmul/kernel.py:23-40)."""
    return _f(a) @ _f(b)


def conv2d(x, w, b=None, stride=(1, 1), padding=(0, 0)) -> np.ndarray:
    """Direct NCHW convolution with zero padding.

    python/dli_ops/aot/conv2d/kernel.py:30-49: out[n,oc,oh,ow] = bias[oc] +
    sum_{ic,kh,kw} x[n,ic,oh*sh+kh-ph,ow*sw+kw-pw] * w[oc,ic,kh,kw], taps outside
    the image read 0; OH = (H + 2*ph - KH)//sh + 1 (template.cc:13-14).
    """
    x, w = _f(x), _f(w)
    n, c, h, wd = x.shape
    oc, ic, kh, kw = w.shape
    assert ic == c
    sh, sw = stride
    ph, pw = padding
    oh = (h + 2 * ph - kh) // sh + 1
    ow = (wd + 2 * pw - kw) // sw + 1
    xp = np.zeros((n, c, h + 2 * ph, wd + 2 * pw))
    xp[:, :, ph:ph + h, pw:pw + wd] = x
    out = np.zeros((n, oc, oh, ow))
    for dy in range(kh):
        for dx in range(kw):
            patch = xp[:, :, dy:dy + sh * (oh - 1) + 1:sh, dx:dx + sw * (ow - 1) + 1:sw]
            out += np.einsum("nchw,oc->nohw", patch, w[:, :, dy, dx])
    if b is not None:
        out += _f(b)[None, :, None, None]
    return out


def rms_norm(x, w, eps: float = 1e-6) -> np.ndarray:
    """x * rsqrt(mean(x^2) + eps) * w over the last dim.

    python/dli_ops/aot/rms_norm/kernel.py:11-13; eps attribute default 1e-6
    (python/dli_ops/aot/rms_norm/template.cc:21).
    """
    x = _f(x)
    ms = np.mean(x * x, axis=-1, keepdims=True)
    return x / np.sqrt(ms + eps) * _f(w)


def add_rms_norm(residual, delta, w, eps: float = 1e-6) -> tuple[np.ndarray, np.ndarray]:
    """The exporter's `add` -> `rms_norm` node pair (python/dli_export/export.py:385-396)."""
    r = _f(residual) + _f(delta)
    return rms_norm(r, w, eps), r


def rotary(q, k, cos, sin, start_pos: int = 0, positions=None) -> tuple[np.ndarray, np.ndarray]:
    """Interleaved-pair rotation of q [B,Hq,S,D] and k [B,Hk,S,D].

    python/dli_ops/aot/rotary/kernel.py:22-35: pair i of token s uses table row
    p = start_pos + s; out[2i] = x[2i] c - x[2i+1] s, out[2i+1] = x[2i] s + x[2i+1] c.
    Elements beyond 2*pairs are copied (the memcpy of rotary/template.cc:11-12).
    `positions` (an extension) gives p = positions[b] + s ([B]) or
    positions[b, s] ([B,S]). k is rotated with its own head count (the reference
    sizes k's loop from q, template.cc:14, which is only correct for Hk == Hq).
    """
    cos, sin = _f(cos), _f(sin)
    pairs = cos.shape[1]

    def rot(x):
        x = _f(x).copy()
        b, h, s, d = x.shape
        if positions is None:
            p = np.broadcast_to(start_pos + np.arange(s)[None, :], (b, s))
        else:
            pos = np.asarray(positions, dtype=np.int64)
            p = pos.reshape(b, 1) + np.arange(s)[None, :] if pos.size == b else pos.reshape(b, s)
        c = cos[p][:, None, :, :]  # [B,1,S,pairs]
        sn = sin[p][:, None, :, :]
        x0 = x[..., 0:2 * pairs:2].copy()
        x1 = x[..., 1:2 * pairs:2].copy()
        x[..., 0:2 * pairs:2] = x0 * c - x1 * sn
        x[..., 1:2 * pairs:2] = x0 * sn + x1 * c
        return x

    return rot(q), rot(k)


def attention(q, k, v, causal: bool = False, scale: float | None = None) -> np.ndarray:
    """softmax(q k^T * scale + mask) v for q [B,Hq,Sq,D], k/v [B,Hkv,Sk,D].

    python/dli_ops/aot/attention/kernel.py:34-62: online softmax; the causal mask
    is bottom-right: key j is visible to query i iff j <= i + (Sk - Sq)
    (kernel.py:35,49-50); scale = 1/sqrt(D) (tools/build_triton_aot_ops.py:283).
    Hq may be a multiple of Hkv (GQA, an extension: head h reads KV head
    h // (Hq/Hkv)). Rows with no visible key return 0.
    """
    q, k, v = _f(q), _f(k), _f(v)
    b, hq, sq, d = q.shape
    hkv, sk = k.shape[1], k.shape[2]
    group = hq // hkv
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    kx = np.repeat(k, group, axis=1)
    vx = np.repeat(v, group, axis=1)
    scores = np.einsum("bhid,bhjd->bhij", q, kx) * scale
    if causal:
        i = np.arange(sq)[:, None]
        j = np.arange(sk)[None, :]
        visible = j <= i + (sk - sq)
        scores = np.where(visible[None, None], scores, -np.inf)
    m = np.max(scores, axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    p = np.exp(scores - m)
    den = np.sum(p, axis=-1, keepdims=True)
    out = np.einsum("bhij,bhjd->bhid", p, vx) / np.where(den > 0, den, 1.0)
    return out


def attention_reference_padded(q, k, v, block_n: int = 32) -> np.ndarray:
    """What the reference kernel computes for NON-causal attention when Sk is not a
    multiple of its key block (BLOCK_N = 32, tools/build_triton_aot_ops.py:292-296).

    python/dli_ops/aot/attention/kernel.py:39-58 loads out-of-range keys as 0
    (`other=0.0`) and masks them only in the causal branch (kernel.py:49-50), so in
    non-causal mode every padded key enters the softmax with score 0 and value 0:
    the denominator gains (ceil(Sk/32)*32 - Sk) terms exp(0 - m). This restates that
    defect so the golden pin can show it; the CUDA kernels implement `attention`.
    """
    q, k, v = _f(q), _f(k), _f(v)
    sk = k.shape[2]
    pad = (-sk) % block_n
    if pad == 0:
        return attention(q, k, v, causal=False)
    kp = np.concatenate([k, np.zeros(k.shape[:2] + (pad, k.shape[3]))], axis=2)
    vp = np.concatenate([v, np.zeros(v.shape[:2] + (pad, v.shape[3]))], axis=2)
    return attention(q, kp, vp, causal=False)


def embedding(ids, table) -> np.ndarray:
    """out[..., :] = table[ids[...], :] (python/dli_ops/aot/embedding/kernel.py:13-23)."""
    return _f(table)[np.asarray(ids, dtype=np.int64)]


def _broadcast(a, b):
    a = _f(a)
    flat_b = _f(b).reshape(-1)
    idx = np.arange(a.size) % flat_b.size
    return a, flat_b[idx].reshape(a.shape)


def add(a, b) -> np.ndarray:
    """out[i] = a[i] + b[i mod numel(b)] (python/dli_ops/aot/add/kernel.py:8-11)."""
    a, bb = _broadcast(a, b)
    return a + bb


def mul(a, b) -> np.ndarray:
    """out[i] = a[i] * b[i mod numel(b)] (python/dli_ops/aot/mul/kernel.py:8-11)."""
    a, bb = _broadcast(a, b)
    return a * bb


def silu(x) -> np.ndarray:
    """x / (1 + exp(-x)) (python/dli_ops/aot/silu/kernel.py:10)."""
    x = _f(x)
    return x / (1.0 + np.exp(-x))


def silu_mul(gate_up) -> np.ndarray:
    """silu(gate) * up for gate_up = [gate | up] along the last dim (export.py:414-415)."""
    gu = _f(gate_up)
    w = gu.shape[-1] // 2
    return silu(gu[..., :w]) * gu[..., w:]


def relu(x) -> np.ndarray:
    """max(x, 0) (python/dli_ops/aot/relu/kernel.py:10)."""
    return np.maximum(_f(x), 0.0)


def softmax(x) -> np.ndarray:
    """Row softmax over the last dim (python/dli_ops/aot/softmax/kernel.py:8-14)."""
    x = _f(x)
    e = np.exp(x - np.max(x, axis=-1, keepdims=True))
    return e / np.sum(e, axis=-1, keepdims=True)


def max_pool2d(x, kernel_size=(2, 2), stride=None, padding=(0, 0)) -> np.ndarray:
    """NCHW max pool; padding taps read -inf (python/dli_ops/aot/max_pool2d/kernel.py:24-41).

    stride defaults to kernel_size (python/dli_ops/aot/max_pool2d/template.cc:10).
    """
    x = _f(x)
    kh, kw = kernel_size
    sh, sw = stride if stride is not None else kernel_size
    ph, pw = padding
    n, c, h, w = x.shape
    oh = (h + 2 * ph - kh) // sh + 1
    ow = (w + 2 * pw - kw) // sw + 1
    xp = np.full((n, c, h + 2 * ph, w + 2 * pw), -np.inf)
    xp[:, :, ph:ph + h, pw:pw + w] = x
    out = np.full((n, c, oh, ow), -np.inf)
    for dy in range(kh):
        for dx in range(kw):
            out = np.maximum(out, xp[:, :, dy:dy + sh * (oh - 1) + 1:sh, dx:dx + sw * (ow - 1) + 1:sw])
    return out


def batch_norm2d(x, weight, bias, running_mean, running_var, eps: float = 1e-5) -> np.ndarray:
    """Inference batch norm (python/dli_ops/aot/batch_norm2d/kernel.py:19-28; eps default
    1e-5, python/dli_ops/aot/batch_norm2d/template.cc:22)."""
    x = _f(x)
    sh = (1, -1, 1, 1)
    return (x - _f(running_mean).reshape(sh)) / np.sqrt(_f(running_var).reshape(sh) + eps) * \
        _f(weight).reshape(sh) + _f(bias).reshape(sh)


def transpose2d(x) -> np.ndarray:
    """out[c, r] = x[r, c] (python/dli_ops/aot/transpose/kernel.py:5-20)."""
    return _f(x).T.copy()


def reshape_shape(shape, target) -> list[int]:
    """Target shape with one -1 inferred (src/utils.cc:54-76); raises ValueError like
    the reference's std::invalid_argument."""
    target = list(target)
    known, infer = 1, -1
    for i, t in enumerate(target):
        if t == -1:
            if infer != -1:
                raise ValueError("reshape has multiple inferred dimensions")
            infer = i
        elif t <= 0:
            raise ValueError("reshape dimension must be positive or -1")
        else:
            known *= t
    numel = int(np.prod(shape)) if len(shape) else 1
    if infer != -1:
        if numel % known != 0:
            raise ValueError("reshape inferred dimension is not integral")
        target[infer] = numel // known
    if int(np.prod(target)) != numel:
        raise ValueError("reshape changes element count")
    return target


def kv_append(cache_k, cache_v, k, v, old_len: int):
    """Writes k/v [B,H,S,D] into rows [old_len, old_len+S) of caches [B,H,cap,D].

    The reference (src/kv_cache.cc:31-42) appends by a flat byte copy, which equals
    concatenation along the sequence axis only when B*H == 1; this restates the
    intended torch.cat(dim=2) semantics.
    """
    ck, cv = _f(cache_k).copy(), _f(cache_v).copy()
    s = _f(k).shape[2]
    ck[:, :, old_len:old_len + s] = _f(k)
    cv[:, :, old_len:old_len + s] = _f(v)
    return ck, cv


def kv_append_reference_flat(old_k, k):
    """The reference's flat append (src/kv_cache.cc:35-42): bytes of the old tensor
    followed by the bytes of the new one, viewed as [B,H,S_old+S_new,D]. Kept to
    document the layout defect the new cache fixes."""
    old_k, k = _f(old_k), _f(k)
    b, h, s0, d = old_k.shape
    flat = np.concatenate([old_k.reshape(-1), k.reshape(-1)])
    return flat.reshape(b, h, s0 + k.shape[2], d)


def argmax(x) -> np.ndarray:
    """Row argmax, lowest index on ties (greedy decoding)."""
    return np.argmax(_f(x), axis=-1).astype(np.int64)
