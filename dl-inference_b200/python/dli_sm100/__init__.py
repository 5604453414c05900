"""ctypes binding of the C ABI in include/dli_sm100.h (libdli_sm100.so).

Thin, allocation-explicit wrappers that take torch CUDA tensors, pass their raw
device pointers and the current torch CUDA stream to the C entry points, and
raise on a non-zero status: ``ValueError`` for DLI_ERR_INVALID_ARGUMENT (the
reference operators raise std::invalid_argument, surfaced by pybind as
ValueError), ``RuntimeError`` otherwise. Outputs are allocated with torch unless
passed in. There is no CPU fallback: loading fails loudly when the library is
missing.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parents[2]
LIB_PATH = Path(os.environ.get("DLI_SM100_LIB", _PKG / "lib" / "libdli_sm100.so"))

DLI_OK = 0
DLI_ERR_INVALID_ARGUMENT = 1
DLI_ERR_UNSUPPORTED = 2
DLI_ERR_CUDA = 3
DLI_ERR_WORKSPACE = 4
DLI_ERR_DEVICE = 5

DTYPE_CODES = {torch.float32: 0, torch.int64: 1, torch.bfloat16: 2, torch.float16: 3,
               torch.int32: 4}

P, I, F, D, Z, N = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int,
                    ctypes.c_size_t, ctypes.c_int)

# name -> (restype, argtypes); mirrors include/dli_sm100.h
SIGNATURES = {
    "dli_sm100_abi_version": (ctypes.c_int, []),
    "dli_sm100_launch_count": (ctypes.c_uint64, []),
    "dli_sm100_last_error": (ctypes.c_char_p, []),
    "dli_sm100_check_device_error": (N, [P]),
    "dli_sm100_linear_workspace_size": (Z, [I, I, I, D]),
    "dli_sm100_linear": (N, [P, P, P, P, I, I, I, D, P, Z, P]),
    "dli_sm100_linear_ex": (N, [P, P, P, P, I, I, I, D, D, P, Z, P]),
    "dli_sm100_matmul": (N, [P, P, P, I, I, I, D, P]),
    "dli_sm100_linear_silu_mul": (N, [P, P, P, I, I, I, D, P]),
    "dli_sm100_conv2d_workspace_size": (Z, [I] * 11 + [D]),
    "dli_sm100_conv2d": (N, [P, P, P, P] + [I] * 11 + [D, P, Z, P]),
    "dli_sm100_rms_norm": (N, [P, P, P, I, I, F, D, P]),
    "dli_sm100_add_rms_norm": (N, [P, P, P, P, P, I, I, F, D, P]),
    "dli_sm100_add_rms_norm_ex": (N, [P, P, P, P, P, I, I, F, D, D, P]),
    "dli_sm100_batch_norm2d": (N, [P, P, P, P, P, P, I, I, I, F, D, P]),
    "dli_sm100_softmax": (N, [P, P, I, I, D, P]),
    "dli_sm100_rotary_embedding": (N, [P, P, P, P, P, P] + [I] * 8 + [P, I, D, P]),
    "dli_sm100_attention_workspace_size": (Z, [I] * 6 + [D]),
    "dli_sm100_attention": (N, [P, P, P, P] + [I] * 7 + [N, F, D, P, Z, P]),
    "dli_sm100_kv_append": (N, [P, P, P, P] + [I] * 6 + [D, P]),
    "dli_sm100_qkv_rotary_cache": (N, [P, P, P, P, P, P, P] + [I] * 8 + [D, P]),
    "dli_sm100_attention_kvcache_workspace_size": (Z, [I] * 6 + [D]),
    "dli_sm100_attention_kvcache": (N, [P, P, P, P, P] + [I] * 6 + [F, D, P, Z, P]),
    "dli_sm100_attention_kvcache_noalloc_max_scratch": (Z, []),
    "dli_sm100_attention_kvcache_noalloc": (N, [P, P, P, P, P] + [I] * 6 + [F, D, P]),
    "dli_sm100_add": (N, [P, P, P, I, I, D, P]),
    "dli_sm100_mul": (N, [P, P, P, I, I, D, P]),
    "dli_sm100_silu": (N, [P, P, I, D, P]),
    "dli_sm100_relu": (N, [P, P, I, D, P]),
    "dli_sm100_silu_mul": (N, [P, P, I, I, D, P]),
    "dli_sm100_embedding": (N, [P, D, P, P, I, I, I, D, P]),
    "dli_sm100_transpose2d": (N, [P, P, I, I, D, P]),
    "dli_sm100_max_pool2d": (N, [P, P] + [I] * 10 + [D, P]),
    "dli_sm100_argmax": (N, [P, P, I, I, D, P]),
    "dli_sm100_select_token": (N, [P, P, I, I, I, I, D, P]),
    "dli_sm100_cast": (N, [P, D, P, D, I, P]),
    "dli_sm100_tp_exchange_bytes": (Z, [D, I, I, D]),
    "dli_sm100_tp_exchange_reset": (N, [P, Z, P]),
    "dli_sm100_allreduce_add_rms_norm": (N, [P, D, D, D, I, I, P, P, P, P, P, I, I, I, F, I, D, P]),
    "dli_sm100_allreduce_add_rms_norm_ex": (N, [P, D, D, D, I, I, P, P, P, P, P, I, I, I, F, I, D, D, P]),
    "dli_sm100_allgather_argmax": (N, [P, D, D, D, I, I, D, P, I, I, I, P, I, D, P]),
    "dli_sm100_linear_exchange_push": (N, [P, P, P, I, I, I, D, P, D, D, I, I, P]),
    "dli_sm100_exchange_add_rms_norm_ex": (N, [P, D, D, D, I, I, P, P, P, P, I, I, I, F, I, D, D, P]),
    "dli_sm100_linear_qkv_rotary_cache": (N, [P] * 9 + [I] * 9 + [D, P]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Loads libdli_sm100.so once and declares every entry point's signature."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"libdli_sm100.so not found at {LIB_PATH}; run dl-inference_b200/build.py")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def launch_count() -> int:
    """Kernels launched (or captured) by libdli_sm100.so in this process so far."""
    return int(lib().dli_sm100_launch_count())


def last_error() -> str:
    return lib().dli_sm100_last_error().decode()


def check(status: int, what: str = "") -> None:
    if status == DLI_OK:
        return
    msg = f"{what}: {last_error()}" if what else last_error()
    if status == DLI_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    raise RuntimeError(msg)


def check_device_error() -> None:
    """Synchronises the current stream and raises if a kernel set the device error word."""
    check(lib().dli_sm100_check_device_error(_stream()), "device")


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _dt(t: torch.Tensor) -> int:
    try:
        return DTYPE_CODES[t.dtype]
    except KeyError as exc:
        raise ValueError(f"unsupported dtype {t.dtype}") from exc


def _workspace(nbytes: int, device) -> torch.Tensor | None:
    if nbytes == 0:
        return None
    return torch.empty(int(nbytes), dtype=torch.uint8, device=device)


def _contig(*ts):
    for t in ts:
        if t is not None and not t.is_contiguous():
            raise ValueError("tensors must be contiguous")


# ---- contractions ---------------------------------------------------------------

def linear(x, w, bias=None, out=None):
    _contig(x, w, bias)
    k = x.shape[-1]
    n = w.shape[0]
    m = x.numel() // k if k else 0
    if w.shape[1] != k:
        raise ValueError("linear: weight K mismatch")
    out = out if out is not None else torch.empty(*x.shape[:-1], n, dtype=x.dtype, device=x.device)
    L = lib()
    ws_bytes = L.dli_sm100_linear_workspace_size(m, n, k, _dt(x))  # stream-K partials (zero-filled)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=x.device) if ws_bytes else None
    check(L.dli_sm100_linear(_ptr(x), _ptr(w), _ptr(bias), _ptr(out), m, n, k, _dt(x), _ptr(ws),
                             ws_bytes, _stream()), "linear")
    return out


def linear_ex(x, w, bias=None, out_dtype=torch.float32):
    """linear with an output dtype wider than the operands (bf16/f16 -> fp32)."""
    _contig(x, w, bias)
    k = x.shape[-1]
    n = w.shape[0]
    m = x.numel() // k if k else 0
    if w.shape[1] != k:
        raise ValueError("linear_ex: weight K mismatch")
    out = torch.empty(*x.shape[:-1], n, dtype=out_dtype, device=x.device)
    L = lib()
    ws_bytes = L.dli_sm100_linear_workspace_size(m, n, k, _dt(x))
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=x.device) if ws_bytes else None
    check(L.dli_sm100_linear_ex(_ptr(x), _ptr(w), _ptr(bias), _ptr(out), m, n, k, _dt(x),
                                DTYPE_CODES[out_dtype], _ptr(ws), ws_bytes, _stream()), "linear_ex")
    return out


def linear_silu_mul(x, w_glu, inter):
    """silu(x @ Wg^T) * (x @ Wu^T); w_glu in the 64-row gate/up block layout
    (dli_export.qwen2.glu_blocked)."""
    _contig(x, w_glu)
    k = x.shape[-1]
    m = x.numel() // k
    out = torch.empty(*x.shape[:-1], inter, dtype=x.dtype, device=x.device)
    check(lib().dli_sm100_linear_silu_mul(_ptr(x), _ptr(w_glu), _ptr(out), m, inter, k, _dt(x), _stream()),
          "linear_silu_mul")
    return out


def matmul(a, b):
    _contig(a, b)
    m, k = a.shape
    n = b.shape[1]
    out = torch.empty(m, n, dtype=a.dtype, device=a.device)
    check(lib().dli_sm100_matmul(_ptr(a), _ptr(b), _ptr(out), m, n, k, _dt(a), _stream()), "matmul")
    return out


def conv2d(x, w, bias=None, stride=(1, 1), padding=(0, 0)):
    _contig(x, w, bias)
    n, c, h, wd = x.shape
    oc, _, kh, kw = w.shape
    oh = (h + 2 * padding[0] - kh) // stride[0] + 1
    ow = (wd + 2 * padding[1] - kw) // stride[1] + 1
    out = torch.empty(n, oc, oh, ow, dtype=x.dtype, device=x.device)
    L = lib()
    dims = (n, c, h, wd, oc, kh, kw, stride[0], stride[1], padding[0], padding[1])
    ws_bytes = L.dli_sm100_conv2d_workspace_size(*dims, _dt(x))
    ws = _workspace(ws_bytes, x.device)
    check(L.dli_sm100_conv2d(_ptr(x), _ptr(w), _ptr(bias), _ptr(out), *dims, _dt(x), _ptr(ws),
                             ws_bytes, _stream()), "conv2d")
    return out


# ---- normalisation --------------------------------------------------------------

def rms_norm(x, w, eps=1e-6):
    _contig(x, w)
    hidden = x.shape[-1]
    out = torch.empty_like(x)
    check(lib().dli_sm100_rms_norm(_ptr(x), _ptr(w), _ptr(out), x.numel() // hidden, hidden,
                                   eps, _dt(x), _stream()), "rms_norm")
    return out


def add_rms_norm(residual, delta, w, eps=1e-6, residual_out=None):
    """(normed, residual + delta). A float32 residual with a bf16/f16 delta keeps
    the residual stream in fp32 (dli_sm100_add_rms_norm_ex); normed has delta's dtype."""
    _contig(residual, delta, w)
    hidden = residual.shape[-1]
    normed = torch.empty_like(delta)
    residual_out = residual_out if residual_out is not None else torch.empty_like(residual)
    check(lib().dli_sm100_add_rms_norm_ex(_ptr(residual), _ptr(delta), _ptr(w), _ptr(normed),
                                          _ptr(residual_out), residual.numel() // hidden, hidden, eps,
                                          _dt(delta), _dt(residual), _stream()), "add_rms_norm")
    return normed, residual_out


class ExchangeGroup:
    """Exchange buffers of a whole tensor-parallel group on ONE device, for
    running every rank of the group in one cooperative launch of
    dli_sm100_allreduce_add_rms_norm (ranks_in_launch = tp). Multi-process
    groups map each rank's buffer through CUDA IPC in the operator plugin."""

    def __init__(self, tp, max_rows, row_elems, dtype=torch.bfloat16, device="cuda"):
        nbytes = lib().dli_sm100_tp_exchange_bytes(tp, max_rows, row_elems, DTYPE_CODES[dtype])
        if nbytes == 0:
            raise ValueError("unsupported exchange shape")
        # torch's allocator returns 512-byte aligned blocks
        self.buffers = [torch.empty(nbytes, dtype=torch.uint8, device=device) for _ in range(tp)]
        self.tp, self.max_rows, self.row_elems, self.dtype = tp, max_rows, row_elems, dtype
        for b in self.buffers:
            check(lib().dli_sm100_tp_exchange_reset(_ptr(b), nbytes, _stream()), "tp_exchange_reset")
        self._ptrs = (ctypes.c_void_p * tp)(*[b.data_ptr() for b in self.buffers])

    def allreduce_add_rms_norm(self, residual, delta, w, eps=1e-6, timeout_ns=0, ranks=None):
        """residual/delta [tp, rows, hidden] (rank-major); returns (normed, residual_out).
        ranks < tp launches only ranks 0..ranks-1 (their waits for the others run out)."""
        _contig(residual, delta, w)
        tp, rows, hidden = delta.shape
        ranks = tp if ranks is None else ranks
        normed, residual_out = torch.empty_like(delta), torch.empty_like(residual)
        st = lib().dli_sm100_allreduce_add_rms_norm_ex(
            self._ptrs, self.tp, 0, ranks, self.max_rows, self.row_elems, _ptr(delta), _ptr(residual),
            _ptr(w), _ptr(normed), _ptr(residual_out), rows * hidden, rows, hidden, eps, timeout_ns,
            _dt(delta), _dt(residual), _stream())
        check(st, "allreduce_add_rms_norm")
        return normed, residual_out

    def linear_allreduce_add_rms_norm(self, x, w, residual, norm_w, eps=1e-6, timeout_ns=0):
        """The fused row-split projection: x [tp, rows, k], w [tp, n, k] (each
        rank's shard), residual [tp, rows, n]. Every rank's GEMM pushes its
        partial rows into the buffers (dli_sm100_linear_exchange_push, one launch
        per rank), then one launch over all ranks sums, adds and normalises
        (dli_sm100_exchange_add_rms_norm_ex). Returns (normed, residual_out), or
        None when the shape is outside the fused path (DLI_ERR_UNSUPPORTED)."""
        _contig(x, w, residual, norm_w)
        tp, rows, k = x.shape
        n = w.shape[1]
        L = lib()
        for r in range(tp):
            st = L.dli_sm100_linear_exchange_push(_ptr(x[r]), _ptr(w[r]), None, rows, n, k, _dt(x), self._ptrs,
                                                  self.tp, r, self.max_rows, self.row_elems, _stream())
            if st == 2 and r == 0:  # DLI_ERR_UNSUPPORTED: nothing was launched on any rank
                return None
            check(st, "linear_exchange_push")
        normed = torch.empty(tp, rows, n, dtype=x.dtype, device=x.device)
        residual_out = torch.empty_like(residual)
        st = L.dli_sm100_exchange_add_rms_norm_ex(
            self._ptrs, self.tp, 0, tp, self.max_rows, self.row_elems, _ptr(residual), _ptr(norm_w), _ptr(normed),
            _ptr(residual_out), rows * n, rows, n, eps, timeout_ns, _dt(x), _dt(residual), _stream())
        check(st, "exchange_add_rms_norm")
        return normed, residual_out

    def allgather_argmax(self, logits, timeout_ns=0, ranks=None):
        """logits [tp, rows, width] (rank i holds ids [i*width, (i+1)*width));
        returns [tp, rows] int64 global argmax ids (the same row on every rank)."""
        _contig(logits)
        tp, rows, width = logits.shape
        ranks = tp if ranks is None else ranks
        out = torch.empty(tp, rows, dtype=torch.int64, device=logits.device)
        st = lib().dli_sm100_allgather_argmax(self._ptrs, self.tp, 0, ranks, self.max_rows, self.row_elems,
                                              DTYPE_CODES[self.dtype], _ptr(logits), rows, width, rows * width,
                                              _ptr(out), timeout_ns, _dt(logits), _stream())
        check(st, "allgather_argmax")
        return out


def batch_norm2d(x, weight, bias, running_mean, running_var, eps=1e-5):
    _contig(x)
    out = torch.empty_like(x)
    check(lib().dli_sm100_batch_norm2d(_ptr(x), _ptr(weight), _ptr(bias), _ptr(running_mean),
                                       _ptr(running_var), _ptr(out), x.numel(), x.shape[1],
                                       x.shape[2] * x.shape[3], eps, _dt(x), _stream()),
          "batch_norm2d")
    return out


def softmax(x):
    _contig(x)
    width = x.shape[-1]
    out = torch.empty_like(x)
    check(lib().dli_sm100_softmax(_ptr(x), _ptr(out), x.numel() // width, width, _dt(x), _stream()),
          "softmax")
    return out


# ---- positional / attention -----------------------------------------------------

def rotary_embedding(q, k, cos, sin, start_pos=0, positions=None):
    _contig(q, k, cos, sin)
    b, hq, s, d = q.shape
    hk = k.shape[1]
    out_q, out_k = torch.empty_like(q), torch.empty_like(k)
    pos_n = positions.numel() if positions is not None else 0
    check(lib().dli_sm100_rotary_embedding(_ptr(q), _ptr(k), _ptr(cos), _ptr(sin), _ptr(out_q),
                                           _ptr(out_k), b, hq, hk, s, d, cos.shape[1],
                                           cos.shape[0], start_pos, _ptr(positions), pos_n,
                                           _dt(q), _stream()), "rotary_embedding")
    return out_q, out_k


def attention(q, k, v, causal=False, scale=0.0, kv_capacity=None, seq_k=None):
    _contig(q, k, v)
    b, hq, sq, d = q.shape
    hkv = k.shape[1]
    cap = kv_capacity if kv_capacity is not None else k.shape[2]
    sk = seq_k if seq_k is not None else k.shape[2]
    out = torch.empty_like(q)
    L = lib()
    ws_bytes = L.dli_sm100_attention_workspace_size(b, hq, hkv, sq, sk, d, _dt(q))
    ws = _workspace(ws_bytes, q.device)
    check(L.dli_sm100_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(out), b, hq, hkv, sq, sk, cap, d,
                                1 if causal else 0, scale, _dt(q), _ptr(ws), ws_bytes, _stream()),
          "attention")
    return out


def kv_append(cache_k, cache_v, k, v, old_len):
    _contig(cache_k, cache_v, k, v)
    b, h, s, d = k.shape
    check(lib().dli_sm100_kv_append(_ptr(cache_k), _ptr(cache_v), _ptr(k), _ptr(v), b, h,
                                    cache_k.shape[2], old_len, s, d, _dt(k), _stream()), "kv_append")


def qkv_rotary_cache(qkv, cos, sin, positions, cache_k, cache_v, batch, seq, q_heads, kv_heads,
                     head_dim, q_out=None):
    _contig(qkv, cos, sin, positions, cache_k, cache_v)
    q_out = q_out if q_out is not None else torch.empty(batch, seq, q_heads, head_dim,
                                                        dtype=qkv.dtype, device=qkv.device)
    check(lib().dli_sm100_qkv_rotary_cache(_ptr(qkv), _ptr(cos), _ptr(sin), _ptr(positions),
                                           _ptr(q_out), _ptr(cache_k), _ptr(cache_v), batch, seq,
                                           q_heads, kv_heads, head_dim, cos.shape[1], cos.shape[0],
                                           cache_k.shape[2], _dt(qkv), _stream()),
          "qkv_rotary_cache")
    return q_out


def linear_qkv_rotary_cache(x, wqkv, bqkv, cos, sin, positions, cache_k, cache_v, batch, seq, q_heads, kv_heads,
                            head_dim, q_out=None):
    """The q|k|v projection with rotary + KV-cache write in its GEMM epilogue.
    Returns q_out, or None when the shape is outside the fused path
    (DLI_ERR_UNSUPPORTED: nothing launched)."""
    _contig(x, wqkv, bqkv, cos, sin, positions, cache_k, cache_v)
    q_out = q_out if q_out is not None else torch.empty(batch, seq, q_heads, head_dim, dtype=x.dtype, device=x.device)
    st = lib().dli_sm100_linear_qkv_rotary_cache(
        _ptr(x), _ptr(wqkv), _ptr(bqkv), _ptr(cos), _ptr(sin), _ptr(positions), _ptr(q_out), _ptr(cache_k),
        _ptr(cache_v), batch, seq, x.shape[-1], q_heads, kv_heads, head_dim, cos.shape[1], cos.shape[0],
        cache_k.shape[2], _dt(x), _stream())
    if st == 2:  # DLI_ERR_UNSUPPORTED
        return None
    check(st, "linear_qkv_rotary_cache")
    return q_out


def attention_kvcache(q, cache_k, cache_v, positions, scale=0.0, out=None):
    _contig(q, cache_k, cache_v, positions)
    b, s, hq, d = q.shape
    hkv, cap = cache_k.shape[1], cache_k.shape[2]
    out = out if out is not None else torch.empty_like(q)
    L = lib()
    ws_bytes = L.dli_sm100_attention_kvcache_workspace_size(b, s, hq, hkv, cap, d, _dt(q))
    ws = _workspace(ws_bytes, q.device)
    check(L.dli_sm100_attention_kvcache(_ptr(q), _ptr(cache_k), _ptr(cache_v), _ptr(positions),
                                        _ptr(out), b, s, hq, hkv, cap, d, scale, _dt(q), _ptr(ws),
                                        ws_bytes, _stream()), "attention_kvcache")
    return out


# ---- elementwise / data movement ------------------------------------------------

def add(a, b):
    _contig(a, b)
    out = torch.empty_like(a)
    check(lib().dli_sm100_add(_ptr(a), _ptr(b), _ptr(out), a.numel(), b.numel(), _dt(a), _stream()),
          "add")
    return out


def mul(a, b):
    _contig(a, b)
    out = torch.empty_like(a)
    check(lib().dli_sm100_mul(_ptr(a), _ptr(b), _ptr(out), a.numel(), b.numel(), _dt(a), _stream()),
          "mul")
    return out


def silu(x):
    _contig(x)
    out = torch.empty_like(x)
    check(lib().dli_sm100_silu(_ptr(x), _ptr(out), x.numel(), _dt(x), _stream()), "silu")
    return out


def relu(x):
    _contig(x)
    out = torch.empty_like(x)
    check(lib().dli_sm100_relu(_ptr(x), _ptr(out), x.numel(), _dt(x), _stream()), "relu")
    return out


def silu_mul(gate_up):
    _contig(gate_up)
    width = gate_up.shape[-1] // 2
    out = torch.empty(*gate_up.shape[:-1], width, dtype=gate_up.dtype, device=gate_up.device)
    check(lib().dli_sm100_silu_mul(_ptr(gate_up), _ptr(out), gate_up.numel() // (2 * width), width,
                                   _dt(gate_up), _stream()), "silu_mul")
    return out


def embedding(ids, table):
    _contig(ids, table)
    hidden = table.shape[1]
    out = torch.empty(*ids.shape, hidden, dtype=table.dtype, device=table.device)
    check(lib().dli_sm100_embedding(_ptr(ids), _dt(ids), _ptr(table), _ptr(out), ids.numel(),
                                    hidden, table.shape[0], _dt(table), _stream()), "embedding")
    return out


def transpose2d(x):
    _contig(x)
    rows, cols = x.shape
    out = torch.empty(cols, rows, dtype=x.dtype, device=x.device)
    check(lib().dli_sm100_transpose2d(_ptr(x), _ptr(out), rows, cols, _dt(x), _stream()), "transpose")
    return out


def max_pool2d(x, kernel_size=(2, 2), stride=None, padding=(0, 0)):
    _contig(x)
    stride = stride if stride is not None else kernel_size
    n, c, h, w = x.shape
    oh = (h + 2 * padding[0] - kernel_size[0]) // stride[0] + 1
    ow = (w + 2 * padding[1] - kernel_size[1]) // stride[1] + 1
    out = torch.empty(n, c, oh, ow, dtype=x.dtype, device=x.device)
    check(lib().dli_sm100_max_pool2d(_ptr(x), _ptr(out), n, c, h, w, kernel_size[0],
                                     kernel_size[1], stride[0], stride[1], padding[0], padding[1],
                                     _dt(x), _stream()), "max_pool2d")
    return out


def argmax(x):
    _contig(x)
    width = x.shape[-1]
    out = torch.empty(*x.shape[:-1], dtype=torch.int64, device=x.device)
    check(lib().dli_sm100_argmax(_ptr(x), _ptr(out), x.numel() // width, width, _dt(x), _stream()),
          "argmax")
    return out


def select_token(x, index):
    _contig(x)
    b, s, w = x.shape
    out = torch.empty(b, w, dtype=x.dtype, device=x.device)
    check(lib().dli_sm100_select_token(_ptr(x), _ptr(out), b, s, w, index, _dt(x), _stream()),
          "select_token")
    return out


def cast(x, dtype):
    _contig(x)
    out = torch.empty(x.shape, dtype=dtype, device=x.device)
    check(lib().dli_sm100_cast(_ptr(x), _dt(x), _ptr(out), DTYPE_CODES[dtype], x.numel(), _stream()),
          "cast")
    return out
