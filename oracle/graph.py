"""CPU interpreter of dli.graph.v1 graphs over oracle/ops.py — TEST INFRASTRUCTURE ONLY.

Executes a graph dict node by node with the numpy oracle (float64), keeping a
position-addressed KV cache for the fused `qkv_rotary_cache` /
`attention_kvcache` operators and an appending cache for the reference's
`attention` with a `kv_cache` attribute (python/dli_ops/aot/attention/
template.cc:10-18). Used to check exported graphs against the source model on
CPU; never used by the product path.
"""
from __future__ import annotations

import numpy as np

from . import ops as O


class GraphOracle:
    def __init__(self, graph: dict, constants: dict[str, np.ndarray], all_reduce=None, all_gather=None):
        """all_reduce: callable summing an array over the ranks of a tensor-parallel
        group (for instance a torch.distributed gloo all_reduce); all_gather:
        callable returning the list of every rank's array in rank order; None =
        one rank."""
        self.graph = graph
        self.constants = constants
        self.all_reduce = all_reduce
        self.all_gather = all_gather
        self.cache: dict[str, dict[str, np.ndarray]] = {}

    def run(self, inputs: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
        env = dict(self.constants)
        env.update(inputs)
        for node in self.graph["nodes"]:
            ins = [env[n] for n in node["inputs"]]
            outs = self._op(node["op"], ins, node.get("attrs", {}))
            for name, val in zip(node["outputs"], outs):
                env[name] = val
        names = self.graph.get("outputs") or list(env)
        return {n: env[n] for n in names}

    def _op(self, op, x, a):
        if op == "embedding":
            return [O.embedding(x[0], x[1])]
        if op == "rms_norm":
            return [O.rms_norm(x[0], x[1], a.get("eps", 1e-6))]
        if op == "add_rms_norm":
            n, r = O.add_rms_norm(x[0], x[1], x[2], a.get("eps", 1e-6))
            return [n, r]
        if op == "linear":
            return [O.linear(x[0], x[1], x[2] if len(x) > 2 else None)]
        if op == "linear_silu_mul":
            # weights in 64-row gate/up blocks (dli_export.qwen2.glu_blocked)
            w = np.asarray(x[1], dtype=np.float64)
            inter, k = int(a["intermediate"]), w.shape[-1]
            b = w.reshape(-1, 2, 64, k)
            gate, up = b[:, 0].reshape(-1, k)[:inter], b[:, 1].reshape(-1, k)[:inter]
            return [O.silu_mul(np.concatenate([O.linear(x[0], gate), O.linear(x[0], up)], -1))]
        if op == "silu_mul":
            return [O.silu_mul(x[0])]
        if op == "last_token":
            return [np.asarray(x[0])[:, a.get("index", np.asarray(x[0]).shape[1] - 1)]]
        if op == "argmax":
            return [O.argmax(x[0])]
        if op == "tp_argmax":
            # vocab-parallel greedy pick: every rank's slice, concatenated in rank order
            if self.all_gather is None:
                return [O.argmax(x[0])]
            return [O.argmax(np.concatenate(self.all_gather(np.asarray(x[0], dtype=np.float64)), -1))]
        if op == "all_reduce_add_rms_norm":
            d = x[1] if self.all_reduce is None else self.all_reduce(np.asarray(x[1]))
            n, r = O.add_rms_norm(x[0], d, x[2], a.get("eps", 1e-6))
            return [n, r]
        if op == "linear_all_reduce_add_rms_norm":
            # (residual, x, w, norm weight): the row-split projection, its
            # all-reduce and the residual add + RMSNorm of one Megatron block
            part = O.linear(x[1], x[2], None)
            d = part if self.all_reduce is None else self.all_reduce(np.asarray(part))
            n, r = O.add_rms_norm(x[0], d, x[3], a.get("eps", 1e-6))
            return [n, r]
        if op == "all_reduce":
            return [x[0] if self.all_reduce is None else self.all_reduce(np.asarray(x[0]))]
        if op == "qkv_rotary_cache":
            return [self._qkv_rotary_cache(x, a)]
        if op == "linear_qkv_rotary_cache":
            # (x, wqkv, bqkv, cos, sin, positions): the projection, then rotary + cache write
            return [self._qkv_rotary_cache([O.linear(x[0], x[1], x[2])] + list(x[3:]), a)]
        if op == "attention_kvcache":
            return [self._attention_kvcache(x, a)]
        if op in ("add", "mul", "silu", "relu", "softmax"):
            return [getattr(O, op)(*x)]
        if op == "reshape":
            return [np.asarray(x[0]).reshape(O.reshape_shape(np.asarray(x[0]).shape, a["shape"]))]
        if op == "cast":  # float64 throughout: a dtype change is the identity here
            return [np.asarray(x[0], dtype=np.float64)]
        raise KeyError(f"oracle graph interpreter: unsupported op {op}")

    def _qkv_rotary_cache(self, x, a):
        qkv, cos, sin, pos = (np.asarray(t) for t in x)
        hq, hkv, d, cap = a["q_heads"], a["kv_heads"], a["head_dim"], a["capacity"]
        b, s = qkv.shape[:2]
        t = qkv.astype(np.float64).reshape(b, s, hq + 2 * hkv, d)
        q = t[:, :, :hq].transpose(0, 2, 1, 3)
        k = t[:, :, hq:hq + hkv].transpose(0, 2, 1, 3)
        v = t[:, :, hq + hkv:].transpose(0, 2, 1, 3)
        rq, rk = O.rotary(q, k, cos, sin, positions=pos)
        entry = self.cache.setdefault(a["kv_cache"], {"k": np.zeros((b, hkv, cap, d)),
                                                      "v": np.zeros((b, hkv, cap, d))})
        for i in range(b):
            p = int(pos[i])
            entry["k"][i, :, p:p + s] = rk[i]
            entry["v"][i, :, p:p + s] = v[i]
        return rq.transpose(0, 2, 1, 3)

    def _attention_kvcache(self, x, a):
        q, pos = np.asarray(x[0], dtype=np.float64), np.asarray(x[1])
        entry = self.cache[a["kv_cache"]]
        b, s, hq, d = q.shape
        out = np.zeros((b, s, hq * d))
        for i in range(b):
            n = int(pos[i]) + s
            o = O.attention(q[i:i + 1].transpose(0, 2, 1, 3), entry["k"][i:i + 1, :, :n],
                            entry["v"][i:i + 1, :, :n], causal=True, scale=a.get("scale"))
            out[i] = o[0].transpose(1, 0, 2).reshape(s, hq * d)
        return out
