"""Maps a golden case (op name, named inputs, attrs) onto the oracle and onto the
C-ABI wrappers, so one fixture drives both the CPU oracle pin and the GPU
parity test."""
from __future__ import annotations

import numpy as np

from oracle import ops as O


def oracle_outputs(op: str, inp: dict, attrs: dict) -> dict[str, np.ndarray]:
    if op == "linear":
        return {"output": O.linear(inp["x"], inp["weight"], inp.get("bias"))}
    if op == "matmul":
        return {"output": O.matmul(inp["a"], inp["b"])}
    if op == "rms_norm":
        return {"output": O.rms_norm(inp["x"], inp["weight"], attrs.get("eps", 1e-6))}
    if op == "rotary_embedding":
        q, k = O.rotary(inp["q"], inp["k"], inp["cos"], inp["sin"], attrs.get("start_pos", 0))
        return {"out_q": q, "out_k": k}
    if op == "attention":
        return {"output": O.attention(inp["q"], inp["k"], inp["v"], attrs.get("causal", False))}
    if op == "embedding":
        return {"output": O.embedding(inp["ids"], inp["table"])}
    if op in ("add", "mul"):
        a, b = list(inp.values())
        return {"output": getattr(O, op)(a, b)}
    if op in ("silu", "relu", "softmax"):
        return {"output": getattr(O, op)(inp["x"])}
    if op == "max_pool2d":
        return {"output": O.max_pool2d(inp["x"], attrs.get("kernel_size", [2, 2]),
                                       attrs.get("stride"), attrs.get("padding", [0, 0]))}
    if op == "batch_norm2d":
        return {"output": O.batch_norm2d(inp["x"], inp["weight"], inp["bias"], inp["running_mean"],
                                         inp["running_var"], attrs.get("eps", 1e-5))}
    if op == "transpose":
        return {"output": O.transpose2d(inp["x"])}
    if op == "conv2d":
        return {"output": O.conv2d(inp["x"], inp["weight"], inp.get("bias"),
                                   attrs.get("stride", [1, 1]), attrs.get("padding", [0, 0]))}
    if op == "reshape":
        x = np.asarray(inp["x"])
        return {"output": x.reshape(O.reshape_shape(x.shape, attrs["shape"]))}
    raise KeyError(op)


def capi_outputs(op: str, inp: dict, attrs: dict, dtype) -> dict:
    """Runs the op through libdli_sm100.so on cuda:0 with float inputs cast to `dtype`."""
    import torch

    import dli_sm100 as C

    def t(name):
        a = inp[name]
        x = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        return x.to(dtype) if x.is_floating_point() else x

    if op == "linear":
        return {"output": C.linear(t("x"), t("weight"), t("bias") if "bias" in inp else None)}
    if op == "matmul":
        return {"output": C.matmul(t("a"), t("b"))}
    if op == "rms_norm":
        return {"output": C.rms_norm(t("x"), t("weight"), float(attrs.get("eps", 1e-6)))}
    if op == "rotary_embedding":
        cos = torch.from_numpy(inp["cos"]).cuda().float()
        sin = torch.from_numpy(inp["sin"]).cuda().float()
        q, k = C.rotary_embedding(t("q"), t("k"), cos, sin, int(attrs.get("start_pos", 0)))
        return {"out_q": q, "out_k": k}
    if op == "attention":
        return {"output": C.attention(t("q"), t("k"), t("v"), bool(attrs.get("causal", False)))}
    if op == "embedding":
        return {"output": C.embedding(t("ids"), t("table"))}
    if op in ("add", "mul"):
        a, b = list(inp)
        return {"output": getattr(C, op)(t(a), t(b))}
    if op in ("silu", "relu", "softmax"):
        return {"output": getattr(C, op)(t("x"))}
    if op == "max_pool2d":
        return {"output": C.max_pool2d(t("x"), tuple(attrs.get("kernel_size", [2, 2])),
                                       tuple(attrs["stride"]) if "stride" in attrs else None,
                                       tuple(attrs.get("padding", [0, 0])))}
    if op == "batch_norm2d":
        return {"output": C.batch_norm2d(t("x"), t("weight"), t("bias"), t("running_mean"),
                                         t("running_var"), float(attrs.get("eps", 1e-5)))}
    if op == "transpose":
        return {"output": C.transpose2d(t("x"))}
    if op == "conv2d":
        return {"output": C.conv2d(t("x"), t("weight"), t("bias") if "bias" in inp else None,
                                   tuple(attrs.get("stride", [1, 1])),
                                   tuple(attrs.get("padding", [0, 0])))}
    if op == "reshape":
        return {"output": t("x").reshape(O.reshape_shape(inp["x"].shape, attrs["shape"]))}
    raise KeyError(op)
