"""The AlexNet-style CNN of the benchmark configurations as a dli.graph.v1 graph.

Batch of 3x32x32 images; convolutions k3 s1 p1 3->64, ReLU, max-pool 2;
64->192, ReLU, pool; 192->384, ReLU; 384->256, ReLU; 256->256, ReLU, pool;
flatten 4096; linear 4096->4096, ReLU; 4096->4096, ReLU; 4096->10. The graph
uses only the reference's own operator strings (conv2d, relu, max_pool2d,
reshape, linear), as the reference's FX exporter would emit them
(python/dli_export/export.py:54-206), so the same graph runs on the reference
plugin where it has specialisations. Weights are random N(0, 0.02).
"""
from __future__ import annotations

from typing import Any

import torch

CONVS = [(3, 64, True), (64, 192, True), (192, 384, False), (384, 256, False), (256, 256, True)]
FCS = [(4096, 4096, True), (4096, 4096, True), (4096, 10, False)]


def alexnet_graph(batch: int = 64) -> tuple[dict[str, Any], str]:
    """(graph dict, name of its output) for `batch` images."""
    nodes: list[dict[str, Any]] = []
    x = "x"

    def node(op, inputs, attrs=None):
        nonlocal x
        out = f"t{len(nodes)}"
        nodes.append({"name": out, "op": op, "inputs": inputs, "outputs": [out], "attrs": attrs or {}})
        x = out

    for i, (_, _, pool) in enumerate(CONVS):
        node("conv2d", [x, f"conv{i}.w", f"conv{i}.b"], {"stride": [1, 1], "padding": [1, 1]})
        node("relu", [x])
        if pool:
            node("max_pool2d", [x], {"kernel_size": [2, 2], "stride": [2, 2]})
    node("reshape", [x], {"shape": [batch, 4096]})
    for i, (_, _, act) in enumerate(FCS):
        node("linear", [x, f"fc{i}.w", f"fc{i}.b"])
        if act:
            node("relu", [x])
    return {"format": "dli.graph.v1", "model_type": "alexnet_style", "inputs": ["x"], "outputs": [x],
            "nodes": nodes}, x


def alexnet_params(dtype=torch.float16, batch: int = 64, seed: int = 0, device="cpu"):
    """(weights dict, input batch) with N(0, 0.02) weights and N(0, 1) images."""
    g = torch.Generator(device=device).manual_seed(seed)
    p = {}
    for i, (c, oc, _) in enumerate(CONVS):
        p[f"conv{i}.w"] = (torch.randn(oc, c, 3, 3, generator=g, device=device) * 0.02).to(dtype)
        p[f"conv{i}.b"] = (torch.randn(oc, generator=g, device=device) * 0.02).to(dtype)
    for i, (k, n, _) in enumerate(FCS):
        p[f"fc{i}.w"] = (torch.randn(n, k, generator=g, device=device) * 0.02).to(dtype)
        p[f"fc{i}.b"] = (torch.randn(n, generator=g, device=device) * 0.02).to(dtype)
    x = torch.randn(batch, 3, 32, 32, generator=g, device=device).to(dtype)
    return p, x


def alexnet_forward(p, x):
    """The same network in PyTorch eager (the CPU baseline and the test reference)."""
    F = torch.nn.functional
    h = x
    for i, (_, _, pool) in enumerate(CONVS):
        h = F.relu(F.conv2d(h, p[f"conv{i}.w"], p[f"conv{i}.b"], padding=1))
        if pool:
            h = F.max_pool2d(h, 2)
    h = h.reshape(x.shape[0], 4096)
    for i, (_, _, act) in enumerate(FCS):
        h = F.linear(h, p[f"fc{i}.w"], p[f"fc{i}.b"])
        if act:
            h = F.relu(h)
    return h


def alexnet_flops(batch: int = 64) -> float:
    """Multiply-add FLOPs of one forward (2 per MAC; pooling and ReLU excluded)."""
    flops, hw = 0.0, 32
    for c, oc, pool in CONVS:
        flops += 2.0 * batch * oc * hw * hw * c * 9
        if pool:
            hw //= 2
    for k, n, _ in FCS:
        flops += 2.0 * batch * k * n
    return flops
