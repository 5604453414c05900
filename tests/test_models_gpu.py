"""GPU parity of the benchmark's model configurations end to end, through
dli.Engine and the plugin (not operator by operator):

* the AlexNet-style CNN at batch 64 (3x32x32 inputs; convs k3 s1 p1
  3->64, pool, 64->192, pool, 192->384, 384->256, 256->256, pool; FC
  4096->4096->4096->10; weights N(0, 0.02)) as a dli.graph.v1 graph of the
  reference's own operator strings (conv2d, relu, max_pool2d, reshape,
  linear), in fp16 (its benchmark dtype) and fp32 (the reference's),
  against the same network in float64 on the CPU. Tolerances as the operator
  tests: fp32 rel <= 1e-4, fp16 rel <= 1e-2 over eight chained layers;
* the Qwen2 configurations against transformers' Qwen2ForCausalLM (eager,
  fp32, the same bf16-representable random N(0, 0.02) weights), teacher-forced
  through 256 CUDA-graph decode steps (tests/model_parity.py states the
  criteria):
  - the Qwen2-0.5B shape (24 layers, 14/2 heads, D 64, I 4864, vocab 151936,
    tied embeddings) at its workload's batch 8 and 512-token prompts: logits
    rel <= 2e-2 at every step, >= 99% greedy agreement over positions that are
    not near-ties;
  - the Qwen2-7B shape (28 layers, 28/4 heads, D 128, I 18944) at batch 4: at
    least as close to the fp32 source model as the source model run in bf16.
"""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

import dli
import model_parity

pytestmark = pytest.mark.gpu

CONVS = [(3, 64, True), (64, 192, True), (192, 384, False), (384, 256, False), (256, 256, True)]
FCS = [(4096, 4096, True), (4096, 4096, True), (4096, 10, False)]


def _alexnet_graph():
    nodes, x = [], "x"

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
    node("reshape", [x], {"shape": [64, 4096]})
    for i, (_, _, act) in enumerate(FCS):
        node("linear", [x, f"fc{i}.w", f"fc{i}.b"])
        if act:
            node("relu", [x])
    return {"format": "dli.graph.v1", "model_type": "alexnet_style", "inputs": ["x"], "outputs": [x],
            "nodes": nodes}, x


def _alexnet_params(dtype):
    g = torch.Generator().manual_seed(0)
    p = {}
    for i, (c, oc, _) in enumerate(CONVS):
        p[f"conv{i}.w"] = (torch.randn(oc, c, 3, 3, generator=g) * 0.02).to(dtype)
        p[f"conv{i}.b"] = (torch.randn(oc, generator=g) * 0.02).to(dtype)
    for i, (k, n, _) in enumerate(FCS):
        p[f"fc{i}.w"] = (torch.randn(n, k, generator=g) * 0.02).to(dtype)
        p[f"fc{i}.b"] = (torch.randn(n, generator=g) * 0.02).to(dtype)
    x = torch.randn(64, 3, 32, 32, generator=g).to(dtype)
    return p, x


def _alexnet_reference(p, x):
    F = torch.nn.functional
    h = x.double()
    for i, (_, _, pool) in enumerate(CONVS):
        h = F.relu(F.conv2d(h, p[f"conv{i}.w"].double(), p[f"conv{i}.b"].double(), padding=1))
        if pool:
            h = F.max_pool2d(h, 2)
    h = h.reshape(64, 4096)
    for i, (_, _, act) in enumerate(FCS):
        h = F.linear(h, p[f"fc{i}.w"].double(), p[f"fc{i}.b"].double())
        if act:
            h = F.relu(h)
    return h


@pytest.mark.parametrize("dtype,tol", [(torch.float16, 1e-2), (torch.float32, 1e-4)], ids=["f16", "f32"])
def test_alexnet_config_through_engine(dtype, tol):
    graph, out_name = _alexnet_graph()
    p, x = _alexnet_params(dtype)
    ref = _alexnet_reference(p, x)
    e = dli.Engine()
    e.load_library(dli.PLUGIN_PATH)
    inputs = {k: v.cuda() for k, v in p.items()}
    inputs["x"] = x.cuda()
    g = dli.Graph.from_json(json.dumps(graph))
    out = e.run(g, inputs)[out_name]
    again = e.run(g, inputs)[out_name]  # second run through the cached plan
    torch.cuda.synchronize()
    got = out.double().cpu()
    assert got.shape == (64, 10)
    rel = ((got - ref).norm() / ref.norm()).item()
    assert rel <= tol, rel
    assert torch.equal(out, again)


def _qwen2_parity(shape, batch, prompt, steps, seed, name, vs_bf16):
    from dli.qwen2 import Qwen2Runner
    from dli_export.qwen2 import random_state, transform_weights

    dev = torch.device("cuda:0")
    st = random_state(shape, device=dev, dtype=torch.bfloat16, seed=seed, std=0.02)
    hf = model_parity.hf_model(shape, dev, st)
    hf_bf16 = model_parity.hf_model(shape, dev, st, dtype=torch.bfloat16)
    runner = Qwen2Runner(shape, transform_weights(st, shape, dtype=torch.bfloat16),
                         capacity=prompt + steps + 64)
    del st
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    ids = torch.randint(0, shape.vocab, (batch, prompt), device=dev, generator=g)
    stats = model_parity.teacher_forced(runner, hf, ids, steps, hf_bf16=hf_bf16)
    model_parity.report(name, stats)
    runner.release_graphs()
    del hf, hf_bf16, runner
    torch.cuda.empty_cache()
    if vs_bf16:
        model_parity.check_vs_bf16_eager(stats)
    else:
        model_parity.check_absolute(stats)
    assert np.isfinite(stats["max_logits_rel_err"])


def test_qwen2_0_5b_config_matches_source_model():
    """The 0.5B configuration exactly: batch 8, 512-token prompts, 256 greedy
    steps, held to the absolute tolerances (logits rel-err <= 2e-2 at every step,
    >= 99% decidable greedy agreement)."""
    from dli_export.qwen2 import QWEN2_0_5B

    _qwen2_parity(QWEN2_0_5B, batch=8, prompt=512, steps=256, seed=11, name="qwen2-0.5b b8 s512 +256",
                  vs_bf16=False)


def test_qwen2_7b_shape_matches_source_model():
    """The benchmarked 7B shape, all 28 layers: batch 4, 512-token prompts, 256
    steps. With random weights this model turns a 2^-9 change of its input into
    ~2.5% of its logits, so the bf16 bound is out of reach for any bf16
    implementation; the engine must be at least as faithful to the fp32 source
    model as the source model run eagerly in bf16 (tests/model_parity.py)."""
    from dli_export.qwen2 import QWEN2_7B

    _qwen2_parity(QWEN2_7B, batch=4, prompt=512, steps=256, seed=21, name="qwen2-7b b4 s512 +256",
                  vs_bf16=True)
