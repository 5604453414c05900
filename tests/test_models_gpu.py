"""GPU parity of two BASELINE model configs end to end, through dli.Engine and
the plugin (not operator by operator):

* config 2, the AlexNet-style CNN at batch 64 (3x32x32 inputs; convs k3 s1 p1
  3->64, pool, 64->192, pool, 192->384, 384->256, 256->256, pool; FC
  4096->4096->4096->10; weights N(0, 0.02)) as a dli.graph.v1 graph of the
  reference's own operator strings (conv2d, relu, max_pool2d, reshape,
  linear), in fp16 (the BASELINE dtype for it) and fp32 (the reference's),
  against the same network in float64 on the CPU. Tolerances as the operator
  tests: fp32 rel <= 1e-4, fp16 rel <= 1e-2 over eight chained layers;
* config 3, the Qwen2-0.5B shape (24 layers, 14/2 heads, D 64, I 4864, vocab
  151936, tied embeddings) with random N(0, 0.02) bf16 weights: prefill and
  teacher-forced decode logits against transformers' Qwen2ForCausalLM (eager,
  fp32, the same bf16-representable weights), bf16 logits rel <= 2e-2 as
  BASELINE states, and greedy ids that agree at least 90% of the time (random
  weights leave near-ties that a 1-ulp difference can flip).
"""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

import dli

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


def test_qwen2_0_5b_config_matches_source_model():
    from transformers import Qwen2Config, Qwen2ForCausalLM

    from dli.qwen2 import Qwen2Runner
    from dli_export.qwen2 import QWEN2_0_5B as shape
    from dli_export.qwen2 import random_state, transform_weights

    dev = torch.device("cuda:0")
    st = random_state(shape, device=dev, dtype=torch.bfloat16, seed=11, std=0.02)
    cfg = Qwen2Config(vocab_size=shape.vocab, hidden_size=shape.hidden, intermediate_size=shape.intermediate,
                      num_hidden_layers=shape.layers, num_attention_heads=shape.q_heads,
                      num_key_value_heads=shape.kv_heads, max_position_embeddings=4096,
                      rms_norm_eps=shape.rms_eps, rope_theta=shape.rope_theta,
                      tie_word_embeddings=shape.tie_embeddings, attn_implementation="eager")
    hf = Qwen2ForCausalLM(cfg).to(dev).float().eval()
    hf.load_state_dict({k: v.float() for k, v in st.items()}, strict=False)
    runner = Qwen2Runner(shape, transform_weights(st, shape, dtype=torch.bfloat16), capacity=256)
    del st

    batch, prompt, steps = 4, 96, 12
    g = torch.Generator(device=dev).manual_seed(5)
    ids = torch.randint(0, shape.vocab, (batch, prompt), device=dev, generator=g)
    logits, nxt = runner.prefill(ids)
    with torch.no_grad():
        ref = hf(ids).logits[:, -1].float()
    worst = ((logits.float() - ref).norm() / ref.norm()).item()
    agree, total = int((nxt == ref.argmax(-1)).sum()), batch
    hf_ids = torch.cat([ids, ref.argmax(-1, keepdim=True)], 1)
    pos = torch.full((batch,), prompt, dtype=torch.int64, device=dev)
    for _ in range(steps):
        logits, nxt = runner.forward(hf_ids[:, -1:].contiguous(), pos)
        with torch.no_grad():
            ref = hf(hf_ids).logits[:, -1].float()
        worst = max(worst, ((logits.float() - ref).norm() / ref.norm()).item())
        agree += int((nxt == ref.argmax(-1)).sum())
        total += batch
        hf_ids = torch.cat([hf_ids, ref.argmax(-1, keepdim=True)], 1)
        pos += 1
    assert worst <= 2e-2, worst
    assert agree / total >= 0.9, (agree, total)
    assert np.isfinite(worst)
