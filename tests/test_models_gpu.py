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

def _alexnet_graph():
    from dli_export.cnn import alexnet_graph

    return alexnet_graph(64)


def _alexnet_params(dtype):
    from dli_export.cnn import alexnet_params

    return alexnet_params(dtype, 64, seed=0)


def _alexnet_reference(p, x):
    from dli_export.cnn import alexnet_forward

    return alexnet_forward({k: v.double() for k, v in p.items()}, x.double())


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
