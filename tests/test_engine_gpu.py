"""GPU tests through the reference-facing boundary: dli.Engine + the dlopen'ed
plugin (libdli_sm100_ops.so) running dli.graph.v1 graphs.

* every golden case as a one-node graph, the way the reference's operator tests
  drive their runner (tests/operators/operator_test_support.py:108-137);
* attention with a `kv_cache` attribute over several runs at B*H > 1;
* a tiny GQA Qwen2 exported by dli_export.qwen2, checked against the source
  model (transformers Qwen2ForCausalLM, eager attention, fp32) on the same
  bf16-representable weights, teacher-forced through CUDA-graph decode steps
  with the criteria of tests/model_parity.py.
"""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

import dli
import model_parity
from golden_io import all_cases
from op_cases import oracle_outputs
from oracle import ops as O

pytestmark = pytest.mark.gpu

CASES = list(all_cases())


def engine():
    e = dli.Engine()
    e.load_library(dli.PLUGIN_PATH)
    return e


def one_node(op, inputs, outputs, attrs):
    return dli.Graph.from_json(json.dumps({
        "format": "dli.graph.v1", "model_type": "operator_numeric_test", "inputs": list(inputs),
        "outputs": list(outputs),
        "nodes": [{"name": op, "op": op, "inputs": list(inputs), "outputs": list(outputs),
                   "attrs": attrs}]}))


@pytest.mark.parametrize("op,idx,case", CASES, ids=[f"{op}-{i}" for op, i, _ in CASES])
def test_golden_case_through_engine(op, idx, case):
    outs = list(case["outputs"])
    g = one_node(op, case["inputs"], outs, case["attrs"])
    inputs = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in case["inputs"].items()}
    got = engine().run(g, inputs)
    want = oracle_outputs(op, case["inputs"], case["attrs"])
    for name in outs:
        ref = want[name]
        res = got[name].cpu().double().numpy()
        assert res.shape == tuple(np.asarray(ref).shape)
        np.testing.assert_allclose(res, ref, rtol=1e-4, atol=1e-5, err_msg=f"{op}[{idx}].{name}")
        if case["expected"].get(name) is not None:  # the reference test's own expected tensor
            np.testing.assert_allclose(res, case["expected"][name], rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_attention_kv_cache_attr_multi_step(dtype):
    """Reference contract (attention/template.cc:10-18): append k/v to the named cache,
    then attend over all cached rows, bottom-right causal. B*H > 1 across 3 runs."""
    e = engine()
    g = one_node("attention", ["q", "k", "v"], ["out"], {"causal": True, "kv_cache": "layer_0"})
    rng = torch.Generator().manual_seed(0)
    b, h, d = 2, 4, 64
    ks, vs = [], []
    for step, s in enumerate((5, 1, 3)):
        q = torch.randn(b, h, s, d, generator=rng)
        k = torch.randn(b, h, s, d, generator=rng)
        v = torch.randn(b, h, s, d, generator=rng)
        ks.append(k)
        vs.append(v)
        out = e.run(g, {"q": q.to(dtype).cuda(), "k": k.to(dtype).cuda(), "v": v.to(dtype).cuda()})["out"]
        kc = torch.cat(ks, 2).to(dtype).double()
        vc = torch.cat(vs, 2).to(dtype).double()
        ref = O.attention(q.to(dtype).double().numpy(), kc.numpy(), vc.numpy(), causal=True)
        err = np.linalg.norm(out.cpu().double().numpy() - ref) / np.linalg.norm(ref)
        assert err < (1e-5 if dtype == torch.float32 else 1.5e-2), (step, err)
    assert e.kv_cache_length("layer_0") == 9


@pytest.mark.parametrize("batch,prompt,steps", [(2, 37, 64), (4, 128, 256)])
def test_tiny_qwen2_matches_source_model(batch, prompt, steps):
    from dli.qwen2 import Qwen2Runner
    from dli_export.qwen2 import Qwen2Shape, random_state, transform_weights

    shape = Qwen2Shape(hidden=512, layers=2, q_heads=8, kv_heads=2, head_dim=64, intermediate=1024,
                       vocab=4096)
    dev = torch.device("cuda:0")
    st = random_state(shape, device=dev, dtype=torch.bfloat16, seed=7, std=0.05)
    hf = model_parity.hf_model(shape, dev, st)
    runner = Qwen2Runner(shape, transform_weights(st, shape, dtype=torch.bfloat16), capacity=512)

    g = torch.Generator(device=dev).manual_seed(1)
    ids = torch.randint(0, shape.vocab, (batch, prompt), device=dev, generator=g)
    stats = model_parity.teacher_forced(runner, hf, ids, steps)
    model_parity.report(f"tiny qwen2 b{batch} s{prompt} +{steps}", stats)
    model_parity.check(stats)

    # CUDA-graph decode reproduces eager engine decode exactly
    runner.reset()
    out_graph = runner.generate(ids, 8, use_graph=True)
    out_eager = runner.generate(ids, 8, use_graph=False)
    assert torch.equal(out_graph, out_eager)


def test_exported_files_run_through_load_weights(tmp_path):
    from dli_export.qwen2 import Qwen2Shape, export_qwen2, random_state

    shape = Qwen2Shape(hidden=256, layers=1, q_heads=4, kv_heads=2, head_dim=64, intermediate=512,
                       vocab=1000)
    st = random_state(shape, dtype=torch.bfloat16, seed=2)
    gpath, wpath = export_qwen2(st, tmp_path, "q", shape=shape, capacity=128)
    e = engine()
    inputs = dli.load_weights(str(wpath), "cuda")
    inputs["input_ids"] = torch.randint(0, 1000, (3, 9), device="cuda")
    inputs["positions"] = torch.zeros(3, dtype=torch.int64, device="cuda")
    out = e.run(dli.Graph.from_json_file(str(gpath)), inputs)
    assert out["logits"].shape == (3, 1000) and out["next_ids"].shape == (3,)
    assert torch.equal(out["next_ids"], out["logits"].float().argmax(-1))


def test_load_weights_to_device_matches_host_copy(tmp_path):
    """The device loader (mapped file -> pinned staging ring -> device) gives the
    bytes the host loader gives, for tensors larger than one staging chunk (the
    ring wraps several times) and for small and empty ones."""
    from dli_export.qwen2 import write_weights

    g = torch.Generator().manual_seed(4)
    tensors = {"big": torch.randn(9, 1 << 22, generator=g).to(torch.bfloat16),   # 72 MB
               "mid": torch.randn(3000, 777, generator=g),
               "ids": torch.arange(17, dtype=torch.int64),
               "empty": torch.zeros(0, 8),
               "half": torch.randn(5, 3, generator=g).half()}
    path = write_weights(tensors, tmp_path, "w")
    on_host = dli.load_weights(str(path), "cpu")
    on_dev = dli.load_weights(str(path), "cuda")
    assert set(on_dev) == set(tensors)
    for name, t in tensors.items():
        d = on_dev[name]
        assert d.is_cuda and d.dtype == t.dtype and d.shape == t.shape, name
        assert torch.equal(d.cpu(), on_host[name]) and torch.equal(d.cpu(), t), name
