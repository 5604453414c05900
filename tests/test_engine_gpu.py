"""GPU tests through the reference-facing boundary: dli.Engine + the dlopen'ed
plugin (libdli_sm100_ops.so) running dli.graph.v1 graphs.

* every golden case as a one-node graph, the way the reference's operator tests
  drive their runner (tests/operators/operator_test_support.py:108-137);
* attention with a `kv_cache` attribute over several runs at B*H > 1;
* a tiny GQA Qwen2 exported by dli_export.qwen2, checked against the source
  model (transformers Qwen2ForCausalLM, eager attention, fp32) on the same
  bf16-representable weights: last-token logits rel-err <= 2e-2 (bf16 bound)
  and teacher-forced greedy-token agreement.
"""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

import dli
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


def _tiny_hf(shape, device):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(vocab_size=shape.vocab, hidden_size=shape.hidden,
                      intermediate_size=shape.intermediate, num_hidden_layers=shape.layers,
                      num_attention_heads=shape.q_heads, num_key_value_heads=shape.kv_heads,
                      max_position_embeddings=4096, rms_norm_eps=shape.rms_eps,
                      rope_theta=shape.rope_theta, tie_word_embeddings=shape.tie_embeddings,
                      attn_implementation="eager")
    return Qwen2ForCausalLM(cfg).to(device).float().eval()


@pytest.mark.parametrize("batch,prompt,steps", [(2, 37, 24), (4, 128, 16)])
def test_tiny_qwen2_matches_source_model(batch, prompt, steps):
    from dli.qwen2 import Qwen2Runner
    from dli_export.qwen2 import Qwen2Shape, random_state, transform_weights

    shape = Qwen2Shape(hidden=512, layers=2, q_heads=8, kv_heads=2, head_dim=64, intermediate=1024,
                       vocab=4096)
    dev = torch.device("cuda:0")
    st = random_state(shape, device=dev, dtype=torch.bfloat16, seed=7, std=0.05)
    hf = _tiny_hf(shape, dev)
    hf.load_state_dict({k: v.float() for k, v in st.items()}, strict=False)
    runner = Qwen2Runner(shape, transform_weights(st, shape, dtype=torch.bfloat16), capacity=512)

    g = torch.Generator(device=dev).manual_seed(1)
    ids = torch.randint(0, shape.vocab, (batch, prompt), device=dev, generator=g)
    logits, nxt = runner.prefill(ids)
    with torch.no_grad():
        ref = hf(ids).logits[:, -1].float()
    rel = ((logits.float() - ref).norm() / ref.norm()).item()
    assert rel < 2e-2, rel

    # teacher-forced decode: both models see the source model's greedy tokens
    agree, total = int((nxt == ref.argmax(-1)).sum()), batch
    hf_ids = torch.cat([ids, ref.argmax(-1, keepdim=True)], 1)
    pos = torch.full((batch,), prompt, dtype=torch.int64, device=dev)
    worst = rel
    for _ in range(steps):
        logits, nxt = runner.forward(hf_ids[:, -1:].contiguous(), pos)
        with torch.no_grad():
            ref = hf(hf_ids).logits[:, -1].float()
        worst = max(worst, ((logits.float() - ref).norm() / ref.norm()).item())
        agree += int((nxt == ref.argmax(-1)).sum())
        total += batch
        hf_ids = torch.cat([hf_ids, ref.argmax(-1, keepdim=True)], 1)
        pos += 1
    assert worst < 2e-2, worst
    assert agree / total >= 0.9, (agree, total)

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
