"""CPU tests of the host runtime (C++ core behind `import dli`): graph JSON
round trip and attribute typing, operator registry and plugin loading errors,
engine input validation, weights manifest loading. Mirrors the reference's
tests/cpp/test_{graph,operator_registry,engine,weights}.cc contracts."""
from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

import dli

REFERENCE_OPS = ["embedding", "rms_norm", "linear", "matmul", "add", "mul", "relu", "silu", "max_pool2d",
                 "softmax", "reshape", "transpose", "conv2d", "attention", "rotary_embedding",
                 "batch_norm2d"]


def graph_json(nodes, inputs=("x",), outputs=("y",)):
    return json.dumps({"format": "dli.graph.v1", "model_type": "t", "inputs": list(inputs),
                       "outputs": list(outputs), "nodes": nodes})


def test_graph_round_trip_and_attribute_types():
    src = graph_json([{"name": "n", "op_type": "reshape", "inputs": ["x"], "outputs": ["y"],
                       "attrs": {"shape": [2, -1], "eps": 1e-6, "causal": True, "kv_cache": "layer_0",
                                 "mixed": [1, 2.5], "names": ["a", "b"], "empty": []}}])
    g = dli.Graph.from_json(src)
    assert g.format == "dli.graph.v1" and g.model_type == "t"
    assert g.node_ops() == ["reshape"]
    again = dli.Graph.from_json(g.to_json())
    assert again.to_json() == g.to_json()
    attrs = json.loads(g.to_json())["nodes"][0]["attrs"]
    assert attrs["shape"] == [2, -1] and attrs["mixed"] == [1.0, 2.5] and attrs["causal"] is True
    assert attrs["names"] == ["a", "b"] and attrs["empty"] == [] and attrs["eps"] == 1e-6


def test_graph_rejects_bad_documents():
    with pytest.raises(ValueError):
        dli.Graph.from_json('{"format": "dli.graph.v2", "nodes": []}')
    with pytest.raises(ValueError):
        dli.Graph.from_json('{"format": "dli.graph.v1"}')
    with pytest.raises(ValueError):
        dli.Graph.from_json('{"format": "dli.graph.v1", "nodes": [{"name": "a"}]}')
    with pytest.raises(ValueError):
        dli.Graph.from_json('{"nodes": [}')


def test_registry_before_and_after_plugin_load():
    e = dli.Engine()
    for op in REFERENCE_OPS:
        assert not e.has_operator(op)
    e.load_library(dli.PLUGIN_PATH)
    for op in REFERENCE_OPS:
        assert e.has_operator(op), op
    assert e.has_operator("all_reduce")


def test_reference_plugin_file_name_alias_registers_the_same_ops():
    alias = Path(dli.PLUGIN_PATH).with_name("libdli_triton_aot_ops.so")
    e = dli.Engine()
    e.load_library(str(alias))
    assert sorted(e.registered_operators()) == sorted(dli.Engine().load_library(dli.PLUGIN_PATH)
                                                      .registered_operators())


def test_plugin_load_errors(tmp_path):
    e = dli.Engine()
    with pytest.raises(RuntimeError, match="failed to load operator library"):
        e.load_library(str(tmp_path / "missing.so"))
    # a real shared object without the registration symbol
    core = Path(dli.PLUGIN_PATH).with_name("libdli_sm100.so")
    with pytest.raises(RuntimeError, match="missing dli_register_operators"):
        e.load_library(str(core))


def test_engine_reports_missing_input_and_unknown_op():
    e = dli.Engine()
    e.load_library(dli.PLUGIN_PATH)
    g = dli.Graph.from_json(graph_json([{"name": "n", "op": "relu", "inputs": ["nope"], "outputs": ["y"]}]))
    with pytest.raises(ValueError, match="missing input tensor: nope"):
        e.run(g, {"x": torch.zeros(2)})
    g2 = dli.Graph.from_json(graph_json([{"name": "n", "op": "frobnicate", "inputs": ["x"], "outputs": ["y"]}]))
    with pytest.raises(ValueError, match="not registered"):
        e.run(g2, {"x": torch.zeros(2)})


def test_operators_reject_host_tensors_like_the_reference():
    e = dli.Engine()
    e.load_library(dli.PLUGIN_PATH)
    g = dli.Graph.from_json(graph_json([{"name": "n", "op": "relu", "inputs": ["x"], "outputs": ["y"]}]))
    with pytest.raises(ValueError, match="expects CUDA tensors"):
        e.run(g, {"x": torch.zeros(2)})


def test_load_weights_manifest(tmp_path):
    from dli_export.qwen2 import write_weights

    tensors = {"a": torch.arange(6, dtype=torch.float32).reshape(2, 3),
               "b": torch.tensor([1, 2, 3], dtype=torch.int64),
               "c": torch.randn(4, 4).to(torch.bfloat16), "d": torch.randn(3).half()}
    path = write_weights(tensors, tmp_path, "w")
    loaded = dli.load_weights(str(path), "cpu")
    assert set(loaded) == set(tensors)
    for k, v in tensors.items():
        assert loaded[k].dtype == v.dtype and torch.equal(loaded[k], v)
    manifest = json.loads(path.read_text())
    manifest["tensors"]["a"]["nbytes"] = 8
    bad = tmp_path / "bad.json"
    bad.write_text(json.dumps(manifest))
    with pytest.raises(ValueError, match="byte count"):
        dli.load_weights(str(bad), "cpu")
