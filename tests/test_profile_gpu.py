"""dli.ProfileSession on the GPU: per-node CUDA-event times of real runs.

* eager engine runs of a small GQA Qwen2 graph: one event per node per run,
  every node with CUDA tensors timed, the per-node device times adding up to
  no more than the run's own device time between two events around it;
* a decode step captured into a CUDA graph with the markers inside
  (external event-record nodes) and replayed once: every node timed;
* the analyzer summarises the file.
"""
from __future__ import annotations

import json

import pytest
import torch

import dli
from dli import profile as P

pytestmark = pytest.mark.gpu


def _runner():
    from dli.qwen2 import Qwen2Runner
    from dli_export.qwen2 import Qwen2Shape, random_state, transform_weights

    shape = Qwen2Shape(hidden=512, layers=2, q_heads=8, kv_heads=2, head_dim=64, intermediate=1024, vocab=4096)
    st = random_state(shape, device="cuda", dtype=torch.bfloat16, seed=3)
    return Qwen2Runner(shape, transform_weights(st, shape, dtype=torch.bfloat16), capacity=256)


def test_eager_runs_time_every_node(tmp_path):
    runner = _runner()
    nodes = len(runner.graph.node_ops())
    ids = torch.randint(0, 4096, (4, 64), device="cuda")
    runner.prefill(ids)
    prof = dli.ProfileSession(record_shapes=True)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pos = torch.full((4,), 64, dtype=torch.int64, device="cuda")
    ev0.record()
    for step in range(3):
        runner.forward(ids[:, :1].contiguous(), pos + step, profile=prof)
    ev1.record()
    prof.finalize()
    doc = json.loads(prof.to_json())
    P.validate(doc)
    assert len(doc["runs"]) == 3 and all(r["status"] == "ok" for r in doc["runs"])
    assert len(doc["events"]) == 3 * nodes
    assert all(e["gpu_duration_ns"] is not None and e["gpu_duration_ns"] > 0 for e in doc["events"])
    assert all(e["device"] == 0 and e["status"] == "ok" for e in doc["events"])
    total_gpu_ms = sum(e["gpu_duration_ns"] for e in doc["events"]) / 1e6
    assert total_gpu_ms <= ev0.elapsed_time(ev1) * 1.01
    lin = next(e for e in doc["events"] if e["node_name"] == "layers.0.qkv_proj")
    assert lin["shapes"][0].startswith("in:bfloat16@cuda:0[4,1,512]")
    prof.write_json(str(tmp_path / "p.json"))
    summary = P.summarize(P.load(str(tmp_path / "p.json")), group_by="op")
    assert summary["unmeasured"] == 0 and summary["rows"][0]["gpu_ns"]["total"] > 0


def test_captured_decode_step_times_every_node():
    runner = _runner()
    prof = dli.ProfileSession()
    runner.profile_decode_step(4, prof)
    prof.finalize()
    doc = json.loads(prof.to_json())
    assert len(doc["events"]) == len(runner.graph.node_ops())
    assert all(e["gpu_duration_ns"] is not None and e["gpu_duration_ns"] > 0 for e in doc["events"])
