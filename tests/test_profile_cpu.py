"""dli.profile.v1: the native ProfileSession around Engine.run and the analyzer
(dl-inference_b200/python/dli/profile.py), without a GPU.

The reference designs this profiler (.codex/profiling_design.md:141-330 of
dl-inference) but ships none; these tests pin the schema, the error path (a
node that raises is recorded with status "error" and so is its run), the
session's misuse errors, and the analyzer's statistics (nearest-rank
percentiles, CPU and GPU kept apart, --skip-runs) on a synthetic document.
"""
from __future__ import annotations

import csv
import io
import json

import pytest
import torch

import dli
from dli import profile as P


def _doc():
    ev = []
    eid = 0
    for run in range(3):
        for i, (name, op, cpu, gpu) in enumerate([("a", "linear", 10, 100), ("b", "linear", 20, 300),
                                                  ("c", "rms_norm", 5, None)]):
            ev.append({"event_id": eid, "run_id": run, "parent_id": None, "category": "graph_operator",
                       "node_index": i, "node_name": name, "op_type": op, "host_thread_id": 1,
                       "cpu_start_ns": 1000 * run + 10 * i, "cpu_duration_ns": cpu * (run + 1),
                       "gpu_duration_ns": None if gpu is None else gpu * (run + 1),
                       "device": 0, "stream": "0x1", "status": "ok"})
            eid += 1
    return {"schema": "dli.profile.v1", "clock": "steady_clock", "metadata": {"dropped_events": 0},
            "runs": [{"run_id": r, "start_ns": 1000 * r, "duration_ns": 500 + r, "status": "ok"} for r in range(3)],
            "events": ev, "future_field": 1}


def test_summarize_nearest_rank_and_separate_metrics():
    s = P.summarize(_doc(), group_by="node")
    rows = {r["key"][0]: r for r in s["rows"]}
    assert [r["key"][0] for r in s["rows"]][:2] == ["b", "a"]  # sorted by GPU total
    b = rows["b"]
    assert b["count"] == 3 and b["gpu_ns"]["total"] == 300 * 6 and b["cpu_ns"]["total"] == 20 * 6
    assert b["gpu_ns"]["p50"] == 600 and b["gpu_ns"]["p95"] == 900  # nearest rank over [300, 600, 900]
    assert rows["c"]["gpu_unmeasured"] == 3 and rows["c"]["gpu_ns"]["total"] == 0
    assert s["gpu_total_ns"] == 400 * 6 and s["cpu_total_ns"] == 35 * 6  # never added together
    assert abs(rows["b"]["gpu_pct"] - 75.0) < 1e-9
    by_op = P.summarize(_doc(), group_by="op", skip_runs=1)
    lin = next(r for r in by_op["rows"] if r["key"] == ["linear"])
    assert by_op["runs"] == 2 and lin["count"] == 4 and lin["gpu_ns"]["total"] == 400 * 5
    assert "nearest" in P.format_table(s)


def test_compare_export_trace_and_validation(tmp_path):
    before, after = _doc(), _doc()
    for ev in after["events"]:
        if ev["gpu_duration_ns"] is not None:
            ev["gpu_duration_ns"] //= 2
    rows = {tuple(r["key"]): r for r in P.compare(before, after, group_by="op")}
    assert rows[("linear",)]["ratio"] == pytest.approx(0.5)
    buf = io.StringIO()
    P.export_csv(before, buf)
    table = list(csv.reader(io.StringIO(buf.getvalue())))
    assert table[0][3] == "node_name" and len(table) == 1 + 9
    trace = P.chrome_trace(before)
    gpu = [e for e in trace["traceEvents"] if e.get("tid") == 1 and e["ph"] == "X"]
    assert len(gpu) == 6 and gpu[1]["ts"] == pytest.approx(gpu[0]["ts"] + gpu[0]["dur"])  # laid end to end
    path = tmp_path / "p.json"
    path.write_text(json.dumps(before))
    assert P.main(["summarize", str(path), "--json"]) == 0
    assert P.main(["trace", str(path), "-o", str(tmp_path / "t.json")]) == 0
    bad = dict(before, schema="dli.profile.v2")
    with pytest.raises(ValueError, match="schema"):
        P.validate(bad)
    broken = _doc()
    del broken["events"][0]["op_type"]
    with pytest.raises(ValueError, match="lacks"):
        P.validate(broken)


def test_native_session_records_failed_node_and_run():
    g = dli.Graph.from_json(json.dumps({
        "format": "dli.graph.v1", "model_type": "t", "inputs": ["x"], "outputs": ["y"],
        "nodes": [{"name": "view", "op": "reshape", "inputs": ["x"], "outputs": ["y"], "attrs": {"shape": [6]}}]}))
    e = dli.Engine()
    e.load_library(dli.PLUGIN_PATH)
    prof = dli.ProfileSession(gpu=False, record_shapes=True)
    with pytest.raises(ValueError, match="CUDA"):  # the plugin's operators reject host tensors
        e.run(g, {"x": torch.zeros(2, 3)}, profile=prof)
    with pytest.raises(RuntimeError, match="finalize"):
        prof.to_json()
    prof.finalize()
    prof.finalize()  # harmless
    doc = json.loads(prof.to_json())
    P.validate(doc)
    assert doc["runs"][0]["status"] == "error" and len(doc["events"]) == 1
    ev = doc["events"][0]
    assert ev["status"] == "error" and ev["gpu_duration_ns"] is None and ev["device"] is None
    assert ev["node_name"] == "view" and ev["op_type"] == "reshape" and ev["cpu_duration_ns"] >= 0
    assert ev["shapes"] == ["in:float32@cpu[2,3]"]
    with pytest.raises(RuntimeError, match="finalized"):
        e.run(g, {"x": torch.zeros(2, 3)}, profile=prof)
