"""Analyzer for ``dli.profile.v1`` files written by ``dli.ProfileSession``.

    python -m dli.profile summarize profile.json [--group-by node|op] [--skip-runs N] [--json]
    python -m dli.profile compare before.json after.json [--group-by node|op] [--skip-runs N]
    python -m dli.profile export profile.json --format csv -o profile.csv
    python -m dli.profile trace profile.json -o trace.json

The command set and the rules follow the reference's profiling design
(.codex/profiling_design.md:272-330 of dl-inference): CPU submit time and GPU
execution time are separate metrics and never added; percentiles are
nearest-rank; the table sorts by GPU total when GPU samples exist, otherwise by
CPU total; ``--skip-runs`` drops warm-up runs from the statistics without
changing the file. The trace is Chrome/Perfetto JSON: host spans on one track,
and per run the GPU spans laid end to end on another (CUDA events give device
durations and stream order, not host-aligned start times). Only the standard
library is used; unknown fields are ignored, a missing required field or
another schema is an error.
"""
from __future__ import annotations

import argparse
import csv
import json
import math
import sys
from collections import OrderedDict

SCHEMA = "dli.profile.v1"
_REQUIRED_EVENT = ("event_id", "run_id", "node_index", "node_name", "op_type", "cpu_duration_ns",
                   "gpu_duration_ns", "status")


def load(path: str) -> dict:
    with open(path) as f:
        doc = json.load(f)
    validate(doc)
    return doc


def validate(doc: dict) -> None:
    if doc.get("schema") != SCHEMA:
        raise ValueError(f"not a {SCHEMA} document: schema={doc.get('schema')!r}")
    for key in ("runs", "events", "metadata"):
        if key not in doc:
            raise ValueError(f"{SCHEMA}: missing '{key}'")
    for ev in doc["events"]:
        missing = [k for k in _REQUIRED_EVENT if k not in ev]
        if missing:
            raise ValueError(f"{SCHEMA}: event {ev.get('event_id')} lacks {missing}")


def percentile(sorted_vals: list, q: float):
    """Nearest-rank percentile of an ascending list (None when empty)."""
    if not sorted_vals:
        return None
    rank = max(1, math.ceil(q / 100.0 * len(sorted_vals)))
    return sorted_vals[rank - 1]


def _stats(vals: list) -> dict:
    vals = sorted(vals)
    if not vals:
        return {"total": 0, "mean": None, "p50": None, "p95": None, "max": None}
    return {"total": sum(vals), "mean": sum(vals) / len(vals), "p50": percentile(vals, 50),
            "p95": percentile(vals, 95), "max": vals[-1]}


def summarize(doc: dict, group_by: str = "node", skip_runs: int = 0) -> dict:
    runs = [r for r in doc["runs"] if r["run_id"] >= skip_runs]
    keep = {r["run_id"] for r in runs}
    groups: "OrderedDict[tuple, dict]" = OrderedDict()
    failed = unmeasured = 0
    for ev in doc["events"]:
        if ev["run_id"] not in keep or ev.get("category", "graph_operator") != "graph_operator":
            continue
        key = (ev["node_name"], ev["op_type"]) if group_by == "node" else (ev["op_type"],)
        g = groups.setdefault(key, {"count": 0, "cpu": [], "gpu": [], "gpu_unmeasured": 0, "failed": 0})
        g["count"] += 1
        if ev["cpu_duration_ns"] is not None:
            g["cpu"].append(ev["cpu_duration_ns"])
        if ev["gpu_duration_ns"] is not None:
            g["gpu"].append(ev["gpu_duration_ns"])
        elif ev.get("device") is not None:
            g["gpu_unmeasured"] += 1
            unmeasured += 1
        if ev["status"] != "ok":
            g["failed"] += 1
            failed += 1
    cpu_all = sum(sum(g["cpu"]) for g in groups.values())
    gpu_all = sum(sum(g["gpu"]) for g in groups.values())
    rows = []
    for key, g in groups.items():
        cpu, gpu = _stats(g["cpu"]), _stats(g["gpu"])
        rows.append({"key": list(key), "count": g["count"], "cpu_ns": cpu, "gpu_ns": gpu,
                     "cpu_pct": 100.0 * cpu["total"] / cpu_all if cpu_all else None,
                     "gpu_pct": 100.0 * gpu["total"] / gpu_all if gpu_all else None,
                     "gpu_unmeasured": g["gpu_unmeasured"], "failed": g["failed"]})
    rows.sort(key=lambda r: -(r["gpu_ns"]["total"] if gpu_all else r["cpu_ns"]["total"]))
    walls = _stats([r["duration_ns"] for r in runs])
    return {"group_by": group_by, "runs": len(runs), "skipped_runs": skip_runs, "rows": rows,
            "cpu_total_ns": cpu_all, "gpu_total_ns": gpu_all, "run_wall_ns": walls,
            "unmeasured": unmeasured, "failed": failed,
            "dropped": doc["metadata"].get("dropped_events", 0), "percentiles": "nearest-rank"}


def _fmt(ns) -> str:
    return "-" if ns is None else f"{ns / 1e3:10.1f}"


def format_table(summary: dict) -> str:
    head = (f"{'operator':48s} {'n':>5s} {'CPU submit us (tot/p50/p95)':>33s} "
            f"{'GPU execution us (tot/p50/p95)':>33s} {'GPU %':>6s}")
    out = [head, "-" * len(head)]
    for r in summary["rows"]:
        name = "/".join(r["key"])[:48]
        c, g = r["cpu_ns"], r["gpu_ns"]
        pct = "-" if r["gpu_pct"] is None else f"{r['gpu_pct']:6.1f}"
        out.append(f"{name:48s} {r['count']:5d} {_fmt(c['total'])}{_fmt(c['p50'])}{_fmt(c['p95'])} "
                   f"{_fmt(g['total'])}{_fmt(g['p50'])}{_fmt(g['p95'])} {pct}")
    w = summary["run_wall_ns"]
    out.append(f"runs {summary['runs']} (skipped {summary['skipped_runs']}), run wall mean {_fmt(w['mean'])} us "
               f"p50 {_fmt(w['p50'])} p95 {_fmt(w['p95'])}; unmeasured {summary['unmeasured']}, "
               f"failed {summary['failed']}, dropped {summary['dropped']}; percentiles: nearest-rank")
    return "\n".join(out)


def compare(before: dict, after: dict, group_by: str = "op", skip_runs: int = 0) -> list:
    a = {tuple(r["key"]): r for r in summarize(before, group_by, skip_runs)["rows"]}
    b = {tuple(r["key"]): r for r in summarize(after, group_by, skip_runs)["rows"]}
    rows = []
    for key in list(a) + [k for k in b if k not in a]:
        ga = a[key]["gpu_ns"]["total"] if key in a else None
        gb = b[key]["gpu_ns"]["total"] if key in b else None
        rows.append({"key": list(key), "before_gpu_ns": ga, "after_gpu_ns": gb,
                     "ratio": (gb / ga) if ga and gb is not None else None})
    return rows


def export_csv(doc: dict, out) -> None:
    w = csv.writer(out)
    cols = ["event_id", "run_id", "node_index", "node_name", "op_type", "cpu_start_ns", "cpu_duration_ns",
            "gpu_duration_ns", "device", "stream", "status"]
    w.writerow(cols)
    for ev in doc["events"]:
        w.writerow(["" if ev.get(c) is None else ev.get(c) for c in cols])


def chrome_trace(doc: dict) -> dict:
    events = []
    gpu_cursor = {}
    for ev in doc["events"]:
        name = f"{ev['node_name']} ({ev['op_type']})"
        if ev["cpu_duration_ns"] is not None:
            events.append({"name": name, "ph": "X", "pid": 0, "tid": 0, "ts": ev.get("cpu_start_ns", 0) / 1e3,
                           "dur": ev["cpu_duration_ns"] / 1e3, "args": {"run": ev["run_id"], "status": ev["status"]}})
        if ev["gpu_duration_ns"] is not None:
            run = ev["run_id"]
            if run not in gpu_cursor:
                start = next((r["start_ns"] for r in doc["runs"] if r["run_id"] == run), 0)
                gpu_cursor[run] = start
            events.append({"name": name, "ph": "X", "pid": 0, "tid": 1, "ts": gpu_cursor[run] / 1e3,
                           "dur": ev["gpu_duration_ns"] / 1e3, "args": {"run": run, "device": ev.get("device")}})
            gpu_cursor[run] += ev["gpu_duration_ns"]
    meta = [{"name": "thread_name", "ph": "M", "pid": 0, "tid": 0, "args": {"name": "CPU submit"}},
            {"name": "thread_name", "ph": "M", "pid": 0, "tid": 1,
             "args": {"name": "GPU execution (stream order, per run from its host start)"}}]
    return {"traceEvents": meta + events, "displayTimeUnit": "ns"}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m dli.profile")
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("summarize")
    s.add_argument("path")
    s.add_argument("--group-by", choices=("node", "op"), default="node")
    s.add_argument("--skip-runs", type=int, default=0)
    s.add_argument("--json", action="store_true")
    c = sub.add_parser("compare")
    c.add_argument("before")
    c.add_argument("after")
    c.add_argument("--group-by", choices=("node", "op"), default="op")
    c.add_argument("--skip-runs", type=int, default=0)
    e = sub.add_parser("export")
    e.add_argument("path")
    e.add_argument("--format", choices=("csv",), default="csv")
    e.add_argument("-o", "--output", default="-")
    t = sub.add_parser("trace")
    t.add_argument("path")
    t.add_argument("-o", "--output", required=True)
    args = ap.parse_args(argv)
    if args.cmd == "summarize":
        summary = summarize(load(args.path), args.group_by, args.skip_runs)
        if summary["runs"] < 3:
            print(f"warning: {summary['runs']} run(s) measured; percentiles are rough", file=sys.stderr)
        print(json.dumps(summary, indent=1) if args.json else format_table(summary))
    elif args.cmd == "compare":
        for r in compare(load(args.before), load(args.after), args.group_by, args.skip_runs):
            ratio = "-" if r["ratio"] is None else f"{r['ratio']:.3f}"
            print(f"{'/'.join(r['key']):48s} {_fmt(r['before_gpu_ns'])} {_fmt(r['after_gpu_ns'])} {ratio:>8s}")
    elif args.cmd == "export":
        doc = load(args.path)
        if args.output == "-":
            export_csv(doc, sys.stdout)
        else:
            with open(args.output, "w", newline="") as f:
                export_csv(doc, f)
    else:
        with open(args.output, "w") as f:
            json.dump(chrome_trace(load(args.path)), f)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
