"""Qwen2 serving benchmark of the sm_100a plugin (default workload: the Qwen2-7B shape).

One "step" = one generation request batch: a causal prefill of B x S prompt
tokens followed by D greedy decode steps over the KV cache, all through the
dli.Engine running the exported dli.graph.v1 graph with the sm_100a plugin
(decode replayed from a captured CUDA graph). Weights are random-init
N(0, 0.02) of the named architecture (no checkpoints: synthetic data).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--model 7b|0.5b|72b|linear|alexnet]
  python bench.py --impl reference ...     # the reference's CPU path (PyTorch eager)

Multi-GPU (launched by torchrun, one rank per GPU): tensor parallelism over
tp = min(N, max TP the head counts allow, 4 for 7B) with the all-reduce after
o_proj and down_proj fused into the next RMSNorm (NVLink exchange kernel for
decode rows, NCCL for prefill) and a vocabulary-split LM head; N / tp
data-parallel groups split the batch (strong scaling: total work fixed). Times
are CUDA events on each rank, max over ranks.

Printed JSON (rank 0): value = decode tok/s of the whole job; prefill tok/s,
e2e (decode through the public API with host ids in and out every token),
roofline of the dominant decode kernel (gate/up + SwiGLU GEMM, HBM-bound) and of the
dominant prefill kernel (tensor-bound), clocks sampled during the timed region,
CPU baseline, and the number of this library's kernels launched.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "dl-inference_b200"
sys.path.insert(0, str(PKG / "python"))
sys.path.insert(0, str(ROOT))

METRIC = "Qwen2 decode tok/s + prefill tok/s at 1/2/4/8 B200; % of HBM/tensor roofline"

MODELS = {
    # name: (shape, batch, prompt, decode steps, max tp)
    "7b": ("QWEN2_7B", 32, 2048, 512, 4),
    "0.5b": ("QWEN2_0_5B", 8, 512, 256, 2),
    "72b": ("QWEN2_72B", 64, 4096, 512, 8),
}
# single-GPU operator / CNN workloads (replicas only under torchrun)
SMALL = {
    "linear": "single linear x[64,1024] . W[4096,1024]^T + b, fp32",
    "alexnet": "AlexNet-style CNN forward, batch 64, 3x32x32, fp16",
}



# ncu summaries (profiles/) of the dominant decode kernel per (model, tp, batch per rank)
NCU_SUMMARIES = {("7b", 1, 32): "glu_decode_gate_up_qwen2_7b.md"}
_UNITS = {"byte": 1, "kbyte": 1e3, "mbyte": 1e6, "gbyte": 1e9}


def ncu_traffic(name):
    """dram__bytes_read.sum + dram__bytes_write.sum of the launch an ncu summary
    records (its metric table rows `| metric | value unit |`), or None."""
    path = ROOT / "profiles" / name if name else None
    if path is None or not path.exists():
        return None
    found = {}
    for line in path.read_text().splitlines():
        cells = [c.strip().strip("`") for c in line.strip().strip("|").split("|")]
        if len(cells) >= 2 and cells[0] in ("dram__bytes_read.sum", "dram__bytes_write.sum"):
            value, unit = cells[1].split()
            found[cells[0]] = float(value) * _UNITS[unit.lower()]
    return found["dram__bytes_read.sum"] + found["dram__bytes_write.sum"] if len(found) == 2 else None

def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("sm100", "reference"), default="sm100")
    ap.add_argument("--model", choices=sorted(MODELS) + sorted(SMALL), default="7b")
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--prompt", type=int, default=None)
    ap.add_argument("--decode", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-fused-exchange", action="store_true",
                    help="TP graphs: linear + all_reduce_add_rms_norm nodes instead of the GEMM-epilogue push")
    return ap.parse_args()


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks + throttle reasons sampled every 200 ms while active."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        if self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------------
# CPU baseline: the reference's CPU path (PyTorch-eager forward of the exported model)
# ---------------------------------------------------------------------------------

def cpu_baseline(shape, batch: int, prompt: int, seconds: float = 20.0) -> dict:
    """Times transformers' Qwen2 (eager, bf16) on the host cores on a slice of the
    workload: ONE decoder layer of the named shape, decode steps of the full batch
    over a `prompt`-token cache, scaled to the full model (layers x per-layer time +
    the LM head)."""
    import torch
    from transformers import Qwen2Config
    from transformers.models.qwen2.modeling_qwen2 import Qwen2DecoderLayer, Qwen2RotaryEmbedding
    from transformers.cache_utils import DynamicCache

    threads = torch.get_num_threads()
    cfg = Qwen2Config(vocab_size=shape.vocab, hidden_size=shape.hidden,
                      intermediate_size=shape.intermediate, num_hidden_layers=1,
                      num_attention_heads=shape.q_heads, num_key_value_heads=shape.kv_heads,
                      max_position_embeddings=prompt + 64, rms_norm_eps=shape.rms_eps,
                      rope_theta=shape.rope_theta, attn_implementation="eager")
    torch.manual_seed(0)
    with torch.no_grad():
        layer = Qwen2DecoderLayer(cfg, 0).to(torch.bfloat16).eval()
        for p in layer.parameters():
            p.normal_(0, 0.02)
        rot = Qwen2RotaryEmbedding(cfg)
        lm = torch.randn(shape.vocab, shape.hidden, dtype=torch.bfloat16) * 0.02
        # KV cache of `prompt` tokens for the full batch (filled directly)
        cache = DynamicCache()
        kv = torch.randn(batch, shape.kv_heads, prompt, shape.head_dim, dtype=torch.bfloat16)
        cache.update(kv, kv.clone(), 0)
        x = torch.randn(batch, 1, shape.hidden, dtype=torch.bfloat16)
        steps, t_layer = 0, 0.0
        start = time.perf_counter()
        while time.perf_counter() - start < seconds * 0.8 or steps < 2:
            pos = torch.full((batch, 1), prompt + steps, dtype=torch.int64)
            emb = rot(x, pos)
            t0 = time.perf_counter()
            layer(x, attention_mask=None, position_ids=pos, past_key_values=cache,
                  use_cache=True, position_embeddings=emb)
            t_layer += time.perf_counter() - t0
            steps += 1
        t0 = time.perf_counter()
        reps = 0
        while reps < 2 or time.perf_counter() - t0 < seconds * 0.1:
            torch.nn.functional.linear(x[:, 0], lm)
            reps += 1
        t_head = (time.perf_counter() - t0) / reps
    step_s = shape.layers * (t_layer / steps) + t_head
    return {"value": batch / step_s, "unit": "tok/s (decode)", "cores": threads, "kind": "reference",
            "sample": (f"transformers Qwen2 eager bf16 on {threads} host threads: {steps} decode steps "
                       f"of 1 of {shape.layers} decoder layers (batch {batch}, {prompt}-token cache) "
                       f"+ LM head, scaled x{shape.layers} layers"),
            "ms_per_step": step_s * 1e3}


def cpu_prefill(shape, prompt: int, seconds: float = 5.0) -> dict:
    """Times the prefill half of the reference's CPU path: transformers' Qwen2
    (eager, bf16) runs ONE decoder layer of the named shape over one full
    `prompt`-token sequence with the causal mask, repeated within `seconds`
    (at least once, after a short warm-up), plus the LM head on the last token; scaled to the full
    model. The host cores are busy with one sequence already, so a batch of B
    sequences takes B times as long and the rate is tokens per second either way."""
    import torch
    from transformers import Qwen2Config
    from transformers.models.qwen2.modeling_qwen2 import Qwen2DecoderLayer, Qwen2RotaryEmbedding

    threads = torch.get_num_threads()
    cfg = Qwen2Config(vocab_size=shape.vocab, hidden_size=shape.hidden,
                      intermediate_size=shape.intermediate, num_hidden_layers=1,
                      num_attention_heads=shape.q_heads, num_key_value_heads=shape.kv_heads,
                      max_position_embeddings=prompt + 64, rms_norm_eps=shape.rms_eps,
                      rope_theta=shape.rope_theta, attn_implementation="eager")
    torch.manual_seed(1)
    with torch.no_grad():
        layer = Qwen2DecoderLayer(cfg, 0).to(torch.bfloat16).eval()
        for p in layer.parameters():
            p.normal_(0, 0.02)
        rot = Qwen2RotaryEmbedding(cfg)
        lm = torch.randn(shape.vocab, shape.hidden, dtype=torch.bfloat16) * 0.02
        x = torch.randn(1, prompt, shape.hidden, dtype=torch.bfloat16)
        pos = torch.arange(prompt, dtype=torch.int64)[None]
        emb = rot(x, pos)
        mask = torch.full((prompt, prompt), float("-inf")).triu(1)[None, None].to(torch.bfloat16)
        n0 = min(prompt, 64)  # untimed warm-up on a short prefix
        layer(x[:, :n0], attention_mask=mask[..., :n0, :n0], position_ids=pos[:, :n0],
              position_embeddings=tuple(e[:, :n0] for e in emb))
        reps, t_layer = 0, 0.0
        start = time.perf_counter()
        while reps < 1 or time.perf_counter() - start < seconds:
            t0 = time.perf_counter()
            layer(x, attention_mask=mask, position_ids=pos, position_embeddings=emb)
            t_layer += time.perf_counter() - t0
            reps += 1
        t0 = time.perf_counter()
        torch.nn.functional.linear(x[:, -1], lm)
        t_head = time.perf_counter() - t0
    seq_s = shape.layers * (t_layer / reps) + t_head
    return {"value": prompt / seq_s, "unit": "tok/s (prefill)", "cores": threads, "kind": "reference",
            "ms_per_sequence": seq_s * 1e3,
            "sample": (f"transformers Qwen2 eager bf16 on {threads} host threads: {reps} causal forwards of "
                       f"1 of {shape.layers} decoder layers over one {prompt}-token sequence + LM head of the "
                       f"last token, scaled x{shape.layers} layers")}


def workload_config(model: str, batch: int, prompt: int, dsteps: int) -> dict:
    """The `config` keys both arms report for the same workload."""
    return {"workload": f"qwen2-{model}: prefill {batch}x{prompt} + {dsteps} greedy decode steps",
            "model": f"Qwen2-{model.upper()}-shape", "global_batch": batch, "seq_len": prompt,
            "decode_steps": dsteps}


# ---------------------------------------------------------------------------------
# Single-GPU operator / CNN workloads: the single fp32 linear and the AlexNet-style CNN
# ---------------------------------------------------------------------------------

def _small_case(model: str, device):
    """(engine graph dict, output name, constants, input, flops, algorithmic bytes, unit label)."""
    import torch

    if model == "linear":
        g = torch.Generator(device=device).manual_seed(0)
        x = torch.randn(64, 1024, device=device, generator=g)
        w = torch.randn(4096, 1024, device=device, generator=g) * 0.02
        b = torch.randn(4096, device=device, generator=g) * 0.02
        graph = {"format": "dli.graph.v1", "model_type": "single_linear", "inputs": ["x"], "outputs": ["y"],
                 "nodes": [{"name": "fc", "op": "linear", "inputs": ["x", "w", "b"], "outputs": ["y"], "attrs": {}}]}
        nbytes = 4 * (4096 * 1024 + 64 * 1024 + 64 * 4096 + 4096)
        return graph, "y", {"w": w, "b": b}, x, 2.0 * 64 * 1024 * 4096, nbytes, "calls/s"
    from dli_export.cnn import alexnet_flops, alexnet_graph, alexnet_params

    graph, out = alexnet_graph(64)
    p, x = alexnet_params(torch.float16, 64, seed=0, device=device)
    nbytes = 2 * (sum(t.numel() for t in p.values()) + x.numel() + 64 * 10)
    return graph, out, p, x, alexnet_flops(64), nbytes, "images/s"


def run_small(args, world: int, rank: int, local: int) -> int:
    import torch
    import torch.distributed as dist

    import dli
    import dli_sm100

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    graph, out_name, consts, x, flops, nbytes, unit = _small_case(args.model, dev)
    units_per_step = 1 if args.model == "linear" else x.shape[0]
    engine = dli.Engine()
    engine.load_library(dli.PLUGIN_PATH)
    engine.set_constants(consts)
    g = dli.Graph.from_json(json.dumps(graph))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > the 126 MB L2
    stream = torch.cuda.current_stream(dev)

    def step():
        return engine.run(g, {"x": x})[out_name]

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # The timed step is the engine run captured once as a CUDA graph and replayed:
    # the device time of the forward with its input resident in HBM, free of the
    # host's per-call submission cost (the e2e figure below keeps that cost).
    n0 = dli_sm100.launch_count()
    cuda_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(cuda_graph):
        step()
    launches_per_step = dli_sm100.launch_count() - n0
    for _ in range(args.warmup):
        cuda_graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    evs = []
    with ClockSampler(local) as clocks:
        for _ in range(args.steps):
            flush.zero_()  # L2 flushed between timed steps, outside the timed span
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            cuda_graph.replay()
            b.record(stream)
            evs.append((a, b))
        torch.cuda.synchronize()
    launches = launches_per_step * args.steps
    ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = t.item()
    try:
        dli_sm100.check_device_error()
        device_error = None
    except RuntimeError as exc:
        device_error = str(exc)
    # e2e: input from pinned host memory, result read back, every step
    host_x = x.cpu().pin_memory()
    y0 = step()
    host_y = torch.empty(y0.shape, dtype=y0.dtype, pin_memory=True)
    e2e_ms = []
    for i in range(args.warmup + args.steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        xd = host_x.to(dev, non_blocking=True)
        host_y.copy_(engine.run(g, {"x": xd})[out_name], non_blocking=True)
        b.record(stream)
        stream.synchronize()
        if i >= args.warmup:
            e2e_ms.append(a.elapsed_time(b))
    e2e = sum(e2e_ms) / len(e2e_ms)
    pk = peaks()
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        cpu = small_cpu_baseline(args.model, seconds=15.0)
        cpu.pop("ms_per_step", None)
    if rank == 0:
        tflops = flops / (ms / 1e3) / 1e12
        gbs = nbytes / (ms / 1e3) / 1e9
        fp32 = args.model == "linear"
        line = {
            "metric": f"{args.model} throughput ({unit})", "value": world * units_per_step / (ms / 1e3),
            "unit": unit, "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32" if fp32 else "f16",
            "data": "synthetic (seeded N(0,1) inputs, N(0,0.02) weights)",
            "config": {"workload": SMALL[args.model], "model": args.model, "global_batch": 64 * world,
                       "parallelism": f"replicas{world}" if world > 1 else "none",
                       "l2": "flushed between timed steps (256 MB write outside the timed span)"},
            "e2e": {"value": world * units_per_step / (e2e / 1e3), "unit": unit,
                    "h2d_bytes_per_step": host_x.numel() * host_x.element_size(),
                    "d2h_bytes_per_step": host_y.numel() * host_y.element_size(), "ms": e2e,
                    "path": "dli.Engine.run with the input copied from pinned host memory and the output read back"},
            "roofline": ({"bound": "hbm", "achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                          "frac": gbs / pk["hbm_gbs"], "traffic": None, "algorithmic_bytes": nbytes,
                          "flops": flops, "TFLOP/s": tflops, "peak_source": pk["source"],
                          "note": "fp32 on tcgen05 through a three-term bf16 split (FFMA-level error); "
                                  "the weight stream is the HBM floor"}
                         if fp32 else
                         {"bound": "tensor", "achieved": tflops, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                          "frac": tflops / pk["bf16_tflops"], "traffic": None, "flops": flops,
                          "peak_source": pk["source"],
                          "note": "whole forward (13 nodes) against the dense fp16/bf16 peak; launch-bound at batch 64"}),
            "clocks": clocks.summary(), "cpu_baseline": cpu, "gpu_launches": launches,
            "device_error": device_error,
        }
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 1 if device_error else 0


def small_cpu_baseline(model: str, seconds: float = 15.0) -> dict:
    """The reference's CPU path for these workloads: the linear as the aten::linear
    node dispatches it (torch.nn.functional.linear, fp32) and the CNN as a PyTorch
    eager forward (fp32 on the host: 16-bit convolutions are not a host fast path)."""
    import torch

    threads = torch.get_num_threads()
    graph, out, consts, x, flops, _, unit = _small_case(model, "cpu")
    if model == "linear":
        fn = lambda: torch.nn.functional.linear(x, consts["w"], consts["b"])  # noqa: E731
        per = 1
        what = f"torch.nn.functional.linear fp32 [64,1024]x[4096,1024]^T + b on {threads} host threads"
    else:
        from dli_export.cnn import alexnet_forward

        p32 = {k: v.float() for k, v in consts.items()}
        x32 = x.float()
        fn = lambda: alexnet_forward(p32, x32)  # noqa: E731
        per = x.shape[0]
        what = f"AlexNet-style forward, PyTorch eager fp32, batch 64, on {threads} host threads"
    with torch.no_grad():
        fn()
        n, t0 = 0, time.perf_counter()
        while n < 2 or time.perf_counter() - t0 < seconds:
            fn()
            n += 1
        dt = (time.perf_counter() - t0) / n
    return {"value": per / dt, "unit": unit, "cores": threads, "kind": "reference",
            "sample": f"{what}: {n} calls", "ms_per_step": dt * 1e3}


def run_small_reference(args, world: int, rank: int) -> int:
    if rank != 0:
        return 0
    vals = [small_cpu_baseline(args.model, seconds=max(2.0, 40.0 / (args.steps + args.warmup)))
            for _ in range(args.warmup + args.steps)][args.warmup:]
    value = statistics.median(v["value"] for v in vals)
    unit = vals[0]["unit"]
    line = {"metric": f"{args.model} throughput ({unit})", "impl": "reference", "value": value, "unit": unit,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": statistics.median(v["ms_per_step"] for v in vals), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) inputs, N(0,0.02) weights)",
            "config": {"workload": SMALL[args.model], "model": args.model, "global_batch": 64,
                       "parallelism": "none (host cores)"},
            "cpu_baseline": {k: vals[-1][k] for k in ("kind", "cores", "sample")} | {"value": value, "unit": unit},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


def run_reference_arm(args, world: int, rank: int):
    from dli_export import qwen2 as Q

    name, batch, prompt, dsteps, _ = MODELS[args.model]
    if rank != 0:
        return 0
    shape = getattr(Q, name)
    batch = args.batch or batch
    prompt = args.prompt or prompt
    dsteps = args.decode or dsteps
    vals = []
    per = max(3.0, 60.0 / max(1, args.steps + args.warmup))
    for i in range(args.warmup + args.steps):
        r = cpu_baseline(shape, batch, prompt, seconds=per)
        if i >= args.warmup:
            vals.append(r)
    value = statistics.median(v["value"] for v in vals)
    pre = cpu_prefill(shape, prompt)  # once per run: the decode steps above carry the timing contract
    line = {"metric": METRIC, "impl": "reference", "value": value, "unit": "tok/s (decode)",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": statistics.median(v["ms_per_step"] for v in vals),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init N(0,0.02) weights, seeded)",
            "config": workload_config(args.model, batch, prompt, dsteps) | {
                "parallelism": "none (host cores)",
                "reference_sample": f"decode at a {prompt}-token context, one decoder layer timed and scaled"},
            "prefill": {"value": pre["value"], "unit": pre["unit"], "ms_per_sequence": pre["ms_per_sequence"],
                        "sample": pre["sample"]},
            "cpu_baseline": {k: vals[-1][k] for k in ("kind", "cores", "sample")} | {"value": value,
                                                                                     "unit": "tok/s (decode)"},
            "e2e": {"value": value, "unit": "tok/s (decode)", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


# ---------------------------------------------------------------------------------
# sm_100a arm
# ---------------------------------------------------------------------------------

def main() -> int:
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.model in SMALL:
        if args.impl == "reference":
            return run_small_reference(args, world, rank)
        return run_small(args, world, rank, local)
    if args.impl == "reference":
        return run_reference_arm(args, world, rank)

    import torch
    import torch.distributed as dist

    import dli_sm100
    from dli.parallel import TensorParallelComm, parallel_layout
    from dli.qwen2 import Qwen2Runner
    from dli_export import qwen2 as Q

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)

    name, batch, prompt, dsteps, max_tp = MODELS[args.model]
    shape = getattr(Q, name)
    batch = args.batch or batch
    prompt = args.prompt or prompt
    dsteps = args.decode or dsteps
    lay = parallel_layout(world, rank, max_tp, shape)
    tp, dp, group, tp_rank = lay.tp, lay.dp, lay.group, lay.tp_rank
    try:
        b_local = lay.local_batch(batch)
    except ValueError as exc:
        raise SystemExit(str(exc))
    capacity = (prompt + dsteps + 63) // 64 * 64

    # --- communicator: one NCCL comm per tensor-parallel group, built by the plugin
    dli_sm100.lib()  # kernel library loaded before the plugin
    # NVLink exchange buffers for the fused all-reduce + add_rms_norm of decode steps
    tpc = TensorParallelComm(lay, local, exchange=(256, shape.hidden, 2))
    comm = tpc.handle

    # --- weights: random N(0, 0.02), generated on the device layer by layer, sharded
    weights = {}
    for i in range(shape.layers):
        st = Q.random_state(shape, device=dev, dtype=torch.bfloat16, seed=1000 + i,
                            layers=range(i, i + 1), embeddings=False)
        weights.update(Q.transform_weights(st, shape, tp, tp_rank, torch.bfloat16, layers=range(i, i + 1)))
        del st
    g = torch.Generator(device=dev).manual_seed(7)
    weights["embed"] = (torch.randn(shape.vocab, shape.hidden, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    lm = weights["embed"] if shape.tie_embeddings else \
        (torch.randn(shape.vocab, shape.hidden, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    if Q.vocab_parallel(shape, tp):  # this rank's vocabulary rows (the graph picks with tp_argmax)
        vs = shape.vocab // tp
        lm = lm[tp_rank * vs:(tp_rank + 1) * vs].contiguous()
    weights["lm_head"] = lm
    weights["norm"] = torch.ones(shape.hidden, device=dev, dtype=torch.bfloat16)
    cos, sin = Q.rotary_tables(shape, capacity)
    weights["rotary_cos"], weights["rotary_sin"] = cos.to(dev), sin.to(dev)
    torch.cuda.synchronize()

    runner = Qwen2Runner(shape, weights, capacity, tp_size=tp, tp_rank=tp_rank, communicator=comm or 0,
                         fused_exchange=not args.no_fused_exchange)
    gen = torch.Generator(device=dev).manual_seed(100 + group)
    prompts = torch.randint(0, shape.vocab, (b_local, prompt), device=dev, generator=gen)

    def barrier():
        if world > 1:
            dist.barrier()

    # capture the decode graph once (counts the launches of one decode step)
    n0 = dli_sm100.launch_count()
    runner.decode_graph(b_local)
    launches_decode = (dli_sm100.launch_count() - n0) // 3  # 2 warm runs + the captured run
    n0 = dli_sm100.launch_count()
    runner.prefill(prompts)
    launches_prefill = dli_sm100.launch_count() - n0
    torch.cuda.synchronize()

    g_, ids_buf, pos_buf, _, next_buf = runner.decode_graph(b_local)
    stream = torch.cuda.current_stream(dev)

    def one_step():
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record(stream)
        _, nxt = runner.prefill(prompts)
        ids_buf.copy_(nxt.view(-1, 1))
        pos_buf.fill_(prompt)
        ev[1].record(stream)
        for _ in range(dsteps):
            g_.replay()
        ev[2].record(stream)
        return ev

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        events = [one_step() for _ in range(args.steps)]
        torch.cuda.synchronize()
    barrier()
    pre_ms = sum(e[0].elapsed_time(e[1]) for e in events)
    dec_ms = sum(e[1].elapsed_time(e[2]) for e in events)
    t = torch.tensor([pre_ms, dec_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    pre_ms, dec_ms = t.tolist()
    # A kernel whose bounded wait ran out (or that met an out-of-range index)
    # returns early and sets the device error word: such a run is not a measurement.
    try:
        dli_sm100.check_device_error()
        device_error = None
    except RuntimeError as exc:
        device_error = str(exc)
    total_seqs = b_local * dp
    decode_tok_s = total_seqs * dsteps * args.steps / (dec_ms / 1e3)
    prefill_tok_s = total_seqs * prompt * args.steps / (pre_ms / 1e3)
    clock = clocks.summary()

    # --- e2e: decode through the public API, ids from pinned host memory each token,
    #     next ids read back to host each token (same metric, host buffers included)
    host_ids = torch.empty(b_local, 1, dtype=torch.int64, pin_memory=True)
    host_out = torch.empty(b_local, dtype=torch.int64, pin_memory=True)
    host_ids.copy_(prompts[:, -1:].cpu())
    e2e_steps = min(dsteps, 128)
    _, nxt = runner.prefill(prompts)
    pos_buf.fill_(prompt)
    torch.cuda.synchronize()
    barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    wall0 = time.perf_counter()
    for _ in range(e2e_steps):
        ids_buf.copy_(host_ids, non_blocking=True)
        g_.replay()
        host_out.copy_(next_buf, non_blocking=True)
        stream.synchronize()
        host_ids[:, 0] = host_out
    t1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([max(t0.elapsed_time(t1), (time.perf_counter() - wall0) * 1e3)], device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_tok_s = total_seqs * e2e_steps / (e2e_ms.item() / 1e3)

    # --- roofline of the dominant kernels, timed live with CUDA events: the fused
    #     gate/up + SwiGLU GEMM (linear_silu_mul) the decode and prefill graphs run
    pk = peaks()
    inter_local = shape.intermediate // tp
    k_gu = shape.hidden
    w_gu = weights["layers.0.wgu"]  # 64-row gate/up blocks, [2*ceil(I/64)*64, K]
    rows_w = w_gu.shape[0]
    x_dec = torch.randn(b_local, k_gu, device=dev).to(torch.bfloat16)
    reps = 20
    for _ in range(3):
        dli_sm100.linear_silu_mul(x_dec, w_gu, inter_local)
    ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ea.record(stream)
    for _ in range(reps):
        dli_sm100.linear_silu_mul(x_dec, w_gu, inter_local)
    eb.record(stream)
    torch.cuda.synchronize()
    gemm_ms = ea.elapsed_time(eb) / reps
    gemm_bytes = (rows_w * k_gu + b_local * (k_gu + inter_local)) * 2  # weights + x + act
    achieved = gemm_bytes / (gemm_ms / 1e3) / 1e9
    # DRAM bytes (read + write) of one launch of this kernel, parsed from the
    # committed ncu summary of the same launch shape; null for shapes without one
    traffic = ncu_traffic(NCU_SUMMARIES.get((args.model, tp, b_local)))
    # prefill: the same kernel at M = b_local * prompt (capped for memory)
    m_pre = min(b_local * prompt, 16384)
    x_pre = torch.randn(m_pre, k_gu, device=dev).to(torch.bfloat16)
    dli_sm100.linear_silu_mul(x_pre, w_gu, inter_local)
    ea.record(stream)
    for _ in range(5):
        dli_sm100.linear_silu_mul(x_pre, w_gu, inter_local)
    eb.record(stream)
    torch.cuda.synchronize()
    pre_gemm_ms = ea.elapsed_time(eb) / 5
    pre_tflops = 2.0 * m_pre * 2 * inter_local * k_gu / (pre_gemm_ms / 1e3) / 1e12
    step_bytes = Q.decode_bytes_per_step(shape, b_local, prompt + dsteps // 2) / tp
    step_ms = dec_ms / (args.steps * dsteps)
    launches = args.steps * (launches_prefill + dsteps * launches_decode)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:  # timed at N=1 only (all host threads)
        try:
            cpu = cpu_baseline(shape, total_seqs, prompt, seconds=20.0)
            cpu.pop("ms_per_step", None)
            cpu["prefill"] = cpu_prefill(shape, prompt)
        except Exception as exc:  # report, do not fail the GPU measurement
            cpu = {"value": None, "unit": "tok/s (decode)", "cores": os.cpu_count(), "kind": "reference",
                   "sample": f"failed: {exc!r}"[:200]}

    if rank == 0:
        line = {
            "metric": METRIC, "value": decode_tok_s, "unit": "tok/s (decode)", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": (pre_ms + dec_ms) / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init N(0,0.02) weights of the named architecture, uniform token ids; seeded)",
            "config": workload_config(args.model, batch, prompt, dsteps) | {
                       "parallelism": f"tp{tp}" + (f"xdp{dp}" if dp > 1 else ""),
                       "l2": "inputs larger than L2 (weights stream from HBM every step)",
                       "kv_capacity": capacity} | ({"tp_exchange": "exchange kernel" if args.no_fused_exchange
                                                    else "GEMM-epilogue push"} if tp > 1 else {}),
            "prefill": {"value": prefill_tok_s, "unit": "tok/s (prefill)", "ms_per_step": pre_ms / args.steps},
            "decode_ms_per_token_step": step_ms,
            "e2e": {"value": e2e_tok_s, "unit": "tok/s (decode)", "h2d_bytes_per_step": 8 * b_local,
                    "d2h_bytes_per_step": 8 * b_local, "steps": e2e_steps,
                    "path": "Qwen2Runner decode graph fed from pinned host ids, next ids read to host every token"},
            "roofline": {"bound": "hbm",
                         "kernel": f"tcgen05 swap-AB GEMM gate/up + SwiGLU epilogue [{b_local}x{k_gu}]x[{rows_w}x{k_gu}]^T",
                         "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / pk["hbm_gbs"], "traffic": traffic,
                         "algorithmic_bytes": gemm_bytes, "ms": gemm_ms, "peak_source": pk["source"]},
            "roofline_decode_step": {"bound": "hbm", "bytes": step_bytes, "ms": step_ms,
                                     "achieved": step_bytes / (step_ms / 1e3) / 1e9, "peak": pk["hbm_gbs"],
                                     "unit": "GB/s", "frac": step_bytes / (step_ms / 1e3) / 1e9 / pk["hbm_gbs"]},
            "roofline_prefill": {"bound": "tensor",
                                 "kernel": f"tcgen05 GEMM gate/up + SwiGLU epilogue [{m_pre}x{k_gu}]x[{rows_w}x{k_gu}]^T",
                                 "achieved": pre_tflops, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                                 "frac": pre_tflops / pk["bf16_tflops"]},
            "clocks": clock,
            "cpu_baseline": cpu,
            "gpu_launches": launches,
            "launches_per_decode_step": launches_decode,
            "device_error": device_error,
        }
        print(json.dumps(line))
    # graphs holding NCCL launches go before the communicator, which goes before the process group
    del g_, ids_buf, pos_buf, next_buf
    runner.release_graphs()
    del runner
    torch.cuda.synchronize()
    tpc.destroy()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 1 if device_error else 0


if __name__ == "__main__":
    sys.exit(main())
