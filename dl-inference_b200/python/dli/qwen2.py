"""Greedy generation over a Qwen2 graph exported by dli_export.qwen2.

Qwen2Runner drives one tensor-parallel rank: it binds the weights to the
engine once (Engine.set_constants), runs prefill through Engine.run, and
replays the decode step from a captured CUDA graph. Token ids and positions
stay on the device between steps: each decode step writes the argmax ids and
advances the positions inside the graph's static input buffers.
"""
from __future__ import annotations

import json
from typing import Any

import torch

from . import PLUGIN_PATH, Engine, Graph


class Qwen2Runner:
    def __init__(self, shape: Any, weights: dict[str, torch.Tensor], capacity: int,
                 tp_size: int = 1, tp_rank: int = 0, communicator: int = 0,
                 plugin: str = PLUGIN_PATH, fused_glu: bool = True, fused_exchange: bool = True):
        """`weights` come from dli_export.qwen2.transform_weights with the same
        `fused_glu` (the fused SwiGLU GEMM serves bfloat16/float16 weights).
        `fused_exchange`: tensor-parallel projections push their partial rows
        from the GEMM epilogue (linear_all_reduce_add_rms_norm nodes)."""
        from dli_export.qwen2 import build_graph, rotary_tables

        self.shape = shape
        self.capacity = capacity
        self.device = next(iter(weights.values())).device
        self.engine = Engine()
        self.engine.load_library(plugin)
        if tp_size > 1:
            self.engine.set_communicator(communicator, tp_rank, tp_size)
        self.graph = Graph.from_json(json.dumps(build_graph(shape, capacity, tp_size, fused_glu=fused_glu,
                                                            fused_exchange=fused_exchange)))
        consts = dict(weights)
        if "rotary_cos" not in consts:
            cos, sin = rotary_tables(shape, capacity)
            consts["rotary_cos"], consts["rotary_sin"] = cos.to(self.device), sin.to(self.device)
        self.engine.set_constants(consts)
        self._graphs: dict[int, tuple] = {}

    # -- plain engine calls -------------------------------------------------------
    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor, profile=None):
        """input_ids [B,S] int64, positions [B] int64 (cache row of the first token).
        Returns (logits of the last token, next ids). With tensor parallelism over a
        vocabulary that divides evenly, the logits are this rank's slice of the
        vocabulary (ids [rank*V/tp, (rank+1)*V/tp)); the next ids are global.
        `profile` (a dli.ProfileSession) times every node of the run."""
        out = self.engine.run(self.graph, {"input_ids": input_ids, "positions": positions}, profile=profile)
        return out["logits"], out["next_ids"]

    def check_device_error(self) -> None:
        """Raises RuntimeError when a kernel of this process reported an error
        through the device error word: a bounded wait that ran out (a
        tensor-parallel peer that never arrived, a tensor-core pipeline stall) or
        an out-of-range id or position. Such a kernel returns early, so the
        outputs of the run are not valid. Synchronises the current stream. After
        an exchange timeout every rank must reset its exchange buffer
        (dli_sm100_tp_exchange_reset) before the group runs again."""
        import dli_sm100

        dli_sm100.check_device_error()

    def reset(self) -> None:
        """Forgets cached sequences (rows are rewritten by position, so nothing to clear)."""
        self.engine.kv_cache_reset()

    # -- CUDA-graph decode ----------------------------------------------------------
    def profile_decode_step(self, batch: int, profile) -> None:
        """Captures one decode step with every node between CUDA-event markers,
        replays it once and leaves the session holding that replay's per-node
        device times (call profile.finalize() next). The step runs at the last
        cache row, like the warm-up of the decode graph, so live sequences are
        not disturbed. The markers make the step slower than the decode graph."""
        ids = torch.zeros(batch, 1, dtype=torch.int64, device=self.device)
        pos = torch.full((batch,), self.capacity - 1, dtype=torch.int64, device=self.device)
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            self.forward(ids, pos)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        profile.reserve(len(self.graph.node_ops()))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.forward(ids, pos, profile=profile)
        g.replay()
        torch.cuda.synchronize(self.device)
        del g

    def _capture(self, batch: int):
        # Warm-up and capture write one cache row per sequence; the last row is only
        # read after a later step has rewritten it, so live sequences are not disturbed.
        ids = torch.zeros(batch, 1, dtype=torch.int64, device=self.device)
        pos = torch.full((batch,), self.capacity - 1, dtype=torch.int64, device=self.device)
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            for _ in range(2):  # warm the caching allocator and per-kernel attributes
                self.forward(ids, pos)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            logits, next_ids = self.forward(ids, pos)
            ids.copy_(next_ids.view(batch, 1))
            pos.add_(1)
        self._graphs[batch] = (g, ids, pos, logits, next_ids)
        return self._graphs[batch]

    def decode_graph(self, batch: int):
        return self._graphs.get(batch) or self._capture(batch)

    def release_graphs(self) -> None:
        """Drops the captured decode graphs. A graph captured with tensor
        parallelism holds NCCL launches on the runner's communicator: release it
        before that communicator (or the process group) is destroyed."""
        torch.cuda.synchronize(self.device)
        self._graphs.clear()

    def prefill(self, prompt: torch.Tensor, start: torch.Tensor | None = None):
        """prompt [B,S] on the device; returns (logits of the last token, next ids)."""
        b = prompt.shape[0]
        if start is None:
            start = torch.zeros(b, dtype=torch.int64, device=self.device)
        return self.forward(prompt, start)

    def generate(self, prompt: torch.Tensor, steps: int, use_graph: bool = True) -> torch.Tensor:
        """Greedy decoding: returns [B, steps] device ids (the first from prefill)."""
        b, s = prompt.shape
        if s + steps > self.capacity:
            raise ValueError("prompt + steps exceeds the KV-cache capacity")
        out = torch.empty(b, steps, dtype=torch.int64, device=self.device)
        _, nxt = self.prefill(prompt)
        out[:, 0] = nxt
        if steps == 1:
            return out
        if use_graph:
            g, ids, pos, _, next_ids = self.decode_graph(b)
            ids.copy_(nxt.view(b, 1))
            pos.fill_(s)
            for t in range(1, steps):
                g.replay()
                out[:, t] = next_ids
        else:
            ids = nxt.view(b, 1)
            pos = torch.full((b,), s, dtype=torch.int64, device=self.device)
            for t in range(1, steps):
                _, nxt = self.forward(ids, pos)
                out[:, t] = nxt
                ids = nxt.view(b, 1)
                pos = pos + 1
        self.check_device_error()
        return out
