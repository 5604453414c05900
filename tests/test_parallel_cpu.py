"""CPU tests of the multi-rank host logic: the tensor-parallel x data-parallel
layout that bench.py and Qwen2Runner use, and the sharded Qwen2 graph run
rank by rank as separate gloo processes (world size 2 and 4). A real
torch.distributed all_reduce stands in for the NCCL all_reduce operator and an
all_gather for the vocab-parallel greedy pick; each rank's logits must equal
the single-rank graph's logits for its share of the batch and its slice of the
vocabulary, and every rank's next ids the single-rank ids (float64 oracle, so
the only difference is summation order)."""
from __future__ import annotations

import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dli.parallel import parallel_layout
from dli_export.qwen2 import (QWEN2_0_5B, QWEN2_7B, QWEN2_72B, Qwen2Shape, build_graph, random_state,
                              rotary_tables, transform_weights)

TINY = Qwen2Shape(hidden=64, layers=2, q_heads=4, kv_heads=2, head_dim=16, intermediate=96, vocab=50)
BATCH, PROMPT, CAP = 4, 6, 32


@pytest.mark.parametrize("shape,max_tp,world,tp,dp", [
    (QWEN2_7B, 4, 1, 1, 1), (QWEN2_7B, 4, 2, 2, 1), (QWEN2_7B, 4, 4, 4, 1), (QWEN2_7B, 4, 8, 4, 2),
    (QWEN2_0_5B, 2, 8, 2, 4), (QWEN2_72B, 8, 8, 8, 1), (TINY, 4, 4, 2, 2), (TINY, 8, 6, 2, 3),
])
def test_parallel_layout(shape, max_tp, world, tp, dp):
    seen = set()
    for r in range(world):
        lay = parallel_layout(world, r, max_tp, shape)
        assert (lay.tp, lay.dp) == (tp, dp)
        assert lay.group * tp + lay.tp_rank == r and r in lay.group_ranks()
        seen.add((lay.group, lay.tp_rank))
    assert len(seen) == world
    assert parallel_layout(world, 0, max_tp, shape).local_batch(dp * 8) == 8
    with pytest.raises(ValueError):
        parallel_layout(world, world, max_tp, shape)
    if dp > 1:
        with pytest.raises(ValueError):
            parallel_layout(world, 0, max_tp, shape).local_batch(dp * 8 + 1)


def _inputs():
    g = torch.Generator().manual_seed(11)
    ids = torch.randint(0, TINY.vocab, (BATCH, PROMPT), generator=g).numpy()
    nxt = torch.randint(0, TINY.vocab, (BATCH, 1), generator=g).numpy()
    return ids, nxt


def _oracle(tp, tp_rank, all_reduce=None, all_gather=None):
    from oracle.graph import GraphOracle

    st = random_state(TINY, dtype=torch.float32, seed=5, std=0.2)
    w = {k: v.double().numpy() for k, v in transform_weights(st, TINY, tp, tp_rank).items()}
    cos, sin = rotary_tables(TINY, CAP)
    w["rotary_cos"], w["rotary_sin"] = cos.double().numpy(), sin.double().numpy()
    return GraphOracle(build_graph(TINY, capacity=CAP, tp_size=tp), w, all_reduce=all_reduce,
                       all_gather=all_gather)


def _run(o, ids, nxt):
    b = ids.shape[0]
    pre = o.run({"input_ids": ids, "positions": np.zeros(b, dtype=np.int64)})
    dec = o.run({"input_ids": nxt, "positions": np.full(b, ids.shape[1], dtype=np.int64)})
    return pre["logits"], dec["logits"], dec["next_ids"]


def _rank_main(rank, world, port, max_tp, out_dir):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        lay = parallel_layout(world, rank, max_tp, TINY)
        # every rank creates every group, in the same order
        groups = [dist.new_group(list(range(g * lay.tp, (g + 1) * lay.tp))) for g in range(lay.dp)]
        pg = groups[lay.group]
        calls = []

        def all_reduce(a):
            t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float64))
            dist.all_reduce(t, group=pg)
            calls.append(t.numel())
            return t.numpy()

        def all_gather(a):
            t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float64))
            parts = [torch.empty_like(t) for _ in range(lay.tp)]
            dist.all_gather(parts, t, group=pg)
            return [x.numpy() for x in parts]

        ids, nxt = _inputs()
        bl = lay.local_batch(BATCH)
        rows = slice(lay.group * bl, (lay.group + 1) * bl)
        tp_hooks = (all_reduce, all_gather) if lay.tp > 1 else (None, None)
        o = _oracle(lay.tp, lay.tp_rank, *tp_hooks)
        pre, dec, next_ids = _run(o, ids[rows], nxt[rows])
        # the bench's timing rule: every rank's time, max over ranks
        t = torch.tensor([float(rank + 1)])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        np.savez(f"{out_dir}/rank{rank}.npz", pre=pre, dec=dec, next_ids=next_ids, tp=lay.tp,
                 tp_rank=lay.tp_rank, group=lay.group, calls=len(calls), tmax=t.item())
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,max_tp", [(2, 2), (4, 4)])
def test_sharded_graph_over_gloo_matches_single_rank(tmp_path, world, max_tp):
    mp.start_processes(_rank_main, args=(world, _free_port(), max_tp, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    ids, nxt = _inputs()
    ref_pre, ref_dec, ref_next = _run(_oracle(1, 0), ids, nxt)
    for r in range(world):
        res = np.load(tmp_path / f"rank{r}.npz")
        tp, group, tp_rank = int(res["tp"]), int(res["group"]), int(res["tp_rank"])
        bl = BATCH // (world // tp)
        rows = slice(group * bl, (group + 1) * bl)
        # vocab-parallel LM head: each rank holds its slice of the logits
        vs = TINY.vocab // tp
        cols = slice(tp_rank * vs, (tp_rank + 1) * vs)
        np.testing.assert_allclose(res["pre"], ref_pre[rows][:, cols], rtol=1e-10, atol=1e-12)
        np.testing.assert_allclose(res["dec"], ref_dec[rows][:, cols], rtol=1e-10, atol=1e-12)
        np.testing.assert_array_equal(res["next_ids"], ref_next[rows])
        # two all_reduce nodes per layer (after o_proj and after down_proj), prefill + decode
        assert int(res["calls"]) == (2 * TINY.layers * 2 if tp > 1 else 0)
        assert float(res["tmax"]) == world
