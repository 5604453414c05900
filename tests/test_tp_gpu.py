"""Tensor parallelism on two GPUs: the sharded Qwen2 graph with the plugin's
tensor-parallel operators (fused all-reduce + RMSNorm, vocab-parallel argmax),
against the same model on one GPU.

Each of two spawned ranks (one per GPU, NCCL process group, 127.0.0.1
rendezvous) runs a tp=2 Qwen2Runner on its half of the weights, and a tp=1
runner with the full weights on the same GPU. The all-reduce after o_proj and
down_proj runs as the fused NVLink exchange kernel for decode-sized rows and as
NCCL all_reduce + add_rms_norm for prefill; the LM head is split by vocabulary
and the greedy pick exchanges (value, id) candidates (each rank's logits are
compared with its slice of the single-GPU logits). Prefill logits, eager decode
logits and CUDA-graph decode ids (the graph captures the exchange kernels) are
compared: bf16 with a different summation order across ranks, so logits within
2e-2 relative Frobenius error and at least 90% of teacher-forced greedy ids
equal; free-running CUDA-graph generation on two GPUs must equal eager
generation on two GPUs exactly. Skipped on boxes with fewer than two GPUs.
"""
from __future__ import annotations

import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, port, out_dir):
    import os
    from datetime import timedelta

    import torch.distributed as dist

    from dli.parallel import TensorParallelComm, parallel_layout
    from dli.qwen2 import Qwen2Runner
    from dli_export.qwen2 import Qwen2Shape, random_state, transform_weights

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                            timeout=timedelta(seconds=120), device_id=dev)
    shape = Qwen2Shape(hidden=512, layers=2, q_heads=8, kv_heads=2, head_dim=64, intermediate=1024,
                       vocab=4096)
    lay = parallel_layout(2, rank, 2, shape)
    # exchange rows capped at 64: decode (4 rows) takes the fused NVLink kernel,
    # prefill (4 x 40 rows) the NCCL all_reduce + add_rms_norm branch
    tpc = TensorParallelComm(lay, rank, exchange=(64, shape.hidden, 2))
    res = {}
    try:
        st = random_state(shape, device=dev, dtype=torch.bfloat16, seed=7, std=0.05)
        full = Qwen2Runner(shape, transform_weights(st, shape, dtype=torch.bfloat16), capacity=256)
        shard = Qwen2Runner(shape, transform_weights(st, shape, 2, lay.tp_rank, torch.bfloat16), capacity=256,
                            tp_size=2, tp_rank=lay.tp_rank, communicator=tpc.handle)
        g = torch.Generator(device=dev).manual_seed(3)
        ids = torch.randint(0, shape.vocab, (4, 40), device=dev, generator=g)
        rel, agree = [], []
        vs = shape.vocab // 2  # vocab-parallel LM head: this rank's logits columns
        cols = slice(lay.tp_rank * vs, (lay.tp_rank + 1) * vs)
        lf, nf = full.prefill(ids)
        ls, ns = shard.prefill(ids)
        lf = lf[:, cols]
        rel.append(((ls.float() - lf.float()).norm() / lf.float().norm()).item())
        agree.append((nf == ns).float().mean().item())
        pos = torch.full((4,), 40, dtype=torch.int64, device=dev)
        step_ids = nf.view(4, 1)
        for _ in range(6):  # teacher-forced: both see the single-GPU model's tokens
            lf, nf = full.forward(step_ids, pos)
            ls, ns = shard.forward(step_ids, pos)
            lf = lf[:, cols]
            rel.append(((ls.float() - lf.float()).norm() / lf.float().norm()).item())
            agree.append((nf == ns).float().mean().item())
            step_ids, pos = nf.view(4, 1), pos + 1
        full.reset()
        shard.reset()
        gen_graph = shard.generate(ids, 12, use_graph=True)
        gen_eager = shard.generate(ids, 12, use_graph=False)
        torch.cuda.synchronize()
        res = {"rel": rel, "agree": sum(agree) / len(agree),
               "graph_eq_eager": bool(torch.equal(gen_graph, gen_eager))}
        shard.release_graphs()
        full.release_graphs()
        del shard, full
        torch.cuda.synchronize()
    finally:
        tpc.destroy()
        dist.barrier()
        dist.destroy_process_group()
    torch.save(res, f"{out_dir}/rank{rank}.pt")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp2_matches_single_gpu(tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_rank_main, args=(_free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        res = torch.load(tmp_path / f"rank{r}.pt")
        assert max(res["rel"]) < TOL, res
        assert res["agree"] >= 0.9, res
        assert res["graph_eq_eager"], res
