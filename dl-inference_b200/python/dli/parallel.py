"""Multi-GPU plumbing for one process per GPU: where a rank sits in a
tensor-parallel x data-parallel job, and the NCCL communicator that the
plugin's `all_reduce` operator runs on.

The reference has no multi-GPU path; its `all_reduce`-free graphs run on one
device. Here a tensor-parallel graph (dli_export.qwen2.build_graph with
tp_size > 1) carries `all_reduce` nodes, and `Engine.set_communicator` hands the
plugin an `ncclComm_t` created by the plugin itself, so the same NCCL library
that launches the collective also owns the communicator.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Any

from . import PLUGIN_PATH


@dataclass(frozen=True)
class ParallelLayout:
    """Where one rank sits in a tensor-parallel x data-parallel job.

    Ranks r = group * tp + tp_rank: consecutive ranks share one tensor-parallel
    group (one NCCL communicator, all_reduce after o_proj and down_proj); the
    `dp` groups each serve batch / dp sequences with a full copy of the weights."""
    world: int
    rank: int
    tp: int
    dp: int
    group: int
    tp_rank: int

    def local_batch(self, batch: int) -> int:
        if batch % self.dp:
            raise ValueError(f"batch {batch} not divisible by {self.dp} data-parallel groups")
        return batch // self.dp

    def group_ranks(self) -> list[int]:
        return list(range(self.group * self.tp, (self.group + 1) * self.tp))


def parallel_layout(world: int, rank: int, max_tp: int, shape: Any | None = None) -> ParallelLayout:
    """The largest power-of-two tensor-parallel degree <= max_tp that divides the
    world size (and, given a shape, the q/kv head counts and the intermediate
    size, which the Megatron column/row split needs); the rest is data parallel."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    tp = 1
    while tp * 2 <= min(world, max_tp) and world % (tp * 2) == 0:
        if shape is not None and (shape.q_heads % (tp * 2) or shape.kv_heads % (tp * 2)
                                  or shape.intermediate % (tp * 2)):
            break
        tp *= 2
    return ParallelLayout(world, rank, tp, world // tp, rank // tp, rank % tp)


class TensorParallelComm:
    """One NCCL communicator per tensor-parallel group, created by the plugin
    (dli_sm100_nccl_unique_id / dli_sm100_nccl_comm_init). Rank 0 makes one
    unique id per group and broadcasts them over the torch.distributed default
    group, so every rank takes the same collective steps whatever its group.

    `handle` is the ncclComm_t as an integer for Engine.set_communicator (0 when
    tp == 1). With `exchange=(max_rows, row_elems, dtype_code)` it also creates
    the group's NVLink exchange buffers (dli_sm100_tp_exchange_create), which
    the `all_reduce_add_rms_norm` operator uses for rows <= max_rows. Call
    destroy() after every CUDA graph that captured a collective on it has been
    released; it synchronises the device and the group first."""

    def __init__(self, layout: ParallelLayout, device_index: int, plugin: str = PLUGIN_PATH,
                 exchange: tuple[int, int, int] | None = None):
        import torch.distributed as dist

        self.layout = layout
        self.handle = 0
        self._lib = None
        if layout.tp == 1:
            return
        lib = ctypes.CDLL(plugin)
        lib.dli_sm100_nccl_unique_id.restype = ctypes.c_int
        lib.dli_sm100_nccl_unique_id.argtypes = [ctypes.c_void_p, ctypes.c_int]
        lib.dli_sm100_nccl_comm_init.restype = ctypes.c_void_p
        lib.dli_sm100_nccl_comm_init.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        lib.dli_sm100_nccl_comm_destroy.argtypes = [ctypes.c_void_p]
        lib.dli_sm100_tp_exchange_create.restype = ctypes.c_int
        lib.dli_sm100_tp_exchange_create.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64,
                                                     ctypes.c_int64, ctypes.c_int]
        lib.dli_sm100_tp_exchange_destroy.argtypes = [ctypes.c_void_p]
        ids: list[Any] = [None] * layout.dp
        if layout.rank == 0:
            for g in range(layout.dp):
                buf = ctypes.create_string_buffer(256)
                n = lib.dli_sm100_nccl_unique_id(buf, 256)
                ids[g] = buf.raw[:n] if n > 0 else None
        dist.broadcast_object_list(ids, src=0)
        if any(i is None for i in ids):
            raise RuntimeError("operator plugin built without NCCL: tensor parallelism unavailable")
        mine = ctypes.create_string_buffer(ids[layout.group], len(ids[layout.group]))
        handle = lib.dli_sm100_nccl_comm_init(mine, layout.tp, layout.tp_rank, device_index)
        if not handle:
            raise RuntimeError(f"ncclCommInitRank failed on rank {layout.rank} (group {layout.group})")
        self.handle, self._lib = int(handle), lib
        self.exchange = None
        if exchange is not None:
            rc = lib.dli_sm100_tp_exchange_create(ctypes.c_void_p(self.handle), device_index, *exchange)
            # every rank learns whether every rank succeeded (the operator must take
            # the same branch on all of them)
            import torch
            flag = torch.tensor([1 if rc == 0 else 0], device=f"cuda:{device_index}")
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            if int(flag.item()) != 1:
                if rc == 0:
                    lib.dli_sm100_tp_exchange_destroy(ctypes.c_void_p(self.handle))
                raise RuntimeError(f"tensor-parallel exchange buffers unavailable (rank {layout.rank}: code {rc})")
            self.exchange = exchange
        self._device = device_index

    def destroy(self) -> None:
        if self.handle and self._lib is not None:
            import torch
            import torch.distributed as dist

            torch.cuda.synchronize(self._device)
            dist.barrier()  # no rank still pushes into a buffer about to be unmapped
            self._lib.dli_sm100_tp_exchange_destroy(ctypes.c_void_p(self.handle))
            self._lib.dli_sm100_nccl_comm_destroy(ctypes.c_void_p(self.handle))
        self.handle = 0
