"""Batch-sharded data parallelism for the depthwise Conv1D path.

The reference is single-GPU; on an 8xB200 box the batch dimension shards
naturally: FWD and dX are independent per (b, h) sequence and need no
communication, and dK is a sum over b, so each rank computes dK of its batch
slice and one all-reduce (sum) of the [H, K] filter gradient -- 24,576 bytes
at H=128, K=48 -- combines them.  One process per GPU, ``torch.distributed``
over NCCL (NVLink / NVSwitch) for that all-reduce; each rank reads only its
own HBM.

Batch split: rank r of n owns rows [b0, b1) with the first ``B % n`` ranks
holding one extra batch (``shard_range``); uneven splits are allowed, a rank
may own zero batches.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

from . import ops

ComputeFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], tuple[torch.Tensor, torch.Tensor, torch.Tensor]]


def shard_range(B: int, rank: int, world: int) -> tuple[int, int]:
    """[b0, b1) of the batch owned by `rank` (remainder spread over the first ranks)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} for world size {world}")
    if B < 0:
        raise ValueError("B must be non-negative")
    base, extra = divmod(B, world)
    b0 = rank * base + min(rank, extra)
    return b0, b0 + base + (1 if rank < extra else 0)


def native_compute(x: torch.Tensor, k: torch.Tensor, dy: torch.Tensor):
    """FWD, dX and this shard's dK on the GPU through the native library (the
    backward as one ops.dx_dk call: the fused kernel where the shape allows)."""
    y = ops.fwd(x, k)
    gk = torch.empty_like(k)
    gx = ops.dx_dk(dy, x, k, gk, mode="deterministic")
    return y, gx, gk


def allreduce_dk(gk: torch.Tensor, group=None) -> torch.Tensor:
    """Sum the per-rank filter gradients in place (the only collective of the path)."""
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(gk, op=dist.ReduceOp.SUM, group=group)
    return gk


def data_parallel_step(x_local: torch.Tensor, k: torch.Tensor, dy_local: torch.Tensor,
                       compute: ComputeFn | None = None, group=None):
    """One training-path step on this rank's batch shard.

    Returns (y_local, dx_local, dk) where dk is already summed over all ranks.
    ``compute`` defaults to the native GPU kernels; it is injectable so the
    sharding and reduction logic can be exercised on CPU ranks.
    """
    fn = compute or native_compute
    y, gx, gk = fn(x_local, k, dy_local)
    allreduce_dk(gk, group)
    return y, gx, gk
