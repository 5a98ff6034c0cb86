"""Batch-sharded data parallelism for the depthwise Conv1D path.

The reference is single-GPU; on an 8xB200 box the batch dimension shards
naturally: FWD and dX are independent per (b, h) sequence and need no
communication, and dK is a sum over b, so each rank computes dK of its batch
slice and the [H, K] filter gradients -- 24,576 bytes at H=128, K=48 -- are
summed over the ranks.  One process per GPU with ``torch.distributed`` for the
plumbing.  The sum runs either as an NCCL all-reduce after the backward, or
(``PeerExchange``) inside the backward kernel itself: the CTA that computed a
channel's dK row stores it into every other GPU's exchange buffer over NVLink
and adds the ranks' rows (pt_dx_dk_allreduce).  Each rank reads only its own
HBM; the exchange writes into the peers' buffers.

Batch split: rank r of n owns rows [b0, b1) with the first ``B % n`` ranks
holding one extra batch (``shard_range``); uneven splits are allowed, a rank
may own zero batches.
"""
from __future__ import annotations

import ctypes
from typing import Callable

import torch
import torch.distributed as dist

from . import _lib, ops

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
                       compute: ComputeFn | None = None, group=None, exchange: "PeerExchange | None" = None):
    """One training-path step on this rank's batch shard.

    Returns (y_local, dx_local, dk) where dk is already summed over all ranks:
    through ``exchange`` (peer memory, inside the backward kernel where it
    applies) when given, else by an NCCL all-reduce.  ``compute`` defaults to
    the native GPU kernels; it is injectable so the sharding and reduction logic
    can be exercised on CPU ranks.
    """
    if exchange is not None and compute is None:
        y = ops.fwd(x_local, k)
        gk = torch.empty_like(k)
        gx = dx_dk_allreduce(dy_local, x_local, k, gk, exchange)
        return y, gx, gk
    fn = compute or native_compute
    y, gx, gk = fn(x_local, k, dy_local)
    allreduce_dk(gk, group)
    return y, gx, gk


class PeerExchangeUnavailable(RuntimeError):
    """Some rank could not allocate, export or map an exchange buffer (raised on
    every rank alike)."""


class PeerExchange:
    """Exchange buffers for summing dK over the ranks through peer memory.

    Every rank allocates one buffer on its GPU (``pt_peer_alloc``, zeroed),
    exports its CUDA IPC handle, gathers the others' over ``torch.distributed``
    and maps them; ``group()`` returns the ``pt_peer_group`` of the next call
    (the epoch advances by one per call on every rank).  Collective: every rank
    of the process group constructs it, in the same order.  ``close()`` unmaps
    the peers' buffers and frees the own one once every rank is done with it.
    """

    def __init__(self, H: int, K: int, device: torch.device, group=None) -> None:
        self.lib = _lib.load()
        self.group_ = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if not 2 <= self.world <= _lib.PT_MAX_PEERS:
            raise ValueError(f"peer exchange needs 2..{_lib.PT_MAX_PEERS} ranks, got {self.world}")
        self.H, self.K, self.device = H, K, device
        self.nbytes = int(self.lib.pt_peer_buffer_bytes(self.world, H, K))
        self._own = ctypes.c_void_p()
        self._imported: list[ctypes.c_void_p] = []
        bufs = (ctypes.c_void_p * _lib.PT_MAX_PEERS)()
        failure = ""
        with torch.cuda.device(device):
            # Every rank takes part in the same collectives whatever fails locally;
            # the outcome is agreed on with one all-reduce, so either every rank
            # has the exchange or every rank raises PeerExchangeUnavailable.
            handle = ctypes.create_string_buffer(_lib.PT_IPC_HANDLE_BYTES)
            st = self.lib.pt_peer_alloc(self.nbytes, ctypes.byref(self._own))
            if st == _lib.PT_OK:
                st = self.lib.pt_ipc_export(self._own, handle)
            if st != _lib.PT_OK:
                failure = f"rank {self.rank}: exchange buffer: {_lib.status_string(st)}"
            handles: list = [None] * self.world
            dist.all_gather_object(handles, handle.raw if not failure else None, group=group)
            for r, h in enumerate(handles):
                if failure:
                    break
                if r == self.rank:
                    bufs[r] = self._own.value
                    continue
                if h is None:
                    failure = f"rank {r} has no exchange buffer"
                    break
                ptr = ctypes.c_void_p()
                hb = ctypes.create_string_buffer(bytes(h), _lib.PT_IPC_HANDLE_BYTES)
                st = self.lib.pt_ipc_import(hb, ctypes.byref(ptr))
                if st != _lib.PT_OK:
                    failure = f"rank {self.rank} cannot map rank {r}'s buffer: {_lib.status_string(st)}"
                    break
                self._imported.append(ptr)
                bufs[r] = ptr.value
            ok = torch.tensor([0 if failure else 1], device=device, dtype=torch.int32)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
            if int(ok.item()) == 0:
                self.close()
                raise PeerExchangeUnavailable(failure or "another rank could not set up its exchange")
        self._grp = _lib.PeerGroup(self.rank, self.world, bufs, 0)

    def group(self) -> ctypes.c_void_p:
        """The pt_peer_group of the next call (advances the epoch)."""
        self._grp.epoch += 1
        return ctypes.cast(ctypes.pointer(self._grp), ctypes.c_void_p)

    def close(self) -> None:
        """Collective: unmap the peers' buffers, then free the own one once every
        rank has unmapped it."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group_)
        with torch.cuda.device(self.device):
            for ptr in self._imported:
                self.lib.pt_ipc_close(ptr)
            self._imported = []
            dist.barrier(group=self.group_)
            if self._own.value:
                self.lib.pt_peer_free(self._own)
        self._own = None


def dx_dk_allreduce(dy: torch.Tensor, x: torch.Tensor, k: torch.Tensor, gk: torch.Tensor, exchange: PeerExchange,
                    gx: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """dX of this shard into gx and dK summed over the ranks into gk (deterministic:
    gk = the sum), the sum done through the peers' exchange buffers -- inside the
    fused backward kernel where it runs with one CTA per channel."""
    B, H, L, K = ops.check_shapes(x, k)
    if tuple(dy.shape) != (B, H, L) or tuple(gk.shape) != (H, K):
        raise ValueError("gy must be shaped like x and gk like k")
    if (H, K) != (exchange.H, exchange.K):
        raise ValueError("the exchange was built for another [H, K]")
    if gx is None:
        gx = torch.empty_like(dy, memory_format=torch.contiguous_format)
    for t, n in ((dy, "gy"), (x, "x"), (k, "k"), (gk, "gk"), (gx, "gx")):
        ops._ensure_cuda_f32(t, n)
        ops._ensure_raw(t, n)
    lib = _lib.load()
    dev = x.device
    with torch.cuda.device(dev):
        ws_ptr, ws_bytes = ctypes.c_void_p(0), 0
        need = int(lib.pt_dx_dk_workspace_bytes(B, H, L, K)) if B > 0 else 0
        if need > 0:
            ws = workspace if workspace is not None else ops.WORKSPACES.get(dev, need)
            ws_ptr, ws_bytes = ops._ptr(ws), ws.numel() * ws.element_size()
        st = lib.pt_dx_dk_allreduce(ops._ptr(dy), ops._ptr(x), ops._ptr(k), ops._ptr(gx), ops._ptr(gk), B, H, L, K,
                                    ws_ptr, ws_bytes, exchange.group(), ops._stream(dev))
    _lib.check(st, "pt_dx_dk_allreduce")
    return gx


def peer_fused(B: int, H: int, L: int, K: int) -> bool:
    """True when dx_dk_allreduce sums dK inside the backward kernel at this shape."""
    return bool(_lib.load().pt_dx_dk_allreduce_fused(B, H, L, K))
