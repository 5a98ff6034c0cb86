"""GPU, 2 or more ranks: the batch-sharded path matches the full-batch oracle.

Each rank owns one GPU and its slice of the batch, runs FWD / dX / dK through the
native kernels, and the per-rank dK is summed over NCCL (2 ranks) or through the
peers' exchange buffers (every visible GPU, up to 8).  Skipped when fewer than
two GPUs are visible.  NVLS is disabled for these tests (they check the data
path, not the transport).
"""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str, shape) -> None:
    import sys

    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from oracle import reference_torch
        from pathtile_b200.distributed import data_parallel_step, shard_range

        B, H, L, K = shape
        x, k, dy = reference_torch.make_inputs(B, H, L, K, seed=77)
        b0, b1 = shard_range(B, rank, world)
        y, gx, gk = data_parallel_step(x[b0:b1].to(dev), k.to(dev), dy[b0:b1].to(dev))
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"r{rank}_y.npy"), y.cpu().numpy())
        np.save(os.path.join(out_dir, f"r{rank}_gx.npy"), gx.cpu().numpy())
        np.save(os.path.join(out_dir, f"r{rank}_gk.npy"), gk.cpu().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("shape", [(1025, 128, 48, 48), (301, 64, 37, 13)])
def test_two_rank_batch_sharding_matches_oracle(tmp_path, shape):
    import torch.multiprocessing as mp

    from oracle import c_oracle, reference_torch

    mp.spawn(_rank_main, args=(2, _free_port(), str(tmp_path), shape), nprocs=2, join=True)
    B, H, L, K = shape
    x, k, dy = reference_torch.make_inputs(B, H, L, K, seed=77)
    y = np.concatenate([np.load(tmp_path / f"r{r}_y.npy") for r in range(2)])
    gx = np.concatenate([np.load(tmp_path / f"r{r}_gx.npy") for r in range(2)])
    np.testing.assert_allclose(y, c_oracle.fwd(x, k), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(gx, c_oracle.dx(dy, k), rtol=1e-5, atol=1e-5)
    ref = c_oracle.dk(dy, x, K)
    scale = float(np.abs(ref).max())
    for r in range(2):
        np.testing.assert_allclose(np.load(tmp_path / f"r{r}_gk.npy"), ref, rtol=1e-4, atol=1e-4 * scale)


def _peer_world() -> int:
    return min(torch.cuda.device_count(), 8)


def _rank_main_peer(rank: int, world: int, port: int, out_dir: str, shape, calls: int) -> None:
    """The sharded step with dK summed through the peers' exchange buffers,
    `calls` times in a row (the epochs alternate the exchange slots)."""
    import sys

    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    ex = None
    try:
        from oracle import reference_torch
        from pathtile_b200 import ops
        from pathtile_b200.distributed import PeerExchange, data_parallel_step, peer_fused, shard_range

        B, H, L, K = shape
        ex = PeerExchange(H, K, dev)
        b0, b1 = shard_range(B, rank, world)
        for call in range(calls):
            x, k, dy = reference_torch.make_inputs(B, H, L, K, seed=100 + call)
            y, gx, gk = data_parallel_step(x[b0:b1].to(dev), k.to(dev), dy[b0:b1].to(dev), exchange=ex)
            torch.cuda.synchronize()
            np.save(os.path.join(out_dir, f"c{call}_r{rank}_gx.npy"), gx.cpu().numpy())
            np.save(os.path.join(out_dir, f"c{call}_r{rank}_gk.npy"), gk.cpu().numpy())
        with open(os.path.join(out_dir, f"r{rank}_info.txt"), "w") as f:
            f.write(f"{int(peer_fused(b1 - b0, H, L, K))} {ops.device_error()}")
    finally:
        if ex is not None:
            ex.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("shape,fused", [((2048, 128, 48, 48), 1), ((301, 64, 37, 13), 0), ("mixed", None)])
def test_peer_memory_dk_sum_matches_oracle(tmp_path, shape, fused):
    """dK summed over every visible GPU's rank inside the fused backward kernel (one CTA per
    channel) or by the standalone peer kernel after the backward: every rank gets
    the same bits, equal to the full-batch FP64 dK within 1e-4, on four calls in
    a row.  "mixed": at H = 64 a shard of 128 rows runs the fused kernel with one
    CTA per channel and a shard of 129 rows needs two CTAs per channel, so with
    B = 128 * world + 1 rank 0 takes the separate path (backward, then the peer
    kernel) while the others sum inside the backward kernel, through the same slots."""
    import torch.multiprocessing as mp

    from oracle import c_oracle, reference_torch

    calls = 4
    world = _peer_world()
    if shape == "mixed":
        shape = (128 * world + 1, 64, 48, 48)
    mp.spawn(_rank_main_peer, args=(world, _free_port(), str(tmp_path), shape, calls), nprocs=world, join=True)
    B, H, L, K = shape
    for r in range(world):
        kind, err = (int(v) for v in (tmp_path / f"r{r}_info.txt").read_text().split())
        assert err == 0
        if torch.cuda.get_device_properties(0).multi_processor_count == 148:
            assert kind == (fused if fused is not None else int(r > 0))
    for call in range(calls):
        x, k, dy = reference_torch.make_inputs(B, H, L, K, seed=100 + call)
        gx = np.concatenate([np.load(tmp_path / f"c{call}_r{r}_gx.npy") for r in range(world)])
        np.testing.assert_allclose(gx, c_oracle.dx(dy, k), rtol=1e-5, atol=1e-5)
        ref = c_oracle.dk(dy, x, K)
        scale = float(np.abs(ref).max())
        gk0 = np.load(tmp_path / f"c{call}_r0_gk.npy")
        for r in range(1, world):  # rank-ordered sum: the same bits on every rank
            assert np.array_equal(gk0, np.load(tmp_path / f"c{call}_r{r}_gk.npy"))
        np.testing.assert_allclose(gk0, ref, rtol=1e-4, atol=1e-4 * scale)
