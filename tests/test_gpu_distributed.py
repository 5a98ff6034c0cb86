"""GPU, 2 ranks: the batch-sharded path over NCCL matches the full-batch oracle.

Each rank owns one GPU and its slice of the batch, runs FWD / dX / dK through the
native kernels, and the per-rank dK is all-reduced over NCCL.  Skipped when
fewer than two GPUs are visible.  NVLS is disabled for this test (it checks the
data path, not the transport).
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
