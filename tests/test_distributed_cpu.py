"""CPU (gloo) tests of the batch-sharded path: sharding, the dK all-reduce, and
a rank failure detected on the host.  Per-rank work is the FP64 C oracle
injected as the compute function, so no GPU is touched."""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from pathtile_b200.distributed import data_parallel_step, shard_range


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("B,world", [(10, 2), (7, 3), (16384, 8), (3, 4), (0, 2)])
def test_shard_range_covers_batch(B, world):
    spans = [shard_range(B, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == B
    for (a0, a1), (b0, _) in zip(spans, spans[1:]):
        assert a1 == b0 and a1 >= a0
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


def _oracle_compute(x, k, dy):
    from oracle import c_oracle

    K = int(k.shape[1])
    y = torch.from_numpy(c_oracle.fwd(x, k))
    gx = torch.from_numpy(c_oracle.dx(dy, k))
    gk = torch.from_numpy(c_oracle.dk(dy, x, K))
    return y, gx, gk


def _worker(rank, world, port, B, H, L, K, out_dir, fail_rank):
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        from oracle import reference_torch

        x, k, dy = reference_torch.make_inputs(B, H, L, K, seed=5)
        b0, b1 = shard_range(B, rank, world)
        if rank == fail_rank:
            raise RuntimeError("injected rank failure before the dK all-reduce")
        try:
            y, gx, gk = data_parallel_step(x[b0:b1], k, dy[b0:b1], compute=_oracle_compute)
            np.save(os.path.join(out_dir, f"r{rank}_y.npy"), y.numpy())
            np.save(os.path.join(out_dir, f"r{rank}_gx.npy"), gx.numpy())
            np.save(os.path.join(out_dir, f"r{rank}_gk.npy"), gk.numpy())
        except Exception as exc:  # the surviving rank records how it learned of the failure
            with open(os.path.join(out_dir, f"r{rank}_error.txt"), "w") as f:
                f.write(repr(exc))
    finally:
        if rank != fail_rank:
            dist.destroy_process_group()


@pytest.mark.parametrize("world,B", [(2, 9), (3, 16)])
def test_gloo_ranks_match_full_batch_oracle(tmp_path, world, B):
    H, L, K = 6, 20, 7
    mp.spawn(_worker, args=(world, _free_port(), B, H, L, K, str(tmp_path), -1), nprocs=world, join=True)
    from oracle import c_oracle, reference_torch

    x, k, dy = reference_torch.make_inputs(B, H, L, K, seed=5)
    y = np.concatenate([np.load(tmp_path / f"r{r}_y.npy") for r in range(world)])
    gx = np.concatenate([np.load(tmp_path / f"r{r}_gx.npy") for r in range(world)])
    np.testing.assert_allclose(y, c_oracle.fwd(x, k), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(gx, c_oracle.dx(dy, k), rtol=1e-12, atol=1e-12)
    ref = c_oracle.dk(dy, x, K)
    for r in range(world):  # every rank holds the all-reduced dK
        np.testing.assert_allclose(np.load(tmp_path / f"r{r}_gk.npy"), ref, rtol=1e-12, atol=1e-12)


def test_rank_failure_surfaces_as_error_on_survivor(tmp_path):
    ctx = mp.start_processes(_worker, args=(2, _free_port(), 8, 4, 16, 5, str(tmp_path), 1), nprocs=2,
                             join=False, start_method="spawn")
    with pytest.raises(Exception):
        while not ctx.join(timeout=60):
            pass
    # Rank 0 did not hang: its all-reduce ended with an error within the group timeout.
    err = (tmp_path / "r0_error.txt")
    assert err.exists(), "survivor did not report the failed collective"
