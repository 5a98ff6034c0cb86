"""TEST INFRASTRUCTURE ONLY -- the reference's PyTorch CPU path, restated.

The reference times and validates its kernels against a PyTorch function,
``pytorch_depthwise_same`` (benchmark/benchmark_shape_sweep_ampere.py:220-239;
twin ``depthwise_conv1d_same``, benchmark/benchmark_pytorch.py:61-77): pad the
sequence by (K//2, K-1-K//2) and run a grouped ``conv1d`` with one group per
channel; dX and dK come from autograd (benchmark/benchmark_pytorch.py:97-144).
That module cannot be imported on a machine without pycuda (its import chain
pulls in kernels.warp_tiled_ampere), so the same few torch calls are restated
here.  ``dk_fp64`` restates the tap-by-tap FP64 filter-gradient reference of
benchmark/check_dk_fp64_seeds.py:33-43.

Used by tests/, __graft_entry__.smoke() and bench.py (CPU baseline and the
``--impl reference`` arm) as the checker / baseline; never by the product.
"""
from __future__ import annotations

import zlib

import torch
import torch.nn.functional as F


def depthwise_same(x: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
    """y = conv1d(pad(x, (K//2, K-1-K//2)), k[:,None,:], groups=H): length-L output."""
    K = int(k.shape[1])
    left = K // 2
    xp = F.pad(x, (left, K - 1 - left))
    return F.conv1d(xp, k.unsqueeze(1), bias=None, stride=1, padding=0, groups=int(x.shape[1]))


def fwd_dx_dk(x: torch.Tensor, k: torch.Tensor, dy: torch.Tensor):
    """(y, dX, dK) of the reference path through autograd, in the inputs' dtype."""
    xr = x.detach().clone().requires_grad_(True)
    kr = k.detach().clone().requires_grad_(True)
    y = depthwise_same(xr, kr)
    gx, gk = torch.autograd.grad(y, (xr, kr), dy)
    return y.detach(), gx.detach(), gk.detach()


def dk_fp64(x: torch.Tensor, dy: torch.Tensor, K: int) -> torch.Tensor:
    """dK[h,j] = sum_{b,t} dy[b,h,t] x[b,h,t+j-K//2] in float64, one tap at a time."""
    L = int(x.shape[2])
    left = K // 2
    xp = F.pad(x.double(), (left, K - 1 - left))
    d = dy.double()
    return torch.stack([(xp[:, :, j:j + L] * d).sum(dim=(0, 2)) for j in range(K)], dim=1)


def make_inputs(B: int, H: int, L: int, K: int, seed: int):
    """Seeded CPU inputs in the order x, k, dy: x, dy ~ N(0,1), k ~ N(0,1)/sqrt(K)."""
    g = torch.Generator().manual_seed(int(seed))
    x = torch.randn(B, H, L, generator=g, dtype=torch.float32)
    k = torch.randn(H, K, generator=g, dtype=torch.float32) / (K ** 0.5)
    dy = torch.randn(B, H, L, generator=g, dtype=torch.float32)
    return x, k, dy


def case_seed(base_seed: int, config_id: str) -> int:
    """Per-shape seed: base + crc32(config id) (benchmark_pathtile_candidate_sweep.py:109-110)."""
    return int(base_seed + zlib.crc32(config_id.encode("utf-8")))
