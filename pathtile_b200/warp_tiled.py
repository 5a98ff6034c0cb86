"""Drop-in replacement of the reference module ``kernels/warp_tiled.py``.

Same public names (``__all__``, kernels/warp_tiled.py:1020-1031) and the same
argument checks and exceptions (:796-830: ValueError for non-CUDA tensors,
wrong rank and channel mismatch; TypeError for non-FP32), but the kernels
behind ``DepthwiseConvShared`` are the B200 native FWD / dX / dK kernels, not
the reference's shared-memory family.  As in the reference, every launch is
bracketed by CUDA events with a synchronize on both sides and its duration is
appended to ``FWD_TIMES`` / ``BWD_IN_TIMES`` / ``BWD_K_TIMES`` (:736-780);
this serialises the op, exactly like the reference.  The dK output is written
(not accumulated), matching the reference's ``empty_like`` gradient (:902).

Differences: the reference raises RuntimeError at import when CUDA is absent
(:15-18); this module imports anywhere and raises at call time instead, and it
accepts L <= 48 and K <= 48 only (the reference's shared kernels took any L).
The shared-memory helpers describe the reference's tile geometry and are kept
for callers that print them.
"""
from __future__ import annotations

import torch

from . import ops

TTILE = 32
HTILE = 16
THREADS_PER_BLOCK = TTILE * HTILE  # 512
BWD_K_B_TILE = 64


def bwd_kernel_shared_memory_bytes(L: int) -> int:
    """Bytes of the reference dK batch tile: x and gy for BWD_K_B_TILE rows of L floats."""
    return 2 * BWD_K_B_TILE * L * 4


def shared_memory_bytes(K: int) -> int:
    """Bytes of the reference FWD / dX tile: HTILE rows of TTILE + K - 1 floats."""
    return HTILE * (TTILE + K - 1) * 4


FWD_TIMES: list[float] = []
BWD_IN_TIMES: list[float] = []
BWD_K_TIMES: list[float] = []


def reset_timing_collectors() -> None:
    FWD_TIMES.clear()
    BWD_IN_TIMES.clear()
    BWD_K_TIMES.clear()


class CudaContextGuard:
    """No-op context manager kept for callers of the reference's PyCUDA guard
    (kernels/warp_tiled.py:30-38); launches here need no context push."""

    def __enter__(self):
        return self

    def __exit__(self, exc_type, exc_val, exc_tb):
        return False


def _time_launch(fn) -> float:
    """Synchronous CUDA-event timing of one launch on the current stream."""
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    fn()
    end.record()
    end.synchronize()
    return float(start.elapsed_time(end))


def _require_cuda() -> None:
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA GPU is required.")


class DepthwiseConvShared(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: torch.Tensor, kernel: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda or not kernel.is_cuda:
            raise ValueError("x and kernel must be CUDA tensors")
        if x.dtype != torch.float32:
            raise TypeError("x must be float32")
        if kernel.dtype != torch.float32:
            raise TypeError("kernel must be float32")
        if x.ndim != 3:
            raise ValueError(f"x must be [B,H,L], got {tuple(x.shape)}")
        if kernel.ndim != 2:
            raise ValueError(f"kernel must be [H,K], got {tuple(kernel.shape)}")
        _require_cuda()
        x = x.contiguous()
        kernel = kernel.contiguous()
        B, H, L = x.shape
        Hk, K = kernel.shape
        if H != Hk:
            raise ValueError(f"Channel mismatch: x H={H}, kernel H={Hk}")
        ops.check_shapes(x, kernel)
        ctx.save_for_backward(x, kernel)
        ctx.params = (B, H, L, K)
        y = torch.empty_like(x)
        FWD_TIMES.append(_time_launch(lambda: ops.fwd(x, kernel, y)))
        return y

    @staticmethod
    def backward(ctx, grad_y: torch.Tensor):
        x, kernel = ctx.saved_tensors
        grad_y = grad_y.contiguous()
        gx = torch.empty_like(x)
        gk = torch.empty_like(kernel)
        BWD_IN_TIMES.append(_time_launch(lambda: ops.dx(grad_y, kernel, gx)))
        BWD_K_TIMES.append(_time_launch(lambda: ops.dk(grad_y, x, gk, mode="deterministic")))
        return gx, gk


def depthwise_conv_shared(x: torch.Tensor, kernel: torch.Tensor) -> torch.Tensor:
    return DepthwiseConvShared.apply(x, kernel)


__all__ = [
    "DepthwiseConvShared",
    "depthwise_conv_shared",
    "THREADS_PER_BLOCK",
    "TTILE",
    "HTILE",
    "shared_memory_bytes",
    "FWD_TIMES",
    "BWD_IN_TIMES",
    "BWD_K_TIMES",
    "reset_timing_collectors",
]
