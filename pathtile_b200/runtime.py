"""Runtime and autograd operator of the B200 warp-tiled depthwise Conv1D path.

Mirrors the reference runtime surface of kernels/warp_tiled_ampere.py so a
caller can switch by changing the import:

* :class:`B200WarpRuntime` (alias ``AmpereWarpRuntime``) -- the counterpart of
  ``AmpereWarpRuntime`` (:625-846): ``launch_fwd``, ``launch_bwd_input``,
  ``launch_bwd_weight``, ``resource_report``, ``close``;
* ``install_runtime`` / ``get_runtime`` (:849-860);
* :class:`DepthConvB200` (alias ``DepthConvAmpere``) and
  ``depthwise_conv_b200`` (alias ``depthwise_conv_ampere``) (:863-898);
* ``KernelEventCollector`` / ``KERNEL_EVENTS`` (:278-333), the GPU profile
  table (:76-256) with a compute-capability 10.0 entry, and the measurement
  helpers ``minimum_algorithmic_bytes`` / ``algorithmic_bandwidth_gbps``
  (:263-272) and ``summarize_kernel_times`` (:990-1018).

Differences that follow from the design: there is no PyCUDA context (launches
go through the C ABI on the caller's current stream, so ``close`` only
synchronises); launch parameters are runtime values of the native library
(no recompilation per candidate); ``bwdk_block`` means rows (threads) per dK
tile and ``warps_per_block`` means 32-row FWD/dX tiles.
"""
from __future__ import annotations

import threading
import warnings
from dataclasses import dataclass
from typing import Any, Callable

import torch

from . import ops

WARP_SIZE = 32
MAX_L = 48
MAX_K = 48

DEFAULT_B = 16_384
DEFAULT_H = 128
DEFAULT_L = 48
DEFAULT_K = 48

# Reference launch constants (kernels/warp_tiled_ampere.py:71-74).  On B200 the
# frozen table inside the native library decides; None below means "frozen".
DEFAULT_WARPS_PER_BLOCK = 16
DEFAULT_BWDK_BTILE = 64
DEFAULT_BWDK_KPACK = 4
DEFAULT_BWDK_BLOCK = 128


@dataclass(frozen=True)
class GPUProfile:
    key: str
    display_name: str
    compute_capability: tuple[int, int]
    peak_bandwidth_gbps: float
    max_threads_per_sm: int
    max_blocks_per_sm: int
    max_regs_per_sm: int
    max_smem_per_sm: int
    max_warps_per_sm: int

    @property
    def limits(self) -> dict[str, int]:
        return {
            "max_threads_per_sm": self.max_threads_per_sm,
            "max_blocks_per_sm": self.max_blocks_per_sm,
            "max_regs_per_sm": self.max_regs_per_sm,
            "max_smem_per_sm": self.max_smem_per_sm,
            "max_warps_per_sm": self.max_warps_per_sm,
        }


# Compute capability 10.0 (B200): 148 SMs, 64K registers, 228 KB shared memory
# and 64 warps per SM; 8 TB/s nominal HBM3e.  The kernels are sm_100a-only.
GPU_PROFILES = {
    (10, 0): GPUProfile(
        key="b200",
        display_name="NVIDIA B200",
        compute_capability=(10, 0),
        peak_bandwidth_gbps=8000.0,
        max_threads_per_sm=2048,
        max_blocks_per_sm=32,
        max_regs_per_sm=65_536,
        max_smem_per_sm=228 * 1024,
        max_warps_per_sm=64,
    ),
}


def detect_gpu_profile(device_id: int) -> GPUProfile:
    """Profile of a supported device; raises RuntimeError otherwise (as the
    reference does for unsupported capabilities, kernels/warp_tiled_ampere.py:139-146)."""
    capability = tuple(torch.cuda.get_device_capability(device_id))
    if capability not in GPU_PROFILES:
        raise RuntimeError(
            "The B200 path requires compute capability 10.0 (sm_100a); detected CC "
            f"{capability[0]}.{capability[1]}."
        )
    return GPU_PROFILES[capability]


def ceil_div(a: int, b: int) -> int:
    return (a + b - 1) // b


def round_up(value: int, quantum: int) -> int:
    return ceil_div(value, quantum) * quantum


def max_abs_diff(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a - b).abs().max().item())


def normalized_max_abs(a: torch.Tensor, b: torch.Tensor, eps: float = 1e-12) -> float:
    scale = max(float(b.abs().max().item()), eps)
    return max_abs_diff(a, b) / scale


def estimate_gpu_occupancy(
    threads_per_block: int, regs_per_thread: int, smem_per_block: int, profile: GPUProfile
) -> dict[str, Any]:
    """Analytic resident-CTA estimate from per-CTA resources (registers rounded
    to 256 per warp, shared memory to 256 bytes); the occupancy API value is
    reported beside it by :meth:`B200WarpRuntime.resource_report`."""
    if threads_per_block <= 0 or threads_per_block > 1024:
        raise ValueError("threads_per_block must be in [1, 1024]")
    lim = profile.limits
    warps = ceil_div(threads_per_block, WARP_SIZE)
    regs_block = round_up(regs_per_thread * WARP_SIZE, 256) * warps
    smem = round_up(smem_per_block, 256) if smem_per_block else 0
    cons = {
        "threads": lim["max_threads_per_sm"] // threads_per_block,
        "warps": lim["max_warps_per_sm"] // warps,
        "registers": lim["max_regs_per_sm"] // regs_block if regs_block else lim["max_blocks_per_sm"],
        "shared_memory": lim["max_smem_per_sm"] // smem if smem else lim["max_blocks_per_sm"],
        "architectural_block_limit": lim["max_blocks_per_sm"],
    }
    blocks = max(0, min(cons.values()))
    active = min(blocks * warps, lim["max_warps_per_sm"])
    lowest = min(cons.values())
    return {
        "threads_per_block": threads_per_block,
        "warps_per_block": warps,
        "regs_per_thread": regs_per_thread,
        "allocated_regs_per_block": regs_block,
        "static_smem_bytes": smem_per_block,
        "allocated_smem_bytes_est": smem,
        "resident_blocks_per_sm_est": blocks,
        "active_warps_per_sm_est": active,
        "occupancy_est": active / lim["max_warps_per_sm"],
        "limiting_resources_est": ",".join(k for k, v in cons.items() if v == lowest),
        "gpu_profile": profile.key,
        "compute_capability": f"{profile.compute_capability[0]}.{profile.compute_capability[1]}",
    }


estimate_ampere_occupancy = estimate_gpu_occupancy


def minimum_algorithmic_bytes(B: int, H: int, L: int, K: int) -> int:
    """Unique bytes one phase must move: two [B,H,L] FP32 tensors plus [H,K]
    (kernels/warp_tiled_ampere.py:263-266)."""
    return (2 * B * H * L + H * K) * 4


def algorithmic_bandwidth_gbps(num_bytes: int, time_ms: float) -> float:
    if time_ms <= 0:
        return float("nan")
    return num_bytes / (time_ms / 1000.0) / 1e9


def in_range_pairs(L: int, K: int) -> int:
    """(t, j) pairs with 0 <= t+j-K//2 < L for one sequence: the FMAs a phase needs."""
    pad = K // 2
    return sum(max(0, min(L, L + pad - j) - max(0, pad - j)) for j in range(K))


def algorithmic_flops(B: int, H: int, L: int, K: int) -> int:
    """2 x in-range FMAs over all sequences (padded taps are not counted)."""
    return 2 * in_range_pairs(L, K) * B * H


class KernelEventCollector:
    """CUDA-event timing of launches without per-launch synchronisation
    (kernels/warp_tiled_ampere.py:278-333): events are recorded on the current
    stream around each launch and resolved after one synchronize."""

    def __init__(self) -> None:
        self.enabled = False
        self._context: dict[str, Any] = {}
        self._events: list[tuple[str, torch.cuda.Event, torch.cuda.Event, dict[str, Any]]] = []

    def set_context(self, **context: Any) -> None:
        self._context = dict(context)

    def clear(self) -> None:
        self._events.clear()
        self._context.clear()

    def launch(self, phase: str, launch_fn: Callable[[], None], metadata: dict[str, Any] | None = None) -> None:
        if not self.enabled:
            launch_fn()
            return
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        launch_fn()
        end.record()
        row = dict(self._context)
        if metadata:
            row.update(metadata)
        self._events.append((phase, start, end, row))

    def resolve_rows(self, synchronize: bool = True) -> list[dict[str, Any]]:
        if synchronize:
            torch.cuda.synchronize()
        rows: list[dict[str, Any]] = []
        counts: dict[str, int] = {}
        for phase, start, end, meta in self._events:
            counts[phase] = counts.get(phase, 0) + 1
            rows.append({**meta, "phase": phase, "run_id": counts[phase],
                         "runtime_ms": float(start.elapsed_time(end))})
        return rows

    def resolve(self, synchronize: bool = True):
        """Rows as a pandas DataFrame (the reference's return type)."""
        import pandas as pd

        return pd.DataFrame(self.resolve_rows(synchronize))


KERNEL_EVENTS = KernelEventCollector()


def summarize_kernel_times(rows) -> list[dict[str, Any]]:
    """Per-phase mean/median/std/p05/p95 of ``runtime_ms`` rows
    (kernels/warp_tiled_ampere.py:990-1018)."""
    import numpy as np

    if hasattr(rows, "to_dict"):
        rows = rows.to_dict("records")
    phases: dict[str, list[float]] = {}
    for r in rows:
        phases.setdefault(r["phase"], []).append(float(r["runtime_ms"]))
    out = []
    for phase, vals in phases.items():
        v = np.asarray(vals, dtype=float)
        out.append({
            "phase": phase,
            "runs": int(v.size),
            "mean_ms": float(v.mean()),
            "median_ms": float(np.median(v)),
            "std_ms": float(v.std(ddof=1)) if v.size > 1 else 0.0,
            "p05_ms": float(np.quantile(v, 0.05)),
            "p95_ms": float(np.quantile(v, 0.95)),
        })
    return out


class B200WarpRuntime:
    """Launcher for the native FWD / dX / dK kernels.

    ``warps_per_block`` (FWD/dX rows per tile / 32), ``bwdk_block`` (dK rows
    per tile), ``stages`` and ``ctas_per_sm`` override the frozen PathTile
    table of the native library for every shape; leave them None to use the
    frozen choice.  The overrides belong to this runtime object: they travel
    with each of its launches as per-call options (``pt_*_ex``), so two
    runtimes in one process, a tuner beside a training job for instance, never
    see each other's choices (the reference compiles one kernel module per
    runtime, kernels/warp_tiled_ampere.py:636-691).
    ``dk_mode`` selects the dK reduction: "deterministic" (two-pass, default)
    or "atomic".  Both accumulate into ``gk`` in ``launch_bwd_weight`` so the
    reference contract -- the caller zero-fills gk -- holds for either.
    ``fuse_backward`` (B200 addition, default on): when autograd needs both
    gradients at a shape the fused kernel covers, backward is one
    ``launch_bwd_fused`` (phase "bwd_fused") instead of the reference's two
    launches; the explicit ``launch_bwd_input`` / ``launch_bwd_weight`` calls
    are unchanged.
    """

    def __init__(
        self,
        warps_per_block: int | None = None,
        bwdk_btile: int = DEFAULT_BWDK_BTILE,
        bwdk_block: int | None = None,
        fast_math: bool = False,
        stages: int | None = None,
        ctas_per_sm: int | None = None,
        threads_per_row: int = 1,
        dk_mode: str = "deterministic",
        device: int | None = None,
        fuse_backward: bool = True,
    ) -> None:
        if warps_per_block is not None and warps_per_block not in {1, 2, 4, 8}:
            raise ValueError("warps_per_block must be one of 1,2,4,8 (32..256 rows per tile)")
        if bwdk_btile != 64:
            raise ValueError("This paper-confirmed version fixes BWDK_BTILE=64")
        if bwdk_block is not None and (bwdk_block < 32 or bwdk_block > 256 or bwdk_block % 32):
            raise ValueError("bwdk_block must be a multiple of 32 in [32, 256]")
        if stages is not None and stages not in (2, 3, 4):
            raise ValueError("stages must be 2, 3 or 4")
        if ctas_per_sm is not None and ctas_per_sm not in (1, 2, 3, 4):
            raise ValueError("ctas_per_sm must be 1, 2, 3 or 4")
        if fast_math:
            warnings.warn("fast_math is ignored: the B200 kernels are always strict FP32", stacklevel=2)
        if dk_mode not in ops.DK_MODES:
            raise ValueError(f"dk_mode must be one of {sorted(ops.DK_MODES)}")
        if not torch.cuda.is_available():
            raise RuntimeError("CUDA GPU is required")
        self.device_id = torch.cuda.current_device() if device is None else int(device)
        self.profile = detect_gpu_profile(self.device_id)
        self.technique = f"WarpThread-{self.profile.key}"
        self.warps_per_block = warps_per_block
        self.bwdk_btile = bwdk_btile
        self.bwdk_block = bwdk_block
        self.stages = stages
        self.ctas_per_sm = ctas_per_sm
        if threads_per_row not in (1, 2):
            raise ValueError("threads_per_row must be 1 or 2")
        self.threads_per_row = threads_per_row
        self.dk_mode = dk_mode
        self.fuse_backward = bool(fuse_backward)
        self.fast_math = False
        self._closed = False
        self.opts = launch_options(warps_per_block, bwdk_block, stages, ctas_per_sm, threads_per_row)

    @staticmethod
    def _check_shapes(x: torch.Tensor, k: torch.Tensor) -> tuple[int, int, int, int]:
        return ops.check_shapes(x, k)

    def _check_open(self) -> None:
        if self._closed:
            raise RuntimeError("runtime is closed")

    def launch_fwd(self, x: torch.Tensor, k: torch.Tensor, y: torch.Tensor,
                   collector: KernelEventCollector | None = None) -> None:
        self._check_open()
        B, H, L, K = self._check_shapes(x, k)
        (collector or KERNEL_EVENTS).launch("fwd", lambda: ops.fwd(x, k, y, opts=self.opts),
                                            {"B": B, "H": H, "L": L, "K": K})

    def launch_bwd_input(self, gy: torch.Tensor, k: torch.Tensor, gx: torch.Tensor,
                         collector: KernelEventCollector | None = None) -> None:
        self._check_open()
        B, H, L, K = self._check_shapes(gy, k)
        (collector or KERNEL_EVENTS).launch("bwd_input", lambda: ops.dx(gy, k, gx, opts=self.opts),
                                            {"B": B, "H": H, "L": L, "K": K})

    def launch_bwd_weight(self, gy: torch.Tensor, x: torch.Tensor, gk: torch.Tensor, K: int,
                          collector: KernelEventCollector | None = None) -> None:
        """gk += dK (gk zero-filled by the caller, as in the reference)."""
        self._check_open()
        for t, n in ((gy, "gy"), (x, "x"), (gk, "gk")):
            if not t.is_cuda:
                raise ValueError("gy, x, and gk must be CUDA tensors")
            if t.dtype != torch.float32:
                raise ValueError("Only FP32 is supported")
        if gy.shape != x.shape:
            raise ValueError("gy and x must have the same [B,H,L] shape")
        B, H, L = map(int, x.shape)
        if tuple(gk.shape) != (H, K):
            raise ValueError(f"gk must have shape {(H, K)}")
        if L > MAX_L or K > MAX_K:
            raise ValueError(f"Specialized kernels require L<={MAX_L}, K<={MAX_K}")
        mode = self.dk_mode
        (collector or KERNEL_EVENTS).launch(
            "bwd_weight", lambda: ops.dk(gy, x, gk, mode=mode, accumulate=True, opts=self.opts),
            {"B": B, "H": H, "L": L, "K": K})

    def launch_bwd_fused(self, gy: torch.Tensor, x: torch.Tensor, k: torch.Tensor, gx: torch.Tensor,
                         gk: torch.Tensor, collector: KernelEventCollector | None = None) -> None:
        """gx = dX and gk += dK in one call (ops.dx_dk; one fused kernel where it
        applies, else the two kernels); gk zero-filled by the caller, as for
        launch_bwd_weight."""
        self._check_open()
        B, H, L, K = self._check_shapes(x, k)
        mode = self.dk_mode
        (collector or KERNEL_EVENTS).launch(
            "bwd_fused", lambda: ops.dx_dk(gy, x, k, gk, gx=gx, mode=mode, accumulate=True, opts=self.opts),
            {"B": B, "H": H, "L": L, "K": K})

    def resource_report(self, B: int = DEFAULT_B, H: int = DEFAULT_H, L: int = DEFAULT_L,
                        K: int = DEFAULT_K) -> list[dict[str, Any]]:
        """Registers, shared memory, spills and occupancy of the kernels this runtime
        launches at one shape: FWD, dX and dK, plus the fused backward where
        autograd would use it."""
        rows = []
        names = ["fwd", "bwd_input", "bwd_weight"]
        if self.fuse_backward and ops.fused_backward(B, H, L, K, opts=self.opts):
            names.append("bwd_fused")
        for name in names:
            info = ops.kernel_info(name, B, H, L, K, device=self.device_id, opts=self.opts)
            est = estimate_gpu_occupancy(info["threads_per_block"], info["regs_per_thread"],
                                         info["static_smem_bytes"] + info["dynamic_smem_bytes"], self.profile)
            rows.append({"kernel": name, **est, **info})
        return rows

    def close(self) -> None:
        """Synchronise the device; later launches through this runtime raise."""
        if self._closed:
            return
        torch.cuda.synchronize(self.device_id)
        self._closed = True


def launch_options(warps_per_block: int | None = None, bwdk_block: int | None = None, stages: int | None = None,
                   ctas_per_sm: int | None = None, threads_per_row: int = 1):
    """Per-call launch options (``pt_launch_opts``) for the reference's runtime
    arguments: FWD/dX take ``warps_per_block`` 32-row warps per tile, dK
    ``bwdk_block`` rows per tile; unset values keep the frozen table for that
    path, unless another argument is set (it then fills in the defaults of the
    reference runtime's launch: 4 warps, 3 stages, 2 CTAs per SM for FWD/dX;
    128 rows, 2 stages, 2 CTAs per SM for dK)."""
    from ._lib import LaunchOpts

    o = LaunchOpts.frozen()
    if warps_per_block is not None or stages is not None or ctas_per_sm is not None:
        for p in (0, 1):
            o.rows_per_tile[p] = 32 * (warps_per_block or 4)
            o.stages[p] = stages or 3
            o.ctas_per_sm[p] = ctas_per_sm or 2
            o.threads_per_row[p] = threads_per_row
    if bwdk_block is not None or stages is not None or ctas_per_sm is not None:
        o.rows_per_tile[2] = bwdk_block or 128
        o.stages[2] = stages or 2
        o.ctas_per_sm[2] = ctas_per_sm or 2
        o.threads_per_row[2] = threads_per_row
    return o


AmpereWarpRuntime = B200WarpRuntime

_RUNTIME: B200WarpRuntime | None = None
_RUNTIME_LOCK = threading.Lock()


def install_runtime(runtime: B200WarpRuntime) -> None:
    global _RUNTIME
    _RUNTIME = runtime


def get_runtime() -> B200WarpRuntime:
    if _RUNTIME is None:
        raise RuntimeError("CUDA runtime has not been installed")
    return _RUNTIME


def default_runtime() -> B200WarpRuntime:
    """The installed runtime, installing a frozen-table one on first use."""
    global _RUNTIME
    if _RUNTIME is None:
        with _RUNTIME_LOCK:
            if _RUNTIME is None:
                _RUNTIME = B200WarpRuntime()
    return _RUNTIME


class DepthConvB200(torch.autograd.Function):
    """Autograd op: forward launches FWD; backward launches dX and dK for the
    inputs that need gradients (kernels/warp_tiled_ampere.py:863-894), as one
    fused launch when both are needed, the runtime's fuse_backward is on and
    the shape is one the fused kernel covers."""

    @staticmethod
    def forward(ctx: Any, x: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
        runtime = get_runtime()
        x_c = x.contiguous()
        k_c = k.contiguous()
        B, H, L, K = runtime._check_shapes(x_c, k_c)
        y = torch.empty_like(x_c)
        runtime.launch_fwd(x_c, k_c, y)
        ctx.save_for_backward(x_c, k_c)
        ctx.params = (B, H, L, K)
        return y

    @staticmethod
    def backward(ctx: Any, gy: torch.Tensor):
        runtime = get_runtime()
        x_c, k_c = ctx.saved_tensors
        B, H, L, K = ctx.params
        gy_c = gy.contiguous()
        if tuple(gy_c.shape) != (B, H, L):
            raise ValueError("Unexpected gradient shape")
        gx = gk = None
        if (ctx.needs_input_grad[0] and ctx.needs_input_grad[1] and runtime.fuse_backward
                and ops.fused_backward(B, H, L, K)):
            gx = torch.empty_like(x_c)
            if runtime.dk_mode == "atomic":
                gk = torch.zeros_like(k_c)
                runtime.launch_bwd_fused(gy_c, x_c, k_c, gx, gk)
            else:
                gk = torch.empty_like(k_c)
                KERNEL_EVENTS.launch("bwd_fused", lambda: ops.dx_dk(gy_c, x_c, k_c, gk, gx=gx),
                                     {"B": B, "H": H, "L": L, "K": K})
            return gx, gk
        if ctx.needs_input_grad[0]:
            gx = torch.empty_like(x_c)
            runtime.launch_bwd_input(gy_c, k_c, gx)
        if ctx.needs_input_grad[1]:
            # Atomic mode accumulates, so it needs the zero fill (outside the
            # dK kernel, as in the reference); deterministic mode overwrites.
            if runtime.dk_mode == "atomic":
                gk = torch.zeros_like(k_c)
                runtime.launch_bwd_weight(gy_c, x_c, gk, K)
            else:
                gk = torch.empty_like(k_c)
                KERNEL_EVENTS.launch("bwd_weight", lambda: ops.dk(gy_c, x_c, gk, mode="deterministic"),
                                     {"B": B, "H": H, "L": L, "K": K})
        return gx, gk


DepthConvAmpere = DepthConvB200


def depthwise_conv_b200(x: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
    """Differentiable same-length depthwise Conv1D, x[B,H,L] * k[H,K] -> y[B,H,L]."""
    default_runtime()
    return DepthConvB200.apply(x, k)


def depthwise_conv_ampere(x: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
    """Reference-named entry (kernels/warp_tiled_ampere.py:897); requires install_runtime."""
    return DepthConvB200.apply(x, k)


class DepthConvCL(torch.autograd.Function):
    """Channels-last autograd op: x[B,L,H] * k[H,K] -> y[B,L,H] on the [B,L,H]
    kernels (ops.fwd_cl / dx_cl / dk_cl), for callers such as the S4 block that
    hold activations channels-last (kernels/warp_tiled_ampere.py:1186-1190)."""

    @staticmethod
    def forward(ctx: Any, x: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
        x_c = x.contiguous()
        k_c = k.contiguous()
        y = ops.fwd_cl(x_c, k_c)
        ctx.save_for_backward(x_c, k_c)
        return y

    @staticmethod
    def backward(ctx: Any, gy: torch.Tensor):
        x_c, k_c = ctx.saved_tensors
        gy_c = gy.contiguous()
        gx = ops.dx_cl(gy_c, k_c) if ctx.needs_input_grad[0] else None
        gk = None
        if ctx.needs_input_grad[1]:
            gk = torch.empty_like(k_c)
            ops.dk_cl(gy_c, x_c, gk)
        return gx, gk


def depthwise_conv_b200_cl(x: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
    """Differentiable same-length depthwise Conv1D on channels-last x[B,L,H] with k[H,K]."""
    return DepthConvCL.apply(x, k)


depthwise_conv_b200_cl.channels_last = True


def roofline_ms(B: int, H: int, L: int, K: int, hbm_gbs: float, fma_tflops: float) -> float:
    """Per-phase roofline time: max(bytes / HBM bandwidth, FLOPs / FP32 FMA peak)."""
    t_mem = minimum_algorithmic_bytes(B, H, L, K) / (hbm_gbs * 1e9)
    t_fma = algorithmic_flops(B, H, L, K) / (fma_tflops * 1e12)
    return 1e3 * max(t_mem, t_fma)


def fp32_fma_peak_tflops(sm_count: int = 148, sm_mhz: float = 1965.0) -> float:
    """FP32 FMA peak: SMs x 128 lanes x 2 FLOP x clock."""
    return sm_count * 128 * 2 * sm_mhz * 1e6 / 1e12


__all__ = [
    "B200WarpRuntime", "AmpereWarpRuntime", "DepthConvB200", "DepthConvAmpere", "DepthConvCL",
    "depthwise_conv_b200_cl",
    "depthwise_conv_b200", "depthwise_conv_ampere", "install_runtime", "get_runtime",
    "default_runtime", "KernelEventCollector", "KERNEL_EVENTS", "GPUProfile", "GPU_PROFILES",
    "detect_gpu_profile", "estimate_gpu_occupancy", "minimum_algorithmic_bytes",
    "algorithmic_bandwidth_gbps", "algorithmic_flops", "in_range_pairs", "summarize_kernel_times",
    "max_abs_diff", "normalized_max_abs", "roofline_ms", "fp32_fma_peak_tflops",
    "WARP_SIZE", "MAX_L", "MAX_K", "DEFAULT_B", "DEFAULT_H", "DEFAULT_L", "DEFAULT_K",
    "DEFAULT_WARPS_PER_BLOCK", "DEFAULT_BWDK_BTILE", "DEFAULT_BWDK_KPACK", "DEFAULT_BWDK_BLOCK",
    "ceil_div", "round_up",
]

