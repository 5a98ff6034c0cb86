"""Tensor-level launches of the native FWD / dX / dK kernels.

Each function validates its tensors the way the reference runtime does
(``AmpereWarpRuntime._check_shapes``, kernels/warp_tiled_ampere.py:704-717:
ValueError for device, dtype, rank, channel mismatch and L/K > 48), then calls
the C ABI on the tensors' device and on ``torch.cuda.current_stream()`` of
that device (the reference launched on PyCUDA's default stream,
kernels/warp_tiled_ampere.py:734-744; here the caller's stream is honoured).
No computation happens on the host and there is no fallback path.
"""
from __future__ import annotations

import contextlib
import ctypes
import threading

import torch

from . import _lib
from ._lib import (
    PT_DK_ATOMIC,
    PT_DK_DETERMINISTIC,
    PT_DK_DETERMINISTIC_ACCUMULATE,
    PT_MAX_K,
    PT_MAX_L,
    PT_PATH_DK,
    PT_PATH_DX,
    PT_PATH_FWD,
)

DK_MODES = {
    "atomic": PT_DK_ATOMIC,
    "deterministic": PT_DK_DETERMINISTIC,
}


def _ensure_cuda_f32(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != torch.float32:
        raise ValueError(f"{name}: only FP32 is supported, got {t.dtype}")


def _ensure_raw(t: torch.Tensor, name: str) -> None:
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if t.numel() and t.data_ptr() % 16:
        raise ValueError(f"{name} must be 16-byte aligned")


def check_shapes(x: torch.Tensor, k: torch.Tensor) -> tuple[int, int, int, int]:
    """Validate x[B,H,L] and k[H,K]; return (B, H, L, K)."""
    _ensure_cuda_f32(x, "x")
    _ensure_cuda_f32(k, "k")
    if x.ndim != 3 or k.ndim != 2:
        raise ValueError("Expected x[B,H,L] and k[H,K]")
    B, H, L = map(int, x.shape)
    Hk, K = map(int, k.shape)
    if H != Hk:
        raise ValueError("x and k channel dimensions do not match")
    if L > PT_MAX_L or K > PT_MAX_K:
        raise ValueError(f"Specialized kernels require L<={PT_MAX_L}, K<={PT_MAX_K}")
    if H < 1 or L < 1 or K < 1:
        raise ValueError("H, L and K must be positive")
    if x.device != k.device:
        raise ValueError("x and k must be on the same device")
    return B, H, L, K


def _ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _opts_ptr(opts: "_lib.LaunchOpts | None") -> ctypes.c_void_p | None:
    return None if opts is None else ctypes.cast(ctypes.pointer(opts), ctypes.c_void_p)


def _launch_rows(path: int, inp: torch.Tensor, k: torch.Tensor, out: torch.Tensor, what: str,
                 opts: "_lib.LaunchOpts | None" = None) -> None:
    B, H, L, K = check_shapes(inp, k)
    _ensure_cuda_f32(out, "out")
    if tuple(out.shape) != (B, H, L):
        raise ValueError(f"out must have shape {(B, H, L)}")
    if out.device != inp.device:
        raise ValueError("out must be on the input's device")
    for t, n in ((inp, "input"), (k, "k"), (out, "out")):
        _ensure_raw(t, n)
    if B == 0:
        return
    lib = _lib.load()
    with torch.cuda.device(inp.device):
        if opts is None:
            fn = lib.pt_fwd if path == PT_PATH_FWD else lib.pt_dx
            st = fn(_ptr(inp), _ptr(k), _ptr(out), B, H, L, K, _stream(inp.device))
        else:
            fn = lib.pt_fwd_ex if path == PT_PATH_FWD else lib.pt_dx_ex
            st = fn(_ptr(inp), _ptr(k), _ptr(out), B, H, L, K, _opts_ptr(opts), _stream(inp.device))
    _lib.check(st, what)


def fwd(x: torch.Tensor, k: torch.Tensor, y: torch.Tensor | None = None,
        opts: "_lib.LaunchOpts | None" = None) -> torch.Tensor:
    """y[b,h,t] = sum_j x[b,h,t+j-K//2] k[h,j] (same length L).  ``opts``: per-call
    launch options (None: the process-wide choice, by default the frozen table)."""
    if y is None:
        check_shapes(x, k)
        y = torch.empty_like(x, memory_format=torch.contiguous_format)
    _launch_rows(PT_PATH_FWD, x, k, y, "pt_fwd", opts)
    return y


def dx(dy: torch.Tensor, k: torch.Tensor, gx: torch.Tensor | None = None,
       opts: "_lib.LaunchOpts | None" = None) -> torch.Tensor:
    """gx[b,h,t] = sum_j dy[b,h,t-j+K//2] k[h,j]."""
    if gx is None:
        check_shapes(dy, k)
        gx = torch.empty_like(dy, memory_format=torch.contiguous_format)
    _launch_rows(PT_PATH_DX, dy, k, gx, "pt_dx", opts)
    return gx


class _WorkspaceCache:
    """One reusable deterministic-dK workspace per (device, stream) (the reference
    caches its [H,K,num_btiles] partials per runtime,
    kernels/warp_tiled_noatomic_optimized.py:1448-1471).

    Launches on one stream run in order, so they can share a buffer; launches on
    two streams of one device may run at the same time, so each stream gets its
    own buffer (a shared one would let one launch reduce the other's partials).
    Allocation happens on the launch stream (the caching allocator ties the block
    to it), so the allocator never hands the memory to other work while a
    launch still reads it."""

    def __init__(self) -> None:
        self._lock = threading.Lock()
        self._bufs: dict[tuple[int, int], torch.Tensor] = {}

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        stream = torch.cuda.current_stream(idx)
        key = (idx, int(stream.cuda_stream))
        with self._lock:
            buf = self._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                n = max(nbytes, 1 << 20)
                with torch.cuda.stream(stream):
                    buf = torch.empty(n, dtype=torch.uint8, device=torch.device("cuda", idx))
                self._bufs[key] = buf
            return buf

    def clear(self) -> None:
        """Release every cached workspace (after the streams that used them are done)."""
        with self._lock:
            self._bufs.clear()


WORKSPACES = _WorkspaceCache()


def dk_workspace_bytes(B: int, H: int, L: int, K: int, device: torch.device | None = None,
                       opts: "_lib.LaunchOpts | None" = None) -> int:
    lib = _lib.load()
    with torch.cuda.device(device) if device is not None else _nullctx():
        return int(lib.pt_dk_workspace_bytes_ex(B, H, L, K, _opts_ptr(opts)))


def dx_dk_workspace_bytes(B: int, H: int, L: int, K: int, device: torch.device | None = None,
                          opts: "_lib.LaunchOpts | None" = None) -> int:
    lib = _lib.load()
    with torch.cuda.device(device) if device is not None else _nullctx():
        return int(lib.pt_dx_dk_workspace_bytes_ex(B, H, L, K, _opts_ptr(opts)))


def _nullctx() -> contextlib.AbstractContextManager:
    return contextlib.nullcontext()


def dk(
    dy: torch.Tensor,
    x: torch.Tensor,
    gk: torch.Tensor,
    mode: str = "deterministic",
    accumulate: bool = False,
    workspace: torch.Tensor | None = None,
    opts: "_lib.LaunchOpts | None" = None,
) -> torch.Tensor:
    """Filter gradient dk[h,j] = sum_{b,t} dy[b,h,t] x[b,h,t+j-K//2] into gk[H,K].

    mode "atomic": gk += dK through float atomics (gk must be zeroed first for a
    plain gradient; the reference's contract, kernels/warp_tiled_ampere.py:890-893).
    mode "deterministic": two passes through a workspace; gk = dK, or gk += dK
    with accumulate=True; bit-reproducible for a fixed launch configuration.
    Without ``workspace`` the cached buffer of the current stream is used:
    calls on one stream run in order, calls on different streams get
    different buffers.  A caller-provided ``workspace`` must not be in use by a
    launch on another stream at the same time.
    """
    _ensure_cuda_f32(dy, "gy")
    _ensure_cuda_f32(x, "x")
    _ensure_cuda_f32(gk, "gk")
    if tuple(dy.shape) != tuple(x.shape):
        raise ValueError("gy and x must have the same [B,H,L] shape")
    if x.ndim != 3 or gk.ndim != 2:
        raise ValueError("Expected gy/x [B,H,L] and gk [H,K]")
    B, H, L = map(int, x.shape)
    K = int(gk.shape[1])
    if tuple(gk.shape) != (H, K):
        raise ValueError(f"gk must have shape {(H, K)}")
    if L > PT_MAX_L or K > PT_MAX_K:
        raise ValueError(f"Specialized kernels require L<={PT_MAX_L}, K<={PT_MAX_K}")
    if H < 1 or L < 1 or K < 1:
        raise ValueError("H, L and K must be positive")
    if not (dy.device == x.device == gk.device):
        raise ValueError("gy, x and gk must be on one device")
    if mode not in DK_MODES:
        raise ValueError(f"mode must be one of {sorted(DK_MODES)}")
    for t, n in ((dy, "gy"), (x, "x"), (gk, "gk")):
        _ensure_raw(t, n)
    code = DK_MODES[mode]
    if code == PT_DK_DETERMINISTIC and accumulate:
        code = PT_DK_DETERMINISTIC_ACCUMULATE
    lib = _lib.load()
    dev = x.device
    with torch.cuda.device(dev):
        ws_ptr, ws_bytes = ctypes.c_void_p(0), 0
        if code != PT_DK_ATOMIC and B > 0:
            ws_bytes = int(lib.pt_dk_workspace_bytes_ex(B, H, L, K, _opts_ptr(opts)))
            if ws_bytes == 0:
                raise _lib.PathTileError(_lib.PT_ERR_WORKSPACE, "pt_dk_workspace_bytes")
            ws = workspace if workspace is not None else WORKSPACES.get(dev, ws_bytes)
            if ws.device != dev or ws.numel() * ws.element_size() < ws_bytes:
                raise ValueError(f"workspace must be on {dev} and hold {ws_bytes} bytes")
            ws.record_stream(torch.cuda.current_stream(dev))
            ws_ptr = _ptr(ws)
            ws_bytes = ws.numel() * ws.element_size()
        st = lib.pt_dk_ex(_ptr(dy), _ptr(x), _ptr(gk), B, H, L, K, code, ws_ptr, ws_bytes, _opts_ptr(opts),
                          _stream(dev))
    _lib.check(st, "pt_dk")
    return gk


def dx_dk(
    dy: torch.Tensor,
    x: torch.Tensor,
    k: torch.Tensor,
    gk: torch.Tensor,
    gx: torch.Tensor | None = None,
    mode: str = "deterministic",
    accumulate: bool = False,
    workspace: torch.Tensor | None = None,
    opts: "_lib.LaunchOpts | None" = None,
) -> torch.Tensor:
    """Both backward products in one call: returns gx = dX(dy, k) and writes the
    filter gradient into gk with dk()'s modes (and its workspace rules).  Where a
    fused kernel applies (see backward_kind) dy and x are read once: the
    tensor-core one for 32 < L <= 48 (L % 4 == 0) on grids that give each CTA one
    channel, else the CUDA-core one for the specialised (L, K) shapes; other
    shapes run dx() then dk().  The reference's backward launches the two
    separately (kernels/warp_tiled_ampere.py:882-898).
    """
    _ensure_cuda_f32(dy, "gy")
    _ensure_cuda_f32(x, "x")
    _ensure_cuda_f32(k, "k")
    _ensure_cuda_f32(gk, "gk")
    if tuple(dy.shape) != tuple(x.shape):
        raise ValueError("gy and x must have the same [B,H,L] shape")
    B, H, L, K = check_shapes(x, k)
    if tuple(gk.shape) != (H, K):
        raise ValueError(f"gk must have shape {(H, K)}")
    if gx is None:
        gx = torch.empty_like(dy, memory_format=torch.contiguous_format)
    _ensure_cuda_f32(gx, "gx")
    if tuple(gx.shape) != tuple(dy.shape):
        raise ValueError("gx must have the shape of gy")
    if not (dy.device == x.device == k.device == gk.device == gx.device):
        raise ValueError("gy, x, k, gk and gx must be on one device")
    if mode not in DK_MODES:
        raise ValueError(f"mode must be one of {sorted(DK_MODES)}")
    for t, n in ((dy, "gy"), (x, "x"), (k, "k"), (gk, "gk"), (gx, "gx")):
        _ensure_raw(t, n)
    code = DK_MODES[mode]
    if code == PT_DK_DETERMINISTIC and accumulate:
        code = PT_DK_DETERMINISTIC_ACCUMULATE
    lib = _lib.load()
    dev = x.device
    with torch.cuda.device(dev):
        ws_ptr, ws_bytes = ctypes.c_void_p(0), 0
        need = int(lib.pt_dx_dk_workspace_bytes_ex(B, H, L, K, _opts_ptr(opts))) if B > 0 else 0
        if need > 0:
            ws = workspace if workspace is not None else WORKSPACES.get(dev, need)
            if ws.device != dev or ws.numel() * ws.element_size() < need:
                raise ValueError(f"workspace must be on {dev} and hold {need} bytes")
            ws.record_stream(torch.cuda.current_stream(dev))
            ws_ptr = _ptr(ws)
            ws_bytes = ws.numel() * ws.element_size()
        st = lib.pt_dx_dk_ex(_ptr(dy), _ptr(x), _ptr(k), _ptr(gx), _ptr(gk), B, H, L, K, code, ws_ptr, ws_bytes,
                             _opts_ptr(opts), _stream(dev))
    _lib.check(st, "pt_dx_dk")
    return gx


BACKWARD_KINDS = {0: "separate", 1: "tensor_fused", 2: "ffma_fused"}


def backward_kind(B: int, H: int, L: int, K: int, opts: "_lib.LaunchOpts | None" = None) -> str:
    """What dx_dk() runs at this shape on the current device: "tensor_fused" (one
    kernel, dX on tcgen05, dK on the CUDA cores), "ffma_fused" (one kernel on the
    CUDA cores) or "separate" (dx() then dk())."""
    return BACKWARD_KINDS[int(_lib.load().pt_dx_dk_fused_ex(B, H, L, K, _opts_ptr(opts)))]


def fused_backward(B: int, H: int, L: int, K: int, opts: "_lib.LaunchOpts | None" = None) -> bool:
    """True when dx_dk() reads dy and x once (one fused kernel) at this shape on the current device."""
    return backward_kind(B, H, L, K, opts) != "separate"


def dx_dk_launches(B: int, H: int, L: int, K: int, opts: "_lib.LaunchOpts | None" = None,
                   mode: str = "deterministic") -> int:
    """Kernel launches of one dx_dk() at this shape: the fused kernel (plus a partial
    reduce where the deterministic dK needs one), or dX + the dK kernels."""
    if B <= 0:
        return 0
    lib = _lib.load()
    kind = int(lib.pt_dx_dk_fused_ex(B, H, L, K, _opts_ptr(opts)))
    if kind == 1:
        return 1 if int(lib.pt_dx_dk_workspace_bytes_ex(B, H, L, K, _opts_ptr(opts))) == 0 else 2
    if kind == 2:
        return 1 if mode == "atomic" else 2
    return 2 if mode == "atomic" else 3


# ---------------- channels-last [B, L, H] ----------------
def _check_cl(x: torch.Tensor, k: torch.Tensor) -> tuple[int, int, int, int]:
    """Validate x[B,L,H] (channels last) and k[H,K]; return (B, L, H, K)."""
    _ensure_cuda_f32(x, "x")
    _ensure_cuda_f32(k, "k")
    if x.ndim != 3 or k.ndim != 2:
        raise ValueError("Expected x[B,L,H] and k[H,K]")
    B, L, H = map(int, x.shape)
    Hk, K = map(int, k.shape)
    if H != Hk:
        raise ValueError("x and k channel dimensions do not match")
    if L > PT_MAX_L or K > PT_MAX_K:
        raise ValueError(f"Specialized kernels require L<={PT_MAX_L}, K<={PT_MAX_K}")
    if H < 1 or L < 1 or K < 1:
        raise ValueError("H, L and K must be positive")
    if x.device != k.device:
        raise ValueError("x and k must be on the same device")
    for tt, n in ((x, "x"), (k, "k")):
        if not tt.is_contiguous():
            raise ValueError(f"{n} must be contiguous")
    return B, L, H, K


def _conv_cl(fn_name: str, inp: torch.Tensor, k: torch.Tensor, out: torch.Tensor | None) -> torch.Tensor:
    B, L, H, K = _check_cl(inp, k)
    if out is None:
        out = torch.empty_like(inp, memory_format=torch.contiguous_format)
    _ensure_cuda_f32(out, "out")
    if tuple(out.shape) != (B, L, H) or out.device != inp.device or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous {(B, L, H)} tensor on the input's device")
    if B == 0:
        return out
    with torch.cuda.device(inp.device):
        st = getattr(_lib.load(), fn_name)(_ptr(inp), _ptr(k), _ptr(out), B, L, H, K, _stream(inp.device))
    _lib.check(st, fn_name)
    return out


def fwd_cl(x: torch.Tensor, k: torch.Tensor, y: torch.Tensor | None = None) -> torch.Tensor:
    """Channels-last FWD: y[b,t,h] = sum_j x[b,t+j-K//2,h] k[h,j] for x, y [B,L,H]."""
    return _conv_cl("pt_fwd_cl", x, k, y)


def dx_cl(dy: torch.Tensor, k: torch.Tensor, gx: torch.Tensor | None = None) -> torch.Tensor:
    """Channels-last input gradient: gx[b,t,h] = sum_j dy[b,t-j+K//2,h] k[h,j]."""
    return _conv_cl("pt_dx_cl", dy, k, gx)


def dk_cl(dy: torch.Tensor, x: torch.Tensor, gk: torch.Tensor, accumulate: bool = False,
          workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Channels-last filter gradient into gk[H,K] (deterministic: gk = dK, or gk += dK)."""
    B, L, H, K = _check_cl(x, gk)
    _ensure_cuda_f32(dy, "gy")
    if tuple(dy.shape) != (B, L, H) or dy.device != x.device or not dy.is_contiguous():
        raise ValueError("gy must be a contiguous tensor shaped and placed like x")
    lib = _lib.load()
    dev = x.device
    with torch.cuda.device(dev):
        ws_ptr, ws_bytes = ctypes.c_void_p(0), 0
        if B > 0:
            need = int(lib.pt_dk_cl_workspace_bytes(B, L, H, K))
            ws = workspace if workspace is not None else WORKSPACES.get(dev, need)
            if ws.device != dev or ws.numel() * ws.element_size() < need:
                raise ValueError(f"workspace must be on {dev} and hold {need} bytes")
            ws.record_stream(torch.cuda.current_stream(dev))
            ws_ptr, ws_bytes = _ptr(ws), ws.numel() * ws.element_size()
        st = lib.pt_dk_cl(_ptr(dy), _ptr(x), _ptr(gk), B, L, H, K, 1 if accumulate else 0, ws_ptr, ws_bytes,
                          _stream(dev))
    _lib.check(st, "pt_dk_cl")
    return gk


def config(path: str, B: int, H: int, L: int, K: int, opts: "_lib.LaunchOpts | None" = None) -> dict[str, int]:
    """Launch choice of one path at one shape (C ABI pt_config): the frozen table,
    or ``opts`` / the process-wide overrides where they are set."""
    code = {"fwd": PT_PATH_FWD, "bwd_input": PT_PATH_DX, "bwd_weight": PT_PATH_DK}[path]
    out = (ctypes.c_int * 9)()
    _lib.check(_lib.load().pt_config_ex(code, B, H, L, K, out, 9, _opts_ptr(opts)), "pt_config")
    return {"rows_per_tile": out[0], "stages": out[1], "ctas_per_sm": out[2], "specialised": out[3],
            "intensity_class": ("light", "medium", "heavy")[out[4]], "threads_per_row": out[5],
            "engine": ENGINES[out[6]], "bwd_kernel": out[7], "helper_channels": out[8]}


KERNEL_PATHS = {"fwd": PT_PATH_FWD, "bwd_input": PT_PATH_DX, "bwd_weight": PT_PATH_DK,
                "bwd_fused": _lib.PT_PATH_BWD_FUSED}


def kernel_info(path: str, B: int, H: int, L: int, K: int, device: torch.device | int | None = None,
                opts: "_lib.LaunchOpts | None" = None) -> dict[str, int]:
    """Registers, shared memory, occupancy and grid of the kernel a path launches (C ABI
    pt_kernel_info); path "bwd_fused" is the fused dX + dK kernel (PathTileError with
    status PT_ERR_UNSUPPORTED where dx_dk() does not fuse)."""
    code = KERNEL_PATHS[path]
    out = (ctypes.c_int * 8)()
    lib = _lib.load()
    with torch.cuda.device(device) if device is not None else _nullctx():
        st = lib.pt_kernel_info_ex(code, B, H, L, K, out, 8, _opts_ptr(opts))
    _lib.check(st, "pt_kernel_info")
    keys = ("regs_per_thread", "static_smem_bytes", "local_memory_bytes", "threads_per_block",
            "dynamic_smem_bytes", "resident_blocks_per_sm", "grid", "specialised")
    return dict(zip(keys, (int(v) for v in out)))


def set_config(path: str, rows_per_tile: int = 0, stages: int = 3, ctas_per_sm: int = 2,
               threads_per_row: int = 1) -> None:
    """Override one path's launch configuration (rows_per_tile=0 restores the frozen table)."""
    code = {"fwd": PT_PATH_FWD, "bwd_input": PT_PATH_DX, "bwd_weight": PT_PATH_DK}[path]
    _lib.check(_lib.load().pt_set_config(code, rows_per_tile, stages, ctas_per_sm, threads_per_row),
               "pt_set_config")


ENGINES = ("ffma", "tensor")


def set_engine(path: str, engine: str | None) -> None:
    """Select the engine of one path for all shapes: "ffma" (CUDA-core kernels), "tensor"
    (tcgen05 at L % 4 == 0; other shapes, and dK shapes whose accumulators cannot stay
    resident, stay on FFMA), or None for the frozen table."""
    code = {"fwd": PT_PATH_FWD, "bwd_input": PT_PATH_DX, "bwd_weight": PT_PATH_DK}[path]
    eng = -1 if engine is None else ENGINES.index(engine)
    _lib.check(_lib.load().pt_set_engine(code, eng), "pt_set_engine")


def device_error(clear: bool = False, device: torch.device | int | None = None) -> int:
    """Read (and optionally clear) the device error word; synchronises the device."""
    out = ctypes.c_uint(0)
    lib = _lib.load()
    if device is None:
        st = lib.pt_device_error(ctypes.byref(out), int(clear))
    else:
        with torch.cuda.device(device):
            st = lib.pt_device_error(ctypes.byref(out), int(clear))
    _lib.check(st, "pt_device_error")
    return int(out.value)
