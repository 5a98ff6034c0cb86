"""ctypes binding of ``libpathtile_b200.so`` (the C ABI in include/pathtile_b200.h).

The shared library is built in-tree by :mod:`pathtile_b200.build`.  There is
no fallback: if the library is missing or cannot be loaded, every entry point
raises.  The binding exposes the raw functions; tensor-level wrappers live in
:mod:`pathtile_b200.ops`.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libpathtile_b200.so"

PT_OK = 0
PT_ERR_ARGS = -2
PT_ERR_UNSUPPORTED = -3
PT_ERR_ALIGN = -4
PT_ERR_WORKSPACE = -5
PT_ERR_CUDA = -6
PT_ERR_DEVICE = -7
PT_ERR_SCRATCH_LIMIT = -8
PT_DK_NOALLOC_SCRATCH_BYTES = 8 * 1024 * 1024

PT_DK_ATOMIC = 0
PT_DK_DETERMINISTIC = 1
PT_DK_DETERMINISTIC_ACCUMULATE = 2

PT_PATH_FWD = 0
PT_PATH_DX = 1
PT_PATH_DK = 2
PT_PATH_BWD_FUSED = 3  # pt_kernel_info only

PT_ENGINE_FFMA = 0
PT_ENGINE_TENSOR = 1

# pt_launch_opts.bwd_kernel: the kernel pt_dx_dk runs.
PT_BWD_FROZEN = -1
PT_BWD_SEPARATE = 0
PT_BWD_TENSOR_FUSED = 1
PT_BWD_FFMA_FUSED = 2
PT_BWD_ANY_FUSED = 3

PT_MAX_L = 48
PT_MAX_K = 48
PT_MAX_PEERS = 8
PT_IPC_HANDLE_BYTES = 64


class LaunchOpts(ctypes.Structure):
    """``pt_launch_opts``: per-call launch options, one entry per path (FWD, DX, DK).

    rows_per_tile 0 keeps the frozen PathTile table for that path; engine -1
    keeps the frozen engine."""

    _fields_ = [
        ("rows_per_tile", ctypes.c_int * 3),
        ("stages", ctypes.c_int * 3),
        ("ctas_per_sm", ctypes.c_int * 3),
        ("threads_per_row", ctypes.c_int * 3),
        ("engine", ctypes.c_int * 3),
        ("bwd_kernel", ctypes.c_int),
        ("helper_channels", ctypes.c_int),
    ]

    @classmethod
    def frozen(cls) -> "LaunchOpts":
        o = cls()
        for p in range(3):
            o.engine[p] = -1
        o.bwd_kernel = PT_BWD_FROZEN
        o.helper_channels = -1
        return o


class PeerGroup(ctypes.Structure):
    """``pt_peer_group``: this rank, the number of ranks, every rank's exchange
    buffer as mapped into this process, and the call's epoch."""

    _fields_ = [
        ("rank", ctypes.c_int),
        ("world", ctypes.c_int),
        ("bufs", ctypes.c_void_p * PT_MAX_PEERS),
        ("epoch", ctypes.c_uint),
    ]


# Every symbol include/pathtile_b200.h declares, with (restype, argtypes).
_c_int, _c_size, _vp, _fp = ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "pt_fwd": (_c_int, [_fp, _fp, _fp, _c_int, _c_int, _c_int, _c_int, _vp]),
    "pt_dx": (_c_int, [_fp, _fp, _fp, _c_int, _c_int, _c_int, _c_int, _vp]),
    "pt_dk": (_c_int, [_fp, _fp, _fp, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _c_size, _vp]),
    "pt_dk_workspace_bytes": (_c_size, [_c_int, _c_int, _c_int, _c_int]),
    "pt_dx_dk": (_c_int, [_fp, _fp, _fp, _fp, _fp, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _c_size, _vp]),
    "pt_dx_dk_workspace_bytes": (_c_size, [_c_int, _c_int, _c_int, _c_int]),
    "pt_dx_dk_fused": (_c_int, [_c_int, _c_int, _c_int, _c_int]),
    "pt_fwd_cl": (_c_int, [_fp, _fp, _fp, _c_int, _c_int, _c_int, _c_int, _vp]),
    "pt_dx_cl": (_c_int, [_fp, _fp, _fp, _c_int, _c_int, _c_int, _c_int, _vp]),
    "pt_dk_cl": (_c_int, [_fp, _fp, _fp, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _c_size, _vp]),
    "pt_dk_cl_workspace_bytes": (_c_size, [_c_int, _c_int, _c_int, _c_int]),
    "pt_dk_noalloc": (_c_int, [_fp, _fp, _fp, _c_int, _c_int, _c_int, _c_int, _c_int, _vp]),
    "pt_config": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, ctypes.POINTER(ctypes.c_int), _c_int]),
    "pt_set_config": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int]),
    "pt_set_engine": (_c_int, [_c_int, _c_int]),
    "pt_kernel_info": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, ctypes.POINTER(ctypes.c_int), _c_int]),
    "pt_device_error": (_c_int, [ctypes.POINTER(ctypes.c_uint), _c_int]),
    "pt_status_string": (ctypes.c_char_p, [_c_int]),
    "pt_last_cuda_error": (_c_int, []),
    "pt_version": (_c_int, []),
    "pt_fwd_ex": (_c_int, [_fp, _fp, _fp, _c_int, _c_int, _c_int, _c_int, _vp, _vp]),
    "pt_dx_ex": (_c_int, [_fp, _fp, _fp, _c_int, _c_int, _c_int, _c_int, _vp, _vp]),
    "pt_dk_ex": (_c_int, [_fp, _fp, _fp, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _c_size, _vp, _vp]),
    "pt_dx_dk_ex": (_c_int, [_fp, _fp, _fp, _fp, _fp, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _c_size, _vp,
                             _vp]),
    "pt_dk_workspace_bytes_ex": (_c_size, [_c_int, _c_int, _c_int, _c_int, _vp]),
    "pt_dx_dk_workspace_bytes_ex": (_c_size, [_c_int, _c_int, _c_int, _c_int, _vp]),
    "pt_dx_dk_fused_ex": (_c_int, [_c_int, _c_int, _c_int, _c_int, _vp]),
    "pt_config_ex": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, ctypes.POINTER(ctypes.c_int), _c_int, _vp]),
    "pt_kernel_info_ex": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, ctypes.POINTER(ctypes.c_int), _c_int,
                                   _vp]),
    "pt_selftest_wait_timeout": (_c_int, [ctypes.c_ulonglong, _vp, _vp]),
    "pt_peer_buffer_bytes": (_c_size, [_c_int, _c_int, _c_int]),
    "pt_peer_alloc": (_c_int, [_c_size, ctypes.POINTER(ctypes.c_void_p)]),
    "pt_peer_free": (_c_int, [_vp]),
    "pt_ipc_export": (_c_int, [_vp, _vp]),
    "pt_ipc_import": (_c_int, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "pt_ipc_close": (_c_int, [_vp]),
    "pt_dx_dk_allreduce": (_c_int, [_fp, _fp, _fp, _fp, _fp, _c_int, _c_int, _c_int, _c_int, _vp, _c_size, _vp,
                                    _vp]),
    "pt_dx_dk_allreduce_fused": (_c_int, [_c_int, _c_int, _c_int, _c_int]),
    "pt_allreduce_peer": (_c_int, [_fp, _c_int, _c_int, _vp, _vp]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class PathTileError(RuntimeError):
    """A non-zero status from the native library."""

    def __init__(self, status: int, what: str, detail: str = "") -> None:
        self.status = status
        msg = f"{what} failed with status {status}: {status_string(status)}"
        if detail:
            msg += f" ({detail})"
        super().__init__(msg)


def load() -> ctypes.CDLL:
    """Load the native library once; raise if it is absent (no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"native library {LIB_PATH} is missing; build it with "
                "`python -m pathtile_b200.build` (nvcc, sm_100a). There is no CPU fallback."
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def status_string(status: int) -> str:
    return load().pt_status_string(int(status)).decode()


def last_cuda_error() -> int:
    return int(load().pt_last_cuda_error())


def check(status: int, what: str) -> None:
    if status != PT_OK:
        detail = ""
        if status == PT_ERR_CUDA:
            detail = f"cuda error {last_cuda_error()}"
        raise PathTileError(status, what, detail)
