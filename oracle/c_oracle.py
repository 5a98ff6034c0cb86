"""TEST INFRASTRUCTURE ONLY -- ctypes binding of oracle/pt_oracle.c (FP64 loops)."""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"

_lib = None


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            from .build_oracle import build_c_oracle

            build_c_oracle()
        lib = ctypes.CDLL(str(LIB))
        fp, dp, ci = ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int
        for name in ("pto_fwd_f64", "pto_dx_f64", "pto_dk_f64"):
            getattr(lib, name).argtypes = [fp, fp, dp, ci, ci, ci, ci]
            getattr(lib, name).restype = None
        for name in ("pto_fwd_rows_f64", "pto_dx_rows_f64"):
            getattr(lib, name).argtypes = [fp, fp, dp, ci, ci, ci, ctypes.c_void_p, ctypes.c_longlong]
            getattr(lib, name).restype = None
        lib.pto_num_threads.restype = ci
        lib.pto_num_threads.argtypes = []
        _lib = lib
    return _lib


def _f32(a) -> np.ndarray:
    a = np.asarray(a.detach().cpu().numpy() if hasattr(a, "detach") else a)
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data)


def fwd(x, k) -> np.ndarray:
    x, k = _f32(x), _f32(k)
    B, H, L = x.shape
    K = k.shape[1]
    y = np.empty((B, H, L), dtype=np.float64)
    load().pto_fwd_f64(_p(x), _p(k), _p(y), B, H, L, K)
    return y


def dx(dy, k) -> np.ndarray:
    dy, k = _f32(dy), _f32(k)
    B, H, L = dy.shape
    K = k.shape[1]
    gx = np.empty((B, H, L), dtype=np.float64)
    load().pto_dx_f64(_p(dy), _p(k), _p(gx), B, H, L, K)
    return gx


def dk(dy, x, K: int) -> np.ndarray:
    dy, x = _f32(dy), _f32(x)
    B, H, L = x.shape
    gk = np.empty((H, K), dtype=np.float64)
    load().pto_dk_f64(_p(dy), _p(x), _p(gk), B, H, L, K)
    return gk


def fwd_rows(x, k, rows: np.ndarray) -> np.ndarray:
    """FWD of selected flattened rows (b*H+h) only: [len(rows), L]."""
    x, k = _f32(x), _f32(k)
    _, H, L = x.shape
    K = k.shape[1]
    r = np.ascontiguousarray(rows, dtype=np.int64)
    y = np.empty((r.size, L), dtype=np.float64)
    load().pto_fwd_rows_f64(_p(x), _p(k), _p(y), H, L, K, _p(r), r.size)
    return y


def dx_rows(dy, k, rows: np.ndarray) -> np.ndarray:
    dy, k = _f32(dy), _f32(k)
    _, H, L = dy.shape
    K = k.shape[1]
    r = np.ascontiguousarray(rows, dtype=np.int64)
    gx = np.empty((r.size, L), dtype=np.float64)
    load().pto_dx_rows_f64(_p(dy), _p(k), _p(gx), H, L, K, _p(r), r.size)
    return gx


def num_threads() -> int:
    return int(load().pto_num_threads())
