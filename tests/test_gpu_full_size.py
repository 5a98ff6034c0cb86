"""GPU parity at the full BASELINE sizes, every element, every engine.

For the primary workload (B=16384, H=128, L=K=48) and the four edge shapes,
FWD and dX are compared element by element against the FP64 C oracle
(rtol = atol = 1e-5) on each engine that can run the shape -- the frozen
table's choice, the CUDA-core kernels forced, the tensor-core kernels forced
-- and the backward through ops.dx_dk (the fused kernel where it applies) is
compared the same way, dK against the FP64 dK (1e-4 relative).  Each check
reports its accuracy margin, max |err| / (atol + rtol |ref|) for FWD / dX and
max |err| / (rtol |ref| + rtol max |ref|) for dK (1.0 = at the bar); set
PT_PARITY_LOG to a file path to collect them as JSON lines.
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from oracle import c_oracle, reference_torch
from pathtile_b200 import _lib, ops

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-5
DK_RTOL = 1e-4

FULL_SHAPES = [
    (16384, 128, 48, 48),  # primary workload
    (4096, 64, 37, 13),    # edge shapes
    (8192, 256, 16, 4),
    (16384, 128, 48, 3),
    (2048, 512, 33, 33),
]


def _opts(engine: str | None) -> _lib.LaunchOpts | None:
    if engine is None:
        return None
    o = _lib.LaunchOpts.frozen()
    for p in range(3):
        o.engine[p] = _lib.PT_ENGINE_FFMA if engine == "ffma" else _lib.PT_ENGINE_TENSOR
    return o


def conv_margin(got: torch.Tensor, ref64: np.ndarray, chunk: int = 1 << 24) -> float:
    """max |got - ref| / (ATOL + RTOL |ref|) over every element (on the GPU, in FP64)."""
    g = got.reshape(-1)
    r = torch.from_numpy(ref64.reshape(-1))
    worst = 0.0
    for i in range(0, g.numel(), chunk):
        rr = r[i:i + chunk].to(g.device)
        m = ((g[i:i + chunk].double() - rr).abs() / (ATOL + RTOL * rr.abs())).max()
        worst = max(worst, float(m))
    return worst


def dk_margin(got: torch.Tensor, ref64: np.ndarray) -> float:
    r = torch.from_numpy(ref64).to(got.device)
    scale = float(r.abs().max())
    return float(((got.double() - r).abs() / (DK_RTOL * r.abs() + DK_RTOL * scale)).max())


def record(**row) -> None:
    print(json.dumps(row))
    path = os.environ.get("PT_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(row) + "\n")


@pytest.mark.parametrize("B,H,L,K", FULL_SHAPES)
def test_every_element_every_engine_against_fp64(cuda_device, B, H, L, K):
    dev = cuda_device
    x_c, k_c, dy_c = reference_torch.make_inputs(B, H, L, K, 42)
    x, k, dy = x_c.to(dev), k_c.to(dev), dy_c.to(dev)
    y64 = c_oracle.fwd(x_c, k_c)
    gx64 = c_oracle.dx(dy_c, k_c)
    gk64 = c_oracle.dk(dy_c, x_c, K)
    shape = dict(B=B, H=H, L=L, K=K)
    seen = set()
    for engine in (None, "ffma", "tensor"):
        o = _opts(engine)
        ran = tuple(ops.config(p, B, H, L, K, opts=o)["engine"] for p in ("fwd", "bwd_input", "bwd_weight"))
        if ran in seen:
            continue  # this engine does not apply here: it runs what an earlier case ran
        seen.add(ran)
        y = ops.fwd(x, k, opts=o)
        gx = ops.dx(dy, k, opts=o)
        gk = torch.full_like(k, float("nan"))
        ops.dk(dy, x, gk, opts=o)
        torch.cuda.synchronize()
        assert ops.device_error(clear=True) == 0, "a kernel wait expired"
        m = dict(fwd=conv_margin(y, y64), dx=conv_margin(gx, gx64), dk=dk_margin(gk, gk64))
        record(test="full_size", **shape, requested=engine or "frozen", engines=list(ran), margin=m)
        assert m["fwd"] <= 1.0 and m["dx"] <= 1.0 and m["dk"] <= 1.0, m
        del y, gx
    # The backward as autograd runs it: one dx_dk call (the fused kernel where it applies).
    gk = torch.full_like(k, float("nan"))
    gx = ops.dx_dk(dy, x, k, gk)
    torch.cuda.synchronize()
    assert ops.device_error(clear=True) == 0, "a kernel wait expired"
    m = dict(dx=conv_margin(gx, gx64), dk=dk_margin(gk, gk64))
    record(test="full_size", **shape, requested="dx_dk", kind=ops.backward_kind(B, H, L, K), margin=m)
    assert m["dx"] <= 1.0 and m["dk"] <= 1.0, m
