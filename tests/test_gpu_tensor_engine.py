"""GPU parity of the tensor-core FWD / dX / dK kernels (tcgen05, 3xTF32 split).

The tensor engine must meet the same FP32 bar as the CUDA-core kernels:
rtol = atol = 1e-5 against the FP64 C oracle for FWD / dX and 1e-4 relative
of the FP64 dK (|dK - dK64| <= 1e-4 |dK64| + 1e-4 max|dK64|), on every layout class of the
engine (one channel per tile row with L <= 16: one 64-B swizzled box, L <=
32: one 128-B box, L <= 48: both; and packed super-rows of 48 / L channels
for L in {4, 8, 12, 16, 24}, including a partial last group), ragged batch tiles (B not a multiple of 128), K > L, even and odd
taps, H above the 256-channel TMA box limit of the CUDA-core tiles, and the
three Toeplitz operand regimes (one or two resident channels per CTA, or a
rebuild per tile).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import c_oracle, reference_torch
from pathtile_b200 import ops

pytestmark = pytest.mark.gpu

FWD_TOL = dict(rtol=1e-5, atol=1e-5)


DK_RTOL = 1e-4
PATHS = ("fwd", "bwd_input", "bwd_weight")


def assert_dk_close(got: np.ndarray, ref64: np.ndarray) -> None:
    scale = float(np.abs(ref64).max()) if ref64.size else 0.0
    np.testing.assert_allclose(got, ref64, rtol=DK_RTOL, atol=DK_RTOL * max(scale, 1e-30))


@pytest.fixture
def tensor_engine(cuda_device):
    for p in PATHS:
        ops.set_engine(p, "tensor")
    try:
        yield cuda_device
    finally:
        for p in PATHS:
            ops.set_engine(p, None)


def _inputs(B, H, L, K, seed, device):
    x, k, dy = reference_torch.make_inputs(B, H, L, K, seed)
    return x.to(device), k.to(device), dy.to(device), (x, k, dy)


SHAPES = [
    (1000, 128, 48, 48),  # primary shape class, ragged last batch tile
    (130, 20, 40, 40),    # 64-B box half padding (L = 40)
    (300, 3, 44, 13),
    (200, 300, 48, 47),   # H > 256, odd K; no grid keeps operands resident: per-tile rebuild
    (300, 256, 48, 48),   # grid 128: two resident channels per CTA
    (1000, 96, 48, 48),   # grid 144: two resident channels per CTA
    (257, 5, 32, 32),     # one 128-B box
    (129, 7, 20, 7),      # 128-B box, L = 20 (12 zero columns)
    (100, 7, 28, 28),     # 128-B box, L = 28
    (64, 3, 36, 36),      # both boxes, L = 36
    # packed super-rows of 48 / L channels (2-D maps, block-diagonal Toeplitz)
    (500, 10, 24, 24),    # 2 channels per super-row
    (777, 13, 16, 9),     # 3 per super-row, last group partial (13 = 4 * 3 + 1)
    (64, 9, 16, 16),
    (260, 50, 12, 12),    # 4 per super-row, last group partial
    (33, 4, 12, 5),
    (3, 2, 8, 48),        # 6 per super-row, K > L, one partial group
    (129, 31, 8, 3),
    (1, 1, 4, 1),         # 12 per super-row, one channel present
    (300, 40, 4, 4),
]


@pytest.mark.parametrize("B,H,L,K", SHAPES)
def test_tensor_engine_against_fp64_oracle(tensor_engine, B, H, L, K):
    dev = tensor_engine
    assert ops.config("fwd", B, H, L, K)["engine"] == "tensor"
    assert ops.config("bwd_input", B, H, L, K)["engine"] == "tensor"
    x, k, dy, cpu = _inputs(B, H, L, K, 2024, dev)
    y = ops.fwd(x, k)
    gx = ops.dx(dy, k)
    torch.cuda.synchronize()
    assert ops.device_error(clear=True) == 0, "a kernel wait expired"
    np.testing.assert_allclose(y.cpu().numpy(), c_oracle.fwd(cpu[0], cpu[1]), **FWD_TOL)
    np.testing.assert_allclose(gx.cpu().numpy(), c_oracle.dx(cpu[2], cpu[1]), **FWD_TOL)


def test_tensor_engine_matches_ffma_engine(cuda_device):
    x, k, dy, _ = _inputs(2048, 128, 48, 48, 77, cuda_device)
    y_f, gx_f = ops.fwd(x, k), ops.dx(dy, k)
    try:
        ops.set_engine("fwd", "tensor")
        ops.set_engine("bwd_input", "tensor")
        y_t, gx_t = ops.fwd(x, k), ops.dx(dy, k)
    finally:
        ops.set_engine("fwd", None)
        ops.set_engine("bwd_input", None)
    torch.cuda.synchronize()
    assert ops.device_error(clear=True) == 0
    torch.testing.assert_close(y_t, y_f, **FWD_TOL)
    torch.testing.assert_close(gx_t, gx_f, **FWD_TOL)


def test_tensor_engine_is_deterministic_and_stream_ordered(tensor_engine):
    dev = tensor_engine
    x, k, dy, cpu = _inputs(700, 64, 48, 48, 3, dev)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        outs = [ops.fwd(x, k) for _ in range(3)]
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    assert ops.device_error(clear=True) == 0
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    np.testing.assert_allclose(outs[0].cpu().numpy(), c_oracle.fwd(cpu[0], cpu[1]), **FWD_TOL)


def test_tensor_engine_shapes_it_does_not_cover_stay_on_ffma(tensor_engine):
    assert ops.config("fwd", 64, 8, 37, 13)["engine"] == "ffma"  # L % 4 != 0
    assert ops.config("bwd_weight", 64, 8, 37, 13)["engine"] == "ffma"
    # 300 groups on 148 SMs: no grid keeps dK's accumulators resident
    assert ops.config("bwd_weight", 200, 300, 48, 47)["engine"] == "ffma"
    assert ops.config("bwd_weight", 16384, 128, 48, 48)["engine"] == "tensor"


@pytest.mark.parametrize("mode", ["deterministic", "atomic"])
@pytest.mark.parametrize("B,H,L,K", SHAPES)
def test_tensor_dk_against_fp64_oracle(tensor_engine, B, H, L, K, mode):
    dev = tensor_engine
    x, k, dy, cpu = _inputs(B, H, L, K, 404, dev)
    gk = torch.zeros_like(k) if mode == "atomic" else torch.full_like(k, float("nan"))
    ops.dk(dy, x, gk, mode=mode)
    torch.cuda.synchronize()
    assert ops.device_error(clear=True) == 0, "a kernel wait expired"
    assert_dk_close(gk.cpu().numpy(), c_oracle.dk(cpu[2], cpu[0], K))


def test_tensor_dk_primary_workload(tensor_engine):
    dev = tensor_engine
    B, H, L, K = 16384, 128, 48, 48
    x, k, dy, cpu = _inputs(B, H, L, K, 42, dev)
    gk = torch.empty_like(k)
    ops.dk(dy, x, gk)
    torch.cuda.synchronize()
    assert ops.device_error(clear=True) == 0
    assert_dk_close(gk.cpu().numpy(), c_oracle.dk(cpu[2], cpu[0], K))
    # <dK(dy, x), k> = <FWD(x), dy> (size-independent identity)
    y = ops.fwd(x, k)
    a = float((gk.double() * k.double()).sum())
    b = float((y.double() * dy.double()).sum())
    assert abs(a - b) <= 1e-6 * (float(y.double().abs().sum()) + 1.0)


def test_tensor_dk_deterministic_and_accumulate(tensor_engine):
    dev = tensor_engine
    x, k, dy, cpu = _inputs(4096, 96, 48, 48, 8, dev)
    outs = []
    for _ in range(3):
        gk = torch.empty_like(k)
        ops.dk(dy, x, gk, mode="deterministic")
        outs.append(gk.clone())
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    gk = torch.ones_like(k)
    ops.dk(dy, x, gk, mode="deterministic", accumulate=True)
    torch.cuda.synchronize()
    assert ops.device_error(clear=True) == 0
    assert_dk_close(gk.cpu().numpy() - 1.0, c_oracle.dk(cpu[2], cpu[0], 48))
