"""GPU parity of the fused backward reached through ops.dx_dk / pt_dx_dk: the
tensor-core kernel (dX on tcgen05, dK on the CUDA cores) and the CUDA-core
kernel (dX and dK both FFMA, one pass over dy and x).

Bars as for the separate kernels: dX within rtol = atol = 1e-5 of the FP64 C
oracle, dK within 1e-4 relative of the FP64 dK.  Covered: every tensor-core
fused instantiation class (every K <= 48; rows of 32 < L <= 48 columns,
L % 4 == 0, in the kernel's 48-column layout), both dK regimes of that kernel
(one CTA per channel writes dK directly; several CTAs per channel write
partials summed by the reduce kernel); for the CUDA-core kernel both loaders
(TMA tiles at L % 4 == 0, 1-D bulk copies otherwise), channel blocks with a
ragged last block (H > 256), several batches per tile, ragged batch tiles; the
three dK modes; and shapes that fall back to pt_dx + pt_dk.
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
def _fusable_layout(L, K) -> bool:
    return 32 < L <= 48 and L % 4 == 0 and 1 <= K <= 48


def assert_dk_close(got: np.ndarray, ref64: np.ndarray) -> None:
    scale = float(np.abs(ref64).max()) if ref64.size else 0.0
    np.testing.assert_allclose(got, ref64, rtol=DK_RTOL, atol=DK_RTOL * max(scale, 1e-30))


def _inputs(B, H, L, K, seed, device):
    x, k, dy = reference_torch.make_inputs(B, H, L, K, seed)
    return x.to(device), k.to(device), dy.to(device), (x, k, dy)


def _sm_count(dev) -> int:
    return torch.cuda.get_device_properties(dev).multi_processor_count


def tensor_schedule(B, H, sm, helper_limit=None):
    """The host's schedule of the tensor-core fused kernel (None: it does not apply):
    kp = floor(min(tiles, SMs) / H) primary CTAs per channel; the SMs left over
    become helpers taking every channel's tail blocks when that shortens the
    busiest CTA (a channel switch counted as one tile) by >= 3 % and no helper
    owns more than `helper_limit` channels (default: the frozen limit the
    library reports); otherwise the plain grid of kp*H CTAs, which must keep
    >= 3/4 of min(tiles, SMs) busy."""
    if helper_limit is None:
        helper_limit = ops.config("bwd_input", B, H, 48, 48)["helper_channels"]
    nblk = -(-B // 128)
    gmax = min(nblk * H, sm)
    kp = gmax // H
    if kp < 1:
        return None
    plain = -(-nblk // kp)
    E = sm - kp * H
    if E >= 1 and nblk >= 2 and -(-H // E) <= helper_limit:
        m = -(-H // E)
        best, best_p = plain, 0
        for P in range(1, nblk):
            cost = max(-(-P // kp), m * (nblk - P) + (m - 1))
            if cost < best:
                best, best_p = cost, P
        if best_p > 0 and 100 * best <= 97 * plain:
            return {"kp": kp, "E": E, "m": m, "P": best_p, "tiles": best}
    if 4 * kp * H < 3 * gmax:
        return None
    return {"kp": kp, "E": 0, "m": 0, "P": nblk, "tiles": plain}


def _expect_tensor_fused(B, H, L, K, sm) -> bool:
    return _fusable_layout(L, K) and tensor_schedule(B, H, sm) is not None


def _expect_kind(B, H, L, K, sm) -> str:
    """Tensor-core fused where it applies, else the CUDA-core fused kernel where a
    specialised CUDA-core kernel exists for (L, K) with its loader, else separate."""
    if _expect_tensor_fused(B, H, L, K, sm):
        return "tensor_fused"
    if not ops.config("bwd_weight", B, H, L, K)["specialised"]:
        return "separate"
    dx = ops.config("bwd_input", B, H, L, K)
    # Heavy shapes whose separate dX runs on the tensor cores stay separate.
    return "separate" if dx["engine"] == "tensor" and dx["intensity_class"] == "heavy" else "ffma_fused"


def _run(dy, x, k, mode="deterministic", accumulate=False, gk=None):
    if gk is None:
        gk = torch.zeros_like(k) if mode == "atomic" else torch.full_like(k, float("nan"))
    gx = ops.dx_dk(dy, x, k, gk, mode=mode, accumulate=accumulate)
    torch.cuda.synchronize()
    assert ops.device_error(clear=True) == 0, "a kernel wait expired"
    return gx, gk


SHAPES = [
    (1000, 128, 48, 48),  # one CTA per channel: direct dK; ragged last tile
    (1000, 128, 48, 3),
    (700, 128, 48, 8),
    (513, 128, 48, 16),
    (300, 128, 48, 24),
    (129, 128, 48, 32),
    (1000, 64, 48, 48),   # two CTAs per channel: partials + reduce
    (20000, 3, 48, 24),   # 49 CTAs per channel
    (900, 37, 48, 16),    # 4 CTAs per channel
    (100, 128, 48, 48),   # one tile per CTA
    (1, 4, 48, 48),       # one row, four CTAs
    (5000, 74, 48, 32),   # 2 CTAs per channel
    (64, 1, 48, 3),
    (700, 128, 48, 5),    # K not among the CUDA-core kernels' specialisations
    (4096, 128, 48, 48),  # plain grid: one CTA per channel
    (300, 128, 48, 47),   # odd K, the largest register spill
    (250, 128, 48, 1),
    (1000, 128, 44, 44),  # 44-column rows in the 48-column layout
    (513, 64, 40, 40),
    (400, 128, 40, 13),
    (129, 128, 36, 36),
    (600, 128, 36, 8),
]


@pytest.mark.parametrize("mode", ["deterministic", "atomic"])
@pytest.mark.parametrize("B,H,L,K", SHAPES)
def test_fused_backward_against_fp64_oracle(cuda_device, B, H, L, K, mode):
    dev = cuda_device
    if _sm_count(dev) >= 128:
        assert ops.backward_kind(B, H, L, K) == _expect_kind(B, H, L, K, _sm_count(dev))
    x, k, dy, cpu = _inputs(B, H, L, K, 1717, dev)
    gx, gk = _run(dy, x, k, mode=mode)
    np.testing.assert_allclose(gx.cpu().numpy(), c_oracle.dx(cpu[2], cpu[1]), **FWD_TOL)
    assert_dk_close(gk.cpu().numpy(), c_oracle.dk(cpu[2], cpu[0], K))


@pytest.mark.parametrize("B,H,L,K", [(200, 8, 42, 40), (100, 5, 28, 5), (40, 63, 37, 13), (300, 96, 48, 48)])
def test_unfused_shapes_fall_back_to_separate_kernels(cuda_device, B, H, L, K):
    """No specialised CUDA-core kernel for (L, K), odd L with H*L % 4 != 0, or a
    heavy shape whose dX runs on the tensor cores (no whole-channel grid for the
    tensor-core fused kernel at H = 96): dX then dK."""
    dev = cuda_device
    assert ops.backward_kind(B, H, L, K) == "separate"
    x, k, dy, cpu = _inputs(B, H, L, K, 99, dev)
    gx, gk = _run(dy, x, k)
    np.testing.assert_allclose(gx.cpu().numpy(), c_oracle.dx(cpu[2], cpu[1]), **FWD_TOL)
    assert_dk_close(gk.cpu().numpy(), c_oracle.dk(cpu[2], cpu[0], K))


FFMA_FUSED_SHAPES = [
    (300, 96, 48, 24),    # TMA tiles; H = 96 leaves no whole-channel tensor-core grid
    (64, 300, 48, 48),    # H > 256: channel blocks, ragged last block
    (513, 64, 37, 13),    # 1-D bulk tiles (odd L), an edge shape's (L, K)
    (77, 512, 33, 33),    # bulk tiles, channel blocks
    (1000, 256, 16, 4),   # an edge shape's (L, K): several batches per tile
    (130, 20, 32, 32),    # TMA tiles, many batches per tile, ragged last tile
    (257, 64, 31, 16),    # odd L, bulk tiles
    (999, 128, 24, 24),
    (700, 40, 32, 32),
    (5, 4, 16, 8),        # fewer rows than one tile
]


@pytest.mark.parametrize("mode", ["deterministic", "atomic"])
@pytest.mark.parametrize("B,H,L,K", FFMA_FUSED_SHAPES)
def test_ffma_fused_backward_against_fp64_oracle(cuda_device, B, H, L, K, mode):
    dev = cuda_device
    if _sm_count(dev) >= 128:
        assert ops.backward_kind(B, H, L, K) == "ffma_fused"
    x, k, dy, cpu = _inputs(B, H, L, K, 4242, dev)
    gx, gk = _run(dy, x, k, mode=mode)
    np.testing.assert_allclose(gx.cpu().numpy(), c_oracle.dx(cpu[2], cpu[1]), **FWD_TOL)
    assert_dk_close(gk.cpu().numpy(), c_oracle.dk(cpu[2], cpu[0], K))


def test_ffma_fused_backward_accumulate_determinism_and_separate_agreement(cuda_device):
    dev = cuda_device
    B, H, L, K = 2000, 64, 37, 13
    assert ops.backward_kind(B, H, L, K) == "ffma_fused"
    x, k, dy, cpu = _inputs(B, H, L, K, 12, dev)
    outs = [_run(dy, x, k)[1].clone() for _ in range(3)]
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    ref = c_oracle.dk(cpu[2], cpu[0], K)
    gk = torch.ones_like(k)
    gx, gk = _run(dy, x, k, mode="deterministic", accumulate=True, gk=gk)
    assert_dk_close(gk.cpu().numpy() - 1.0, ref)
    # Same dX arithmetic as the separate CUDA-core kernel (the same in-range FMAs in
    # the same order): bit-identical.
    gx_s = ops.dx(dy, k)
    torch.cuda.synchronize()
    assert torch.equal(gx, gx_s)


def test_forcing_a_tensor_engine_keeps_the_cuda_core_fusion_off(cuda_device):
    from pathtile_b200 import _lib

    o = _lib.LaunchOpts.frozen()
    o.engine[2] = _lib.PT_ENGINE_TENSOR
    assert ops.backward_kind(300, 96, 48, 24, opts=o) == "separate"
    assert ops.backward_kind(300, 96, 48, 24) == "ffma_fused"


def _helper_opts(limit: int):
    from pathtile_b200 import _lib

    o = _lib.LaunchOpts.frozen()
    o.bwd_kernel, o.helper_channels = _lib.PT_BWD_TENSOR_FUSED, limit
    return o


@pytest.mark.parametrize("B,H,limit", [(16384, 128, 0), (16384, 64, 4), (16384, 96, 4), (16384, 128, 8)])
def test_fused_schedule_grid(cuda_device, B, H, limit):
    sm = _sm_count(cuda_device)
    sc = tensor_schedule(B, H, sm, helper_limit=limit)
    if sm == 148:
        expect = {(128, 0): {"kp": 1, "E": 0}, (64, 4): {"kp": 2, "E": 20, "m": 4},
                  (96, 4): {"kp": 1, "E": 52, "m": 2}, (128, 8): {"kp": 1, "E": 20, "m": 7, "P": 113}}[(H, limit)]
        assert all(sc[k] == v for k, v in expect.items()), sc
    o = _helper_opts(limit)
    assert ops.backward_kind(B, H, 48, 48, opts=o) == "tensor_fused"
    info = ops.kernel_info("bwd_fused", B, H, 48, 48, opts=o)
    assert info["grid"] == (sm if sc["E"] else sc["kp"] * H)
    assert info["threads_per_block"] == 512 and info["local_memory_bytes"] == 0


HELPER_SHAPES = [
    (4096, 128, 48, 48, 8),   # 20 helpers beside 128 primaries, up to 7 channels each
    (4096, 128, 48, 7, 8),
    (3000, 96, 48, 40, 4),    # 52 helpers with two channels each; no plain grid at H = 96
    (3000, 64, 48, 24, 4),    # two primaries per channel plus helpers
    (5000, 100, 44, 11, 4),   # 44-column rows, helpers with up to three channels
]


@pytest.mark.parametrize("mode", ["deterministic", "atomic"])
@pytest.mark.parametrize("B,H,L,K,limit", HELPER_SHAPES)
def test_helper_schedules_against_fp64_oracle(cuda_device, B, H, L, K, limit, mode):
    """The tensor-core fused kernel with helper CTAs (channel switches, per-segment
    dK partials), selected per call; the frozen table may not use helpers."""
    dev = cuda_device
    o = _helper_opts(limit)
    sm = _sm_count(dev)
    sc = tensor_schedule(B, H, sm, helper_limit=limit)
    if sm == 148:
        assert sc is not None and sc["E"] > 0, sc
        assert ops.kernel_info("bwd_fused", B, H, L, K, opts=o)["grid"] == sm
    x, k, dy, cpu = _inputs(B, H, L, K, 2525, dev)
    gk = torch.zeros_like(k) if mode == "atomic" else torch.full_like(k, float("nan"))
    gx = ops.dx_dk(dy, x, k, gk, mode=mode, opts=o)
    torch.cuda.synchronize()
    assert ops.device_error(clear=True) == 0, "a kernel wait expired"
    np.testing.assert_allclose(gx.cpu().numpy(), c_oracle.dx(cpu[2], cpu[1]), **FWD_TOL)
    assert_dk_close(gk.cpu().numpy(), c_oracle.dk(cpu[2], cpu[0], K))
    # Deterministic: the same partials summed in the same order, run after run.
    if mode == "deterministic":
        gk2 = torch.empty_like(k)
        ops.dx_dk(dy, x, k, gk2, opts=o)
        torch.cuda.synchronize()
        assert torch.equal(gk, gk2)


@pytest.mark.parametrize("H", [128, 64, 96])
def test_fused_backward_accumulate_and_determinism(cuda_device, H):
    dev = cuda_device
    B, L, K = 3000, 48, 48
    x, k, dy, cpu = _inputs(B, H, L, K, 5, dev)
    outs = [_run(dy, x, k)[1].clone() for _ in range(3)]
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    gk = torch.ones_like(k)
    gx, gk = _run(dy, x, k, mode="deterministic", accumulate=True, gk=gk)
    ref = c_oracle.dk(cpu[2], cpu[0], K)
    assert_dk_close(gk.cpu().numpy() - 1.0, ref)
    gk = torch.full_like(k, 2.0)
    _, gk = _run(dy, x, k, mode="atomic", gk=gk)  # atomic adds onto what gk holds
    assert_dk_close(gk.cpu().numpy() - 2.0, ref)


def test_fused_backward_matches_separate_kernels(cuda_device):
    dev = cuda_device
    x, k, dy, _ = _inputs(4096, 128, 48, 48, 31, dev)
    gx_f, gk_f = _run(dy, x, k)
    gx_s = ops.dx(dy, k)
    gk_s = torch.empty_like(k)
    ops.dk(dy, x, gk_s)
    torch.cuda.synchronize()
    assert ops.device_error(clear=True) == 0
    torch.testing.assert_close(gx_f, gx_s, **FWD_TOL)
    torch.testing.assert_close(gk_f, gk_s, rtol=DK_RTOL, atol=DK_RTOL * float(gk_s.abs().max()))


def test_fused_backward_side_stream(cuda_device):
    dev = cuda_device
    x, k, dy, cpu = _inputs(1500, 128, 48, 16, 8, dev)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        gk = torch.empty_like(k)
        gx = ops.dx_dk(dy, x, k, gk)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    assert ops.device_error(clear=True) == 0
    np.testing.assert_allclose(gx.cpu().numpy(), c_oracle.dx(cpu[2], cpu[1]), **FWD_TOL)
    assert_dk_close(gk.cpu().numpy(), c_oracle.dk(cpu[2], cpu[0], 16))


@pytest.mark.parametrize("fuse", [True, False])
def test_autograd_backward_fuses_when_both_gradients_are_needed(cuda_device, fuse):
    from pathtile_b200 import runtime

    prev = runtime._RUNTIME
    rt = runtime.B200WarpRuntime(fuse_backward=fuse)
    runtime.install_runtime(rt)
    try:
        B, H, L, K = 1000, 128, 48, 48
        x, k, dy, cpu = _inputs(B, H, L, K, 77, cuda_device)
        xr = x.clone().requires_grad_(True)
        kr = k.clone().requires_grad_(True)
        runtime.KERNEL_EVENTS.clear()
        runtime.KERNEL_EVENTS.enabled = True
        y = runtime.depthwise_conv_ampere(xr, kr)
        y.backward(dy)
        rows = runtime.KERNEL_EVENTS.resolve_rows()
        phases = [r["phase"] for r in rows]
        expect = ["fwd", "bwd_fused"] if fuse and ops.fused_backward(B, H, L, K) else ["fwd", "bwd_input", "bwd_weight"]
        assert phases == expect
        assert ops.device_error(clear=True) == 0
        np.testing.assert_allclose(xr.grad.cpu().numpy(), c_oracle.dx(cpu[2], cpu[1]), **FWD_TOL)
        assert_dk_close(kr.grad.cpu().numpy(), c_oracle.dk(cpu[2], cpu[0], K))
    finally:
        runtime.KERNEL_EVENTS.enabled = False
        runtime.KERNEL_EVENTS.clear()
        rt.close()
        runtime._RUNTIME = prev
