"""GPU parity of the CUDA path against the oracle (run on a B200).

Tolerances (the spec of this path):
* FWD and dX: rtol = atol = 1e-5 against the reference PyTorch FP32 path
  (golden vectors) and against the FP64 C oracle;
* dK: within 1e-4 relative of an FP64 reference, checked as
  |dK - dK64| <= 1e-4 * |dK64| + 1e-4 * max|dK64| elementwise.
All launches go through the C ABI (pathtile_b200.ops -> libpathtile_b200.so).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_cases, load_golden
from oracle import c_oracle, reference_torch
from pathtile_b200 import ops, runtime, warp_tiled

pytestmark = pytest.mark.gpu

FWD_TOL = dict(rtol=1e-5, atol=1e-5)
DK_RTOL = 1e-4


def assert_dk_close(got: np.ndarray, ref64: np.ndarray) -> None:
    scale = float(np.abs(ref64).max()) if ref64.size else 0.0
    np.testing.assert_allclose(got, ref64, rtol=DK_RTOL, atol=DK_RTOL * max(scale, 1e-30))


def run_path(x, k, dy, mode="deterministic"):
    y = ops.fwd(x, k)
    gx = ops.dx(dy, k)
    gk = torch.zeros_like(k) if mode == "atomic" else torch.full_like(k, float("nan"))
    ops.dk(dy, x, gk, mode=mode)
    torch.cuda.synchronize()
    assert ops.device_error(clear=True) == 0, "a kernel wait expired"
    return y, gx, gk


CASES = golden_cases()


@pytest.mark.parametrize("mode", ["deterministic", "atomic"])
@pytest.mark.parametrize("case", CASES, ids=[c["id"] for c in CASES])
def test_golden_vectors(cuda_device, case, mode):
    g = load_golden(case)
    x, k, dy = (torch.from_numpy(g[n]).to(cuda_device) for n in ("x", "k", "dy"))
    y, gx, gk = run_path(x, k, dy, mode)
    np.testing.assert_allclose(y.cpu().numpy(), g["y"], **FWD_TOL)
    np.testing.assert_allclose(gx.cpu().numpy(), g["gx"], **FWD_TOL)
    np.testing.assert_allclose(y.cpu().numpy(), g["y64"], **FWD_TOL)
    np.testing.assert_allclose(gx.cpu().numpy(), g["gx64"], **FWD_TOL)
    assert_dk_close(gk.cpu().numpy(), g["gk64"])
    # Accuracy margin against the FP64 reference (1.0 = at the 1e-5 bar): the
    # 3xTF32 tensor-core path and the FFMA path both stay at or below half the bar.
    for got, ref in ((y, g["y64"]), (gx, g["gx64"])):
        err = np.abs(got.cpu().numpy().astype(np.float64) - ref)
        margin = float((err / (FWD_TOL["atol"] + FWD_TOL["rtol"] * np.abs(ref))).max()) if ref.size else 0.0
        assert margin <= 0.5, margin


def _inputs(B, H, L, K, seed, device):
    x, k, dy = reference_torch.make_inputs(B, H, L, K, seed)
    return x.to(device), k.to(device), dy.to(device), (x, k, dy)


def _adjoint_checks(x, k, dy, y, gx, gk):
    # <FWD(x), dy> = <x, dX(dy)> = <dK(dy, x), k>: size-independent identities.
    a = float((y.double() * dy.double()).sum())
    b = float((x.double() * gx.double()).sum())
    c = float((gk.double() * k.double()).sum())
    scale = float(y.double().abs().sum()) + 1.0
    assert abs(a - b) <= 1e-6 * scale
    assert abs(a - c) <= 1e-6 * scale


FULL_SHAPES = [
    (16384, 128, 48, 48),  # primary workload
    (4096, 64, 37, 13),    # edge shapes
    (8192, 256, 16, 4),
    (16384, 128, 48, 3),
    (2048, 512, 33, 33),
]
# Every element of FWD, dX and dK at these shapes, on every engine, is compared
# with the FP64 oracle in tests/test_gpu_full_size.py.


@pytest.mark.parametrize("B,H,L,K", FULL_SHAPES)
def test_full_size_adjoint_identities(cuda_device, B, H, L, K):
    x, k, dy, cpu = _inputs(B, H, L, K, 42, cuda_device)
    y, gx, gk = run_path(x, k, dy)
    _adjoint_checks(x, k, dy, y, gx, gk)
    assert ops.device_error() == 0


MID_SHAPES = [
    (1000, 128, 48, 48),   # TMA path, H fits the tile
    (999, 300, 48, 48),    # TMA path, channel blocks with a partial last block
    (513, 64, 37, 13),     # bulk-copy path (odd L)
    (77, 512, 33, 33),     # bulk-copy path, channel blocks
    (130, 20, 40, 40),     # TMA path, several batches per tile, ragged last tile
    (37, 19, 23, 11),      # generic kernels (shape not specialised)
    (40, 63, 37, 13),      # generic kernels (H*L % 4 != 0 for odd L)
    (5, 7, 48, 47),        # even/odd pad asymmetry (unspecialised: tensor engine by default)
    (1, 1, 1, 1),
    (3, 2, 1, 48),         # K > L
]


@pytest.mark.parametrize("B,H,L,K", MID_SHAPES)
@pytest.mark.parametrize("mode", ["deterministic", "atomic"])
def test_mid_shapes_full_oracle(cuda_device, B, H, L, K, mode):
    x, k, dy, cpu = _inputs(B, H, L, K, 1234, cuda_device)
    y, gx, gk = run_path(x, k, dy, mode)
    np.testing.assert_allclose(y.cpu().numpy(), c_oracle.fwd(cpu[0], cpu[1]), **FWD_TOL)
    np.testing.assert_allclose(gx.cpu().numpy(), c_oracle.dx(cpu[2], cpu[1]), **FWD_TOL)
    assert_dk_close(gk.cpu().numpy(), c_oracle.dk(cpu[2], cpu[0], K))


@pytest.mark.parametrize("B,H,L,K", [(5, 7, 48, 47), (64, 24, 44, 44), (100, 16, 20, 7)])
def test_generic_kernels_with_the_cuda_core_engine_forced(cuda_device, B, H, L, K):
    """Shapes without a specialised CUDA-core kernel default to the tensor engine
    where it applies; forced onto the CUDA cores they run the generic kernels."""
    assert ops.config("fwd", B, H, L, K)["specialised"] == 0
    paths = ("fwd", "bwd_input", "bwd_weight")
    try:
        for p in paths:
            ops.set_engine(p, "ffma")
        assert all(ops.config(p, B, H, L, K)["engine"] == "ffma" for p in paths)
        x, k, dy, cpu = _inputs(B, H, L, K, 77, cuda_device)
        y, gx, gk = run_path(x, k, dy)
    finally:
        for p in paths:
            ops.set_engine(p, None)
    np.testing.assert_allclose(y.cpu().numpy(), c_oracle.fwd(cpu[0], cpu[1]), **FWD_TOL)
    np.testing.assert_allclose(gx.cpu().numpy(), c_oracle.dx(cpu[2], cpu[1]), **FWD_TOL)
    assert_dk_close(gk.cpu().numpy(), c_oracle.dk(cpu[2], cpu[0], K))
    assert ops.device_error() == 0


def test_unspecialised_shapes_take_the_tensor_engine(cuda_device):
    assert ops.config("fwd", 4096, 128, 44, 44)["specialised"] == 0
    assert ops.config("fwd", 4096, 128, 44, 44)["engine"] == "tensor"
    assert ops.config("bwd_input", 4096, 128, 44, 44)["engine"] == "tensor"
    assert ops.config("fwd", 4096, 128, 40, 40)["engine"] == "ffma"  # specialised, partial tile
    assert ops.config("fwd", 4096, 128, 37, 17)["engine"] == "ffma"  # L % 4 != 0


@pytest.mark.parametrize("rows", [32, 64, 128, 256])
@pytest.mark.parametrize("stages", [2, 3, 4])
@pytest.mark.parametrize("ctas", [1, 2, 4])
@pytest.mark.parametrize("tpr", [1, 2])
def test_every_launch_configuration(cuda_device, rows, stages, ctas, tpr):
    shapes = [(700, 128, 48, 48), (301, 300, 48, 48), (257, 64, 37, 13), (65, 20, 40, 40), (99, 64, 33, 33)]
    try:
        for path in ("fwd", "bwd_input", "bwd_weight"):
            ops.set_config(path, rows, stages, ctas, tpr)
        for B, H, L, K in shapes:
            x, k, dy, cpu = _inputs(B, H, L, K, 7, cuda_device)
            y, gx, gk = run_path(x, k, dy)
            np.testing.assert_allclose(y.cpu().numpy(), c_oracle.fwd(cpu[0], cpu[1]), **FWD_TOL)
            np.testing.assert_allclose(gx.cpu().numpy(), c_oracle.dx(cpu[2], cpu[1]), **FWD_TOL)
            assert_dk_close(gk.cpu().numpy(), c_oracle.dk(cpu[2], cpu[0], K))
    finally:
        for path in ("fwd", "bwd_input", "bwd_weight"):
            ops.set_config(path, 0)


def test_deterministic_dk_is_bitwise_reproducible(cuda_device):
    x, k, dy, _ = _inputs(4096, 128, 48, 48, 3, cuda_device)
    outs = []
    for _ in range(3):
        gk = torch.empty_like(k)
        ops.dk(dy, x, gk, mode="deterministic")
        outs.append(gk.clone())
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])


def test_accumulate_semantics(cuda_device):
    x, k, dy, cpu = _inputs(300, 64, 48, 24, 5, cuda_device)
    ref = c_oracle.dk(cpu[2], cpu[0], 24)
    for mode in ("atomic", "deterministic"):
        gk = torch.ones_like(k)
        ops.dk(dy, x, gk, mode=mode, accumulate=True)
        assert_dk_close(gk.cpu().numpy() - 1.0, ref)


def test_side_stream(cuda_device):
    x, k, dy, cpu = _inputs(2048, 128, 48, 48, 9, cuda_device)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        y = ops.fwd(x, k)
        gk = torch.empty_like(k)
        ops.dk(dy, x, gk)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    np.testing.assert_allclose(y.cpu().numpy(), c_oracle.fwd(cpu[0], cpu[1]), **FWD_TOL)
    assert_dk_close(gk.cpu().numpy(), c_oracle.dk(cpu[2], cpu[0], 48))


def test_empty_batch(cuda_device):
    x = torch.empty(0, 8, 16, device=cuda_device)
    k = torch.randn(8, 4, device=cuda_device)
    assert ops.fwd(x, k).shape == (0, 8, 16)
    gk = torch.full_like(k, 3.0)
    ops.dk(x, x, gk)
    torch.cuda.synchronize()
    assert torch.count_nonzero(gk) == 0


def test_autograd_operator(cuda_device):
    x, k, dy, cpu = _inputs(512, 128, 48, 48, 11, cuda_device)
    xr = x.clone().requires_grad_(True)
    kr = k.clone().requires_grad_(True)
    y = runtime.depthwise_conv_b200(xr, kr)
    y.backward(dy)
    torch.cuda.synchronize()
    np.testing.assert_allclose(y.detach().cpu().numpy(), c_oracle.fwd(cpu[0], cpu[1]), **FWD_TOL)
    np.testing.assert_allclose(xr.grad.cpu().numpy(), c_oracle.dx(cpu[2], cpu[1]), **FWD_TOL)
    assert_dk_close(kr.grad.cpu().numpy(), c_oracle.dk(cpu[2], cpu[0], 48))


def test_reference_runtime_surface(cuda_device):
    rt = runtime.AmpereWarpRuntime(dk_mode="atomic")
    runtime.install_runtime(rt)
    x, k, dy, cpu = _inputs(256, 64, 32, 16, 13, cuda_device)
    y = torch.empty_like(x)
    gx = torch.empty_like(x)
    gk = torch.zeros_like(k)
    col = runtime.KernelEventCollector()
    col.enabled = True
    rt.launch_fwd(x, k, y, col)
    rt.launch_bwd_input(dy, k, gx, col)
    rt.launch_bwd_weight(dy, x, gk, 16, col)
    rows = col.resolve_rows()
    assert [r["phase"] for r in rows] == ["fwd", "bwd_input", "bwd_weight"]
    assert all(r["runtime_ms"] > 0 for r in rows)
    np.testing.assert_allclose(y.cpu().numpy(), c_oracle.fwd(cpu[0], cpu[1]), **FWD_TOL)
    np.testing.assert_allclose(gx.cpu().numpy(), c_oracle.dx(cpu[2], cpu[1]), **FWD_TOL)
    assert_dk_close(gk.cpu().numpy(), c_oracle.dk(cpu[2], cpu[0], 16))
    xr = x.clone().requires_grad_(True)
    out = runtime.depthwise_conv_ampere(xr, k)
    out.backward(dy)
    np.testing.assert_allclose(xr.grad.cpu().numpy(), c_oracle.dx(cpu[2], cpu[1]), **FWD_TOL)
    report = {r["kernel"]: r for r in rt.resource_report()}
    expect = {"fwd", "bwd_input", "bwd_weight"} | ({"bwd_fused"} if ops.fused_backward(16384, 128, 48, 48) else set())
    assert set(report) == expect
    assert all(report[p]["local_memory_bytes"] == 0 for p in ("fwd", "bwd_input", "bwd_weight"))
    assert all(r["regs_per_thread"] > 0 and r["resident_blocks_per_sm"] >= 1 for r in report.values())
    rt.close()
    runtime._RUNTIME = None


def test_two_runtimes_keep_their_own_launch_options(cuda_device):
    """Each runtime's overrides travel with its own launches; neither changes the
    process-wide (frozen) choice nor the other runtime's."""
    B, H, L, K = 700, 128, 48, 48
    frozen = ops.config("fwd", B, H, L, K)
    a = runtime.B200WarpRuntime(warps_per_block=2, stages=2, ctas_per_sm=1, bwdk_block=64)
    b = runtime.B200WarpRuntime()
    assert ops.config("fwd", B, H, L, K) == frozen
    assert ops.config("fwd", B, H, L, K, opts=a.opts)["rows_per_tile"] == 64
    assert ops.config("bwd_weight", B, H, L, K, opts=a.opts)["rows_per_tile"] == 64
    assert ops.config("fwd", B, H, L, K, opts=b.opts) == frozen
    x, k, dy, cpu = _inputs(B, H, L, K, 17, cuda_device)
    outs = {}
    for name, rt in (("a", a), ("b", b), ("a2", a)):
        y, gx, gk = torch.empty_like(x), torch.empty_like(x), torch.zeros_like(k)
        rt.launch_fwd(x, k, y)
        rt.launch_bwd_input(dy, k, gx)
        rt.launch_bwd_weight(dy, x, gk, K)
        torch.cuda.synchronize()
        outs[name] = (y, gx, gk)
    assert ops.device_error(clear=True) == 0
    y64, gx64, gk64 = c_oracle.fwd(cpu[0], cpu[1]), c_oracle.dx(cpu[2], cpu[1]), c_oracle.dk(cpu[2], cpu[0], K)
    for y, gx, gk in outs.values():
        np.testing.assert_allclose(y.cpu().numpy(), y64, **FWD_TOL)
        np.testing.assert_allclose(gx.cpu().numpy(), gx64, **FWD_TOL)
        assert_dk_close(gk.cpu().numpy(), gk64)
    a.close()
    assert ops.config("fwd", B, H, L, K) == frozen


def test_legacy_warp_tiled_surface(cuda_device):
    warp_tiled.reset_timing_collectors()
    x, k, dy, cpu = _inputs(64, 128, 48, 48, 42, cuda_device)
    xr = x.clone().requires_grad_(True)
    kr = k.clone().requires_grad_(True)
    y = warp_tiled.depthwise_conv_shared(xr, kr)
    y.backward(dy)
    assert len(warp_tiled.FWD_TIMES) == len(warp_tiled.BWD_IN_TIMES) == len(warp_tiled.BWD_K_TIMES) == 1
    np.testing.assert_allclose(y.detach().cpu().numpy(), c_oracle.fwd(cpu[0], cpu[1]), **FWD_TOL)
    np.testing.assert_allclose(xr.grad.cpu().numpy(), c_oracle.dx(cpu[2], cpu[1]), **FWD_TOL)
    assert_dk_close(kr.grad.cpu().numpy(), c_oracle.dk(cpu[2], cpu[0], 48))
    with pytest.raises(TypeError):
        warp_tiled.depthwise_conv_shared(x.double(), k)
    with pytest.raises(ValueError, match="Channel mismatch"):
        warp_tiled.depthwise_conv_shared(x, k[:64])


def test_default_path_kernels_have_no_spills(cuda_device):
    """Every kernel the frozen table launches at the BASELINE shapes -- the
    tensor-core FWD / dX kernels where they apply, the CUDA-core kernels, and the
    fused backward of dx_dk -- keeps its working set in registers."""
    for B, H, L, K in FULL_SHAPES:
        for path in ("fwd", "bwd_input", "bwd_weight"):
            info = ops.kernel_info(path, B, H, L, K)
            assert info["specialised"] == 1
            assert info["local_memory_bytes"] == 0, (path, B, H, L, K, info)
            assert info["resident_blocks_per_sm"] >= 1
        assert ops.fused_backward(B, H, L, K)
        info = ops.kernel_info("bwd_fused", B, H, L, K)
        assert info["local_memory_bytes"] == 0, ("bwd_fused", B, H, L, K, info)
        assert info["resident_blocks_per_sm"] >= 1
    # Every K of the tensor-core fused kernel (its register split is per K).
    for K in range(1, 49):
        info = ops.kernel_info("bwd_fused", 16384, 128, 48, K)
        assert info["threads_per_block"] == 512 and info["regs_per_thread"] == 128, (K, info)
        assert info["local_memory_bytes"] == 0, (K, info)


def test_reference_kernels_agree_when_built(cuda_device):
    """Cross-check against the reference's own CUDA kernels compiled for sm_100a
    (oracle/_ref, built from the reference checkout where it exists)."""
    import ctypes
    from pathlib import Path

    lib_path = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libref_warptile.so"
    if not lib_path.exists():
        pytest.skip("reference kernels not built (reference checkout absent when building)")
    lib = ctypes.CDLL(str(lib_path))
    x, k, dy, _ = _inputs(1024, 128, 48, 48, 21, cuda_device)
    y_ref, gx_ref, gk_ref = torch.empty_like(x), torch.empty_like(x), torch.zeros_like(k)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.ref_fwd(p(x), p(k), p(y_ref), 1024, 128, 48, 48, s) == 0
    assert lib.ref_dx(p(dy), p(k), p(gx_ref), 1024, 128, 48, 48, s) == 0
    assert lib.ref_dk(p(dy), p(x), p(gk_ref), 1024, 128, 48, 48, s) == 0
    y, gx, gk = run_path(x, k, dy)
    torch.testing.assert_close(y, y_ref, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(gx, gx_ref, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(gk, gk_ref, rtol=1e-4, atol=1e-3)


def test_no_device_errors_recorded(cuda_device):
    assert ops.device_error(clear=True) == 0
