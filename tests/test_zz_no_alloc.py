"""GPU: pt_dk_noalloc, the filter-gradient entry point that allocates nothing.

Callers that may not allocate device memory -- a runtime that owns a fixed
memory budget and every allocation in it, or a steady-state loop where
cudaMalloc/cudaFree would block on the device -- cannot provide the workspace
that pt_dk's deterministic mode needs.  pt_dk_noalloc keeps those partial sums
in a fixed 8 MiB scratch array inside the library instead.  This test calls it
through the C ABI twice in a row (different inputs each time, so a call cannot
lean on what the previous one left in the shared scratch), on both dK engines,
and checks every result against pt_dk with a caller workspace (bit-identical:
the same kernels sum the same partials in the same order) and against an FP64
dK within the tolerance of the parity tests (1e-4 relative to the FP64
scale).  It is collected last and needs nothing from earlier tests.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import reference_torch
from pathtile_b200 import _lib, ops

pytestmark = pytest.mark.gpu

SHAPES = [
    (4096, 128, 48, 48),  # specialised TMA kernels
    (513, 64, 37, 13),    # specialised bulk-copy kernels
    (61, 19, 23, 11),     # generic kernels
]


def _p(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _close(got: torch.Tensor, ref: np.ndarray) -> None:
    scale = float(np.abs(ref).max())
    np.testing.assert_allclose(got.double().cpu().numpy(), ref, rtol=1e-4, atol=1e-4 * scale)


def _fp64_dk(dy: torch.Tensor, x: torch.Tensor, K: int) -> np.ndarray:
    """dk[h,j] = sum_{b,t} dy[b,h,t] x[b,h,t+j-K//2] in FP64, on the GPU (plain torch)."""
    B, H, L = x.shape
    xp = torch.nn.functional.pad(x.double(), (K // 2, K - 1 - K // 2))
    d = dy.double()
    return torch.stack([(xp[:, :, j:j + L] * d).sum(dim=(0, 2)) for j in range(K)], dim=1).cpu().numpy()


@pytest.fixture(scope="module")
def lib():
    from pathtile_b200 import build

    if not torch.cuda.is_available():
        pytest.fail("needs a CUDA device")
    build.build()
    return _lib.load()


@pytest.mark.parametrize("B,H,L,K", SHAPES)
def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(lib, B, H, L, K):
    dev = torch.device("cuda", 0)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    assert lib.pt_dk_workspace_bytes(B, H, L, K) <= _lib.PT_DK_NOALLOC_SCRATCH_BYTES
    for call, seed in enumerate((101, 202)):
        x, k, dy = (t.to(dev) for t in reference_torch.make_inputs(B, H, L, K, seed))
        ref = torch.empty_like(k)
        ops.dk(dy, x, ref, mode="deterministic")  # existing entry point, caller workspace
        got = torch.full_like(k, float("nan"))
        st = lib.pt_dk_noalloc(_p(dy), _p(x), _p(got), B, H, L, K, 0, stream)
        assert st == _lib.PT_OK, _lib.status_string(st)
        acc = torch.ones_like(k)
        st = lib.pt_dk_noalloc(_p(dy), _p(x), _p(acc), B, H, L, K, 1, stream)
        assert st == _lib.PT_OK, _lib.status_string(st)
        torch.cuda.synchronize()
        # Same kernels, same partial order: bit-identical to pt_dk, and the
        # accumulate mode adds dK onto what dk held with one FP32 add, as
        # torch's `ref + 1` does.
        assert torch.equal(got, ref)
        assert torch.equal(acc, ref + 1.0)
        _close(got, _fp64_dk(dy, x, K))
    assert ops.device_error(clear=True) == 0


def test_noalloc_tensor_core_dk_engine_on_consecutive_calls(lib):
    """The tensor-core dK keeps a different partial layout (per-CTA partials
    plus a slot -> channel-group table) in the same scratch array."""
    dev = torch.device("cuda", 0)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    B, H, L, K = 4096, 128, 48, 48
    ops.set_engine("bwd_weight", "tensor")
    try:
        assert ops.config("bwd_weight", B, H, L, K)["engine"] == "tensor"
        assert lib.pt_dk_workspace_bytes(B, H, L, K) <= _lib.PT_DK_NOALLOC_SCRATCH_BYTES
        for seed in (303, 404):
            x, k, dy = (t.to(dev) for t in reference_torch.make_inputs(B, H, L, K, seed))
            ref = torch.empty_like(k)
            ws = torch.empty(ops.dk_workspace_bytes(B, H, L, K), dtype=torch.uint8, device=dev)
            ops.dk(dy, x, ref, mode="deterministic", workspace=ws)
            got = torch.full_like(k, float("nan"))
            st = lib.pt_dk_noalloc(_p(dy), _p(x), _p(got), B, H, L, K, 0, stream)
            assert st == _lib.PT_OK, _lib.status_string(st)
            torch.cuda.synchronize()
            assert torch.equal(got, ref)
            _close(got, _fp64_dk(dy, x, K))
    finally:
        ops.set_engine("bwd_weight", None)
    assert ops.device_error(clear=True) == 0


def test_noalloc_scratch_holds_the_primary_workload(lib):
    """The documented primary shape (B=16384, H=128, L=K=48) fits the fixed
    scratch under the frozen launch table on this device (no launch needed)."""
    assert 0 < lib.pt_dk_workspace_bytes(16384, 128, 48, 48) <= _lib.PT_DK_NOALLOC_SCRATCH_BYTES


def test_noalloc_rejects_shapes_beyond_its_scratch(lib):
    dev = torch.device("cuda", 0)
    B, H, L, K = 600, 512, 23, 11  # generic kernels: partials [CTAs][K][H] exceed 8 MiB
    need = lib.pt_dk_workspace_bytes(B, H, L, K)
    assert need > _lib.PT_DK_NOALLOC_SCRATCH_BYTES
    x = torch.zeros(B, H, L, device=dev)
    gk = torch.zeros(H, K, device=dev)
    st = lib.pt_dk_noalloc(_p(x), _p(x), _p(gk), B, H, L, K, 0, ctypes.c_void_p(0))
    assert st == _lib.PT_ERR_SCRATCH_LIMIT
    assert "8 MiB" in _lib.status_string(st)
