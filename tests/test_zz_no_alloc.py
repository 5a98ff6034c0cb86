"""GPU: pt_dk_noalloc, the filter-gradient entry point that allocates nothing.

Callers that may not allocate device memory -- a runtime that owns a fixed
memory budget and every allocation in it, or a steady-state loop where
cudaMalloc/cudaFree would block on the device -- cannot provide the workspace
that pt_dk's deterministic mode needs.  pt_dk_noalloc keeps those partial sums
in a fixed 8 MiB scratch array inside the library instead.  This test calls it
through the C ABI twice in a row (different inputs each time, so a call cannot
lean on what the previous one left in the shared scratch) and checks every
result against pt_dk with a caller workspace, within the dK tolerance of the
parity tests (1e-4 relative to the FP64 scale).  It is collected last and
needs nothing from earlier tests.
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


def _close(got: torch.Tensor, ref: torch.Tensor) -> None:
    r = ref.double().cpu().numpy()
    scale = float(np.abs(r).max())
    np.testing.assert_allclose(got.double().cpu().numpy(), r, rtol=1e-4, atol=1e-4 * scale)


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
        _close(got, ref)
        _close(acc - 1.0, ref)
    assert ops.device_error(clear=True) == 0


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
