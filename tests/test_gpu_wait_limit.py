"""GPU: a bounded device-side wait runs out, reports, and leaves the context usable.

Every pipeline kernel waits on mbarriers through one bounded routine (2 s
limit); when a wait runs out the kernel sets a bit in the device error word and
returns instead of spinning.  pt_selftest_wait_timeout launches one warp that
waits, through that same routine with a 1 ms limit, on an mbarrier nothing ever
arrives on -- no copy is issued and no memory outside the kernel's own shared
memory is touched, so the only thing that can happen is the timeout.  The test
checks that the wait gave up after about the limit, that the error word holds
the consumer-wait bit, and that a regular launch right after is correct.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import c_oracle, reference_torch
from pathtile_b200 import _lib, ops

pytestmark = pytest.mark.gpu

LIMIT_NS = 1_000_000  # 1 ms


def _p(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def test_wait_runs_out_sets_the_error_bit_and_returns(cuda_device):
    lib = _lib.load()
    assert ops.device_error(clear=True) == 0
    out = torch.full((2,), -1, dtype=torch.int64, device=cuda_device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    st = lib.pt_selftest_wait_timeout(LIMIT_NS, _p(out), stream)
    assert st == _lib.PT_OK, _lib.status_string(st)
    torch.cuda.synchronize()
    waited_ns, succeeded = out.tolist()
    assert succeeded == 0
    assert LIMIT_NS <= waited_ns < 1_000_000_000
    assert ops.device_error(clear=True) == 1  # bit 0: a consumer's wait ran out
    assert ops.device_error() == 0

    # The context is intact: the next regular launches are correct.
    B, H, L, K = 256, 128, 48, 48
    x, k, dy = reference_torch.make_inputs(B, H, L, K, 5)
    y = ops.fwd(x.to(cuda_device), k.to(cuda_device))
    gk = torch.empty(H, K, device=cuda_device)
    gx = ops.dx_dk(dy.to(cuda_device), x.to(cuda_device), k.to(cuda_device), gk)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    np.testing.assert_allclose(y.cpu().numpy(), c_oracle.fwd(x, k), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(gx.cpu().numpy(), c_oracle.dx(dy, k), rtol=1e-5, atol=1e-5)
    ref = c_oracle.dk(dy, x, K)
    np.testing.assert_allclose(gk.cpu().numpy(), ref, rtol=1e-4, atol=1e-4 * float(np.abs(ref).max()))


def test_wait_that_is_satisfied_reports_nothing(cuda_device):
    """Many waits that do complete (a full pipeline run) leave the word at zero."""
    x, k, _ = reference_torch.make_inputs(4096, 64, 48, 48, 6)
    for _ in range(3):
        ops.fwd(x.to(cuda_device), k.to(cuda_device))
    assert ops.device_error() == 0
