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


def _group_with_a_silent_peer(H: int, K: int):
    """A two-rank pt_peer_group on this one GPU whose second rank never runs: both
    exchange buffers are local allocations, so this rank's rows and flags land in
    both, while the flags rank 1 would publish into this rank's buffer stay zero."""
    lib = _lib.load()
    nbytes = lib.pt_peer_buffer_bytes(2, H, K)
    own, other = ctypes.c_void_p(), ctypes.c_void_p()
    assert lib.pt_peer_alloc(nbytes, ctypes.byref(own)) == _lib.PT_OK
    assert lib.pt_peer_alloc(nbytes, ctypes.byref(other)) == _lib.PT_OK
    bufs = (ctypes.c_void_p * _lib.PT_MAX_PEERS)()
    bufs[0], bufs[1] = own.value, other.value
    return _lib.PeerGroup(0, 2, bufs, 1), (own, other)


def _check_peer_wait_ran_out(dk: torch.Tensor, fill: float, t0: float) -> None:
    import time

    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert 1.5 <= elapsed < 60.0  # the 2 s limit, then the kernel returned
    assert ops.device_error(clear=True) == 64  # bit 6: a peer's row never arrived
    assert bool((dk == fill).all())  # rows whose sum is incomplete are left unwritten


@pytest.mark.parametrize("fused", [False, True])
def test_peer_wait_runs_out_sets_the_error_bit_and_returns(cuda_device, fused):
    """The peer exchange's bounded wait (a flag that nothing sets: the second rank
    does not exist) gives up after its limit, sets the peer-wait bit and leaves dK
    untouched -- in the standalone peer kernel and inside the fused backward kernel
    -- and the next regular launches are correct."""
    import time

    lib = _lib.load()
    assert ops.device_error(clear=True) == 0
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    B, H, L, K = (1024, 128, 48, 48) if fused else (64, 8, 37, 13)
    grp, bufs = _group_with_a_silent_peer(H, K)
    grp_p = ctypes.cast(ctypes.pointer(grp), ctypes.c_void_p)
    try:
        fill = 7.0
        dk = torch.full((H, K), fill, device=cuda_device)
        x, k, dy = reference_torch.make_inputs(B, H, L, K, 11)
        x, k, dy = x.to(cuda_device), k.to(cuda_device), dy.to(cuda_device)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        if fused:
            if torch.cuda.get_device_properties(cuda_device).multi_processor_count == 148:
                assert lib.pt_dx_dk_allreduce_fused(B, H, L, K) == 1
            gx = torch.empty_like(x)
            st = lib.pt_dx_dk_allreduce(_p(dy), _p(x), _p(k), _p(gx), _p(dk), B, H, L, K, None, 0, grp_p, stream)
        else:
            st = lib.pt_allreduce_peer(_p(dk), H, K, grp_p, stream)
        assert st == _lib.PT_OK, _lib.status_string(st)
        _check_peer_wait_ran_out(dk, fill, t0)
        if fused:  # dX does not depend on the exchange
            np.testing.assert_allclose(gx.cpu().numpy(), c_oracle.dx(dy.cpu(), k.cpu()), rtol=1e-5, atol=1e-5)
    finally:
        torch.cuda.synchronize()
        for b in bufs:
            lib.pt_peer_free(b)
    # The context is intact.
    y = ops.fwd(x, k)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    np.testing.assert_allclose(y.cpu().numpy(), c_oracle.fwd(x.cpu(), k.cpu()), rtol=1e-5, atol=1e-5)
