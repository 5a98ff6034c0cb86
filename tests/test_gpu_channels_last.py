"""GPU parity of the channels-last ([B, L, H]) kernels: pt_fwd_cl / pt_dx_cl /
pt_dk_cl through ops.fwd_cl / dx_cl / dk_cl and the DepthConvCL autograd op.

Same bars as the [B, H, L] kernels: FWD / dX within rtol = atol = 1e-5 of the
FP64 C oracle (run on the transposed tensors), dK within 1e-4 relative of the
FP64 dK.  Shapes cover every compiled (L, K) bucket (maxima 16 / 32 / 48, runtime
L and K below them), H not a multiple of the 32-channel CTA width, ragged
batches, K > L, even and odd K, and the S4 model's shape.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import c_oracle, reference_torch
from pathtile_b200 import ops, runtime, s4conv

pytestmark = pytest.mark.gpu

FWD_TOL = dict(rtol=1e-5, atol=1e-5)
DK_RTOL = 1e-4


def assert_dk_close(got: np.ndarray, ref64: np.ndarray) -> None:
    scale = float(np.abs(ref64).max()) if ref64.size else 0.0
    np.testing.assert_allclose(got, ref64, rtol=DK_RTOL, atol=DK_RTOL * max(scale, 1e-30))


def _inputs_cl(B, H, L, K, seed, device):
    """Oracle inputs in [B, H, L] and their channels-last copies on the device."""
    x, k, dy = reference_torch.make_inputs(B, H, L, K, seed)
    to_cl = lambda t: t.transpose(1, 2).contiguous().to(device)
    return to_cl(x), k.to(device), to_cl(dy), (x, k, dy)


def _hl(t: torch.Tensor) -> np.ndarray:
    return t.transpose(1, 2).cpu().numpy()


SHAPES = [
    (300, 128, 48, 48),   # the S4 block's shape class
    (77, 33, 20, 7),      # L bucket 32, K bucket 16, H = 32 + 1
    (5, 3, 16, 16),
    (64, 70, 33, 33),     # L and K bucket 48 just above 32
    (1, 1, 4, 1),
    (129, 40, 48, 3),
    (200, 64, 30, 47),    # K > L
    (31, 300, 12, 12),
    (16, 8, 8, 48),       # K bucket 48, L bucket 16
]


@pytest.mark.parametrize("B,H,L,K", SHAPES)
def test_channels_last_against_fp64_oracle(cuda_device, B, H, L, K):
    x, k, dy, cpu = _inputs_cl(B, H, L, K, 606, cuda_device)
    y = ops.fwd_cl(x, k)
    gx = ops.dx_cl(dy, k)
    gk = torch.full_like(k, float("nan"))
    ops.dk_cl(dy, x, gk)
    torch.cuda.synchronize()
    np.testing.assert_allclose(_hl(y), c_oracle.fwd(cpu[0], cpu[1]), **FWD_TOL)
    np.testing.assert_allclose(_hl(gx), c_oracle.dx(cpu[2], cpu[1]), **FWD_TOL)
    assert_dk_close(gk.cpu().numpy(), c_oracle.dk(cpu[2], cpu[0], K))


def test_channels_last_dk_accumulate_and_determinism(cuda_device):
    x, k, dy, cpu = _inputs_cl(3000, 128, 48, 48, 7, cuda_device)
    outs = []
    for _ in range(3):
        gk = torch.empty_like(k)
        ops.dk_cl(dy, x, gk)
        outs.append(gk.clone())
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    gk = torch.ones_like(k)
    ops.dk_cl(dy, x, gk, accumulate=True)
    torch.cuda.synchronize()
    assert_dk_close(gk.cpu().numpy() - 1.0, c_oracle.dk(cpu[2], cpu[0], 48))


def test_channels_last_autograd_matches_channels_first_op(cuda_device):
    B, H, L, K = 500, 128, 48, 48
    x, k, dy, _ = _inputs_cl(B, H, L, K, 9, cuda_device)
    xr = x.clone().requires_grad_(True)
    kr = k.clone().requires_grad_(True)
    y = runtime.depthwise_conv_b200_cl(xr, kr)
    y.backward(dy)
    xh = x.transpose(1, 2).contiguous().requires_grad_(True)
    kh = k.clone().requires_grad_(True)
    yh = runtime.depthwise_conv_b200(xh, kh)
    yh.backward(dy.transpose(1, 2).contiguous())
    torch.cuda.synchronize()
    torch.testing.assert_close(y, yh.transpose(1, 2), **FWD_TOL)
    torch.testing.assert_close(xr.grad, xh.grad.transpose(1, 2), **FWD_TOL)
    torch.testing.assert_close(kr.grad, kh.grad, rtol=DK_RTOL, atol=DK_RTOL * float(kh.grad.abs().max()))


def test_channels_last_s4_model_matches_channels_first(cuda_device):
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.manual_seed(4)
    cl = s4conv.Model(dropout=0.0).to(cuda_device)
    cf = s4conv.Model(dropout=0.0).to(cuda_device)
    cf.load_state_dict(cl.state_dict())
    for blk in cf.blocks:
        blk.kernel_layer.conv = runtime.depthwise_conv_b200
    assert cl.blocks[0].kernel_layer.channels_last and not cf.blocks[0].kernel_layer.channels_last
    x, target = s4conv.synthetic_batch(512, device=cuda_device, seed=2)
    lc = s4conv.rmsle(cl(x), target)
    lf = s4conv.rmsle(cf(x), target)
    torch.testing.assert_close(lc, lf, rtol=1e-5, atol=1e-6)
    lc.backward()
    lf.backward()
    for (name, pc), pf in zip(cl.named_parameters(), cf.parameters()):
        scale = float(pf.grad.abs().max()) + 1e-12
        torch.testing.assert_close(pc.grad, pf.grad, rtol=1e-3, atol=1e-4 * scale, msg=name)
