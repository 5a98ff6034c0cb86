"""S4ConvD on the native operator (the path's caller in the reference).

CPU: folding the block's skip term into the centre tap is the reference's
``conv(x, k) + x * skip`` (kernels/warp_tiled_ampere.py:1186-1188).
GPU: the model with the native operator matches the same model (same weights)
on the reference's PyTorch convolution, through a full training step.
"""
from __future__ import annotations

import copy

import pytest
import torch

from oracle import reference_torch
from pathtile_b200 import s4conv


def test_skip_fold_equals_reference_block_on_cpu():
    torch.manual_seed(0)
    kl = s4conv.S4ConvKernel(16, 8, conv=reference_torch.depthwise_same)
    x = torch.randn(3, 16, 48)
    skip = torch.randn(16)
    folded = kl(x, skip)
    k = kl.build_kernel(48, x.device)
    explicit = reference_torch.depthwise_same(x, k) + x * skip.unsqueeze(-1)
    torch.testing.assert_close(folded, explicit, rtol=1e-5, atol=1e-5)


def test_skip_gradient_is_centre_tap_gradient_on_cpu():
    torch.manual_seed(1)
    kl = s4conv.S4ConvKernel(8, 8, conv=reference_torch.depthwise_same)
    x = torch.randn(2, 8, 16)
    skip = torch.randn(8, requires_grad=True)
    dy = torch.randn(2, 8, 16)
    kl(x, skip).backward(dy)
    torch.testing.assert_close(skip.grad, (dy * x).sum(dim=(0, 2)), rtol=1e-5, atol=1e-5)


def test_model_shapes_on_cpu():
    m = s4conv.Model(conv=reference_torch.depthwise_same)
    x, t = s4conv.synthetic_batch(5, device="cpu")
    assert m(x).shape == (5, 1)
    assert s4conv.rmsle(m(x), t).ndim == 0


def test_channels_last_block_matches_channels_first_block_on_cpu():
    """The block's [B, L, H] path (no transposes, 1x1 conv as a linear map over
    the last dimension) computes what its [B, H, L] path computes."""
    def conv_cl(x, k):  # the reference conv, applied to channels-last tensors
        return reference_torch.depthwise_same(x.transpose(1, 2), k).transpose(1, 2).contiguous()
    conv_cl.channels_last = True
    torch.manual_seed(1)
    m_cl = s4conv.Model(hidden_dim=16, state_dim=8, num_blocks=2, dropout=0.0, conv=conv_cl)
    m_cf = copy.deepcopy(m_cl)
    for blk in m_cf.blocks:
        blk.kernel_layer.conv = reference_torch.depthwise_same
    assert m_cl.blocks[0].kernel_layer.channels_last and not m_cf.blocks[0].kernel_layer.channels_last
    x, target = s4conv.synthetic_batch(6, device="cpu", seed=3)
    l_cl = s4conv.rmsle(m_cl(x), target)
    l_cf = s4conv.rmsle(m_cf(x), target)
    torch.testing.assert_close(l_cl, l_cf, rtol=1e-5, atol=1e-6)
    l_cl.backward()
    l_cf.backward()
    for (name, a), b in zip(m_cl.named_parameters(), m_cf.parameters()):
        torch.testing.assert_close(a.grad, b.grad, rtol=1e-4, atol=1e-6, msg=name)


@pytest.mark.gpu
def test_native_model_matches_reference_conv_model_through_a_training_step():
    if not torch.cuda.is_available():
        pytest.fail("needs a CUDA device")
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    dev = torch.device("cuda", 0)
    torch.manual_seed(3)
    ours = s4conv.Model(dropout=0.0).to(dev)
    ref = copy.deepcopy(ours)
    for blk in ref.blocks:
        blk.kernel_layer.conv = reference_torch.depthwise_same
    x, target = s4conv.synthetic_batch(256, device=dev, seed=5)
    loss_o = s4conv.rmsle(ours(x), target)
    loss_r = s4conv.rmsle(ref(x), target)
    torch.testing.assert_close(loss_o, loss_r, rtol=1e-5, atol=1e-6)
    loss_o.backward()
    loss_r.backward()
    for (name, po), pr in zip(ours.named_parameters(), ref.parameters()):
        scale = float(pr.grad.abs().max()) + 1e-12
        torch.testing.assert_close(po.grad, pr.grad, rtol=1e-3, atol=1e-4 * scale, msg=name)
    opt_o, opt_r = s4conv.make_optimizer(ours), s4conv.make_optimizer(ref)
    for _ in range(3):
        lo = s4conv.train_step(ours, opt_o, x, target)
        lr_ = s4conv.train_step(ref, opt_r, x, target)
    torch.testing.assert_close(lo, lr_, rtol=1e-4, atol=1e-5)
    for po, pr in zip(ours.parameters(), ref.parameters()):
        torch.testing.assert_close(po, pr, rtol=1e-4, atol=1e-5)
