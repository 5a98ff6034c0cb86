"""S4ConvD on the B200 depthwise-convolution operator (the path's caller).

The reference trains a four-block S4 model whose every block runs the short
depthwise convolution on [B, H, L] with K = L taps generated from the S4
parameters (kernels/warp_tiled_ampere.py:1122-1215, training loop :1432-1560:
batch 16384, L = 48, H = 128, SGD lr 1e-3 momentum 0.9, RMSLE loss).  This
module rebuilds that model on the native depthwise operator.

Two B200-side changes, neither of which changes the function computed:

* the block's skip term ``y + x * skip`` (:1188) is a convolution with ``skip``
  added to the centre tap (tap K//2 multiplies x[t]), so the block convolves
  with ``k + skip * e_{K//2}`` and the extra elementwise pass disappears;
  autograd routes the centre-tap gradient (which dK computes anyway) to ``skip``;
* the block keeps its activations channels-last: the reference transposes
  [B, L, H] to [B, H, L] for the convolution and back (:1186, :1190); here the
  convolution runs on [B, L, H] directly (:func:`runtime.depthwise_conv_b200_cl`)
  and the 1x1 ``Conv1d`` + GLU over channels becomes the same linear map over
  the last dimension (same parameters).

``conv`` is injectable so a caller can time the same model on another
convolution; a conv function with a true ``channels_last`` attribute gets
[B, L, H] tensors, any other gets [B, H, L] (the reference's layout).  By
default every block uses the native channels-last operator.
"""
from __future__ import annotations

import math
from typing import Callable

import torch
import torch.nn as nn

import torch.nn.functional as F

from .runtime import MAX_L, depthwise_conv_b200_cl

ConvFn = Callable[[torch.Tensor, torch.Tensor], torch.Tensor]


class S4ConvKernel(nn.Module):
    """Diagonal S4 kernel generator: k[h, t] = 2 Re(sum_n C'_hn exp(dt_h A_hn t))."""

    def __init__(self, hidden_dim: int, state_dim: int, conv: ConvFn = depthwise_conv_b200_cl) -> None:
        super().__init__()
        self.H = hidden_dim
        self.N = state_dim
        self.conv = conv
        self.log_dt = nn.Parameter(
            torch.rand(hidden_dim) * (math.log(0.1) - math.log(0.001)) + math.log(0.001))
        self.C_re = nn.Parameter(torch.randn(hidden_dim, state_dim // 2))
        self.C_im = nn.Parameter(torch.randn(hidden_dim, state_dim // 2))
        self.log_A_re = nn.Parameter(torch.randn(hidden_dim, state_dim // 2))
        self.A_im = nn.Parameter(torch.ones(hidden_dim, state_dim // 2))

    def build_kernel(self, taps: int, device: torch.device) -> torch.Tensor:
        dt = torch.exp(self.log_dt)
        C = torch.complex(self.C_re, self.C_im)
        A = torch.complex(-torch.exp(self.log_A_re), self.A_im)
        dtA = A * dt.unsqueeze(-1)
        times = torch.arange(taps, device=device, dtype=torch.float32)
        powers = torch.exp(dtA.unsqueeze(-1) * times)
        C_eff = C * (torch.exp(dtA) - 1.0) / A
        return (2 * torch.einsum("hn,hnk->hk", C_eff, powers).real).contiguous()

    @property
    def channels_last(self) -> bool:
        return bool(getattr(self.conv, "channels_last", False))

    def forward(self, x: torch.Tensor, skip: torch.Tensor | None = None) -> torch.Tensor:
        """x is [B, L, H] for a channels-last conv, else [B, H, L]; the output likewise."""
        if self.channels_last:
            _, L, H = x.shape
        else:
            _, H, L = x.shape
        if H != self.H:
            raise ValueError(f"Expected H={self.H}, got {H}")
        if L > MAX_L:
            raise ValueError(f"The depthwise kernels support L<={MAX_L}")
        k = self.build_kernel(L, x.device)
        if skip is not None:  # y + x*skip == conv with skip added to the centre tap
            centre = torch.zeros_like(k)
            centre[:, L // 2] = 1.0
            k = k + centre * skip.unsqueeze(-1)
        return self.conv(x.contiguous(), k)


class S4ConvBlock(nn.Module):
    def __init__(self, hidden_dim: int, state_dim: int, dropout: float, conv: ConvFn = depthwise_conv_b200_cl) -> None:
        super().__init__()
        self.skip = nn.Parameter(torch.randn(hidden_dim))
        self.kernel_layer = S4ConvKernel(hidden_dim, state_dim, conv)
        self.activation = nn.GELU()
        self.dropout = nn.Dropout(dropout)
        self.output_linear = nn.Sequential(nn.Conv1d(hidden_dim, 2 * hidden_dim, kernel_size=1), nn.GLU(dim=1))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        residual = x  # [B, L, H]
        if self.kernel_layer.channels_last:
            y = self.kernel_layer(x.contiguous(), self.skip)
            y = self.activation(self.dropout(y))
            conv1x1 = self.output_linear[0]
            y = F.glu(F.linear(y, conv1x1.weight.squeeze(-1), conv1x1.bias), dim=-1)
            return y + residual
        x_hl = x.transpose(1, 2).contiguous()
        y = self.kernel_layer(x_hl, self.skip)
        y = self.output_linear(self.activation(self.dropout(y)))
        return y.transpose(1, 2) + residual


class Model(nn.Module):
    """Encoder -> S4 blocks -> decoder; input [B, L, input_dim], output [B, output_dim]."""

    def __init__(self, state_dim: int = 64, hidden_dim: int = 128, input_dim: int = 4, output_dim: int = 1,
                 num_blocks: int = 4, dropout: float = 0.01, conv: ConvFn = depthwise_conv_b200_cl) -> None:
        super().__init__()
        self.encoder = nn.Linear(input_dim, hidden_dim)
        self.blocks = nn.ModuleList([S4ConvBlock(hidden_dim, state_dim, dropout, conv) for _ in range(num_blocks)])
        self.decoder = nn.Linear(hidden_dim, output_dim)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = self.encoder(x)
        for block in self.blocks:
            x = block(x)
        return self.decoder(x)[:, -1, :]


def rmsle(prediction: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """Root mean squared log error on non-negative clamps (the reference's loss)."""
    p = torch.clamp(prediction.reshape(-1), min=0.0)
    t = torch.clamp(target.reshape(-1), min=0.0)
    return torch.sqrt((torch.log1p(p) - torch.log1p(t)).square().mean() + 1e-12)


def make_optimizer(model: nn.Module, lr: float = 1e-3, momentum: float = 0.9) -> torch.optim.Optimizer:
    return torch.optim.SGD(model.parameters(), lr=lr, momentum=momentum)


def train_step(model: nn.Module, optimizer: torch.optim.Optimizer, x: torch.Tensor,
               target: torch.Tensor) -> torch.Tensor:
    """One optimisation step: zero grads, forward, RMSLE, backward, SGD update."""
    optimizer.zero_grad(set_to_none=True)
    loss = rmsle(model(x), target)
    loss.backward()
    optimizer.step()
    return loss.detach()


def synthetic_batch(batch: int, seq_len: int = 48, input_dim: int = 4, device: str | torch.device = "cuda",
                    seed: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Seeded stand-in for the reference's meter-reading windows (the ASHRAE data is not
    shipped): features ~ N(0,1), non-negative targets ~ |N(0,1)| scaled."""
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(batch, seq_len, input_dim, device=device, generator=g)
    target = torch.randn(batch, 1, device=device, generator=g).abs() * 3.0
    return x, target
