"""Mamba-style mixer around a scan layer (drop-in for the reference's models/mixer.py:31-99).

    in_proj (C -> 2 * expand * C) -> split (u, z)
    u: causal depthwise Conv1d (kernel d_conv) -> SiLU -> ssm
    y = ssm(u) * SiLU(z) -> out_proj (expand * C -> C)

Same constructor, parameter names and forward contract as the reference. The projections
and the depthwise convolution are cuDNN / cuBLAS calls; the scan layer (``ssm``) is one
of this package's CUDA layers.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F


class MambaStyleMixer(nn.Module):
    """Shapes: (batch, time, in_features) -> (batch, time, in_features).

    Args:
        in_features: input width.
        ssm: the scan layer, operating on (batch, time, expand * in_features).
        expand: inner width factor. Default 4.
        d_conv: depthwise convolution width along the sequence. Default 4.
        causal_conv: left padding only (position t sees positions <= t). Default True.
    """

    def __init__(self, in_features: int, ssm: nn.Module, expand: int = 4, d_conv: int = 4,
                 causal_conv: bool = True):
        super().__init__()
        inner_dim = expand * in_features
        self.in_features = in_features
        self.inner_dim = inner_dim
        self.d_conv = d_conv
        self.causal_conv = causal_conv
        self.in_proj = nn.Linear(in_features, 2 * inner_dim, bias=False)
        self.conv = nn.Conv1d(inner_dim, inner_dim, kernel_size=d_conv, groups=inner_dim, padding=0)
        self.ssm = ssm
        self.out_proj = nn.Linear(inner_dim, in_features, bias=False)

    def forward(self, x: torch.Tensor, inference_params=None) -> torch.Tensor:
        # ``inference_params`` is accepted for the prenorm Block calling convention; the
        # scan layers have no single-step decoding state here.
        del inference_params
        u, z = self.in_proj(x).chunk(2, dim=-1)
        if self.causal_conv:
            pad = (self.d_conv - 1, 0)
        else:
            left = (self.d_conv - 1) // 2
            pad = (left, self.d_conv - 1 - left)
        u = self.conv(F.pad(u.transpose(1, 2), pad)).transpose(1, 2)
        u = F.silu(u)
        y = self.ssm(u)
        y = y * F.silu(z)
        return self.out_proj(y)
