"""Mamba-style mixer around a scan layer (drop-in for the reference's models/mixer.py:31-99).

    in_proj (C -> 2 * expand * C) -> split (u, z)
    u: causal depthwise Conv1d (kernel d_conv) -> SiLU -> ssm
    y = ssm(u) * SiLU(z) -> out_proj (expand * C -> C)

Same constructor, parameter names and forward contract as the reference. The projections
are cuBLAS GEMMs; the convolution + SiLU and the SiLU gate are this package's
channels-last kernels (``semx_conv_silu``, ``semx_gate_silu``), which read u and z in
place from the in_proj output, so the transposes, padding and split copies of the
reference formulation never materialise; the scan layer (``ssm``) is one of this
package's CUDA layers.

``forward(x, layout=...)`` (not in the reference) runs the mixer on token rows in any
:class:`~semambaxlinoss_b200.layout.TokenLayout` its scan layer accepts: the projections
and the gate are per-token, and the convolution and the scan read the layout in place.
A reversed layout gives ``flip(mixer(flip(x)))`` without the flips.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import _lib
from .layout import TokenLayout, check_rows


class _DxzLink:
    """Gradient buffer of the in_proj output shared by the gate and the convolution of one
    forward call: the gate's backward (which always runs first, since the convolution's
    output gradient flows back through the scan from the gate) writes dz into columns
    [C, 2C); the convolution's backward writes du into columns [0, C) and returns it."""

    __slots__ = ("dxz",)

    def __init__(self):
        self.dxz = None


def _check_xz(xz):
    if not xz.is_cuda:
        raise RuntimeError("MambaStyleMixer requires CUDA tensors.")
    if xz.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError(f"MambaStyleMixer: unsupported dtype {xz.dtype}")


class _ConvSiLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, xz, weight, bias, C, K, left, link, layout):
        check_rows("conv_silu xz", xz, layout)
        w = weight.detach().reshape(C, K).float().contiguous()
        b = None if bias is None else bias.detach().float().contiguous()
        v = torch.empty((*xz.shape[:-1], C), dtype=torch.float32, device=xz.device)
        a = _lib.new_args(_lib.SemxConvSiluArgs)
        a.K, a.left, a.bf16 = K, left, int(xz.dtype == torch.bfloat16)
        a.S, a.L, a.C, a.ld = layout.S, layout.L, C, xz.shape[-1]
        _lib.set_layout(a, layout)
        a.xz, a.w, a.b, a.v = xz.data_ptr(), w.data_ptr(), _lib.ptr(b), v.data_ptr()
        _lib.call("semx_conv_silu_fwd", a, xz.device)
        ctx.save_for_backward(xz, w, b if b is not None else w.new_empty(0))
        ctx.cfg = (C, K, left, bias is not None, weight.shape, link, layout)
        return v

    @staticmethod
    def backward(ctx, dv):
        xz, w, b = ctx.saved_tensors
        C, K, left, has_bias, wshape, link, layout = ctx.cfg
        ld = xz.shape[-1]
        dxz = link.dxz
        if dxz is None:  # no gradient reached the gate: the z half is zero
            dxz = torch.zeros_like(xz)
        link.dxz = None
        dv = dv.float().contiguous()
        dw = torch.empty((C, K), dtype=torch.float32, device=xz.device)
        db = torch.empty(C, dtype=torch.float32, device=xz.device) if has_bias else None
        a = _lib.new_args(_lib.SemxConvSiluArgs)
        a.K, a.left, a.bf16 = K, left, int(xz.dtype == torch.bfloat16)
        a.S, a.L, a.C, a.ld = layout.S, layout.L, C, ld
        _lib.set_layout(a, layout)
        a.xz, a.w, a.b = xz.data_ptr(), w.data_ptr(), (b.data_ptr() if has_bias else None)
        a.dv, a.dxz, a.dw, a.db = dv.data_ptr(), dxz.data_ptr(), dw.data_ptr(), _lib.ptr(db)
        ws = _lib.empty_f32(_lib.load().semx_conv_silu_workspace_bytes(a), xz.device)
        a.workspace = ws.data_ptr()
        _lib.call("semx_conv_silu_bwd", a, xz.device)
        return dxz, dw.reshape(wshape), db, None, None, None, None, None


class _GateSiLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, xz, C, link):
        ld = xz.shape[-1]
        y = y.float().contiguous()
        o = torch.empty((*xz.shape[:-1], C), dtype=xz.dtype, device=xz.device)
        a = _lib.new_args(_lib.SemxGateSiluArgs)
        a.bf16 = int(xz.dtype == torch.bfloat16)
        a.n, a.C, a.ld = xz.numel() // ld, C, ld
        a.y, a.xz, a.o = y.data_ptr(), xz.data_ptr(), o.data_ptr()
        _lib.call("semx_gate_silu_fwd", a, xz.device)
        ctx.save_for_backward(y, xz)
        ctx.cfg = (C, link)
        return o

    @staticmethod
    def backward(ctx, do):
        y, xz = ctx.saved_tensors
        C, link = ctx.cfg
        ld = xz.shape[-1]
        do = do.to(xz.dtype).contiguous()
        dy = torch.empty_like(y)
        dxz = torch.empty_like(xz)  # columns [0, C) are written by the convolution's backward
        a = _lib.new_args(_lib.SemxGateSiluArgs)
        a.bf16 = int(xz.dtype == torch.bfloat16)
        a.n, a.C, a.ld = xz.numel() // ld, C, ld
        a.y, a.xz, a.dout, a.dy, a.dxz = y.data_ptr(), xz.data_ptr(), do.data_ptr(), dy.data_ptr(), dxz.data_ptr()
        _lib.call("semx_gate_silu_bwd", a, xz.device)
        link.dxz = dxz
        return dy, None, None, None


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

    def accepts_layout(self, layout: TokenLayout) -> bool:
        """Whether forward(x, layout=layout) runs without copies: the convolution reads
        any layout, so this is whether the scan layer reads it."""
        if layout.is_default:
            return True
        ok = getattr(self.ssm, "accepts_layout", None)
        return bool(ok is not None and ok(layout))

    def forward(self, x: torch.Tensor, inference_params=None,
                layout: TokenLayout | None = None) -> torch.Tensor:
        # ``inference_params`` is accepted for the prenorm Block calling convention; the
        # scan layers have no single-step decoding state here.
        del inference_params
        xz = self.in_proj(x)
        _check_xz(xz)
        xz = xz.contiguous()
        if layout is None:
            if xz.dim() != 3:
                raise ValueError(f"MambaStyleMixer expects (batch, time, features), got {tuple(x.shape)}")
            layout = TokenLayout.contiguous(xz.shape[0], xz.shape[1])
        elif not self.accepts_layout(layout):
            raise ValueError(f"{type(self.ssm).__name__} does not read the token layout {layout}")
        left = self.d_conv - 1 if self.causal_conv else (self.d_conv - 1) // 2
        link = _DxzLink()
        u = _ConvSiLU.apply(xz, self.conv.weight, self.conv.bias, self.inner_dim, self.d_conv, left, link,
                            layout)
        if layout.is_default:  # any scan layer: (S, L, width) sequences
            y = self.ssm(u.view(layout.S, layout.L, -1)).reshape(u.shape)
        else:
            y = self.ssm(u, layout=layout)
        return self.out_proj(_GateSiLU.apply(y, xz, self.inner_dim, link))
