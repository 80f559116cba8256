"""LinOSS layer (drop-in for models/linoss/linoss.py of the reference).

Same constructor, parameter names, registration order and initial values (so reference
``state_dict``s load and equal seeds give equal parameters), same forward contract
(batch, time, in_features) -> (batch, time, in_features). The computation is arranged
for the GPU:

* ``Bu = B x`` is one real GEMM producing the interleaved complex64 tensor directly;
* the constraints, discretisation and recurrence run in one fused sm_100a scan
  (:func:`linoss_scan_fused`), whose backward recomputes states instead of storing them;
* the readout ``Re(C y2) + D x`` is one fused pass over the token rows
  (``semx_linoss_readout``, P <= 32 oscillators): forward y, backward dx, dC and dD, with
  the state gradient dy2 = dy conj(C) as one GEMM; wider states use a real GEMM plus the
  skip term.

There is one execution path: the CUDA scan. ``use_triton`` is accepted for API
compatibility; CPU tensors raise like the reference's GPU operator does.
"""
from __future__ import annotations

import math
from typing import Literal

import torch
import torch.nn as nn

from .. import _lib
from ..layout import TokenLayout
from .scan import DEFAULT_CHUNK, linoss_scan_fused

#: Largest state the fused readout kernels take (C[h, :] lives in one thread's registers).
_MAX_FUSED_P = 32


def _uniform_init(shape, std: float = 1.0) -> torch.Tensor:
    return torch.empty(*shape).uniform_(-std, std)


def _map_theta_to_A(thetas: torch.Tensor, G_diag: torch.Tensor, steps: torch.Tensor):
    """Closed-form A giving eigenvalue phase ``thetas`` for damping G and step
    (models/linoss/linoss.py:133-145): the root of the damped-IMEX characteristic
    polynomial on the branch that matches the phase quadrant."""
    sec2 = 1.0 / torch.cos(thetas) ** 2
    tan2 = torch.tan(thetas) ** 2
    root = torch.sqrt(steps**4 * sec2 + steps**5 * G_diag * sec2)
    common = steps**2 * (4.0 + 2.0 * steps * G_diag + 4.0 * tan2 + 2.0 * steps * G_diag * tan2)
    denom = 2.0 * steps**4 * (1.0 + tan2)
    return torch.where(thetas > math.pi / 2, (4.0 * root + common) / denom,
                       (common - 4.0 * root) / denom)


def _project_input(B_param: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """Bu = B x, B complex (P, H) stored as (P, H, 2); returns (..., P) complex64.

    One GEMM against the (2P, H) real matrix whose rows are (p, re/im), so the result
    is already the interleaved complex layout."""
    P, H, _ = B_param.shape
    W = B_param.permute(0, 2, 1).reshape(2 * P, H)
    out = torch.matmul(x, W.t()).float()  # fp32 even when autocast ran the GEMM in bf16
    return torch.view_as_complex(out.view(*out.shape[:-1], P, 2))


def _readout(C_param: torch.Tensor, y2: torch.Tensor) -> torch.Tensor:
    """Re(C y2) for C complex (H, P) stored as (H, P, 2): one GEMM with rows
    (C_re[h, p], -C_im[h, p]) against y2 viewed as interleaved reals."""
    H, P, _ = C_param.shape
    W = torch.stack((C_param[..., 0], -C_param[..., 1]), dim=-1).reshape(H, 2 * P)
    y2r = torch.view_as_real(y2).reshape(*y2.shape[:-1], 2 * P)
    return torch.matmul(y2r, W.t())


class _Readout(torch.autograd.Function):
    """semx_linoss_readout_fwd / _bwd: y = Re(C y2) + D x (models/linoss/linoss.py:118-120)
    for y2 (..., P) complex64, x (..., H) fp32, C (H, P, 2), D (H)."""

    @staticmethod
    def forward(ctx, y2, x, C, D):
        H, P, _ = C.shape
        y2c = y2.contiguous()
        xc = x.contiguous()
        Cf, Df = C.detach().float().contiguous(), D.detach().float().contiguous()
        y = torch.empty(xc.shape, dtype=torch.float32, device=x.device)
        a = _lib.new_args(_lib.SemxLinossReadoutArgs)
        a.rows, a.H, a.P = xc.numel() // H, H, P
        a.x, a.y2, a.C, a.D, a.y = xc.data_ptr(), y2c.data_ptr(), Cf.data_ptr(), Df.data_ptr(), y.data_ptr()
        _lib.call("semx_linoss_readout_fwd", a, x.device)
        ctx.save_for_backward(y2c, xc, Cf, Df)
        ctx.dtypes = (C.dtype, D.dtype)
        return y

    @staticmethod
    def backward(ctx, dy):
        y2, x, Cf, Df = ctx.saved_tensors
        H, P, _ = Cf.shape
        dy = dy.float().contiguous()
        dx = torch.empty_like(x)
        dC, dD = torch.empty_like(Cf), torch.empty_like(Df)
        a = _lib.new_args(_lib.SemxLinossReadoutArgs)
        a.rows, a.H, a.P = x.numel() // H, H, P
        a.x, a.y2, a.C, a.D = x.data_ptr(), y2.data_ptr(), Cf.data_ptr(), Df.data_ptr()
        a.dy, a.dx, a.dC, a.dD = dy.data_ptr(), dx.data_ptr(), dC.data_ptr(), dD.data_ptr()
        ws = _lib.empty_f32(_lib.load().semx_linoss_readout_workspace_bytes(a), x.device)
        a.workspace = ws.data_ptr()
        _lib.call("semx_linoss_readout_bwd", a, x.device)
        # dy2[p] = sum_h dy[h] conj(C[h, p]): one GEMM against [C_re | -C_im] as (re, im) pairs.
        W = torch.stack((Cf[..., 0], -Cf[..., 1]), dim=-1).reshape(H, 2 * P)
        dy2 = torch.view_as_complex(torch.mm(dy.view(-1, H), W).view(*y2.shape, 2))
        return dy2, dx, dC.to(ctx.dtypes[0]), dD.to(ctx.dtypes[1])


class LinOSS(nn.Module):
    """LinOSS sequence mixer (LinOSS-IM, LinOSS-IMEX, damped LinOSS-IMEX).

    Shapes:
        Input:  (batch, time, in_features)
        Output: (batch, time, in_features)

    ``chunk_size`` (not in the reference) sets the backward recompute block; it changes
    memory traffic only, never results.
    """

    def __init__(
        self,
        in_features: int,
        state_dim: int = 64,
        discretization: Literal["IM", "IMEX"] = "IMEX",
        damping: bool = True,
        r_min: float = 0.9,
        theta_max: float = math.pi,
        use_triton: bool = False,
        a_from_g: bool = True,
        chunk_size: int = DEFAULT_CHUNK,
    ):
        super().__init__()
        if discretization == "IM" and damping:
            raise NotImplementedError("Discretization=IM with damping=True is not implemented.")
        if discretization not in ("IM", "IMEX"):
            raise NotImplementedError(f"Discretization {discretization} not implemented")
        self.in_features = in_features
        self.state_dim = state_dim
        self.discretization = discretization
        self.damping = damping
        self.A_from_G = a_from_g
        self.use_triton = use_triton
        self.chunk_size = chunk_size

        self.steps = nn.Parameter(torch.randn(state_dim) * 0.5)
        with torch.no_grad():
            step0 = torch.sigmoid(self.steps)
        if discretization == "IMEX" and damping:
            # Eigenvalue radius uniform in area on [r_min, 1), phase uniform on [0, theta_max).
            r_max = 1.0
            radius = torch.sqrt(torch.rand(state_dim) * (r_max**2 - r_min**2) + r_min**2)
            G0 = (1.0 - radius**2) / (step0 * radius**2)
            self.G_diag = nn.Parameter(G0)
            phase = torch.rand(state_dim) * theta_max
            self.A_diag = nn.Parameter(_map_theta_to_A(phase, torch.relu(G0), step0))
        else:
            self.register_parameter("G_diag", None)
            self.A_diag = nn.Parameter(torch.rand(state_dim))
        self.B = nn.Parameter(_uniform_init((state_dim, in_features, 2), 1.0 / math.sqrt(in_features)))
        self.C = nn.Parameter(_uniform_init((in_features, state_dim, 2), 1.0 / math.sqrt(state_dim)))
        self.D = nn.Parameter(torch.randn(in_features))

    @property
    def variant(self) -> str:
        if self.discretization == "IM":
            return "IM"
        return "DAMPED_IMEX" if self.damping else "IMEX"

    def accepts_layout(self, layout: TokenLayout) -> bool:
        """Sequence-major token rows, in either step order (the scan kernels run a chain
        forwards or backwards through its rows)."""
        return layout.is_contiguous

    def forward(self, x: torch.Tensor, layout: TokenLayout | None = None) -> torch.Tensor:
        """``layout`` (not in the reference): x holds layout.rows sequence-major token rows,
        scanned last step first when layout.reverse (the result is flip(layer(flip(x)))
        along time, without the flips)."""
        lead = x.shape[:-1]
        reverse = False
        if layout is not None:
            if not layout.is_contiguous:
                raise ValueError(f"LinOSS reads sequence-major token rows only, got {layout}")
            x3 = x.reshape(layout.S, layout.L, x.shape[-1])
            reverse = layout.reverse
        else:
            x3 = x.reshape(-1, *x.shape[-2:]) if x.dim() != 3 else x
        Bu = _project_input(self.B.float(), x3.float())
        y2 = linoss_scan_fused(
            self.variant, self.steps, self.A_diag, self.G_diag, Bu,
            a_from_g=self.A_from_G, chunk=self.chunk_size, reverse=reverse,
        )
        if self.state_dim <= _MAX_FUSED_P:
            y = _Readout.apply(y2, x3.float(), self.C, self.D)
        else:
            y = _readout(self.C.float(), y2) + x3 * self.D
        return y.reshape(*lead, -1) if x.dim() != 3 else y
