"""SelectiveLRU (SISO) layer — drop-in for models/selective_lru/selective_lru.py:26-276.

Same constructor, parameter names, registration order, initial values and tags
(``_no_weight_decay`` / ``_no_reinit``), so reference ``state_dict``s load and equal
seeds give equal parameters. Forward contract: (batch, time, d_model) ->
(batch, time, d_model) [+ final state]. The token projection ``x_proj`` is a cuBLAS
GEMM; the two low-rank step projections with the softplus and the rate scale run as one
pass over the (batch, time, d_model) step tensors (``semx_step_proj``, reading dnu_r /
dth_r in place from the x_proj rows); the discretisation, scan, readout, envelope and D
skip run in the fused sm_100a scan (:func:`fused_selective_lru`), whose backward
recomputes states chunk by chunk.

There is one execution path (the CUDA scan). ``use_triton`` is kept for API
compatibility; ``chunk_size`` is the checkpoint interval of the backward recompute
(default 64: memory traffic only, never results); ``block_c`` is accepted and unused.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from .. import _lib
from ..layout import TokenLayout
from .scan import fused_selective_lru

GAINS = ("gamma", "mamba", "zoh")


def _inv_softplus(x: torch.Tensor) -> torch.Tensor:
    """Inverse of softplus for x > 0 (stable form): x + log(-expm1(-x))."""
    return x + torch.log(-torch.expm1(-x))


def _step_projection(lin: nn.Linear, z: torch.Tensor) -> torch.Tensor:
    """``lin(z)`` for a rank-r step projection (r -> d_model) as one fp32 GEMM, with the
    bias as the weight row of an appended column of ones.

    The result is the (batch, time, d_model) fp32 tensor the scan reads. Under bf16
    autocast, ``nn.Linear`` on the non-contiguous split of the x_proj output runs a bf16
    matmul plus a separate bias add, and the scan then casts the result to fp32. Each of
    those passes is a full (batch, time, d_model) read and write. Outside autocast the
    value is the same as ``lin(z)`` up to rounding order.
    """
    shp = z.shape
    with torch.autocast(device_type=z.device.type, enabled=False):
        z2 = z.reshape(-1, shp[-1]).float()
        z1 = torch.cat([z2, z2.new_ones(z2.shape[0], 1)], dim=1)
        w1 = torch.cat([lin.weight.t(), lin.bias.unsqueeze(0)], dim=0).float()
        out = torch.mm(z1, w1)
    return out.reshape(*shp[:-1], lin.out_features)


def _z_rows(z: torch.Tensor) -> tuple[torch.Tensor, int]:
    """z (..., r) as a (rows, r) view and its row stride (a contiguous copy if the leading
    dimensions do not collapse to one stride)."""
    r = z.shape[-1]
    try:
        zz = z.view(-1, r)
    except RuntimeError:
        zz = z.contiguous().view(-1, r)
    if zz.stride(1) != 1:
        zz = zz.contiguous()
    return zz, (zz.stride(0) if zz.shape[0] > 1 else r)


class _StepProjections(torch.autograd.Function):
    """semx_step_proj_fwd / _bwd: (delta_nu, delta_theta) from the dnu_r / dth_r columns of
    the token projection rows (models/selective_lru/selective_lru.py:216-220)."""

    @staticmethod
    def forward(ctx, z_nu, z_th, W_nu, b_nu, W_th, b_th, scale):
        if not z_nu.is_cuda:
            raise RuntimeError("SelectiveLRU step projections require CUDA tensors.")
        if z_nu.dtype not in (torch.float32, torch.bfloat16) or z_th.dtype != z_nu.dtype:
            raise ValueError(f"step projections: unsupported z dtypes {z_nu.dtype}, {z_th.dtype}")
        zn, ldn = _z_rows(z_nu)
        zt, ldt = _z_rows(z_th)
        if ldn != ldt:
            zn, zt = zn.contiguous(), zt.contiguous()
            ldn = zn.shape[1]
        rows, r = zn.shape
        C = W_nu.shape[0]
        Wn, bn = W_nu.detach().float().contiguous(), b_nu.detach().float().contiguous()
        Wt, bt = W_th.detach().float().contiguous(), b_th.detach().float().contiguous()
        dnu = torch.empty((*z_nu.shape[:-1], C), dtype=torch.float32, device=z_nu.device)
        dth = torch.empty_like(dnu)
        a = _lib.new_args(_lib.SemxStepProjArgs)
        a.bf16, a.rank, a.scale = int(zn.dtype == torch.bfloat16), r, float(scale)
        a.rows, a.C, a.ldz = rows, C, ldn
        a.z_nu, a.z_th = zn.data_ptr(), zt.data_ptr()
        a.W_nu, a.b_nu, a.W_th, a.b_th = Wn.data_ptr(), bn.data_ptr(), Wt.data_ptr(), bt.data_ptr()
        a.delta_nu, a.delta_th = dnu.data_ptr(), dth.data_ptr()
        _lib.call("semx_step_proj_fwd", a, z_nu.device)
        ctx.save_for_backward(zn, zt, Wn, bn, Wt, bt)
        ctx.cfg = (float(scale), ldn, z_nu.shape, z_th.shape, W_nu.dtype, b_nu.dtype)
        return dnu, dth

    @staticmethod
    def backward(ctx, g_nu, g_th):
        zn, zt, Wn, bn, Wt, bt = ctx.saved_tensors
        scale, ldz, shape_nu, shape_th, wdt, bdt = ctx.cfg
        rows, r = zn.shape
        C = Wn.shape[0]
        dev = zn.device
        g_nu = None if g_nu is None else g_nu.float().contiguous()
        g_th = None if g_th is None else g_th.float().contiguous()
        dzn = torch.empty((rows, r), dtype=zn.dtype, device=dev)
        dzt = torch.empty_like(dzn)
        dWn, dbn = torch.empty_like(Wn), torch.empty_like(bn)
        dWt, dbt = torch.empty_like(Wt), torch.empty_like(bt)
        a = _lib.new_args(_lib.SemxStepProjArgs)
        a.bf16, a.rank, a.scale = int(zn.dtype == torch.bfloat16), r, scale
        a.rows, a.C, a.ldz = rows, C, ldz
        a.z_nu, a.z_th = zn.data_ptr(), zt.data_ptr()
        a.W_nu, a.b_nu, a.W_th, a.b_th = Wn.data_ptr(), bn.data_ptr(), Wt.data_ptr(), bt.data_ptr()
        a.d_delta_nu, a.d_delta_th = _lib.ptr(g_nu), _lib.ptr(g_th)
        a.dz_nu, a.dz_th = dzn.data_ptr(), dzt.data_ptr()
        a.dW_nu, a.db_nu, a.dW_th, a.db_th = dWn.data_ptr(), dbn.data_ptr(), dWt.data_ptr(), dbt.data_ptr()
        ws = _lib.empty_f32(_lib.load().semx_step_proj_workspace_bytes(a), dev)
        a.workspace = ws.data_ptr()
        _lib.call("semx_step_proj_bwd", a, dev)
        return (dzn.view(shape_nu), dzt.view(shape_th), dWn.to(wdt), dbn.to(bdt), dWt.to(wdt),
                dbt.to(bdt), None)


#: Largest dt_rank the fused step-projection kernels take; wider ranks (d_model > 512)
#: use the GEMM formulation of :func:`_step_projection`.
_MAX_FUSED_RANK = 8


def _phase_grid(n_modes: int, n_real_modes: int, theta_max: float) -> torch.Tensor:
    """``n_real_modes`` zero phases, then oscillators evenly spaced on (0, theta_max]."""
    n_osc = n_modes - n_real_modes
    return torch.cat([
        torch.zeros(n_real_modes),
        torch.linspace(theta_max / max(n_osc, 1), theta_max, n_osc),
    ])


class SelectiveLRU(nn.Module):
    """SISO selective SSM with a bank of complex oscillators per channel.

    Per channel c and mode n, with selective step ``delta_nu > 0`` and detuning
    ``delta_theta`` (per token and channel, shared over modes)::

        lam = exp(delta_nu * (-a + j (omega + [s] delta_theta)))
        Bu  = gain * (B_re + j B_im)_t * x_t,   gain in {gamma, mamba, zoh}
        h_t = lam h_{t-1} + Bu_t
        y_t = Re(<C_t, h_t>) [+ <g, |h_t|^2>] + D x_t
    """

    def __init__(
        self,
        d_model: int,
        d_state: int = 16,
        dt_rank: int | None = None,
        dt_min: float = 1e-3,
        dt_max: float = 0.1,
        theta_max: float = math.pi,
        n_real_modes: int = 0,
        envelope_readout: bool = False,
        mode_detune: bool = False,
        rate_scale: float = 1.0,
        input_gain: str = "gamma",
        use_triton: bool = False,
        chunk_size: int = 16,
        block_c: int = 32,
        device=None,
        dtype=None,
    ):
        super().__init__()
        if not 0 <= n_real_modes <= d_state:
            raise ValueError(f"n_real_modes must be in [0, d_state={d_state}], got {n_real_modes}")
        if input_gain not in GAINS:
            raise ValueError(f"input_gain must be 'gamma', 'mamba', or 'zoh', got {input_gain!r}")
        self.input_gain = input_gain
        self.d_model = d_model
        self.d_state = d_state
        self.n_real_modes = n_real_modes
        self.envelope_readout = envelope_readout
        self.mode_detune = mode_detune
        self.rate_scale = float(rate_scale)
        self.use_triton = use_triton
        self.chunk_size = chunk_size
        self.block_c = block_c
        self.dt_rank = dt_rank if dt_rank is not None else max(1, math.ceil(d_model / 64))
        r, N = self.dt_rank, d_state

        # One fused token projection: [dt_nu (r) | dt_theta (r) | B_re B_im (2N) | C_re C_im (2N)].
        self.x_proj = nn.Linear(d_model, 2 * r + 4 * N, bias=False)
        self.dt_nu_up = nn.Linear(r, d_model, bias=True)
        self.dt_theta_up = nn.Linear(r, d_model, bias=True)

        # S4D-real decays a = 1..N per channel; phases realised at a log-uniform baseline step.
        self.A_log = nn.Parameter(torch.log(torch.arange(1, N + 1, dtype=torch.float32).repeat(d_model, 1)))
        dt = torch.exp(torch.rand(d_model) * (math.log(dt_max) - math.log(dt_min)) + math.log(dt_min))
        self.omega = nn.Parameter(_phase_grid(N, n_real_modes, theta_max).expand(d_model, N) / dt.unsqueeze(-1))
        self.D = nn.Parameter(torch.ones(d_model))

        with torch.no_grad():
            # Low-rank up maps start at zero: delta_theta = 0, delta_nu = softplus(bias) = dt.
            self.dt_nu_up.weight.zero_()
            self.dt_theta_up.weight.zero_()
            self.dt_nu_up.bias.copy_(_inv_softplus(dt))
            self.dt_theta_up.bias.zero_()

        if envelope_readout:
            self.env_gain = nn.Parameter(torch.zeros(d_model, N))
            self.env_gain._no_weight_decay = True
        if mode_detune:
            self.detune_gain = nn.Parameter(torch.ones(d_model, N))
            self.detune_gain._no_weight_decay = True

        self.dt_nu_up.bias._no_reinit = True
        self.dt_theta_up.bias._no_reinit = True
        self.A_log._no_weight_decay = True
        self.omega._no_weight_decay = True
        self.D._no_weight_decay = True

    #: Streaming: when set to a step count K, forward() runs sequences longer than K as
    #: consecutive K-step pieces, each starting from the previous piece's final state (the
    #: h_init / return_final_state path), so the layer's (batch, time, d_model) step
    #: tensors exist for one piece at a time. The result equals the unsplit scan's (the
    #: recurrence is the same; only the projection GEMMs' row blocking changes). None: one
    #: piece. Gradients flow through the carried states.
    stream_chunk: int | None = None

    def accepts_layout(self, layout: TokenLayout) -> bool:
        """Every token layout is read in place, except that a streamed layer (stream_chunk
        set) splits (batch, time, d_model) tensors along time and so takes the default one
        only."""
        return layout.is_default or self.stream_chunk is None

    def forward(self, x: torch.Tensor, h_init: torch.Tensor | None = None,
                rate_scale: float | None = None, return_final_state: bool = False,
                layout: TokenLayout | None = None):
        """``h_init``: optional complex (B, C, N) initial state; ``rate_scale``: per-call
        frame-rate factor on the selective step; ``return_final_state``: also return
        h_{T-1} as complex (B, C, N) (gradients flow through it). ``layout`` (not in the
        reference): x is any tensor of layout.rows token rows, read in that
        :class:`TokenLayout` (reversed, or strided); y has x's shape and row order, and
        the states are (layout.S, C, N)."""
        if layout is not None and not layout.is_default:
            if not self.accepts_layout(layout):
                raise ValueError("a streamed SelectiveLRU (stream_chunk set) reads the default layout only")
            return self._forward_piece(x, h_init, rate_scale, return_final_state, layout)
        K = self.stream_chunk
        if K is not None and x.shape[1] > K:
            h, ys = h_init, []
            for t0 in range(0, x.shape[1], K):
                y, h = self._forward_piece(x[:, t0:t0 + K], h, rate_scale, True)
                ys.append(y)
            y = torch.cat(ys, 1)
            return (y, h) if return_final_state else y
        return self._forward_piece(x, h_init, rate_scale, return_final_state)

    def _forward_piece(self, x, h_init, rate_scale, return_final_state, layout=None):
        r, N = self.dt_rank, self.d_state
        x = x.float()
        dnu_r, dth_r, B_sel, C_sel = torch.split(self.x_proj(x), [r, r, 2 * N, 2 * N], dim=-1)
        rs = self.rate_scale if rate_scale is None else float(rate_scale)
        if r <= _MAX_FUSED_RANK:
            delta_nu, delta_theta = _StepProjections.apply(
                dnu_r, dth_r, self.dt_nu_up.weight, self.dt_nu_up.bias, self.dt_theta_up.weight,
                self.dt_theta_up.bias, rs)
        else:
            delta_nu = F.softplus(_step_projection(self.dt_nu_up, dnu_r))
            if rs != 1.0:
                delta_nu = delta_nu * rs
            delta_theta = _step_projection(self.dt_theta_up, dth_r)
        a = torch.exp(self.A_log)
        g = self.env_gain if self.envelope_readout else None
        s = self.detune_gain if self.mode_detune else None
        h0_re = h_init.real if h_init is not None else None
        h0_im = h_init.imag if h_init is not None else None
        y, hf_re, hf_im = fused_selective_lru(
            delta_nu, delta_theta, a, self.omega,
            B_sel[..., :N], B_sel[..., N:], C_sel[..., :N], C_sel[..., N:],
            x, self.D, g, s, h0_re, h0_im,
            block_t=self.chunk_size, want_final_state=return_final_state,
            input_gain=self.input_gain, layout=layout,
        )
        if return_final_state:
            return y, torch.complex(hf_re, hf_im)
        return y


def _uniform_init(shape, std: float = 1.0) -> torch.Tensor:
    return torch.empty(*shape).uniform_(-std, std)


class SelectiveLRUMIMO(nn.Module):
    """Multi-head selective MIMO SSM (drop-in for
    models/selective_lru/selective_lru.py:279-587).

    One bank of ``state_dim`` complex modes split block-diagonally over ``n_heads`` heads;
    head h owns ``state_dim / n_heads`` modes driven by (and read out to) its
    ``in_features / n_heads`` channels through static complex B / C. Per (token, head):
    selective step ``delta_nu`` and detune ``delta_theta``; poles
    ``exp(delta_nu (-a + j (omega + [s] delta_theta)))``; drive
    ``gain * (B_static x [+ rank-r write])`` with gain in {gamma, mamba, zoh, none};
    readout ``Re(C h) [+ <g, |h|^2>] + D x [+ rank-r read]``.

    Same constructor, parameter names, registration order, initial values and tags as the
    reference. All token projections, the static drive B x included, are one GEMM (its
    weight from :meth:`_projection`); poles, gain, scan, readout, D skip and the rank /
    envelope feedthrough run in the sm_100a layer kernels (:func:`mimo_layer`), one per
    direction.
    """

    def __init__(
        self,
        in_features: int,
        state_dim: int = 16,
        n_heads: int = 1,
        rank: int = 0,
        dt_min: float = 1e-3,
        dt_max: float = 0.1,
        theta_max: float = math.pi,
        n_real_modes: int = 0,
        envelope_readout: bool = False,
        mode_detune: bool = False,
        rate_scale: float = 1.0,
        selective_init_std: float = 1e-2,
        input_gain: str = "gamma",
        normalize_input: bool | None = None,
        use_triton: bool = False,
    ):
        super().__init__()
        if in_features % n_heads != 0:
            raise ValueError(f"in_features={in_features} not divisible by n_heads={n_heads}")
        if state_dim % n_heads != 0:
            raise ValueError(f"state_dim={state_dim} not divisible by n_heads={n_heads}")
        if not 0 <= n_real_modes <= state_dim // n_heads:
            raise ValueError(
                f"n_real_modes must be in [0, state_dim/n_heads={state_dim // n_heads}], "
                f"got {n_real_modes}"
            )
        if input_gain not in ("gamma", "mamba", "zoh", "none"):
            raise ValueError(
                f"input_gain must be 'gamma', 'mamba', 'zoh', or 'none', got {input_gain!r}"
            )
        self.in_features = in_features
        self.state_dim = state_dim
        self.n_heads = n_heads
        self.rank = rank
        self.n_real_modes = n_real_modes
        self.envelope_readout = envelope_readout
        self.mode_detune = mode_detune
        self.rate_scale = float(rate_scale)
        self.input_gain = input_gain
        self.use_triton = use_triton
        self.f_head = in_features // n_heads
        self.n_head = state_dim // n_heads
        H, Nh, Fh = n_heads, self.n_head, self.f_head

        self.dt_nu_proj = nn.Linear(in_features, H, bias=True)
        self.dt_theta_proj = nn.Linear(in_features, H, bias=True)
        self.A_log = nn.Parameter(torch.log(torch.arange(1, Nh + 1, dtype=torch.float32).repeat(H, 1)))
        dt = torch.exp(torch.rand(H) * (math.log(dt_max) - math.log(dt_min)) + math.log(dt_min))
        self.omega = nn.Parameter(_phase_grid(Nh, n_real_modes, theta_max).expand(H, Nh) / dt.unsqueeze(-1))
        self.B = nn.Parameter(_uniform_init((H, Nh, Fh, 2), std=1.0 / math.sqrt(Fh)))
        self.C = nn.Parameter(_uniform_init((H, Fh, Nh, 2), std=1.0 / math.sqrt(Nh)))
        self.D = nn.Parameter(torch.ones(in_features))
        if rank > 0:
            self.b_dir = nn.Linear(in_features, H * rank * Nh, bias=False)
            self.b_coef = nn.Linear(in_features, H * rank, bias=False)
            self.c_read = nn.Linear(in_features, 2 * H * rank * Nh, bias=False)
            self.c_coef = nn.Linear(in_features, H * rank, bias=False)
            # (H * rank, Fh) rather than (H, rank, Fh): unambiguous gradient strides for DDP.
            self.c_out = nn.Parameter(_uniform_init((H * rank, Fh), std=1.0 / math.sqrt(Fh)))

        with torch.no_grad():
            self.dt_nu_proj.weight.zero_()
            self.dt_theta_proj.weight.zero_()
            self.dt_nu_proj.bias.copy_(_inv_softplus(dt))
            self.dt_theta_proj.bias.zero_()
            if rank > 0:
                self.b_dir.weight.normal_(0.0, 1.0 / math.sqrt(in_features))
                self.c_read.weight.normal_(0.0, 1.0 / math.sqrt(in_features))
                coef_std = selective_init_std / math.sqrt(in_features)
                self.b_coef.weight.normal_(0.0, coef_std)
                self.c_coef.weight.normal_(0.0, coef_std)

        if envelope_readout:
            self.env_gain = nn.Parameter(torch.zeros(H, Fh, Nh))
            self.env_gain._no_weight_decay = True
        if mode_detune:
            self.detune_gain = nn.Parameter(torch.ones(H, Nh))
            self.detune_gain._no_weight_decay = True

        self.dt_nu_proj.bias._no_reinit = True
        self.dt_theta_proj.bias._no_reinit = True
        self.A_log._no_weight_decay = True
        self.omega._no_weight_decay = True
        self.D._no_weight_decay = True

    def _projection(self):
        """All token projections as one weight matrix, rows in the order the fused layer
        kernels read them: [dt_nu (H) | dt_theta (H) | b_coef (H r) | b_dir (H r Nh) |
        c_coef (H r) | c_read (2 H r Nh) | static drive B (2 H Nh, block-diagonal)], and
        the dt biases [dt_nu (H) | dt_theta (H)], which the kernels add themselves (the
        other projections have none). The static drive B x is computed (and
        back-propagated) in the projection GEMM, so dB comes from its weight gradient."""
        from .mimo import drive_weight

        ws = [self.dt_nu_proj.weight, self.dt_theta_proj.weight]
        if self.rank > 0:
            ws += [self.b_coef.weight, self.b_dir.weight, self.c_coef.weight, self.c_read.weight]
        ws.append(drive_weight(self.B))
        return torch.cat(ws, 0), torch.cat([self.dt_nu_proj.bias, self.dt_theta_proj.bias])

    def accepts_layout(self, layout: TokenLayout) -> bool:
        """The MIMO layer kernels read (batch, time, in_features) tensors in the default
        sequence-major order only."""
        return layout.is_default

    def forward(self, x: torch.Tensor, rate_scale: float | None = None) -> torch.Tensor:
        """Float32 input runs in float32; bfloat16 input (or float32 input under CUDA bf16
        autocast) runs the projections and the kernel's operand reads in bfloat16 with
        float32 state, accumulation and output."""
        from .mimo import mimo_layer_projected

        bf16 = x.dtype == torch.bfloat16 or (
            x.is_cuda and torch.is_autocast_enabled("cuda")
            and torch.get_autocast_dtype("cuda") == torch.bfloat16)
        W, dt_bias = self._projection()
        with torch.autocast("cuda", enabled=False):
            dt = torch.bfloat16 if bf16 else torch.float32
            rs = self.rate_scale if rate_scale is None else float(rate_scale)
            return mimo_layer_projected(
                x.to(dt), W.to(dt), dt_bias, self.A_log, self.omega,
                self.detune_gain if self.mode_detune else None,
                self.C, self.D, self.c_out if self.rank > 0 else None,
                self.env_gain if self.envelope_readout else None, self.n_heads, self.n_head,
                self.f_head, self.rank, self.input_gain, rs)
