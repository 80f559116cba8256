"""TF-block plumbing around the scan layers (drop-in for the reference's
models/mamba_block.py: HybridBlock 41-102, _build_mixer_cls 105-299, create_block 303-344,
MambaBlock 347-396, TFMambaBlock 420-508).

The reference builds its blocks from the third-party ``mamba_ssm`` package (``Block``,
``RMSNorm``, ``_init_weights``, ``layer_norm_fn``), which is not part of the reference
checkout. Their documented behaviour is restated here:

* ``RMSNorm(d, eps)``: y = x / sqrt(mean(x^2) + eps) * weight (weight initialised to 1,
  no bias).
* ``Block(dim, mixer_cls, mlp_cls=nn.Identity, norm_cls, ...)``, the pre-norm residual
  block: ``residual = x + residual`` (or ``x`` when no residual is given),
  ``h = mixer(norm(residual))``; returns ``(h, residual)``; the caller adds the final
  residual.
* ``_init_weights(module, n_layer)``: zero every Linear bias not tagged ``_no_reinit``;
  re-draw every ``out_proj.weight`` / ``fc2.weight`` Kaiming-uniform (a = sqrt(5)) and
  divide it by sqrt(n_layer).

Token layouts (:mod:`semambaxlinoss_b200.layout`): a TF-block keeps its activations as
one (batch, frames, bins, channels) tensor. The frequency-axis scans read it as
contiguous sequences and the time-axis scans read it through a strided row grid, and
the backward branch of a bi-directional block runs its convolution and scan in reverse
step order over the same rows. This replaces the reference's ``torch.flip`` pair and
its permute + contiguous copies (models/mamba_block.py:387-396, 496-507) with reads in
place. A scan layer that cannot read a layout (the MIMO layer; a streamed
SelectiveLRU for strided layouts) falls back to the reference's copies.

Supported mixers: ``selective_lru``, ``selective_lru_mimo``, ``linoss`` (the layers on
this package's scan path). The reference's other backbones (``mamba``, ``mamba2``,
``mamba3`` from mamba_ssm, ``s4d``, ``s5``, and ``selective_linoss``, whose source the
reference does not contain) raise NotImplementedError.
"""
from __future__ import annotations

import math
from functools import partial
from typing import Literal

import torch
from torch import nn
import torch.nn.functional as F

from . import _lib
from .layout import TokenLayout
from .linoss import LinOSS
from .mixer import MambaStyleMixer
from .selective_lru import SelectiveLRU, SelectiveLRUMIMO


class _RmsNorm(torch.autograd.Function):
    """semx_rms_norm_fwd / _bwd: one kernel per direction (fp32 arithmetic, output in the
    input's dtype, fp32 or bf16)."""

    @staticmethod
    def forward(ctx, x, weight, eps):
        if not x.is_cuda:
            raise RuntimeError("RMSNorm requires CUDA tensors.")
        if x.dtype not in (torch.float32, torch.bfloat16):
            raise ValueError(f"RMSNorm: unsupported dtype {x.dtype}")
        shape = x.shape
        x2 = x.contiguous().view(-1, shape[-1])
        w = weight.detach().float().contiguous()
        y = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
        a = _lib.new_args(_lib.SemxRmsNormArgs)
        a.bf16, a.eps, a.n, a.d = int(x.dtype == torch.bfloat16), float(eps), x2.shape[0], x2.shape[1]
        a.x, a.weight, a.y, a.rstd = x2.data_ptr(), w.data_ptr(), y.data_ptr(), rstd.data_ptr()
        _lib.call("semx_rms_norm_fwd", a, x.device)
        ctx.save_for_backward(x2, w, rstd)
        ctx.meta = (shape, float(eps), weight.dtype)
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w, rstd = ctx.saved_tensors
        shape, eps, wdtype = ctx.meta
        dy2 = dy.to(x2.dtype).contiguous().view(-1, shape[-1])
        dx = torch.empty_like(x2)
        dw = torch.empty_like(w)
        a = _lib.new_args(_lib.SemxRmsNormArgs)
        a.bf16, a.eps, a.n, a.d = int(x2.dtype == torch.bfloat16), eps, x2.shape[0], x2.shape[1]
        a.x, a.weight, a.rstd = x2.data_ptr(), w.data_ptr(), rstd.data_ptr()
        a.dy, a.dx, a.dweight = dy2.data_ptr(), dx.data_ptr(), dw.data_ptr()
        ws = _lib.empty_f32(_lib.load().semx_rms_norm_workspace_bytes(a), x2.device)
        a.workspace = ws.data_ptr()
        _lib.call("semx_rms_norm_bwd", a, x2.device)
        return dx.view(shape), dw.to(wdtype), None


class RMSNorm(nn.Module):
    """Root-mean-square normalisation over the last dimension with a learned gain:
    y = x / sqrt(mean(x^2) + eps) * weight, in fp32, returned in x's dtype. Runs the
    semx_rms_norm kernels (CUDA tensors only)."""

    def __init__(self, hidden_size: int, eps: float = 1e-5, device=None, dtype=None):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size, device=device, dtype=dtype))
        self.register_parameter("bias", None)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return _RmsNorm.apply(x, self.weight, self.eps)


class Block(nn.Module):
    """Pre-norm residual block: returns (mixer(norm(x + residual)), x + residual)."""

    def __init__(self, dim, mixer_cls, mlp_cls=nn.Identity, norm_cls=nn.LayerNorm,
                 fused_add_norm=False, residual_in_fp32=False):
        super().__init__()
        self.residual_in_fp32 = residual_in_fp32
        self.fused_add_norm = fused_add_norm
        self.norm = norm_cls(dim)
        self.mixer = mixer_cls(dim)
        if mlp_cls is not nn.Identity:
            self.norm2 = norm_cls(dim)
            self.mlp = mlp_cls(dim)
        else:
            self.mlp = None

    def forward(self, hidden_states, residual=None, inference_params=None, **mixer_kwargs):
        residual = hidden_states + residual if residual is not None else hidden_states
        hidden_states = self.norm(residual.to(dtype=self.norm.weight.dtype))
        if self.residual_in_fp32:
            residual = residual.to(torch.float32)
        hidden_states = self.mixer(hidden_states, inference_params=inference_params, **mixer_kwargs)
        if self.mlp is not None:
            residual = hidden_states + residual
            hidden_states = self.mlp(self.norm2(residual.to(dtype=self.norm2.weight.dtype)))
        return hidden_states, residual


def _init_weights(module, n_layer, initializer_range=0.02, rescale_prenorm_residual=True,
                  n_residuals_per_layer=1):
    if isinstance(module, nn.Linear):
        if module.bias is not None and not getattr(module.bias, "_no_reinit", False):
            nn.init.zeros_(module.bias)
    elif isinstance(module, nn.Embedding):
        nn.init.normal_(module.weight, std=initializer_range)
    if rescale_prenorm_residual:
        for name, p in module.named_parameters():
            if name in ("out_proj.weight", "fc2.weight"):
                nn.init.kaiming_uniform_(p, a=math.sqrt(5))
                with torch.no_grad():
                    p /= math.sqrt(n_residuals_per_layer * n_layer)


def _apply_layer_norm(x, residual, norm_layer):
    """Pre-norm add + norm: returns (norm(x + residual), x + residual)."""
    residual = x + residual if residual is not None else x
    return norm_layer(residual), residual


class HybridBlock(nn.Module):
    """Two backbones in one block: 'sequential' (norm -> b1 -> norm -> b2, residual
    threaded through) or 'parallel' (sigmoid-gated mix of b1 and b2 on the same input)."""

    def __init__(self, dim, backbone_1, backbone_2, mode: Literal["sequential", "parallel"] = "sequential",
                 gate_hidden=None, norm_cls=None):
        super().__init__()
        self.backbone_1 = backbone_1
        self.backbone_2 = backbone_2
        self.mode = mode
        norm_cls = norm_cls if norm_cls is not None else partial(nn.LayerNorm, eps=1e-5)
        self.norm1 = norm_cls(dim)
        self.norm2 = norm_cls(dim) if mode == "sequential" else None
        if mode == "parallel":
            if gate_hidden is None:
                self.gate = nn.Linear(2 * dim, dim)
            else:
                self.gate = nn.Sequential(nn.Linear(2 * dim, gate_hidden), nn.SiLU(), nn.Linear(gate_hidden, dim))

    def accepts_layout(self, layout: TokenLayout) -> bool:
        return all(_accepts(b, layout) for b in (self.backbone_1, self.backbone_2))

    def forward(self, x, residual=None, layout: TokenLayout | None = None):
        kw = {} if layout is None else {"layout": layout}
        if self.mode == "sequential":
            x, residual = _apply_layer_norm(x, residual, self.norm1)
            x = self.backbone_1(x, **kw)
            x, residual = _apply_layer_norm(x, residual, self.norm2)
            x = self.backbone_2(x, **kw)
        elif self.mode == "parallel":
            x, residual = _apply_layer_norm(x, residual, self.norm1)
            x1 = self.backbone_1(x, **kw)
            x2 = self.backbone_2(x, **kw)
            g = torch.sigmoid(self.gate(torch.cat([x1, x2], dim=-1)))
            x = g * x1 + (1.0 - g) * x2
        else:
            raise ValueError(f"Unknown mode {self.mode}. Has to be either 'sequential' or 'parallel'.")
        return x, residual


def _accepts(module, layout: TokenLayout) -> bool:
    """Whether ``module`` (a mixer, a pre-norm Block or a HybridBlock) reads ``layout``
    in place."""
    if isinstance(module, Block):
        module = module.mixer
    ok = getattr(module, "accepts_layout", None)
    return layout.is_default or bool(ok is not None and ok(layout))


_OUT_OF_SCOPE = ("mamba", "mamba2", "mamba3", "selective_linoss", "s4d", "s5")


def _build_mixer_cls(d_model, model_cfg, layer_idx=0):
    """``mixer_cls(d_model)`` partial for one backbone, read from ``model_cfg`` (keys
    ``ssm``, ``d_state``, ``d_conv``, ``expand``, ``ssm_params``, ``causal_conv``)."""
    ssm = model_cfg["ssm"]
    ssm_params = model_cfg.get("ssm_params", {}) or {}
    d_state, d_conv, expand = model_cfg["d_state"], model_cfg["d_conv"], model_cfg["expand"]
    causal = model_cfg.get("causal_conv", True)
    if ssm == "linoss":
        layer = LinOSS(
            in_features=expand * d_model,
            state_dim=d_state,
            discretization=ssm_params.get("discretization", "IMEX"),
            damping=ssm_params.get("damping", True),
            r_min=ssm_params.get("r_min", 0.9),
            theta_max=ssm_params.get("theta_max", math.pi),
            a_from_g=ssm_params.get("a_from_g", True),
            use_triton=ssm_params.get("use_triton", False),
            chunk_size=ssm_params.get("linoss_chunk", 64),
        )
    elif ssm == "selective_lru_mimo":
        layer = SelectiveLRUMIMO(in_features=expand * d_model, state_dim=d_state, **ssm_params)
    elif ssm == "selective_lru":
        layer = SelectiveLRU(
            d_model=expand * d_model,
            d_state=d_state,
            dt_rank=ssm_params.get("dt_rank", None),
            dt_min=ssm_params.get("dt_min", 1e-3),
            dt_max=ssm_params.get("dt_max", 0.1),
            theta_max=ssm_params.get("theta_max", math.pi),
            n_real_modes=ssm_params.get("n_real_modes", 0),
            envelope_readout=ssm_params.get("envelope_readout", False),
            mode_detune=ssm_params.get("mode_detune", False),
            rate_scale=ssm_params.get("rate_scale", 1.0),
            input_gain=ssm_params.get("input_gain", "gamma"),
            use_triton=ssm_params.get("use_triton", False),
            chunk_size=ssm_params.get("chunk_size", 16),
            block_c=ssm_params.get("block_c", 32),
        )
    elif ssm in _OUT_OF_SCOPE:
        raise NotImplementedError(
            f"mixer {ssm!r} is not part of this package (only the selective-LRU and LinOSS "
            "scan layers are)"
        )
    else:
        raise ValueError(
            f"Unknown mixer {ssm!r}; expected 'mamba', 'mamba2', 'mamba3', "
            "'linoss', 'selective_lru', 'selective_lru_mimo', 's4d', or 's5'."
        )
    return partial(MambaStyleMixer, ssm=layer, expand=expand, d_conv=d_conv, causal_conv=causal)


def create_block(d_model, model_cfg, layer_idx=0, rms_norm=True, fused_add_norm=False,
                 residual_in_fp32=False):
    norm_eps = model_cfg.get("norm_epsilon", 1e-5)
    norm_cls = partial(nn.LayerNorm if not rms_norm else RMSNorm, eps=norm_eps)
    if model_cfg["ssm"] == "hybrid":
        hybrid_cfg = model_cfg.get("hybrid", {})
        b1 = _build_mixer_cls(d_model, model_cfg["backbone_1"], layer_idx)(d_model)
        b2 = _build_mixer_cls(d_model, model_cfg["backbone_2"], layer_idx)(d_model)
        block = HybridBlock(dim=d_model, backbone_1=b1, backbone_2=b2,
                            mode=hybrid_cfg.get("mode", "sequential"),
                            gate_hidden=hybrid_cfg.get("gate_hidden", None), norm_cls=norm_cls)
        block.layer_idx = layer_idx
        return block
    mixer_cls = _build_mixer_cls(d_model, model_cfg, layer_idx)
    block = Block(d_model, mixer_cls, nn.Identity, norm_cls=norm_cls,
                  fused_add_norm=fused_add_norm, residual_in_fp32=residual_in_fp32)
    block.layer_idx = layer_idx
    return block


class MambaBlock(nn.Module):
    """Bi- or uni-directional scan block over (batch, length, channels).

    ``cfg["bidirectional"]`` (default True): output is the concat of the forward pass and
    the time-reversed backward pass (2 * channels); unidirectional output keeps channels.
    """

    def __init__(self, in_channels, cfg):
        super().__init__()
        n_layer = 1
        self.bidirectional = cfg.get("bidirectional", True)
        self.forward_blocks = nn.ModuleList(create_block(in_channels, cfg) for _ in range(n_layer))
        if self.bidirectional:
            self.backward_blocks = nn.ModuleList(create_block(in_channels, cfg) for _ in range(n_layer))
        self.apply(partial(_init_weights, n_layer=n_layer))

    def accepts_layout(self, layout: TokenLayout) -> bool:
        """Whether forward(x, layout=layout) reads x in place: the forward blocks take
        the layout and the backward blocks its reverse."""
        if not all(_accepts(b, layout) for b in self.forward_blocks):
            return False
        return not self.bidirectional or all(_accepts(b, layout.flipped()) for b in self.backward_blocks)

    def forward(self, x, layout: TokenLayout | None = None):
        """x: (batch, length, channels), or with ``layout`` (not in the reference) any
        tensor of layout.rows token rows. The backward branch runs its blocks on the
        reversed layout of the same rows when they accept it, which equals the flip /
        blocks / flip of the reference without the copies; otherwise (default layout
        only) it flips."""
        if layout is None:
            layout = TokenLayout.contiguous(x.shape[0], x.shape[1])
        kw = {} if layout.is_default else {"layout": layout}
        xf, rf = x, None
        for layer in self.forward_blocks:
            xf, rf = layer(xf, rf, **kw)
        y_forward = xf + rf if rf is not None else xf
        if not self.bidirectional:
            return y_forward
        back = layout.flipped()
        if all(_accepts(b, back) for b in self.backward_blocks):
            xb, rb = x, None
            for layer in self.backward_blocks:
                xb, rb = layer(xb, rb, layout=back)
            y_backward = xb + rb if rb is not None else xb
        else:
            if not layout.is_default:
                raise ValueError(f"the backward blocks read neither {back} nor flipped copies of it")
            xb, rb = torch.flip(x, [1]), None
            for layer in self.backward_blocks:
                xb, rb = layer(xb, rb)
            y_backward = torch.flip(xb + rb, [1]) if rb is not None else torch.flip(xb, [1])
        return torch.cat([y_forward, y_backward], -1)


def _layer_spec_matches(spec, layer_idx, num_layers):
    """``layers`` override spec: ints (negative from the end) or inclusive 'a-b' ranges."""
    for item in spec:
        if isinstance(item, str) and "-" in item.strip().lstrip("-"):
            lo, hi = item.split("-")
            if int(lo) <= layer_idx <= int(hi):
                return True
        else:
            idx = int(item)
            if idx < 0:
                idx += num_layers
            if idx == layer_idx:
                return True
    return False


def _pointwise_transpose(conv: nn.ConvTranspose1d, y: torch.Tensor) -> torch.Tensor:
    """``conv(y.permute(0, 2, 1)).permute(0, 2, 1)`` for a kernel-1, stride-1
    ConvTranspose1d, evaluated channels-last: out = y W[:, :, 0] + b, one GEMM on the
    (N, L, C_in) rows with no layout conversion or transposed copies."""
    assert conv.kernel_size == (1,) and conv.stride == (1,) and conv.groups == 1
    return F.linear(y, conv.weight[:, :, 0].t(), conv.bias)


class TFMambaBlock(nn.Module):
    """Time-frequency block: a MambaBlock along time over (B*F) sequences, then along
    frequency over (B*T) sequences, each followed by a channel projection and a residual.
    Input / output: (batch, channels, time, freq)."""

    def __init__(self, cfg, layer_idx=0, num_layers=1):
        super().__init__()
        self.cfg = cfg
        self.layer_idx = layer_idx
        self.hid_feature = cfg["model_cfg"]["hid_feature"]
        mcfg = cfg["model_cfg"]
        time_cfg = mcfg.get("time_mixer", mcfg)
        freq_cfg = mcfg.get("freq_mixer", mcfg)
        for override in mcfg.get("layer_overrides") or []:
            if _layer_spec_matches(override.get("layers", []), layer_idx, num_layers):
                time_cfg = override.get("time_mixer", time_cfg)
                freq_cfg = override.get("freq_mixer", freq_cfg)
        self.time_mamba = MambaBlock(in_channels=self.hid_feature, cfg=time_cfg)
        self.freq_mamba = MambaBlock(in_channels=self.hid_feature, cfg=freq_cfg)
        t_width = self.hid_feature * (2 if self.time_mamba.bidirectional else 1)
        f_width = self.hid_feature * (2 if self.freq_mamba.bidirectional else 1)
        self.use_transpose = mcfg.get("use_transpose", True)
        if self.use_transpose:
            self.tlinear = nn.ConvTranspose1d(self.hid_feature * 2, self.hid_feature, 1, stride=1)
            self.flinear = nn.ConvTranspose1d(self.hid_feature * 2, self.hid_feature, 1, stride=1)
        else:
            self.tlinear = nn.Linear(t_width, self.hid_feature)
            self.flinear = nn.Linear(f_width, self.hid_feature)
        n_bins = mcfg.get("freq_emb_bins", None)
        if n_bins:
            self.freq_emb = nn.Parameter(torch.zeros(n_bins, self.hid_feature))
            self.freq_emb._no_weight_decay = True
        else:
            self.freq_emb = None

    def _project(self, lin, y):
        return _pointwise_transpose(lin, y) if self.use_transpose else lin(y)

    def forward(self, x):
        """x: (batch, channels, time, freq) -> the same shape. The activations stay one
        (batch, time, freq, channels) tensor throughout: the time-axis scans read it
        through TokenLayout.time_axis, the frequency-axis scans as contiguous sequences.
        The result is a (b, c, t, f) view of that tensor, so the permute at the start of
        the next block is free. A time mixer that cannot read the strided layout gets the
        reference's (b*f, t, c) copy instead."""
        b, c, t, f = x.size()
        if self.freq_emb is not None:
            assert f == self.freq_emb.shape[0], (
                f"freq_emb_bins={self.freq_emb.shape[0]} but the latent input has {f} bins")
            x = x + self.freq_emb.t().unsqueeze(0).unsqueeze(2)
        tl = TokenLayout.time_axis(b, t, f)
        if self.time_mamba.accepts_layout(tl):
            x = x.permute(0, 2, 3, 1).contiguous()  # (b, t, f, c); no copy after a TF-block
            x = self._project(self.tlinear, self.time_mamba(x, layout=tl)) + x
        else:
            x = x.permute(0, 3, 2, 1).contiguous().view(b * f, t, c)
            x = self._project(self.tlinear, self.time_mamba(x)) + x
            x = x.view(b, f, t, c).permute(0, 2, 1, 3).contiguous()
        x = x.view(b * t, f, c)
        x = self._project(self.flinear, self.freq_mamba(x)) + x
        return x.view(b, t, f, c).permute(0, 3, 1, 2)
