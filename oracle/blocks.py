"""Oracle for the callers around the scans (test infrastructure; see ``oracle/__init__.py``).

Functional float64 restatements, driven by a module's ``state_dict``:
* ``mixer_forward``  — ``MambaStyleMixer.forward`` (reference models/mixer.py:77-99);
* ``block_forward``  — the pre-norm residual block of the third-party ``mamba_ssm``
  package as the reference uses it (models/mamba_block.py:335-342, 374-396): RMSNorm,
  mixer, residual (documented behaviour; the package is not in the reference checkout);
* ``mamba_block_forward`` / ``tf_block_forward`` — ``MambaBlock.forward`` and
  ``TFMambaBlock.forward`` (models/mamba_block.py:374-396, 478-508).
The scan layers inside come from ``oracle.selective_lru`` / ``oracle.linoss``.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from oracle import linoss as olin
from oracle import selective_lru as oslru


def _sub(params: dict, prefix: str) -> dict:
    n = len(prefix)
    return {k[n:]: v for k, v in params.items() if k.startswith(prefix)}


def ssm_forward(kind: str, params: dict, u, cfg: dict):
    """The scan layer inside a mixer: kind in {'selective_lru', 'linoss', 'selective_lru_mimo'}."""
    if kind == "selective_lru":
        return oslru.selective_lru_forward(params, u, cfg)
    if kind == "linoss":
        return olin.linoss_forward(params, u, cfg.get("discretization", "IMEX"), cfg.get("damping", True),
                                   cfg.get("a_from_g", True))
    if kind == "selective_lru_mimo":
        return oslru.selective_lru_mimo_forward(params, u, cfg)
    raise ValueError(kind)


def mixer_forward(params: dict, x, kind: str, ssm_cfg: dict, d_conv=4, causal=True):
    """in_proj -> split -> causal depthwise conv -> SiLU -> ssm -> * SiLU(z) -> out_proj
    (models/mixer.py:82-99)."""
    uz = x @ params["in_proj.weight"].t()
    u, z = uz.chunk(2, dim=-1)
    if causal:
        pad = (d_conv - 1, 0)
    else:
        left = (d_conv - 1) // 2
        pad = (left, d_conv - 1 - left)
    uc = F.pad(u.transpose(1, 2), pad)
    uc = F.conv1d(uc, params["conv.weight"], params["conv.bias"], groups=uc.shape[1])
    u = F.silu(uc.transpose(1, 2))
    y = ssm_forward(kind, _sub(params, "ssm."), u, ssm_cfg)
    y = y * F.silu(z)
    return y @ params["out_proj.weight"].t()


def rms_norm(x, weight, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * weight


def block_forward(params: dict, x, kind, ssm_cfg, eps=1e-5, d_conv=4, causal=True):
    """Pre-norm residual block with no incoming residual: mixer(RMSNorm(x)) + x."""
    h = rms_norm(x, params["norm.weight"], eps)
    return mixer_forward(_sub(params, "mixer."), h, kind, ssm_cfg, d_conv, causal) + x


def mamba_block_forward(params: dict, x, kind, ssm_cfg, bidirectional=True, **kw):
    y = block_forward(_sub(params, "forward_blocks.0."), x, kind, ssm_cfg, **kw)
    if not bidirectional:
        return y
    yb = block_forward(_sub(params, "backward_blocks.0."), torch.flip(x, [1]), kind, ssm_cfg, **kw)
    return torch.cat([y, torch.flip(yb, [1])], -1)


def tf_block_forward(params: dict, x, time_spec, freq_spec, use_transpose=True):
    """x (b, c, t, f); *_spec = (kind, ssm_cfg, extra kwargs of mamba_block_forward)."""
    b, c, t, f = x.shape
    h = x.permute(0, 3, 2, 1).reshape(b * f, t, c)
    ht = mamba_block_forward(_sub(params, "time_mamba."), h, time_spec[0], time_spec[1], **time_spec[2])
    h = _proj(params, "tlinear.", ht, use_transpose) + h
    h = h.view(b, f, t, c).permute(0, 2, 1, 3).reshape(b * t, f, c)
    hf = mamba_block_forward(_sub(params, "freq_mamba."), h, freq_spec[0], freq_spec[1], **freq_spec[2])
    h = _proj(params, "flinear.", hf, use_transpose) + h
    return h.view(b, t, f, c).permute(0, 3, 1, 2)


def _proj(params, prefix, h, use_transpose):
    w, bias = params[prefix + "weight"], params[prefix + "bias"]
    if use_transpose:  # ConvTranspose1d(in, out, 1): weight (in, out, 1)
        return h @ w[..., 0] + bias
    return h @ w.t() + bias
