"""Selective-LRU SISO scan operators backed by libsemx (``semx_selective_lru_fwd/bwd``).

* :func:`fused_selective_lru` — same name, arguments and return value as the
  reference operator (models/selective_lru/selective_lru_triton.py:528-577): the fused
  discretisation + complex diagonal scan + readout (+ envelope) + D skip, with optional
  per-mode detune, initial state and final state (gradients flow through all of them).
* :func:`fused_selective_lru_real` — the real specialisation (omega = delta_theta =
  B_im = C_im = 0): h = exp(-delta_nu a) h + gain B_t x, y = <C_t, h> + D x.

Conventions follow the reference: CUDA tensors only (RuntimeError otherwise), inputs made
contiguous fp32, outputs freshly allocated, unused outputs get ``None`` gradients
(``set_materialize_grads(False)``), a gradient arriving on the final state is injected
into the adjoint. ``block_t`` is the checkpoint interval of the recompute backward (a
multiple of 4, at most 256); ``block_c`` is accepted for API compatibility (the channel
tiling is chosen from N).

``layout`` (a :class:`~semambaxlinoss_b200.layout.TokenLayout`, not in the reference
signature) lets the per-token tensors be any (rows, width) arrangement the kernels read
in place: a reversed step order, or a row grid such as the time axis of a
(batch, frames, bins, width) tensor. The per-token outputs and gradients keep the
inputs' shapes and row order; ``h0`` and the final state stay (S, C, N).
"""
from __future__ import annotations

import torch

from .. import _lib
from ..layout import TokenLayout, check_rows

DEFAULT_CHUNK = 16


def _f32(t):
    if t is None:
        return None
    return t.detach().to(torch.float32).contiguous()


def _check_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("fused selective-LRU scan requires CUDA tensors.")


def _build_args(real, gain_code, chunk, layout, C, N, t):
    a = _lib.new_args(_lib.SemxSelectiveLruArgs)
    a.real, a.input_gain, a.chunk = int(real), gain_code, int(chunk)
    a.S, a.L, a.C, a.N = layout.S, layout.L, C, N
    _lib.set_layout(a, layout)
    for name, tensor in t.items():
        setattr(a, name, _lib.ptr(tensor))
    return a


class _SelectiveLRUScan(torch.autograd.Function):
    # Inputs (in order): delta_nu, delta_theta, a, omega, B_re, B_im, C_re, C_im, x, D, g,
    # s, h0_re, h0_im; then non-tensor block_t, want_final_state, gain_code, real, layout.
    @staticmethod
    def forward(ctx, delta_nu, delta_theta, a, omega, B_re, B_im, C_re, C_im, x, D, g, s,
                h0_re, h0_im, block_t, want_final_state, gain_code, real, layout):
        ctx.set_materialize_grads(False)
        _check_cuda(delta_nu, delta_theta, a, omega, B_re, B_im, C_re, C_im, x, D, g, s,
                    h0_re, h0_im)
        if layout is None:
            if delta_nu.dim() != 3:
                raise ValueError(f"delta_nu must be (B, T, C), got {tuple(delta_nu.shape)}")
            layout = TokenLayout.contiguous(delta_nu.shape[0], delta_nu.shape[1])
        S, L, C = layout.S, layout.L, delta_nu.shape[-1]
        N = a.shape[1]
        if a.shape != (C, N):
            raise ValueError("selective-LRU operand shapes do not agree")
        for name, t, w in (("delta_nu", delta_nu, C), ("x", x, C), ("B_re", B_re, N), ("C_re", C_re, N)):
            check_rows(name, t, layout, w)
        if not real:
            for name, t, w in (("delta_theta", delta_theta, C), ("B_im", B_im, N), ("C_im", C_im, N)):
                check_rows(name, t, layout, w)
        dev = delta_nu.device
        ins = {
            "delta_nu": _f32(delta_nu), "delta_theta": None if real else _f32(delta_theta),
            "a": _f32(a), "omega": None if real else _f32(omega),
            "B_re": _f32(B_re), "B_im": None if real else _f32(B_im),
            "C_re": _f32(C_re), "C_im": None if real else _f32(C_im),
            "x": _f32(x), "D": _f32(D), "g": _f32(g), "s": None if real else _f32(s),
            "h0_re": _f32(h0_re), "h0_im": None if real else _f32(h0_im),
        }
        need = any(ctx.needs_input_grad[:14])
        save_hf = want_final_state or need
        y = torch.empty(delta_nu.shape, dtype=torch.float32, device=dev)
        hf_re = torch.empty((S, C, N), dtype=torch.float32, device=dev) if save_hf else None
        hf_im = (torch.empty((S, C, N), dtype=torch.float32, device=dev)
                 if save_hf and not real else None)
        args = _build_args(real, gain_code, block_t, layout, C, N, dict(ins, y=y, hf_re=hf_re, hf_im=hf_im))
        ckpt = None
        if need:
            ckpt = _lib.empty_f32(_lib.load().semx_selective_lru_ckpt_bytes(args), dev)
            args.ckpt = ckpt.data_ptr()
        _lib.call("semx_selective_lru_fwd", args, dev)
        if need:
            ctx.save_for_backward(*[ins[k] for k in (
                "delta_nu", "delta_theta", "a", "omega", "B_re", "B_im", "C_re", "C_im", "x",
                "D", "g", "s", "h0_re", "h0_im")], ckpt)
            ctx.cfg = (layout, C, N, block_t, gain_code, real, delta_nu.shape, B_re.shape)
        dummy = y.new_zeros(1)
        if not save_hf:
            return y, dummy, dummy
        return y, hf_re, (hf_im if hf_im is not None else torch.zeros_like(hf_re))

    @staticmethod
    def backward(ctx, dy, dhf_re, dhf_im):
        (dnu, dth, a, om, Bre, Bim, Cre, Cim, x, D, g, s, h0r, h0i, ckpt) = ctx.saved_tensors
        layout, C, N, block_t, gain_code, real, tok_shape, sel_shape = ctx.cfg
        S = layout.S
        dev = dnu.device
        if dhf_re is None and dhf_im is not None:
            dhf_re = torch.zeros_like(dhf_im)
        if dhf_im is None and dhf_re is not None:
            dhf_im = torch.zeros_like(dhf_re)
        if dy is None:
            dy = torch.zeros(tok_shape, dtype=torch.float32, device=dev)
        need = ctx.needs_input_grad

        def out(i, shape):
            return torch.empty(shape, dtype=torch.float32, device=dev) if need[i] else None

        def zout(i, shape):
            return torch.zeros(shape, dtype=torch.float32, device=dev) if need[i] else None

        grads = {
            "d_delta_nu": out(0, tok_shape),
            "d_delta_theta": None if real else out(1, tok_shape),
            "da": zout(2, (C, N)),
            "domega": None if real else zout(3, (C, N)),
            "dB_re": zout(4, sel_shape),
            "dB_im": None if real else zout(5, sel_shape),
            "dC_re": zout(6, sel_shape),
            "dC_im": None if real else zout(7, sel_shape),
            "dx": out(8, tok_shape),
            "dD": zout(9, (C,)),
            "dg": zout(10, (C, N)) if g is not None else None,
            "ds": zout(11, (C, N)) if (s is not None and not real) else None,
            "dh0_re": zout(12, (S, C, N)) if h0r is not None else None,
            "dh0_im": zout(13, (S, C, N)) if (h0i is not None and not real) else None,
        }
        t = {"delta_nu": dnu, "delta_theta": dth, "a": a, "omega": om, "B_re": Bre,
             "B_im": Bim, "C_re": Cre, "C_im": Cim, "x": x, "D": D, "g": g, "s": s,
             "h0_re": h0r, "h0_im": h0i, "ckpt": ckpt, "dy": dy.to(torch.float32).contiguous(),
             "dhf_re": None if dhf_re is None else _f32(dhf_re),
             "dhf_im": None if (dhf_im is None or real) else _f32(dhf_im)}
        t.update(grads)
        args = _build_args(real, gain_code, block_t, layout, C, N, t)
        ws = _lib.empty_f32(_lib.load().semx_selective_lru_workspace_bytes(args), dev)
        args.workspace = ws.data_ptr()
        _lib.call("semx_selective_lru_bwd", args, dev)
        order = ["d_delta_nu", "d_delta_theta", "da", "domega", "dB_re", "dB_im", "dC_re",
                 "dC_im", "dx", "dD", "dg", "ds", "dh0_re", "dh0_im"]
        return tuple(grads[k] for k in order) + (None, None, None, None, None)


def fused_selective_lru(
    delta_nu: torch.Tensor,
    delta_theta: torch.Tensor,
    a: torch.Tensor,
    omega: torch.Tensor,
    Bsel_re: torch.Tensor,
    Bsel_im: torch.Tensor,
    Csel_re: torch.Tensor,
    Csel_im: torch.Tensor,
    x: torch.Tensor,
    D: torch.Tensor,
    g: torch.Tensor | None = None,
    s: torch.Tensor | None = None,
    h0_re: torch.Tensor | None = None,
    h0_im: torch.Tensor | None = None,
    block_t: int = DEFAULT_CHUNK,
    block_c: int = 32,
    want_final_state: bool = False,
    input_gain: str = "gamma",
    layout: TokenLayout | None = None,
):
    """Fused selective-LRU scan + readout. Returns ``(y, hf_re, hf_im)``: ``y`` (B, T, C)
    and the final state parts (B, C, N) (1-element dummies unless ``want_final_state``
    or gradients are required)::

        lam  = exp(delta_nu * (-a + j*(omega [+ s*] delta_theta)))
        Bu   = gain * (Bsel_re + j*Bsel_im) * x
        h_t  = lam_t * h_{t-1} + Bu_t      (h_{-1} = h0, default 0)
        y    = Re(<C, h>) [+ <g, |h|^2>] + D * x
    """
    del block_c
    if input_gain not in ("gamma", "mamba", "zoh"):
        raise ValueError(f"input_gain must be 'gamma', 'mamba', or 'zoh', got {input_gain!r}")
    return _SelectiveLRUScan.apply(
        delta_nu, delta_theta, a, omega, Bsel_re, Bsel_im, Csel_re, Csel_im, x, D, g, s,
        h0_re, h0_im, int(block_t), bool(want_final_state), _lib.GAIN_CODES[input_gain], False,
        layout,
    )


def fused_selective_lru_real(
    delta_nu: torch.Tensor,
    a: torch.Tensor,
    B: torch.Tensor,
    C: torch.Tensor,
    x: torch.Tensor,
    D: torch.Tensor,
    input_gain: str = "mamba",
    h0: torch.Tensor | None = None,
    g: torch.Tensor | None = None,
    block_t: int = DEFAULT_CHUNK,
    want_final_state: bool = False,
    layout: TokenLayout | None = None,
):
    """Real selective diagonal scan (the ``fused_selective_lru`` special case with
    omega = delta_theta = B_im = C_im = 0). Returns ``(y, hf)``."""
    if input_gain not in ("gamma", "mamba", "zoh"):
        raise ValueError(f"input_gain must be 'gamma', 'mamba', or 'zoh', got {input_gain!r}")
    y, hf, _ = _SelectiveLRUScan.apply(
        delta_nu, None, a, None, B, None, C, None, x, D, g, None, h0, None,
        int(block_t), bool(want_final_state), _lib.GAIN_CODES[input_gain], True, layout,
    )
    return y, hf
