"""Oracle for the selective-LRU scans (test infrastructure; see ``oracle/__init__.py``).

Restates models/selective_lru/selective_lru.py of the reference:
* ``selective_recurrence``      — ``_selective_recurrence`` (590-599);
* ``selective_lru_op``          — the materialised path of ``SelectiveLRU.forward``
                                  (242-276), taking the operands of the fused op
                                  ``fused_selective_lru`` (selective_lru_triton.py:528-547);
* ``selective_lru_forward``     — the whole ``SelectiveLRU.forward`` (197-276);
* ``mimo_scan_readout``         — the non-fused branch of ``SelectiveLRUMIMO.forward``
                                  (569-574), operands of ``fused_selective_lru_mimo``;
* ``selective_lru_mimo_forward``— the whole ``SelectiveLRUMIMO.forward`` (488-587).
Works in any floating dtype on the CPU.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def selective_recurrence(lam, Bu, h0=None):
    """h_t = lam_t * h_{t-1} + Bu_t (complex, per element); restates selective_lru.py:590-599."""
    B, T, N = Bu.shape
    h = Bu.new_zeros(B, N) if h0 is None else h0
    outs = []
    for t in range(T):
        h = lam[:, t] * h + Bu[:, t]
        outs.append(h)
    if not outs:
        return Bu.new_zeros(B, 0, N)
    return torch.stack(outs, dim=1)


def selective_lru_op(
    delta_nu, delta_theta, a, omega, Bre, Bim, Cre, Cim, x, D,
    g=None, s=None, h0_re=None, h0_im=None, input_gain="gamma", return_final_state=False,
):
    """Materialised SISO scan + readout (selective_lru.py:243-276).

    delta_nu, delta_theta, x: (B,T,C); a, omega, g, s: (C,N); B*/C*: (B,T,N); D: (C,);
    h0_re/h0_im: (B,C,N). Returns y (B,T,C) [and the final state (B,C,N) complex].
    """
    B_, T, C = x.shape
    N = a.shape[1]
    nu = torch.exp(-delta_nu.unsqueeze(-1) * a)
    dth_n = delta_theta.unsqueeze(-1)
    base = omega + (s * dth_n if s is not None else dth_n)
    theta = delta_nu.unsqueeze(-1) * base
    lam = torch.polar(nu, theta)
    Bmat = torch.complex(Bre, Bim).unsqueeze(-2)
    if input_gain == "gamma":
        gain = torch.sqrt((1.0 - nu * nu).clamp_min(1e-6))
        Bu = (gain * x.unsqueeze(-1)) * Bmat
    elif input_gain == "mamba":
        Bu = (delta_nu * x).unsqueeze(-1) * Bmat
    elif input_gain == "zoh":
        dn = delta_nu.unsqueeze(-1)
        lm1_re = torch.expm1(-dn * a) * torch.cos(theta) - 2.0 * torch.sin(0.5 * theta).square()
        lm1_im = nu * torch.sin(theta)
        den = (a * a + base * base).clamp_min(1e-8)
        g_re = (base * lm1_im - a * lm1_re) / den
        g_im = -(a * lm1_im + base * lm1_re) / den
        Bu = (torch.complex(g_re, g_im) * x.unsqueeze(-1)) * Bmat
    else:
        raise ValueError(input_gain)
    h0 = torch.complex(h0_re, h0_im).reshape(B_, C * N) if h0_re is not None else None
    h = selective_recurrence(lam.reshape(B_, T, C * N), Bu.reshape(B_, T, C * N), h0)
    h = h.reshape(B_, T, C, N)
    C_complex = torch.complex(Cre, Cim)
    y = torch.einsum("btn,btcn->btc", C_complex, h).real + x * D
    if g is not None:
        y = y + torch.einsum("cn,btcn->btc", g, h.real**2 + h.imag**2)
    if return_final_state:
        hf = h[:, -1] if T > 0 else torch.complex(h0_re, h0_im) if h0_re is not None else None
        return y, hf
    return y


def selective_lru_real_op(delta_nu, a, B, C, x, D, input_gain="mamba", h0=None,
                          return_final_state=False):
    """Real special case of ``selective_lru_op`` (omega = delta_theta = B_im = C_im = 0):
    lam = exp(-delta_nu * a), Bu = gain * B_t * x, y = <C_t, h> + D x."""
    z_tc = torch.zeros_like(delta_nu)
    z_cn = torch.zeros_like(a)
    z_tn = torch.zeros_like(B)
    out = selective_lru_op(
        delta_nu, z_tc, a, z_cn, B, z_tn, C, z_tn, x, D,
        h0_re=h0, h0_im=None if h0 is None else torch.zeros_like(h0),
        input_gain=input_gain, return_final_state=return_final_state,
    )
    if return_final_state:
        y, hf = out
        return y, hf.real
    return out


def selective_lru_forward(params: dict, x, cfg: dict, h_init=None, rate_scale=None,
                          return_final_state=False):
    """``SelectiveLRU.forward`` (selective_lru.py:197-276) from a parameter dict with the
    reference's names (x_proj.weight, dt_nu_up.weight/bias, dt_theta_up.weight/bias,
    A_log, omega, D, env_gain, detune_gain). cfg: dt_rank, d_state, rate_scale,
    input_gain, envelope_readout, mode_detune."""
    r, N = cfg["dt_rank"], cfg["d_state"]
    proj = x @ params["x_proj.weight"].t()
    dnu_r, dth_r, B_sel, C_sel = torch.split(proj, [r, r, 2 * N, 2 * N], dim=-1)
    delta_nu = F.softplus(dnu_r @ params["dt_nu_up.weight"].t() + params["dt_nu_up.bias"])
    rs = cfg.get("rate_scale", 1.0) if rate_scale is None else float(rate_scale)
    if rs != 1.0:
        delta_nu = delta_nu * rs
    delta_theta = dth_r @ params["dt_theta_up.weight"].t() + params["dt_theta_up.bias"]
    a = torch.exp(params["A_log"])
    g = params["env_gain"] if cfg.get("envelope_readout") else None
    s = params["detune_gain"] if cfg.get("mode_detune") else None
    return selective_lru_op(
        delta_nu, delta_theta, a, params["omega"],
        B_sel[..., :N], B_sel[..., N:], C_sel[..., :N], C_sel[..., N:], x, params["D"], g, s,
        None if h_init is None else h_init.real, None if h_init is None else h_init.imag,
        input_gain=cfg.get("input_gain", "gamma"), return_final_state=return_final_state,
    )


def mimo_scan_readout(lam_re, lam_im, Bu_re, Bu_im, C_re, C_im, x, D, H, Nh, Fh):
    """Scan + block-diagonal readout + D skip (selective_lru.py:569-574).

    Returns (y (B,T,Fd), h_re, h_im (B,T,N)), the outputs of ``fused_selective_lru_mimo``.
    """
    Bsz, T, N = lam_re.shape
    h = selective_recurrence(torch.complex(lam_re, lam_im), torch.complex(Bu_re, Bu_im))
    hh = h.view(Bsz, T, H, Nh)
    C_c = torch.complex(C_re, C_im)
    y = torch.einsum("hfn,bthn->bthf", C_c, hh).real.reshape(Bsz, T, H * Fh)
    y = y + x * D
    return y, h.real, h.imag


def mimo_discretise(delta_nu, delta_theta, x, params: dict, cfg: dict, s_b=None, b_t=None, bx=None):
    """Pole, drive and gain of ``SelectiveLRUMIMO.forward`` (selective_lru.py:502-546).

    delta_nu, delta_theta: (B,T,H) after softplus / rate scale; s_b (B,T,H,r) and b_t
    (B,T,H,r,Nh) the rank-write projections (computed from x when not given); bx
    (B,T,H,Nh,2) the static drive B x (computed from x and B when not given). Returns
    (lam_re, lam_im, Bu_re, Bu_im) each (B,T,N)."""
    Bsz, T, Fdim = x.shape
    H, rank = cfg["n_heads"], cfg.get("rank", 0)
    Nh, Fh = cfg["state_dim"] // H, Fdim // H
    N = H * Nh
    a = torch.exp(params["A_log"])
    dnu_n = delta_nu.unsqueeze(-1)
    dth_n = delta_theta.unsqueeze(-1)
    nu = torch.exp(-dnu_n * a)
    base = params["omega"] + (params["detune_gain"] * dth_n if cfg.get("mode_detune") else dth_n)
    theta = dnu_n * base
    lam_re = (nu * torch.cos(theta)).reshape(Bsz, T, N)
    lam_im = (nu * torch.sin(theta)).reshape(Bsz, T, N)
    if bx is None:
        xh = x.view(Bsz, T, H, Fh)
        Bu_re = torch.einsum("hnf,bthf->bthn", params["B"][..., 0], xh)
        Bu_im = torch.einsum("hnf,bthf->bthn", params["B"][..., 1], xh)
    else:
        Bu_re, Bu_im = bx[..., 0], bx[..., 1]
    if rank > 0:
        if s_b is None:
            s_b = (x @ params["b_coef.weight"].t()).view(Bsz, T, H, rank)
            b_t = (x @ params["b_dir.weight"].t()).view(Bsz, T, H, rank, Nh)
        Bu_re = Bu_re + torch.einsum("bthr,bthrn->bthn", s_b, b_t)
    gain_mode = cfg.get("input_gain", "gamma")
    if gain_mode == "gamma":
        gain = torch.sqrt((1.0 - nu * nu).clamp_min(1e-6))
        Bu_re = Bu_re * gain
        Bu_im = Bu_im * gain
    elif gain_mode == "mamba":
        Bu_re = Bu_re * dnu_n
        Bu_im = Bu_im * dnu_n
    elif gain_mode == "zoh":
        lm1_re = torch.expm1(-dnu_n * a) * torch.cos(theta)
        lm1_re = lm1_re - 2.0 * torch.sin(0.5 * theta).square()
        lm1_im = nu * torch.sin(theta)
        den = (a * a + base * base).clamp_min(1e-8)
        g_re = (base * lm1_im - a * lm1_re) / den
        g_im = -(a * lm1_im + base * lm1_re) / den
        Bu_re, Bu_im = g_re * Bu_re - g_im * Bu_im, g_re * Bu_im + g_im * Bu_re
    return lam_re, lam_im, Bu_re.reshape(Bsz, T, N), Bu_im.reshape(Bsz, T, N)


def mimo_projection(params: dict, x, cfg: dict, drive: bool = False):
    """All token projections of ``SelectiveLRUMIMO`` as one row per token, in the column
    order [dnu_raw (H) | dth (H) | s_b (H r) | b_t (H r Nh) | s_c (H r) | c_t (H r 2Nh)]
    (dt_nu_proj / dt_theta_proj / b_coef / b_dir / c_coef / c_read of selective_lru.py:
    494-498, 528-530, 578-579), followed with ``drive`` by the static drive B x per
    (head, mode) as [re, im] pairs (H 2Nh columns; selective_lru.py:516-517)."""
    ws = [params["dt_nu_proj.weight"], params["dt_theta_proj.weight"]]
    bs = [params["dt_nu_proj.bias"], params["dt_theta_proj.bias"]]
    if cfg.get("rank", 0) > 0:
        for k in ("b_coef", "b_dir", "c_coef", "c_read"):
            w = params[k + ".weight"]
            ws.append(w)
            bs.append(w.new_zeros(w.shape[0]))
    proj = x @ torch.cat(ws, 0).t() + torch.cat(bs)
    if not drive:
        return proj
    Bsz, T, Fdim = x.shape
    H = cfg["n_heads"]
    Nh, Fh = cfg["state_dim"] // H, Fdim // H
    bx = torch.einsum("hnfc,bthf->bthnc", params["B"], x.view(Bsz, T, H, Fh))
    return torch.cat([proj, bx.reshape(Bsz, T, 2 * H * Nh)], -1)


def selective_lru_mimo_from_projection(proj, params: dict, x, cfg: dict, rate_scale=None):
    """``SelectiveLRUMIMO.forward`` (selective_lru.py:488-587) given the projection rows
    of :func:`mimo_projection` (so a caller can fix their rounding, e.g. to bf16); rows
    that carry the drive columns use them in place of B x."""
    Bsz, T, Fdim = x.shape
    H, rank = cfg["n_heads"], cfg.get("rank", 0)
    Nh, Fh = cfg["state_dim"] // H, Fdim // H
    delta_nu = F.softplus(proj[..., :H])
    rs = cfg.get("rate_scale", 1.0) if rate_scale is None else float(rate_scale)
    if rs != 1.0:
        delta_nu = delta_nu * rs
    delta_theta = proj[..., H:2 * H]
    s_b = b_t = s_c = cr = None
    if rank > 0:
        o = 2 * H
        s_b = proj[..., o:o + H * rank].reshape(Bsz, T, H, rank)
        o += H * rank
        b_t = proj[..., o:o + H * rank * Nh].reshape(Bsz, T, H, rank, Nh)
        o += H * rank * Nh
        s_c = proj[..., o:o + H * rank].reshape(Bsz, T, H, rank)
        o += H * rank
        cr = proj[..., o:o + 2 * H * rank * Nh].reshape(Bsz, T, H, rank, 2 * Nh)
    o = 2 * H + 2 * H * rank + 3 * H * rank * Nh
    bx = None
    if proj.shape[-1] == o + 2 * H * Nh:
        bx = proj[..., o:].reshape(Bsz, T, H, Nh, 2)
    elif proj.shape[-1] != o:
        raise ValueError(f"projection rows of width {proj.shape[-1]}: expected {o} or {o + 2 * H * Nh}")
    lam_re, lam_im, Bu_re, Bu_im = mimo_discretise(delta_nu, delta_theta, x, params, cfg, s_b, b_t, bx)
    y, h_re, h_im = mimo_scan_readout(
        lam_re, lam_im, Bu_re, Bu_im, params["C"][..., 0], params["C"][..., 1], x,
        params["D"], H, Nh, Fh,
    )
    hh = torch.complex(h_re, h_im).view(Bsz, T, H, Nh)
    if cfg.get("envelope_readout"):
        p = hh.real**2 + hh.imag**2
        y = y + torch.einsum("hfn,bthn->bthf", params["env_gain"], p).reshape(Bsz, T, Fdim)
    if rank > 0:
        c_t = torch.complex(cr[..., :Nh], cr[..., Nh:])
        read = torch.einsum("bthrn,bthn->bthr", c_t, hh).real
        c_out = params["c_out"].view(H, rank, Fh)
        y = y + torch.einsum("bthr,hrf->bthf", s_c * read, c_out).reshape(Bsz, T, Fdim)
    return y


def selective_lru_mimo_forward(params: dict, x, cfg: dict, rate_scale=None):
    """``SelectiveLRUMIMO.forward`` (selective_lru.py:488-587) from a parameter dict with
    the reference's names. cfg: n_heads, state_dim, rank, rate_scale, input_gain,
    envelope_readout, mode_detune."""
    return selective_lru_mimo_from_projection(mimo_projection(params, x, cfg), params, x, cfg,
                                              rate_scale)
