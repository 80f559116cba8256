"""Complex diagonal scan and MIMO scan + readout operators backed by libsemx.

* :func:`selective_scan_real` / :func:`selective_scan` — the reference operators
  ``selective_scan_triton_real`` / ``selective_scan_triton``
  (models/selective_lru/selective_lru_mimo_triton.py:178-211): h_t = lam_t h_{t-1} + Bu_t
  on split real/imaginary (B, T, N) tensors (or complex tensors), h_{-1} = 0.
* :func:`fused_selective_lru_mimo` — the reference operator of the same name
  (models/selective_lru/selective_lru_mimo_triton.py:441-462): scan + block-diagonal
  readout Re(C h) + D x, returning ``(y, h_re, h_im)``.

The reference names with the ``_triton`` suffix are exported as aliases for drop-in use.
CUDA tensors only (RuntimeError otherwise); ValueError on shape mismatch.
"""
from __future__ import annotations

import torch

from .. import _lib


def _f32(t):
    return None if t is None else t.detach().to(torch.float32).contiguous()


class _ComplexScan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, lam_re, lam_im, Bu_re, Bu_im):
        for t in (lam_re, lam_im, Bu_re, Bu_im):
            if not t.is_cuda:
                raise RuntimeError("selective_scan requires CUDA tensors.")
        if lam_re.shape != Bu_re.shape or lam_im.shape != Bu_im.shape or lam_re.shape != lam_im.shape:
            raise ValueError(f"lam {tuple(lam_re.shape)} != Bu {tuple(Bu_re.shape)}")
        S, L, N = lam_re.shape
        ins = [_f32(t) for t in (lam_re, lam_im, Bu_re, Bu_im)]
        h_re = torch.empty_like(ins[0])
        h_im = torch.empty_like(ins[0])
        a = _lib.new_args(_lib.SemxComplexScanArgs)
        a.S, a.L, a.N = S, L, N
        a.lam_re, a.lam_im, a.Bu_re, a.Bu_im = [t.data_ptr() for t in ins]
        a.h_re, a.h_im = h_re.data_ptr(), h_im.data_ptr()
        _lib.call("semx_complex_scan_fwd", a, lam_re.device)
        ctx.save_for_backward(ins[0], ins[1], h_re, h_im)
        return h_re, h_im

    @staticmethod
    def backward(ctx, dh_re, dh_im):
        lam_re, lam_im, h_re, h_im = ctx.saved_tensors
        S, L, N = lam_re.shape
        dh_re = torch.zeros_like(h_re) if dh_re is None else _f32(dh_re)
        dh_im = torch.zeros_like(h_im) if dh_im is None else _f32(dh_im)
        outs = [torch.empty_like(lam_re) for _ in range(4)]
        a = _lib.new_args(_lib.SemxComplexScanArgs)
        a.S, a.L, a.N = S, L, N
        a.lam_re, a.lam_im, a.h_re, a.h_im = [t.data_ptr() for t in (lam_re, lam_im, h_re, h_im)]
        a.dh_re, a.dh_im = dh_re.data_ptr(), dh_im.data_ptr()
        a.dlam_re, a.dlam_im, a.dBu_re, a.dBu_im = [t.data_ptr() for t in outs]
        _lib.call("semx_complex_scan_bwd", a, lam_re.device)
        return tuple(outs)


def selective_scan_real(lam_re, lam_im, Bu_re, Bu_im):
    """h_k = lam_k h_{k-1} + Bu_k (h_{-1} = 0) on split real/imaginary (B, T, N) tensors.
    Returns (h_re, h_im)."""
    return _ComplexScan.apply(lam_re, lam_im, Bu_re, Bu_im)


def selective_scan(lam: torch.Tensor, Bu: torch.Tensor) -> torch.Tensor:
    """Complex-tensor form of :func:`selective_scan_real`: (B, T, N) complex64 -> h."""
    h_re, h_im = selective_scan_real(lam.real, lam.imag, Bu.real, Bu.imag)
    return torch.complex(h_re, h_im)


selective_scan_triton_real = selective_scan_real
selective_scan_triton = selective_scan


class _FusedMIMO(torch.autograd.Function):
    @staticmethod
    def forward(ctx, lam_re, lam_im, Bu_re, Bu_im, C_re, C_im, x, D, H, Nh, Fh):
        for t in (lam_re, lam_im, Bu_re, Bu_im, C_re, C_im, x, D):
            if not t.is_cuda:
                raise RuntimeError("fused_selective_lru_mimo requires CUDA tensors.")
        S, L, N = lam_re.shape
        Fd = x.shape[2]
        if N != H * Nh or Fd != H * Fh or C_re.shape != (H, Fh, Nh):
            raise ValueError("fused_selective_lru_mimo: head sizes do not match the operands")
        ins = [_f32(t) for t in (lam_re, lam_im, Bu_re, Bu_im, C_re, C_im, x, D)]
        y = torch.empty((S, L, Fd), dtype=torch.float32, device=x.device)
        h_re = torch.empty((S, L, N), dtype=torch.float32, device=x.device)
        h_im = torch.empty_like(h_re)
        a = _lib.new_args(_lib.SemxMimoArgs)
        a.S, a.L, a.H, a.Nh, a.Fh = S, L, H, Nh, Fh
        (a.lam_re, a.lam_im, a.Bu_re, a.Bu_im, a.C_re, a.C_im, a.x, a.D) = [t.data_ptr() for t in ins]
        a.y, a.h_re, a.h_im = y.data_ptr(), h_re.data_ptr(), h_im.data_ptr()
        _lib.call("semx_mimo_fwd", a, x.device)
        ctx.save_for_backward(ins[0], ins[1], h_re, h_im, ins[4], ins[5], ins[6], ins[7])
        ctx.dims = (S, L, H, Nh, Fh)
        return y, h_re, h_im

    @staticmethod
    def backward(ctx, dy, dh_re, dh_im):
        lam_re, lam_im, h_re, h_im, C_re, C_im, x, D = ctx.saved_tensors
        S, L, H, Nh, Fh = ctx.dims
        dev = x.device
        dy = torch.zeros_like(x) if dy is None else _f32(dy)
        if dh_re is not None or dh_im is not None:
            dh_re = torch.zeros_like(h_re) if dh_re is None else _f32(dh_re)
            dh_im = torch.zeros_like(h_im) if dh_im is None else _f32(dh_im)
        dlam_re, dlam_im, dBu_re, dBu_im = [torch.empty_like(h_re) for _ in range(4)]
        dx = torch.empty_like(x)
        dC_re, dC_im = torch.empty_like(C_re), torch.empty_like(C_im)
        dD = torch.empty_like(D)
        a = _lib.new_args(_lib.SemxMimoArgs)
        a.S, a.L, a.H, a.Nh, a.Fh = S, L, H, Nh, Fh
        a.lam_re, a.lam_im, a.C_re, a.C_im = [t.data_ptr() for t in (lam_re, lam_im, C_re, C_im)]
        a.x, a.D, a.h_re, a.h_im, a.dy = [t.data_ptr() for t in (x, D, h_re, h_im, dy)]
        a.dh_re, a.dh_im = _lib.ptr(dh_re), _lib.ptr(dh_im)
        a.dlam_re, a.dlam_im, a.dBu_re, a.dBu_im = [t.data_ptr() for t in (dlam_re, dlam_im, dBu_re, dBu_im)]
        a.dx, a.dC_re, a.dC_im, a.dD = [t.data_ptr() for t in (dx, dC_re, dC_im, dD)]
        ws = _lib.empty_f32(_lib.load().semx_mimo_workspace_bytes(a), dev)
        a.workspace = ws.data_ptr()
        _lib.call("semx_mimo_bwd", a, dev)
        return dlam_re, dlam_im, dBu_re, dBu_im, dC_re, dC_im, dx, dD, None, None, None


def fused_selective_lru_mimo(lam_re, lam_im, Bu_re, Bu_im, C_re, C_im, x, D, n_heads, n_head, f_head):
    """Fused MIMO scan + block-diagonal readout + D skip. ``lam``/``Bu`` are the (B, T, N)
    halves (N = n_heads * n_head), ``C_re``/``C_im`` the (n_heads, f_head, n_head) readout
    halves, ``x`` the (B, T, Fd) input (Fd = n_heads * f_head) and ``D`` (Fd,). Returns
    ``(y, h_re, h_im)`` with y = Re(C h) + D x and the (B, T, N) state halves."""
    return _FusedMIMO.apply(lam_re, lam_im, Bu_re, Bu_im, C_re, C_im, x, D,
                            int(n_heads), int(n_head), int(f_head))


def _layer_fwd(x, proj, dt_bias, params, dims, want_ckpt):
    """semx_mimo_layer_fwd on contiguous x / proj (same dtype) and fp32 parameters
    (A_log, omega, detune_gain, C, D, c_out, env_gain). Returns (y, ckpt or None)."""
    H, Nh, Fh, rank, gain_code, rate_scale = dims
    S, L, Fd = x.shape
    y = torch.empty((S, L, Fd), dtype=torch.float32, device=x.device)
    a = _lib.new_args(_lib.SemxMimoLayerArgs)
    a.input_gain, a.rank, a.rate_scale = gain_code, rank, float(rate_scale)
    a.detune, a.envelope = int(params[2] is not None), int(params[6] is not None)
    a.bf16 = int(x.dtype == torch.bfloat16)
    a.S, a.L, a.H, a.Nh, a.Fh = S, L, H, Nh, Fh
    a.x, a.proj, a.y, a.dt_bias = x.data_ptr(), proj.data_ptr(), y.data_ptr(), _lib.ptr(dt_bias)
    (a.A_log, a.omega, a.detune_gain, a.C, a.D, a.c_out, a.env_gain) = [_lib.ptr(t) for t in params]
    ckpt = None
    if want_ckpt:
        ckpt = _lib.empty_f32(_lib.load().semx_mimo_layer_ckpt_bytes(a), x.device)
        a.ckpt = ckpt.data_ptr()
    _lib.call("semx_mimo_layer_fwd", a, x.device)
    return y, ckpt


def _layer_bwd(x, proj, ckpt, dt_bias, params, dims, dy):
    """semx_mimo_layer_bwd. Returns dx (the skip part D dy, dtype of x), dproj and the
    parameter gradients as a dict (dA_log, domega, ddetune, dC, dD, dc_out, denv,
    d_dt_bias; None where the operand is absent)."""
    A_log, omega, det, C, D, c_out, env = params
    H, Nh, Fh, rank, gain_code, rate_scale = dims
    S, L, Fd = x.shape
    dev = x.device
    dx = torch.empty_like(x)
    dproj = torch.empty_like(proj)
    g = {k: torch.empty_like(v) for k, v in (("dA_log", A_log), ("domega", omega), ("dC", C), ("dD", D))}
    g["ddetune"] = torch.empty_like(det) if det is not None else None
    g["dc_out"] = torch.empty_like(c_out) if rank > 0 else None
    g["denv"] = torch.empty_like(env) if env is not None else None
    g["d_dt_bias"] = torch.empty_like(dt_bias) if dt_bias is not None else None
    a = _lib.new_args(_lib.SemxMimoLayerArgs)
    a.input_gain, a.rank, a.rate_scale = gain_code, rank, float(rate_scale)
    a.detune, a.envelope = int(det is not None), int(env is not None)
    a.bf16 = int(x.dtype == torch.bfloat16)
    a.S, a.L, a.H, a.Nh, a.Fh = S, L, H, Nh, Fh
    a.x, a.proj, a.ckpt, a.dy, a.dx, a.dproj = [t.data_ptr() for t in (x, proj, ckpt, dy, dx, dproj)]
    a.dt_bias = _lib.ptr(dt_bias)
    (a.A_log, a.omega, a.detune_gain, a.C, a.D, a.c_out, a.env_gain) = [_lib.ptr(t) for t in params]
    for k, v in g.items():
        setattr(a, k, _lib.ptr(v))
    ws = _lib.empty_f32(_lib.load().semx_mimo_layer_workspace_bytes(a), dev)
    a.workspace = ws.data_ptr()
    _lib.call("semx_mimo_layer_bwd", a, dev)
    return dx, dproj, g


def _check_layer(x, proj_cols, C, dims, tensors):
    H, Nh, Fh, rank = dims[:4]
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("SelectiveLRUMIMO requires CUDA tensors.")
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError(f"SelectiveLRUMIMO: unsupported dtype {x.dtype}")
    if x.dim() != 3 or x.shape[2] != H * Fh or C.shape != (H, Fh, Nh, 2) or proj_cols != proj_width(H, Nh, rank):
        raise ValueError("SelectiveLRUMIMO operand shapes do not agree")


class _MimoLayer(torch.autograd.Function):
    """The SelectiveLRUMIMO layer after its token projections (semx_mimo_layer_fwd/bwd):
    poles, gain, scan, readout and feedthrough in one kernel per direction."""

    @staticmethod
    def forward(ctx, x, proj, dt_bias, A_log, omega, detune_gain, C, D, c_out, env_gain, dims):
        _check_layer(x, proj.shape[-1], C, dims, (x, proj, A_log, omega, C, D))
        if x.dtype != proj.dtype or proj.shape[:2] != x.shape[:2]:
            raise ValueError("x and proj must have the same dtype and leading shape")
        x, proj = x.contiguous(), proj.contiguous()
        params = [_f32(t) for t in (A_log, omega, detune_gain, C, D, c_out, env_gain)]
        dtb = _f32(dt_bias)
        y, ckpt = _layer_fwd(x, proj, dtb, params, dims, any(ctx.needs_input_grad))
        if ckpt is not None:
            ctx.save_for_backward(x, proj, ckpt, dtb, *params)
            ctx.dims = dims
        return y

    @staticmethod
    def backward(ctx, dy):
        x, proj, ckpt, dtb, *params = ctx.saved_tensors
        dx, dproj, g = _layer_bwd(x, proj, ckpt, dtb, params, ctx.dims, _f32(dy))
        return (dx, dproj, g["d_dt_bias"], g["dA_log"], g["domega"], g["ddetune"], g["dC"], g["dD"],
                g["dc_out"], g["denv"], None)


class _MimoLayerProjected(torch.autograd.Function):
    """The whole SelectiveLRUMIMO layer from its concatenated projection weight W
    (P, H Fh): proj = x W^T (one GEMM), then the layer kernels. The backward's input
    gradient is one accumulating GEMM, dx = D dy + dproj W, and dW = dproj^T x."""

    @staticmethod
    def forward(ctx, x, W, dt_bias, A_log, omega, detune_gain, C, D, c_out, env_gain, dims):
        _check_layer(x, W.shape[0], C, dims, (x, W, A_log, omega, C, D))
        if W.dtype != x.dtype or W.shape[1] != x.shape[2]:
            raise ValueError("W must be (P, in_features) in the dtype of x")
        x, W = x.contiguous(), W.contiguous()
        proj = torch.matmul(x, W.t())
        params = [_f32(t) for t in (A_log, omega, detune_gain, C, D, c_out, env_gain)]
        dtb = _f32(dt_bias)
        y, ckpt = _layer_fwd(x, proj, dtb, params, dims, any(ctx.needs_input_grad))
        if ckpt is not None:
            ctx.save_for_backward(x, W, proj, ckpt, dtb, *params)
            ctx.dims = dims
        return y

    @staticmethod
    def backward(ctx, dy):
        x, W, proj, ckpt, dtb, *params = ctx.saved_tensors
        dx, dproj, g = _layer_bwd(x, proj, ckpt, dtb, params, ctx.dims, _f32(dy))
        P, Fd = W.shape
        dproj2 = dproj.view(-1, P)
        dx.view(-1, Fd).addmm_(dproj2, W)
        dW = dproj2.t().mm(x.view(-1, Fd)) if ctx.needs_input_grad[1] else None
        return (dx, dW, g["d_dt_bias"], g["dA_log"], g["domega"], g["ddetune"], g["dC"], g["dD"],
                g["dc_out"], g["denv"], None)


def proj_width(n_heads, n_head, rank):
    """Columns of the projection row the layer kernels read (see :func:`mimo_layer`)."""
    H, Nh, r = int(n_heads), int(n_head), int(rank)
    return 2 * H + 2 * H * r + 3 * H * r * Nh + 2 * H * Nh


def drive_weight(B):
    """The static input map B (H, Nh, Fh, 2) as the block-diagonal rows of the projection
    weight that produce the drive columns: row h*2Nh + 2n + c, column h*Fh + f holds
    B[h, n, f, c] (c = 0 real, 1 imaginary part)."""
    H, Nh, Fh, _ = B.shape
    return torch.block_diag(*B.permute(0, 1, 3, 2).reshape(H, 2 * Nh, Fh).unbind(0))


def mimo_layer(x, proj, A_log, omega, detune_gain, C, D, c_out, env_gain, n_heads, n_head,
               f_head, rank, input_gain="gamma", rate_scale=1.0, dt_bias=None):
    """SelectiveLRUMIMO after its token projections. ``proj`` (B, T, P) holds, per token,
    [dnu_raw (H) | dth (H) | s_b (H r) | b_t (H r Nh) | s_c (H r) | c_t (H r 2Nh) |
    bx (H 2Nh)] with dnu = softplus(dnu_raw + b_nu) * rate_scale, dth = dth + b_th
    (``dt_bias`` = [b_nu (H) | b_th (H)], optional) and bx the static drive
    (sum_f B[h, n, f] x[h Fh + f], real and imaginary part per mode; :func:`drive_weight`
    gives its weight rows); ``x`` (B, T, H Fh) and ``proj`` are both float32 or both
    bfloat16 (state and outputs are float32). Returns y (B, T, H Fh) float32; the
    gradient reaching x directly is the skip part D dy, the drive's part flows through
    ``proj``."""
    return _MimoLayer.apply(x, proj, dt_bias, A_log, omega, detune_gain, C, D, c_out, env_gain,
                            _dims(n_heads, n_head, f_head, rank, input_gain, rate_scale))


def mimo_layer_projected(x, W, dt_bias, A_log, omega, detune_gain, C, D, c_out, env_gain, n_heads,
                         n_head, f_head, rank, input_gain="gamma", rate_scale=1.0):
    """The whole SelectiveLRUMIMO layer: :func:`mimo_layer` on ``proj = x W^T`` with the
    projection GEMM inside the operator (``W`` (P, H Fh) in the dtype of ``x``, rows in
    the column order of :func:`mimo_layer`), so its backward forms the input gradient in
    one accumulating GEMM."""
    return _MimoLayerProjected.apply(x, W, dt_bias, A_log, omega, detune_gain, C, D, c_out, env_gain,
                                     _dims(n_heads, n_head, f_head, rank, input_gain, rate_scale))


def _dims(n_heads, n_head, f_head, rank, input_gain, rate_scale):
    if input_gain not in _lib.GAIN_CODES:
        raise ValueError(f"input_gain must be 'gamma', 'mamba', 'zoh', or 'none', got {input_gain!r}")
    return (int(n_heads), int(n_head), int(f_head), int(rank), _lib.GAIN_CODES[input_gain], float(rate_scale))
