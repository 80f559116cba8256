"""LinOSS scan operators backed by libsemx (``semx_linoss_fwd`` / ``semx_linoss_bwd``).

Two entry points:

* :func:`linoss_scan` — the reference's generic operator ``linoss_scan_triton(M_11, M_12,
  M_21, M_22, F1, F2) -> Y2`` (models/linoss/triton.py:276-294): given transition
  entries (P,) and forcings (S, L, P) complex64, returns the y2 trajectory. Exported
  under the reference name as well.
* :func:`linoss_scan_fused` — the fused form used by :class:`LinOSS`: Bu in, y2 out, with
  the parameter constraints and the IM / IMEX / damped-IMEX discretisation evaluated
  inside the kernel (models/linoss/linoss.py:81-116, 183-232). Gradients flow to the raw
  ``steps``, ``A_diag``, ``G_diag`` parameters and to Bu.

Conventions follow the reference operators: CUDA tensors only (RuntimeError otherwise),
ValueError on shape mismatch, inputs made contiguous, outputs freshly allocated. The
forward keeps one state checkpoint per ``chunk`` steps when a gradient is needed; the
backward recomputes everything else. ``reverse=True`` (not in the reference) runs every
chain from its last step to its first, in place: the result is
``flip(op(flip(inputs)))`` along the time axis without the two copies.
"""
from __future__ import annotations

import torch

from .. import _lib

DEFAULT_CHUNK = 64

VARIANTS = {
    "IM": _lib.LINOSS_IM,
    "IMEX": _lib.LINOSS_IMEX,
    "DAMPED_IMEX": _lib.LINOSS_DAMPED_IMEX,
}


def _require_cuda(name: str, *tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(f"{name} requires CUDA tensors.")


def _c64(t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.complex64:
        t = t.to(torch.complex64)
    return t.resolve_conj().contiguous()


def _f32(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to(torch.float32).contiguous()


def _call(fn_name: str, args, device):
    lib = _lib.load()
    status = getattr(lib, fn_name)(args, _lib.stream_handle(device))
    _lib.check(fn_name, status)


def _alloc_ckpt(S, L, P, chunk, device):
    nbytes = _lib.load().semx_linoss_ckpt_bytes(S, L, P, chunk)
    return torch.empty(max(nbytes // 4, 1), dtype=torch.float32, device=device)


def _alloc_ws(args, device):
    nbytes = _lib.load().semx_linoss_workspace_bytes(args)
    return torch.empty(max(nbytes // 4, 1), dtype=torch.float32, device=device)


class _LinOSSScanGeneric(torch.autograd.Function):
    @staticmethod
    def forward(ctx, M11, M12, M21, M22, F1, F2, chunk, reverse):
        _require_cuda("linoss_scan", M11, M12, M21, M22, F1, F2)
        if F1.shape != F2.shape:
            raise ValueError(f"F1 {tuple(F1.shape)} != F2 {tuple(F2.shape)}")
        if F1.dim() != 3:
            raise ValueError(f"F1 must be (B, T, N), got {tuple(F1.shape)}")
        S, L, P = F1.shape
        for m in (M11, M12, M21, M22):
            if m.shape != (P,):
                raise ValueError(f"M entries must have shape ({P},), got {tuple(m.shape)}")
        Ms = [_f32(m) for m in (M11, M12, M21, M22)]
        F1c, F2c = _c64(F1), _c64(F2)
        Y2 = torch.empty((S, L, P), dtype=torch.complex64, device=F1.device)
        need = any(ctx.needs_input_grad[:6])
        ckpt = _alloc_ckpt(S, L, P, chunk, F1.device) if need else None
        a = _lib.new_args(_lib.SemxLinossArgs)
        a.variant, a.chunk, a.S, a.L, a.P = _lib.LINOSS_GENERIC, chunk, S, L, P
        a.reverse = int(reverse)
        a.M11, a.M12, a.M21, a.M22 = [m.data_ptr() for m in Ms]
        a.F1, a.F2 = F1c.data_ptr(), F2c.data_ptr()
        a.Y2 = Y2.data_ptr()
        a.ckpt = _lib.ptr(ckpt)
        _call("semx_linoss_fwd", a, F1.device)
        if need:
            ctx.save_for_backward(*Ms, F1c, F2c, ckpt)
            ctx.chunk, ctx.reverse = chunk, int(reverse)
        return Y2

    @staticmethod
    def backward(ctx, dY2):
        M11, M12, M21, M22, F1, F2, ckpt = ctx.saved_tensors
        S, L, P = F1.shape
        dY2 = _c64(dY2)
        dF1 = torch.empty_like(F1)
        dF2 = torch.empty_like(F2)
        dM = torch.empty((4, P), dtype=torch.float32, device=F1.device)
        a = _lib.new_args(_lib.SemxLinossArgs)
        a.variant, a.chunk, a.S, a.L, a.P = _lib.LINOSS_GENERIC, ctx.chunk, S, L, P
        a.reverse = ctx.reverse
        a.M11, a.M12, a.M21, a.M22 = [m.data_ptr() for m in (M11, M12, M21, M22)]
        a.F1, a.F2 = F1.data_ptr(), F2.data_ptr()
        a.ckpt, a.dY2 = ckpt.data_ptr(), dY2.data_ptr()
        a.dF1, a.dF2, a.dM = dF1.data_ptr(), dF2.data_ptr(), dM.data_ptr()
        ws = _alloc_ws(a, F1.device)
        a.workspace = ws.data_ptr()
        _call("semx_linoss_bwd", a, F1.device)
        return dM[0], dM[1], dM[2], dM[3], dF1, dF2, None, None


class _LinOSSScanFused(torch.autograd.Function):
    @staticmethod
    def forward(ctx, steps, A_diag, G_diag, Bu, variant, a_from_g, chunk, reverse):
        _require_cuda("linoss_scan_fused", steps, A_diag, G_diag, Bu)
        if Bu.dim() != 3:
            raise ValueError(f"Bu must be (B, T, N), got {tuple(Bu.shape)}")
        S, L, P = Bu.shape
        code = VARIANTS[variant]
        damped = code == _lib.LINOSS_DAMPED_IMEX
        if damped and G_diag is None:
            raise ValueError("DAMPED_IMEX needs G_diag")
        for name, t in (("steps", steps), ("A_diag", A_diag), ("G_diag", G_diag)):
            if t is not None and t.shape != (P,):
                raise ValueError(f"{name} must have shape ({P},), got {tuple(t.shape)}")
        st, A = _f32(steps), _f32(A_diag)
        G = _f32(G_diag) if damped else None
        Buc = _c64(Bu)
        Y2 = torch.empty((S, L, P), dtype=torch.complex64, device=Bu.device)
        need = any(ctx.needs_input_grad[:4])
        ckpt = _alloc_ckpt(S, L, P, chunk, Bu.device) if need else None
        a = _lib.new_args(_lib.SemxLinossArgs)
        a.variant, a.a_from_g, a.chunk = code, int(bool(a_from_g)), chunk
        a.S, a.L, a.P, a.reverse = S, L, P, int(reverse)
        a.steps, a.A_diag, a.G_diag = st.data_ptr(), A.data_ptr(), _lib.ptr(G)
        a.Bu, a.Y2, a.ckpt = Buc.data_ptr(), Y2.data_ptr(), _lib.ptr(ckpt)
        _call("semx_linoss_fwd", a, Bu.device)
        if need:
            ctx.save_for_backward(st, A, G, Buc, ckpt)
            ctx.cfg = (code, int(bool(a_from_g)), chunk, damped, int(reverse))
        return Y2

    @staticmethod
    def backward(ctx, dY2):
        st, A, G, Bu, ckpt = ctx.saved_tensors
        code, a_from_g, chunk, damped, reverse = ctx.cfg
        S, L, P = Bu.shape
        dY2 = _c64(dY2)
        dBu = torch.empty_like(Bu)
        dparams = torch.zeros((3, P), dtype=torch.float32, device=Bu.device)
        a = _lib.new_args(_lib.SemxLinossArgs)
        a.variant, a.a_from_g, a.chunk = code, a_from_g, chunk
        a.S, a.L, a.P, a.reverse = S, L, P, reverse
        a.steps, a.A_diag, a.G_diag = st.data_ptr(), A.data_ptr(), _lib.ptr(G)
        a.Bu, a.ckpt, a.dY2 = Bu.data_ptr(), ckpt.data_ptr(), dY2.data_ptr()
        a.dBu, a.dparams = dBu.data_ptr(), dparams.data_ptr()
        ws = _alloc_ws(a, Bu.device)
        a.workspace = ws.data_ptr()
        _call("semx_linoss_bwd", a, Bu.device)
        return dparams[0], dparams[1], (dparams[2] if damped else None), dBu, None, None, None, None


def linoss_scan(M_11, M_12, M_21, M_22, F1, F2, chunk: int = DEFAULT_CHUNK, reverse: bool = False):
    """LinOSS scan with a given transition.

    Args:
        M_11, M_12, M_21, M_22: (N,) real float32. Transition entries (block-diagonal,
            N independent 2x2 blocks).
        F1, F2: (B, T, N) complex64. Per-step forcings.
        chunk: checkpoint interval / backward recompute block (multiple of 8, <= 256).
        reverse: scan each chain from its last step to its first.

    Returns:
        Y2: (B, T, N) complex64, the y2 component of the state trajectory.
    """
    return _LinOSSScanGeneric.apply(M_11, M_12, M_21, M_22, F1, F2, int(chunk), bool(reverse))


# Drop-in name of the reference operator (models/linoss/triton.py:276).
linoss_scan_triton = linoss_scan


def linoss_scan_fused(variant: str, steps, A_diag, G_diag, Bu, a_from_g: bool = True,
                      chunk: int = DEFAULT_CHUNK, reverse: bool = False):
    """Fused LinOSS scan: raw parameters (P,) and Bu (B, T, P) complex64 -> y2.

    ``variant`` is "IM", "IMEX" or "DAMPED_IMEX"; ``G_diag`` is used (and required) only
    by DAMPED_IMEX, where ``a_from_g`` selects the constraint direction exactly as
    ``LinOSS(a_from_g=...)`` does.
    """
    if variant not in VARIANTS:
        raise ValueError(f"unknown LinOSS variant {variant!r}")
    return _LinOSSScanFused.apply(steps, A_diag, G_diag, Bu, variant, a_from_g, int(chunk), bool(reverse))
