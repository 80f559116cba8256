"""Token layouts on the GPU: the scans and the convolution read reversed and strided
token rows in place, and the results equal the reference's copies.

* reverse: ``op(x, reverse)`` against the float64 oracle of ``flip(op(flip(x)))`` (the
  reference's bi-directional branch, models/mamba_block.py:387-396), forward and every
  gradient, for the selective-LRU scan (complex with every option, and real), the
  LinOSS scans (fused variants, the generic form, and both IMEX backward paths) and the
  convolution + SiLU (causal and centred windows, short and split-kernel lengths);
* strided: the time axis of a (batch, frames, bins, width) tensor read through
  TokenLayout.time_axis against the oracle of the permuted copy the reference makes
  (models/mamba_block.py:496-507), alone and reversed;
* the blocks: MambaBlock's copy-free backward branch and TFMambaBlock's single-layout
  pass against the same modules run through the reference's flip / permute formulation.
"""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle import linoss as olin
from oracle import selective_lru as oslru
from tests.parity import (BF16_TOL, FP32_TOL, assert_close, crandn, cuda, floor_tol, gen, randn,
                          rel_err, to32)

pytestmark = pytest.mark.gpu

NAMES = ["dnu", "dth", "a", "om", "Bre", "Bim", "Cre", "Cim", "x", "D", "g", "s", "h0r", "h0i"]
TOKEN = {"dnu", "dth", "Bre", "Bim", "Cre", "Cim", "x"}


def _flip_view(b, t, f):
    """(to_seq, from_seq) for the reversed contiguous layout of (S, L, W) tensors."""
    return (lambda v: torch.flip(v, [1])), (lambda v: torch.flip(v, [1]))


def _time_view(b, t, f, reverse):
    """(to_seq, from_seq) between a (b, t, f, W) token tensor and the (b*f, t, W) sequence
    tensor of the time axis (step order reversed when ``reverse``)."""

    def to_seq(v):
        s = v.permute(0, 2, 1, 3).reshape(b * f, t, v.shape[-1])
        return torch.flip(s, [1]) if reverse else s

    def from_seq(s):
        s = torch.flip(s, [1]) if reverse else s
        return s.reshape(b, f, t, s.shape[-1]).permute(0, 2, 1, 3)

    return to_seq, from_seq


# ----------------------------------------------------------------------------- selective LRU

def _slru_inputs(tok_shape, S, C, N, seed, opts):
    g = gen(seed)
    t = {
        "dnu": F.softplus(randn((*tok_shape, C), g)) * 0.3,
        "dth": randn((*tok_shape, C), g),
        "a": torch.exp(randn((C, N), g, scale=0.5)),
        "om": randn((C, N), g),
        "Bre": randn((*tok_shape, N), g), "Bim": randn((*tok_shape, N), g),
        "Cre": randn((*tok_shape, N), g), "Cim": randn((*tok_shape, N), g),
        "x": randn((*tok_shape, C), g), "D": randn(C, g),
        "g": randn((C, N), g, scale=0.1) if "env" in opts else None,
        "s": (1.0 + randn((C, N), g, scale=0.3)) if "detune" in opts else None,
        "h0r": randn((S, C, N), g) if "h0" in opts else None,
        "h0i": randn((S, C, N), g) if "h0" in opts else None,
    }
    gy = randn((*tok_shape, C), g)
    ghf = (randn((S, C, N), g), randn((S, C, N), g))
    return t, gy, ghf


def _slru_oracle(t, gy, ghf, gain, to_seq, from_seq, dtype):
    ins = {k: (v.to(dtype).clone().requires_grad_(True) if v is not None else None) for k, v in t.items()}
    seq = {k: (to_seq(v) if k in TOKEN else v) for k, v in ins.items()}
    y, hf = oslru.selective_lru_op(
        seq["dnu"], seq["dth"], seq["a"], seq["om"], seq["Bre"], seq["Bim"], seq["Cre"], seq["Cim"],
        seq["x"], seq["D"], seq["g"], seq["s"], seq["h0r"], seq["h0i"], input_gain=gain,
        return_final_state=True)
    y = from_seq(y)
    loss = (y * gy.to(dtype)).sum() + (hf.real * ghf[0].to(dtype) + hf.imag * ghf[1].to(dtype)).sum()
    req = [k for k in NAMES if ins[k] is not None]
    return y.detach(), dict(zip(req, torch.autograd.grad(loss, [ins[k] for k in req])))


def _slru_gpu(t, gy, ghf, gain, chunk, layout):
    from semambaxlinoss_b200.selective_lru import fused_selective_lru

    dev = cuda()
    ins = {k: (to32(v, dev).requires_grad_(True) if v is not None else None) for k, v in t.items()}
    y, hf_re, hf_im = fused_selective_lru(
        ins["dnu"], ins["dth"], ins["a"], ins["om"], ins["Bre"], ins["Bim"], ins["Cre"], ins["Cim"],
        ins["x"], ins["D"], ins["g"], ins["s"], ins["h0r"], ins["h0i"], block_t=chunk,
        want_final_state=True, input_gain=gain, layout=layout)
    loss = (y * to32(gy, dev)).sum() + (hf_re * to32(ghf[0], dev) + hf_im * to32(ghf[1], dev)).sum()
    loss.backward()
    return y.detach(), {k: v.grad for k, v in ins.items() if v is not None}


def _slru_check(t, gy, ghf, gain, chunk, layout, to_seq, from_seq):
    y_ref, g_ref = _slru_oracle(t, gy, ghf, gain, to_seq, from_seq, torch.float64)
    y32, g32 = _slru_oracle(t, gy, ghf, gain, to_seq, from_seq, torch.float32)
    y, grads = _slru_gpu(t, gy, ghf, gain, chunk, layout)
    assert y.shape == y_ref.shape
    assert_close(y, y_ref, floor_tol(rel_err(y32, y_ref)), "y")
    for k, ref in g_ref.items():
        assert grads[k].shape == ref.shape, k
        assert_close(grads[k], ref, floor_tol(rel_err(g32[k], ref)), f"d{k}")


@pytest.mark.parametrize("gain", ["gamma", "mamba", "zoh"])
@pytest.mark.parametrize("B,T,C,N,chunk,opts", [
    (2, 23, 6, 8, 8, ("env", "detune", "h0")),
    (3, 45, 40, 16, 20, ("h0",)),      # partial tiles, ragged last chunk, 4 channel groups
    (1, 9, 7, 13, 4, ()),              # N not a multiple of 4
])
def test_selective_lru_reverse_matches_flipped_oracle(B, T, C, N, chunk, opts, gain):
    from semambaxlinoss_b200.layout import TokenLayout

    t, gy, ghf = _slru_inputs((B, T), B, C, N, 31 * B + T + C + N, opts)
    to_seq, from_seq = _flip_view(B, T, 1)
    _slru_check(t, gy, ghf, gain, chunk, TokenLayout.contiguous(B, T, reverse=True), to_seq, from_seq)


@pytest.mark.parametrize("reverse", [False, True])
@pytest.mark.parametrize("b,t,f,C,N,chunk", [(2, 19, 5, 6, 8, 8), (1, 40, 3, 20, 16, 16), (2, 7, 4, 5, 4, 4)])
def test_selective_lru_time_axis_matches_permuted_oracle(b, t, f, C, N, chunk, reverse):
    from semambaxlinoss_b200.layout import TokenLayout

    tv, gy, ghf = _slru_inputs((b, t, f), b * f, C, N, 7 * b + t + f + C, ("env", "detune", "h0"))
    to_seq, from_seq = _time_view(b, t, f, reverse)
    _slru_check(tv, gy, ghf, "gamma", chunk, TokenLayout.time_axis(b, t, f, reverse), to_seq, from_seq)


@pytest.mark.parametrize("layout_kind", ["reverse", "time", "time_reverse"])
@pytest.mark.parametrize("N", [16, 13])
def test_real_selective_lru_layouts_match_oracle(layout_kind, N):
    """The real scan (N <= 16 forward in its register kernel; N = 13 partial) under each
    layout, against the oracle of the copies."""
    from semambaxlinoss_b200.layout import TokenLayout
    from semambaxlinoss_b200.selective_lru import fused_selective_lru_real

    b, t, f, C = 2, 37, 3, 24
    g = gen(900 + N)
    if layout_kind == "reverse":
        tok, S = (b * f, t), b * f
        layout = TokenLayout.contiguous(S, t, reverse=True)
        to_seq, from_seq = _flip_view(S, t, 1)
    else:
        tok, S = (b, t, f), b * f
        layout = TokenLayout.time_axis(b, t, f, reverse=layout_kind == "time_reverse")
        to_seq, from_seq = _time_view(b, t, f, layout.reverse)
    dnu = F.softplus(randn((*tok, C), g, mean=-1.0))
    a = torch.exp(torch.rand(C, N, generator=g, dtype=torch.float64) * 2.7)
    Bt, Ct = randn((*tok, N), g, scale=0.25), randn((*tok, N), g, scale=0.25)
    x, D, h0 = randn((*tok, C), g), randn(C, g), randn((S, C, N), g)
    gy, ghf = randn((*tok, C), g), randn((S, C, N), g)

    def run_oracle(dtype):
        ins = [v.to(dtype).clone().requires_grad_(True) for v in (dnu, a, Bt, Ct, x, D, h0)]
        seq = [to_seq(v) if i in (0, 2, 3, 4) else v for i, v in enumerate(ins)]
        y, hf = oslru.selective_lru_real_op(*seq[:6], input_gain="mamba", h0=seq[6], return_final_state=True)
        y = from_seq(y)
        loss = (y * gy.to(dtype)).sum() + (hf * ghf.to(dtype)).sum()
        return y.detach(), torch.autograd.grad(loss, ins)

    y_ref, g_ref = run_oracle(torch.float64)
    y32, g32 = run_oracle(torch.float32)
    dev = cuda()
    ins = [to32(v, dev).requires_grad_(True) for v in (dnu, a, Bt, Ct, x, D, h0)]
    y, hf = fused_selective_lru_real(*ins[:6], input_gain="mamba", h0=ins[6], block_t=16,
                                     want_final_state=True, layout=layout)
    ((y * to32(gy, dev)).sum() + (hf * to32(ghf, dev)).sum()).backward()
    assert_close(y, y_ref, floor_tol(rel_err(y32, y_ref)), "y")
    for name, v, r, r32 in zip(["dnu", "a", "B", "C", "x", "D", "h0"], ins, g_ref, g32):
        assert_close(v.grad, r, floor_tol(rel_err(r32, r)), f"d{name}")


def test_selective_lru_layout_errors():
    from semambaxlinoss_b200.layout import TokenLayout
    from semambaxlinoss_b200.selective_lru import fused_selective_lru_real

    dev = cuda()
    C, N = 4, 4
    dnu = torch.rand(2, 5, 3, C, device=dev)
    a = torch.rand(C, N, device=dev)
    Bt = torch.rand(2, 5, 3, N, device=dev)
    x, D = torch.rand(2, 5, 3, C, device=dev), torch.rand(C, device=dev)
    with pytest.raises(ValueError):  # 30 token rows, layout of 6 x 4
        fused_selective_lru_real(dnu, a, Bt, Bt, x, D, layout=TokenLayout.time_axis(2, 4, 3))
    # A grid whose rows run past the tensor is refused by the library.
    bad = TokenLayout(S=6, L=5, seq_group=3, group_stride=16, seq_stride=1, step_stride=3)
    with pytest.raises(RuntimeError, match="layout"):
        fused_selective_lru_real(dnu, a, Bt, Bt, x, D, layout=bad)


# ----------------------------------------------------------------------------- LinOSS

VARIANTS = [("IMEX", True, True), ("IMEX", True, False), ("IMEX", False, True), ("IM", False, True)]


def _linoss_params(P, g, variant):
    steps = randn(P, g, scale=1.2)
    if variant == "DAMPED_IMEX":
        return steps, randn(P, g, scale=1.5, mean=0.5), randn(P, g, scale=1.0, mean=0.2)
    return steps, randn(P, g, scale=1.0, mean=0.3), None


def _linoss_oracle(variant, steps, A, G, Bu, gy, afg, dtype):
    cdt = torch.complex128 if dtype == torch.float64 else torch.complex64

    def cast(v):
        return v.to(cdt if v.is_complex() else dtype)

    ins = [cast(v).clone().requires_grad_(True) if v is not None else None for v in (steps, A, G, Bu)]
    y2 = torch.flip(olin.linoss_scan_fused(variant, *ins[:3], torch.flip(ins[3], [1]), a_from_g=afg), [1])
    gyc = cast(gy)
    loss = (y2.real * gyc.real + y2.imag * gyc.imag).sum()
    req = [v for v in ins if v is not None]
    names = [n for n, v in zip(("steps", "A", "G", "Bu"), ins) if v is not None]
    return y2.detach(), dict(zip(names, torch.autograd.grad(loss, req)))


def _linoss_check(variant, steps, A, G, Bu, gy, afg, chunk, slices=None):
    from semambaxlinoss_b200.linoss import linoss_scan_fused

    y_ref, g_ref = _linoss_oracle(variant, steps, A, G, Bu, gy, afg, torch.float64)
    y32, g32 = _linoss_oracle(variant, steps, A, G, Bu, gy, afg, torch.float32)
    dev = cuda()
    ins = [to32(v, dev).requires_grad_(True) if v is not None else None for v in (steps, A, G, Bu)]
    y2 = linoss_scan_fused(variant, *ins, a_from_g=afg, chunk=chunk, reverse=True)
    y2.backward(to32(gy, dev))
    got = {n: v.grad for n, v in zip(("steps", "A", "G", "Bu"), ins) if v is not None}
    for sl in slices or [(...,)]:
        assert_close(y2[sl], y_ref[sl], floor_tol(rel_err(y32[sl], y_ref[sl])), f"y2{sl}")
        for k in g_ref:
            assert_close(got[k][sl], g_ref[k][sl], floor_tol(rel_err(g32[k][sl], g_ref[k][sl])), f"d{k}{sl}")


@pytest.mark.parametrize("disc,damp,afg", VARIANTS)
@pytest.mark.parametrize("S,L,P,chunk", [(3, 17, 16, 8), (2, 70, 37, 16), (2, 130, 200, 64), (2, 1, 3, 8)])
def test_linoss_reverse_matches_flipped_oracle(disc, damp, afg, S, L, P, chunk):
    variant = olin.variant_name(disc, damp)
    g = gen(S * 1000 + L * 10 + P + 5)
    steps, A, G = _linoss_params(P, g, variant)
    _linoss_check(variant, steps, A, G, crandn((S, L, P), g), crandn((S, L, P), g), afg, chunk)


@pytest.mark.parametrize("S,L,P,chunk", [(3, 45, 256, 16), (2, 70, 16, 64)])
def test_linoss_reverse_both_imex_backward_paths(S, L, P, chunk):
    """Reverse scans through the state-reversal backward (stable blocks) and the
    recompute backward (a block with one oscillator growing forward); each block of 128
    oscillators compared on its own."""
    variant = olin.variant_name("IMEX", False)
    g = gen(4343 + P)
    steps, A, _ = _linoss_params(P, g, variant)
    A = A.abs().clamp(max=2.0)
    s9 = torch.logit(torch.tensor(0.9, dtype=torch.float64))
    steps[P - 3], A[P - 3] = s9, 4.05 / 0.81
    if P > 128:
        steps[5], A[5] = s9, 3.95 / 0.81
    slices = [(..., slice(0, 128)), (..., slice(128, P))] if P > 128 else None
    _linoss_check(variant, steps, A, None, crandn((S, L, P), g), crandn((S, L, P), g), True, chunk, slices)


def test_generic_linoss_reverse_matches_flipped_oracle():
    from semambaxlinoss_b200.linoss import linoss_scan

    S, L, P, chunk = 3, 29, 24, 8
    g = gen(77)
    M = [randn(P, g, scale=0.3, mean=m) for m in (0.9, 0.0, 0.0, 0.9)]
    F1, F2, gy = crandn((S, L, P), g), crandn((S, L, P), g), crandn((S, L, P), g)

    def oracle(dtype):
        cdt = torch.complex128 if dtype == torch.float64 else torch.complex64
        ins = [m.to(dtype).clone().requires_grad_(True) for m in M]
        ins += [v.to(cdt).clone().requires_grad_(True) for v in (F1, F2)]
        y = torch.flip(olin.linoss_recurrence(*ins[:4], torch.flip(ins[4], [1]), torch.flip(ins[5], [1])), [1])
        gyc = gy.to(cdt)
        loss = (y.real * gyc.real + y.imag * gyc.imag).sum()
        return y.detach(), torch.autograd.grad(loss, ins)

    y_ref, g_ref = oracle(torch.float64)
    y32, g32 = oracle(torch.float32)
    dev = cuda()
    ins = [to32(m, dev).requires_grad_(True) for m in M] + [to32(v, dev).requires_grad_(True) for v in (F1, F2)]
    y = linoss_scan(*ins, chunk=chunk, reverse=True)
    y.backward(to32(gy, dev))
    assert_close(y, y_ref, floor_tol(rel_err(y32, y_ref)), "y2")
    for name, v, r, r32 in zip(["M11", "M12", "M21", "M22", "F1", "F2"], ins, g_ref, g32):
        assert_close(v.grad, r, floor_tol(rel_err(r32, r)), f"d{name}")


# ----------------------------------------------------------------------------- conv + SiLU

class _IdentityScan(torch.nn.Module):
    """A scan layer that returns its input, reading any layout (isolates the surround)."""

    def accepts_layout(self, layout):
        return True

    def forward(self, u, layout=None):
        return u


def _mixer_reference(params, x, d_conv, causal):
    """Float64 restatement of the reference mixer (models/mixer.py:82-99) with an
    identity scan, on (S, L, F) sequences."""
    xz = x @ params["in_proj.weight"].t()
    u, z = xz.chunk(2, dim=-1)
    pad = (d_conv - 1, 0) if causal else ((d_conv - 1) // 2, d_conv - 1 - (d_conv - 1) // 2)
    C = u.shape[-1]
    u = F.conv1d(F.pad(u.transpose(1, 2), pad), params["conv.weight"], params["conv.bias"], groups=C)
    return (F.silu(u.transpose(1, 2)) * F.silu(z)) @ params["out_proj.weight"].t()


@pytest.mark.parametrize("kind", ["reverse", "time", "time_reverse"])
@pytest.mark.parametrize("b,t,f,F_,d_conv,causal", [(2, 37, 3, 12, 4, True), (1, 5, 2, 5, 3, False),
                                                    (2, 3, 2, 6, 5, False), (1, 300, 2, 8, 4, True)])
@pytest.mark.parametrize("bf16", [False, True])
def test_conv_silu_layouts_match_reference(kind, b, t, f, F_, d_conv, causal, bf16):
    """t = 300 runs the split (quarter-sequence) convolution kernels."""
    from semambaxlinoss_b200.layout import TokenLayout
    from semambaxlinoss_b200.mixer import MambaStyleMixer

    torch.manual_seed(b * 100 + t + F_ + d_conv)
    m = MambaStyleMixer(F_, _IdentityScan(), expand=2, d_conv=d_conv, causal_conv=causal)
    if kind == "reverse":
        tok = (b * f, t)
        layout = TokenLayout.contiguous(b * f, t, reverse=True)
        to_seq, from_seq = _flip_view(b * f, t, 1)
    else:
        tok = (b, t, f)
        layout = TokenLayout.time_axis(b, t, f, reverse=kind == "time_reverse")
        to_seq, from_seq = _time_view(b, t, f, layout.reverse)
    g = gen(7 + t + f)
    x, gy = randn((*tok, F_), g), randn((*tok, F_), g)
    names = [n for n, _ in m.named_parameters()]
    params = {n: p.detach().double().clone().requires_grad_(True) for n, p in m.named_parameters()}
    xr = x.clone().requires_grad_(True)
    yr = from_seq(_mixer_reference(params, to_seq(xr), d_conv, causal))
    ref = [yr.detach()] + list(torch.autograd.grad((yr * gy).sum(), [xr] + [params[n] for n in names]))
    dev = cuda()
    m = m.to(dev)
    xd = x.float().to(dev).requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=bf16):
        y = m(xd, layout=layout)
    (y.float() * gy.float().to(dev)).sum().backward()
    out = [y.detach()] + [xd.grad] + [p.grad for _, p in m.named_parameters()]
    tol = BF16_TOL if bf16 else FP32_TOL
    for name, o, r in zip(["y", "dx"] + ["d" + n for n in names], out, ref):
        assert_close(o, r, tol, name)


# ----------------------------------------------------------------------------- blocks

def _time_cfg(ssm="selective_lru"):
    params = dict(dt_rank=2, n_real_modes=1, chunk_size=8) if ssm == "selective_lru" else \
        dict(n_heads=2, rank=1) if ssm == "selective_lru_mimo" else dict(discretization="IMEX", damping=True)
    return dict(ssm=ssm, d_state=4, d_conv=4, expand=2, bidirectional=True, ssm_params=params)


@pytest.mark.parametrize("ssm", ["selective_lru", "linoss"])
def test_mamba_block_backward_branch_without_flips(ssm):
    """MambaBlock's backward branch on the reversed layout equals the same blocks run on
    flipped copies (the reference formulation), output and every gradient."""
    from semambaxlinoss_b200.mamba_block import MambaBlock

    torch.manual_seed(3)
    dev = cuda()
    m = MambaBlock(8, _time_cfg(ssm)).to(dev)
    with torch.no_grad():
        for p in m.parameters():
            p.add_(0.05 * torch.randn_like(p))
    x = torch.randn(3, 41, 8, device=dev)
    gy = torch.randn(3, 41, 16, device=dev)

    def grads(fn):
        xx = x.clone().requires_grad_(True)
        m.zero_grad()
        y = fn(xx)
        (y * gy).sum().backward()
        return [y.detach(), xx.grad] + [p.grad.clone() for p in m.parameters()]

    def flipped(xx):
        xf, rf = m.forward_blocks[0](xx)
        xb, rb = m.backward_blocks[0](torch.flip(xx, [1]))
        return torch.cat([xf + rf, torch.flip(xb + rb, [1])], -1)

    new, old = grads(m), grads(flipped)
    for i, (a, r) in enumerate(zip(new, old)):
        assert_close(a, r, 1e-5, f"tensor {i}")


@pytest.mark.parametrize("time_ssm", ["selective_lru", "selective_lru_mimo"])
def test_tf_block_single_layout_matches_permuted_copies(time_ssm):
    """TFMambaBlock with its (b, t, f, c) activations read in place (or, for the MIMO
    time mixer, the copies it falls back to) against the same modules run through the
    reference's permute + contiguous formulation; two blocks in a row, so the second
    starts from the first's permuted view."""
    from semambaxlinoss_b200.mamba_block import TFMambaBlock, _pointwise_transpose

    torch.manual_seed(5)
    dev = cuda()
    cfg = {"model_cfg": dict(hid_feature=8, use_transpose=True, time_mixer=_time_cfg(time_ssm),
                             freq_mixer=_time_cfg("linoss"))}
    blocks = torch.nn.ModuleList([TFMambaBlock(cfg), TFMambaBlock(cfg)]).to(dev)
    with torch.no_grad():
        for p in blocks.parameters():
            p.add_(0.05 * torch.randn_like(p))
    x = torch.randn(2, 8, 21, 11, device=dev)
    gy = torch.randn(2, 8, 21, 11, device=dev)

    def reference_block(m, x):
        b, c, t, f = x.shape
        x = x.permute(0, 3, 2, 1).contiguous().view(b * f, t, c)
        x = _pointwise_transpose(m.tlinear, m.time_mamba(x)) + x
        x = x.view(b, f, t, c).permute(0, 2, 1, 3).contiguous().view(b * t, f, c)
        x = _pointwise_transpose(m.flinear, m.freq_mamba(x)) + x
        return x.view(b, t, f, c).permute(0, 3, 1, 2)

    def grads(fn):
        xx = x.clone().requires_grad_(True)
        blocks.zero_grad()
        y = fn(fn(xx, blocks[0]), blocks[1])
        (y * gy).sum().backward()
        return [y.detach(), xx.grad] + [p.grad.clone() for p in blocks.parameters()]

    new = grads(lambda v, m: m(v))
    old = grads(lambda v, m: reference_block(m, v))
    for i, (a, r) in enumerate(zip(new, old)):
        assert_close(a, r, 1e-5, f"tensor {i}")
