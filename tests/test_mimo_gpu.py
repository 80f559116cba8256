"""Complex diagonal scan and MIMO scan + readout on the GPU vs the oracle, and the
SelectiveLRUMIMO layer vs the reference's golden outputs.

Mirrors the reference's tests/test_selective_lru_mimo.py (raw complex scan parity with
gradients through the pole magnitude / phase and the drive; layer parity of outputs and
every gradient; causality, batch independence, zero input) for every input gain, rank
and option.
"""
from __future__ import annotations

import pytest
import torch

from oracle import selective_lru as oslru
from tests.parity import FP32_TOL, assert_close, crandn, cuda, floor_tol, gen, randn, rel_err, to32

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,T,N", [(3, 17, 16), (2, 40, 33), (1, 1, 5), (4, 129, 64)])
def test_complex_scan_matches_oracle(B, T, N):
    from semambaxlinoss_b200.selective_lru import selective_scan_triton

    g = gen(B + T + N)
    nu = torch.rand(B, T, N, generator=g, dtype=torch.float64) * 0.99
    theta = randn((B, T, N), g)
    Bu = crandn((B, T, N), g)
    gh = crandn((B, T, N), g)

    def run(fn, dev, dtype):
        n_ = nu.detach().clone().to(dtype).to(dev).requires_grad_(True)
        th = theta.detach().clone().to(dtype).to(dev).requires_grad_(True)
        cdt = torch.complex128 if dtype == torch.float64 else torch.complex64
        b_ = Bu.detach().clone().to(cdt).to(dev).requires_grad_(True)
        h = fn(torch.polar(n_, th), b_)
        ghd = gh.to(cdt).to(dev)
        (h.real * ghd.real + h.imag * ghd.imag).sum().backward()
        return h.detach(), n_.grad, th.grad, b_.grad

    ref = run(oslru.selective_recurrence, "cpu", torch.float64)
    r32 = run(oslru.selective_recurrence, "cpu", torch.float32)
    out = run(selective_scan_triton, cuda(), torch.float32)
    for name, o, r, q in zip(("h", "dnu", "dtheta", "dBu"), out, ref, r32):
        assert_close(o, r, floor_tol(rel_err(q, r)), name)


def _mimo_case(B, T, H, Nh, Fh, seed, with_dh):
    g = gen(seed)
    N, Fd = H * Nh, H * Fh
    lam = torch.polar(torch.rand(B, T, N, generator=g, dtype=torch.float64) * 0.98, randn((B, T, N), g))
    t = {"lr": lam.real, "li": lam.imag, "br": randn((B, T, N), g), "bi": randn((B, T, N), g),
         "cr": randn((H, Fh, Nh), g, scale=0.3), "ci": randn((H, Fh, Nh), g, scale=0.3),
         "x": randn((B, T, Fd), g), "D": randn(Fd, g)}
    gy = randn((B, T, Fd), g)
    gh = (randn((B, T, N), g), randn((B, T, N), g)) if with_dh else None
    return t, gy, gh


def _mimo_oracle(t, gy, gh, H, Nh, Fh, dtype):
    ins = {k: v.to(dtype).clone().requires_grad_(True) for k, v in t.items()}
    y, hr, hi = oslru.mimo_scan_readout(ins["lr"], ins["li"], ins["br"], ins["bi"], ins["cr"], ins["ci"],
                                        ins["x"], ins["D"], H, Nh, Fh)
    loss = (y * gy.to(dtype)).sum()
    if gh is not None:
        loss = loss + (hr * gh[0].to(dtype) + hi * gh[1].to(dtype)).sum()
    names = list(ins)
    return (y.detach(), hr.detach(), hi.detach()), dict(zip(names, torch.autograd.grad(loss, [ins[k] for k in names])))


@pytest.mark.parametrize("B,T,H,Nh,Fh,with_dh", [(3, 19, 1, 16, 8, False), (2, 70, 2, 8, 32, True),
                                                 (2, 33, 8, 16, 32, True), (1, 5, 3, 5, 7, False)])
def test_fused_mimo_matches_oracle(B, T, H, Nh, Fh, with_dh):
    from semambaxlinoss_b200.selective_lru import fused_selective_lru_mimo

    t, gy, gh = _mimo_case(B, T, H, Nh, Fh, B * T + H + Nh + Fh, with_dh)
    outs_ref, g_ref = _mimo_oracle(t, gy, gh, H, Nh, Fh, torch.float64)
    outs32, g32 = _mimo_oracle(t, gy, gh, H, Nh, Fh, torch.float32)
    dev = cuda()
    ins = {k: to32(v, dev).requires_grad_(True) for k, v in t.items()}
    y, hr, hi = fused_selective_lru_mimo(ins["lr"], ins["li"], ins["br"], ins["bi"], ins["cr"], ins["ci"],
                                         ins["x"], ins["D"], H, Nh, Fh)
    loss = (y * to32(gy, dev)).sum()
    if gh is not None:
        loss = loss + (hr * to32(gh[0], dev) + hi * to32(gh[1], dev)).sum()
    loss.backward()
    for name, o, r, q in zip(("y", "h_re", "h_im"), (y, hr, hi), outs_ref, outs32):
        assert_close(o, r, floor_tol(rel_err(q, r)), name)
    for k in g_ref:
        assert_close(ins[k].grad, g_ref[k], floor_tol(rel_err(g32[k], g_ref[k])), f"d{k}")


def test_module_matches_golden(golden):
    """SelectiveLRUMIMO with the reference's parameters reproduces the reference's float64
    outputs and every gradient (gamma / mamba / zoh / none gains, rank 0-2, envelope,
    detune, rate scale)."""
    from semambaxlinoss_b200.selective_lru import SelectiveLRUMIMO

    dev = cuda()
    for name, rec in golden("mimo").items():
        m = SelectiveLRUMIMO(**rec["config"])
        m.load_state_dict({k: v.float() for k, v in rec["state_dict"].items()})
        m = m.to(dev)
        x = to32(rec["x"], dev).requires_grad_(True)
        y = m(x)
        (y * to32(rec["grad_y"], dev)).sum().backward()
        assert_close(y, rec["y"], FP32_TOL, f"{name} y")
        assert_close(x.grad, rec["grad_x"], FP32_TOL, f"{name} dx")
        for n, p in m.named_parameters():
            assert_close(p.grad, rec["param_grads"][n], FP32_TOL, f"{name} d{n}")


def test_module_properties():
    from semambaxlinoss_b200.selective_lru import SelectiveLRUMIMO

    torch.manual_seed(0)
    m = SelectiveLRUMIMO(in_features=8, state_dim=16, n_heads=2, rank=2).to(cuda()).eval()
    with torch.no_grad():
        for p in m.parameters():
            p.add_(0.1 * torch.randn_like(p))
        x = torch.randn(1, 10, 8, device="cuda")
        y = m(x)
        xp = x.clone()
        xp[:, 5:] += torch.randn_like(xp[:, 5:])
        yp = m(xp)
        assert torch.allclose(y[:, :5], yp[:, :5], atol=1e-6)
        assert not torch.allclose(y[:, 5:], yp[:, 5:])
        x0, x1 = torch.randn(1, 6, 8, device="cuda"), torch.randn(1, 6, 8, device="cuda")
        assert torch.allclose(m(torch.cat([x0, x1])), torch.cat([m(x0), m(x1)]), atol=1e-6)
        z = m(torch.zeros(2, 5, 8, device="cuda"))
        assert torch.allclose(z, torch.zeros_like(z), atol=1e-7)
