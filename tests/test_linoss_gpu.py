"""LinOSS scan on the GPU vs the oracle (float64 restatement of the reference).

Mirrors the reference's tests/test_linoss.py (parity of forward and all gradients at the
reference's shapes and tolerances, causality, batch independence, zero input) and adds
chunk-boundary edge cases, every constraint branch, determinism, and full-size
property checks at the 404-sequence x 321-step, P = 256 shape.
"""
from __future__ import annotations

import pytest
import torch

from oracle import linoss as olin
from tests.parity import FP32_TOL, assert_close, crandn, cuda, floor_tol, gen, randn, rel_err, to32

pytestmark = pytest.mark.gpu

VARIANTS = [("IMEX", True, True), ("IMEX", True, False), ("IMEX", False, True), ("IM", False, True)]


def _variant(disc, damp):
    return olin.variant_name(disc, damp)


def _params(P, g, variant):
    steps = randn(P, g, scale=1.2)
    if variant == "DAMPED_IMEX":
        A = randn(P, g, scale=1.5, mean=0.5)
        G = randn(P, g, scale=1.0, mean=0.2)
    else:
        A = randn(P, g, scale=1.0, mean=0.3)  # about a third of the oscillators at A = 0
        G = None
    return steps, A, G


def _oracle_fused(variant, steps, A, G, Bu, gy, a_from_g, dtype=torch.float64):
    cdt = torch.complex128 if dtype == torch.float64 else torch.complex64

    def cast(t):
        return t.to(cdt if t.is_complex() else dtype)

    ins = [cast(t).clone().requires_grad_(True) if t is not None else None for t in (steps, A, G, Bu)]
    y2 = olin.linoss_scan_fused(variant, *ins, a_from_g=a_from_g)
    gy = cast(gy)
    loss = (y2.real * gy.real + y2.imag * gy.imag).sum()
    req = [t for t in ins if t is not None]
    grads = torch.autograd.grad(loss, req)
    out = dict(zip([n for n, t in zip(("steps", "A", "G", "Bu"), ins) if t is not None], grads))
    return y2.detach(), out


def _tolerances(variant, steps, A, G, Bu, gy, a_from_g, y_ref, g_ref):
    """Per-tensor tolerance: max(1e-4, 2 x error of the reference algorithm in fp32)."""
    y32, g32 = _oracle_fused(variant, steps, A, G, Bu, gy, a_from_g, dtype=torch.float32)
    tol = {"y2": floor_tol(rel_err(y32, y_ref))}
    for k in g_ref:
        tol[k] = floor_tol(rel_err(g32[k], g_ref[k]))
    return tol


def _gpu_fused(variant, steps, A, G, Bu, gy, a_from_g, chunk):
    from semambaxlinoss_b200.linoss import linoss_scan_fused

    dev = cuda()
    ins = [to32(t, dev).requires_grad_(True) if t is not None else None for t in (steps, A, G, Bu)]
    y2 = linoss_scan_fused(variant, *ins, a_from_g=a_from_g, chunk=chunk)
    y2.backward(to32(gy, dev))
    names = ("steps", "A", "G", "Bu")
    return y2.detach(), {n: t.grad for n, t in zip(names, ins) if t is not None}


@pytest.mark.parametrize("disc,damp,afg", VARIANTS)
@pytest.mark.parametrize("S,L,P,chunk", [(3, 17, 16, 8), (2, 40, 5, 16), (1, 33, 37, 8),
                                         (4, 64, 32, 64), (2, 1, 3, 8), (5, 130, 24, 64)])
def test_fused_scan_matches_oracle(disc, damp, afg, S, L, P, chunk):
    variant = _variant(disc, damp)
    g = gen(S * 1000 + L * 10 + P)
    steps, A, G = _params(P, g, variant)
    Bu = crandn((S, L, P), g)
    gy = crandn((S, L, P), g)
    y_ref, g_ref = _oracle_fused(variant, steps, A, G, Bu, gy, afg)
    tol = _tolerances(variant, steps, A, G, Bu, gy, afg, y_ref, g_ref)
    y_gpu, g_gpu = _gpu_fused(variant, steps, A, G, Bu, gy, afg, chunk)
    assert_close(y_gpu, y_ref, tol["y2"], "y2")
    for k in g_ref:
        assert_close(g_gpu[k], g_ref[k], tol[k], f"d{k}")


@pytest.mark.parametrize("S,L,P,chunk", [(3, 45, 256, 16), (2, 70, 16, 64)])
def test_imex_unstable_oscillators_take_the_recompute_backward(S, L, P, chunk):
    """The IMEX backward runs the state backwards in time only for oscillators whose
    transition has both eigenvalues on the unit circle; a thread block holding one with
    step^2 A above 4 (growing forward) goes to the recompute backward. P = 256: of the two
    128-oscillator blocks per sequence, the first (stable, one oscillator at step^2 A =
    3.95) takes the reversal, the second (one at step^2 A = 4.05) the recompute; P = 16:
    every block falls back. Each block's oscillators are compared on their own, since the
    growing one dominates any norm over all of them."""
    variant = _variant("IMEX", False)
    g = gen(4242 + P)
    steps, A, _ = _params(P, g, variant)
    A = A.abs().clamp(max=2.0)  # step^2 A <= 2 elsewhere
    s9 = torch.logit(torch.tensor(0.9, dtype=torch.float64))
    bad = P - 3
    steps[bad], A[bad] = s9, 4.05 / 0.81
    if P > 128:
        steps[5], A[5] = s9, 3.95 / 0.81
    Bu = crandn((S, L, P), g)
    gy = crandn((S, L, P), g)
    y_ref, g_ref = _oracle_fused(variant, steps, A, None, Bu, gy, True)
    y32, g32 = _oracle_fused(variant, steps, A, None, Bu, gy, True, dtype=torch.float32)
    y_gpu, g_gpu = _gpu_fused(variant, steps, A, None, Bu, gy, True, chunk)
    for lo, hi in ((0, min(P, 128)), (128, P)) if P > 128 else ((0, P),):
        sl = (..., slice(lo, hi))
        assert_close(y_gpu[sl], y_ref[sl], floor_tol(rel_err(y32[sl], y_ref[sl])), f"y2[{lo}:{hi}]")
        for k in g_ref:
            tol = floor_tol(rel_err(g32[k][sl], g_ref[k][sl]))
            assert_close(g_gpu[k][sl], g_ref[k][sl], tol, f"d{k}[{lo}:{hi}]")


@pytest.mark.parametrize("S,L,P,chunk", [(3, 17, 16, 8), (2, 29, 64, 16), (1, 100, 7, 64)])
def test_generic_scan_matches_oracle(S, L, P, chunk):
    from semambaxlinoss_b200.linoss import linoss_scan

    g = gen(7 + S + L + P)
    M = [randn(P, g, scale=0.3, mean=m) for m in (0.9, 0.0, 0.0, 0.9)]
    F1, F2, gy = crandn((S, L, P), g), crandn((S, L, P), g), crandn((S, L, P), g)
    ins = [t.clone().requires_grad_(True) for t in (*M, F1, F2)]
    y_ref = olin.linoss_recurrence(*ins)
    loss = (y_ref.real * gy.real + y_ref.imag * gy.imag).sum()
    g_ref = torch.autograd.grad(loss, ins)
    dev = cuda()
    gins = [to32(t, dev).requires_grad_(True) for t in (*M, F1, F2)]
    y = linoss_scan(*gins, chunk=chunk)
    y.backward(to32(gy, dev))
    assert_close(y, y_ref, FP32_TOL, "Y2")
    for name, a, b in zip(("M11", "M12", "M21", "M22", "F1", "F2"), gins, g_ref):
        assert_close(a.grad, b, FP32_TOL, f"d{name}")


def test_generic_scan_matches_golden(golden):
    """Against the reference's own _linoss_recurrence outputs (golden fixture)."""
    from semambaxlinoss_b200.linoss import linoss_scan_triton

    rec = golden("linoss")["linoss_recurrence"]
    dev = cuda()
    ins = [to32(t, dev).requires_grad_(True) for t in (*rec["M"], rec["F1"], rec["F2"])]
    y = linoss_scan_triton(*ins, chunk=8)
    y.backward(to32(rec["grad_Y2"], dev))
    assert_close(y, rec["Y2"], FP32_TOL, "Y2")
    for a, b in zip(ins, rec["grads"]):
        assert_close(a.grad, b, FP32_TOL, "grad")


def _load_module(rec, chunk=8):
    from semambaxlinoss_b200.linoss import LinOSS

    cfg = rec["config"]
    m = LinOSS(cfg["in_features"], cfg["state_dim"], cfg["discretization"], cfg["damping"],
               a_from_g=cfg["a_from_g"], chunk_size=chunk)
    m.load_state_dict({k: v.float() for k, v in rec["state_dict"].items()})
    return m.to(cuda())


def _module_fp32_tolerances(rec):
    """Floors from the reference algorithm evaluated in fp32 (oracle in float32) against
    the reference's own float64 outputs."""
    cfg = rec["config"]
    params = {k: v.float().clone().requires_grad_(True) for k, v in rec["state_dict"].items()}
    x = rec["x"].float().clone().requires_grad_(True)
    y = olin.linoss_forward(params, x, cfg["discretization"], cfg["damping"], cfg["a_from_g"])
    names = list(params)
    grads = torch.autograd.grad((y * rec["grad_y"].float()).sum(), [x] + [params[n] for n in names])
    tol = {"y": floor_tol(rel_err(y, rec["y"])), "x": floor_tol(rel_err(grads[0], rec["grad_x"]))}
    for n, g in zip(names, grads[1:]):
        tol[n] = floor_tol(rel_err(g, rec["param_grads"][n]))
    return tol


@pytest.mark.parametrize("chunk", [8, 64])
def test_module_matches_golden(golden, chunk):
    """LinOSS layer with the reference's parameters reproduces the reference's float64
    outputs and every gradient (all variants)."""
    for name, rec in golden("linoss").items():
        if name == "linoss_recurrence":
            continue
        m = _load_module(rec, chunk)
        x = to32(rec["x"], cuda()).requires_grad_(True)
        y = m(x)
        y.backward(to32(rec["grad_y"], cuda()))
        tol = _module_fp32_tolerances(rec)
        assert_close(y, rec["y"], tol["y"], f"{name} y")
        assert_close(x.grad, rec["grad_x"], tol["x"], f"{name} dx")
        for n, p in m.named_parameters():
            assert_close(p.grad, rec["param_grads"][n], tol[n], f"{name} d{n}")


@pytest.mark.parametrize("disc,damp", [("IMEX", True), ("IMEX", False), ("IM", False)])
def test_module_properties(disc, damp):
    """Causality, batch independence, zero input -> zero output, determinism."""
    from semambaxlinoss_b200.linoss import LinOSS

    torch.manual_seed(0)
    m = LinOSS(in_features=4, state_dim=16, discretization=disc, damping=damp).to(cuda()).eval()
    x = torch.randn(1, 12, 4, device="cuda")
    with torch.no_grad():
        y = m(x)
        xp = x.clone()
        xp[:, 6:] += torch.randn_like(xp[:, 6:])
        yp = m(xp)
        assert torch.allclose(y[:, :6], yp[:, :6], atol=1e-6)
        assert not torch.allclose(y[:, 6:], yp[:, 6:])
        x0, x1 = torch.randn(1, 6, 4, device="cuda"), torch.randn(1, 6, 4, device="cuda")
        assert torch.allclose(m(torch.cat([x0, x1])), torch.cat([m(x0), m(x1)]), atol=1e-6)
        z = m(torch.zeros(2, 5, 4, device="cuda"))
        assert torch.equal(z, torch.zeros_like(z))
    xg = torch.randn(3, 50, 4, device="cuda", requires_grad=True)
    outs = []
    for _ in range(2):
        m.zero_grad()
        xg.grad = None
        m(xg).square().sum().backward()
        outs.append([xg.grad.clone()] + [p.grad.clone() for p in m.parameters()])
    for a, b in zip(*outs):
        assert torch.equal(a, b), "backward is not bitwise deterministic"


def test_empty_and_errors():
    from semambaxlinoss_b200 import _lib
    from semambaxlinoss_b200.linoss import linoss_scan, linoss_scan_fused

    dev = cuda()
    P = 8
    st, A = torch.randn(P, device=dev), torch.rand(P, device=dev)
    for shape in [(0, 5, P), (2, 0, P)]:
        Bu = torch.zeros(shape, dtype=torch.complex64, device=dev, requires_grad=True)
        y = linoss_scan_fused("IMEX", st.requires_grad_(True), A, None, Bu)
        assert y.shape == shape
        y.sum().abs().backward()
    with pytest.raises(RuntimeError):
        linoss_scan_fused("IMEX", st.cpu(), A.cpu(), None, torch.zeros(1, 2, P, dtype=torch.complex64))
    with pytest.raises(ValueError):
        F = torch.zeros(1, 4, P, dtype=torch.complex64, device=dev)
        linoss_scan(A, A, A, A, F, torch.zeros(1, 5, P, dtype=torch.complex64, device=dev))
    with pytest.raises(_lib.SemxError):
        F = torch.zeros(1, 4, P, dtype=torch.complex64, device=dev)
        linoss_scan(A, A, A, A, F, F, chunk=12)


def test_full_size_linoss_workload_properties():
    """The LinOSS-IMEX workload shapes (time pass 404 x 321, frequency pass 1284 x 101, P = 256):
    a sequence slice agrees with the float64 oracle, the forward is linear in Bu, and
    forward + backward are bitwise deterministic."""
    from semambaxlinoss_b200.linoss import linoss_scan_fused

    dev = cuda()
    P = 256
    g = gen(0)
    steps = randn(P, g)
    A = torch.relu(randn(P, g))
    for S, L in [(404, 321), (1284, 101)]:
        Bu = crandn((S, L, P), g)
        gy = crandn((S, L, P), g)
        st32, A32 = to32(steps, dev).requires_grad_(True), to32(A, dev).requires_grad_(True)
        Bu32 = to32(Bu, dev).requires_grad_(True)
        y = linoss_scan_fused("IMEX", st32, A32, None, Bu32)
        y.backward(to32(gy, dev))
        sl = [0, S // 2, S - 1]
        y_ref, g_ref = _oracle_fused("IMEX", steps, A, None, Bu[sl], gy[sl], True)
        assert_close(y[sl], y_ref, FP32_TOL, "y2 slice")
        assert_close(Bu32.grad[sl], g_ref["Bu"], FP32_TOL, "dBu slice")
        # determinism (bitwise) of outputs and reductions
        st2, A2 = st32.detach().clone().requires_grad_(True), A32.detach().clone().requires_grad_(True)
        Bu2 = Bu32.detach().clone().requires_grad_(True)
        y2 = linoss_scan_fused("IMEX", st2, A2, None, Bu2)
        y2.backward(to32(gy, dev))
        assert torch.equal(y, y2) and torch.equal(Bu32.grad, Bu2.grad)
        assert torch.equal(st32.grad, st2.grad) and torch.equal(A32.grad, A2.grad)
        # linearity in Bu (fixed parameters)
        with torch.no_grad():
            B1 = Bu32.detach()
            B2 = to32(crandn((S, L, P), g), dev)
            lhs = linoss_scan_fused("IMEX", st32, A32, None, B1 + B2)
            rhs = linoss_scan_fused("IMEX", st32, A32, None, B1) + linoss_scan_fused(
                "IMEX", st32, A32, None, B2)
            assert_close(lhs, rhs, 1e-4, "linearity")
        del y, y2, Bu32, Bu2


@pytest.mark.parametrize("rows,H,P", [(700, 256, 16), (1100, 300, 32), (37, 5, 3), (513, 64, 8), (1, 7, 1)])
def test_fused_readout_matches_reference(rows, H, P):
    """semx_linoss_readout (the LinOSS layer's y = Re(C y2) + D x, models/linoss/linoss.py:
    118-120) against the float64 expression: output, dy2, dx, dC, dD, and the same bits on
    a second call (fixed reduction order)."""
    from semambaxlinoss_b200.linoss.linoss import _Readout

    g = gen(rows * 3 + H + P)
    y2 = crandn((rows, P), g)
    x = randn((rows, H), g)
    C = randn((H, P, 2), g, scale=0.3)
    D = randn(H, g)
    gy = randn((rows, H), g)
    ins = [t.clone().requires_grad_(True) for t in (y2, x, C, D)]
    Cc = torch.complex(ins[2][..., 0], ins[2][..., 1])
    ref = torch.einsum("fn,bn->bf", Cc, ins[0]).real + ins[1] * ins[3]
    ref_g = torch.autograd.grad((ref * gy).sum(), ins)
    dev = cuda()
    got_in = [to32(t, dev).requires_grad_(True) for t in (y2, x, C, D)]

    def run():
        for t in got_in:
            t.grad = None
        y = _Readout.apply(*got_in)
        (y * to32(gy, dev)).sum().backward()
        return [y.detach()] + [t.grad.clone() for t in got_in]

    out = run()
    assert_close(out[0], ref, FP32_TOL, "y")
    for name, o, r in zip(["dy2", "dx", "dC", "dD"], out[1:], ref_g):
        assert_close(o, r, FP32_TOL, name)
    for a, b in zip(out[2:], run()[2:]):
        assert torch.equal(a, b)


def test_fused_readout_empty_rows():
    from semambaxlinoss_b200.linoss.linoss import _Readout

    dev = cuda()
    y2 = torch.zeros(0, 4, dtype=torch.complex64, device=dev, requires_grad=True)
    x = torch.zeros(0, 6, device=dev, requires_grad=True)
    C = torch.randn(6, 4, 2, device=dev, requires_grad=True)
    D = torch.randn(6, device=dev, requires_grad=True)
    y = _Readout.apply(y2, x, C, D)
    y.sum().backward()
    assert y.shape == (0, 6)
    assert torch.equal(C.grad, torch.zeros_like(C)) and torch.equal(D.grad, torch.zeros_like(D))
