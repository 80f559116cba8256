"""Selective-LRU SISO scan on the GPU vs the oracle (float64 restatement of the
reference's materialised path).

Mirrors the reference's tests/test_selective_lru.py (direct fused-op parity of forward and
all input gradients at its (B, T, C, N, chunk) shapes, module parity, causality, batch
independence, zero input) for every input gain and option, and adds: the real
specialisation, N not a multiple of 4, N = 32, channel counts that need one
and several thread-block clusters, final-state gradients, determinism, and full-size
property checks on the 404 x 321, C = 256, N = 16 real scan.
"""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle import selective_lru as oslru
from tests.parity import FP32_TOL, assert_close, cuda, floor_tol, gen, randn, rel_err, to32

pytestmark = pytest.mark.gpu

NAMES = ["dnu", "dth", "a", "om", "Bre", "Bim", "Cre", "Cim", "x", "D", "g", "s", "h0r", "h0i"]


def _inputs(B, T, C, N, seed, opts):
    g = gen(seed)
    t = {
        "dnu": F.softplus(randn((B, T, C), g)) * 0.3,
        "dth": randn((B, T, C), g),
        "a": torch.exp(randn((C, N), g, scale=0.5)),
        "om": randn((C, N), g),
        "Bre": randn((B, T, N), g), "Bim": randn((B, T, N), g),
        "Cre": randn((B, T, N), g), "Cim": randn((B, T, N), g),
        "x": randn((B, T, C), g), "D": randn(C, g),
        "g": randn((C, N), g, scale=0.1) if "env" in opts else None,
        "s": (1.0 + randn((C, N), g, scale=0.3)) if "detune" in opts else None,
        "h0r": randn((B, C, N), g) if "h0" in opts else None,
        "h0i": randn((B, C, N), g) if "h0" in opts else None,
    }
    gy = randn((B, T, C), g)
    ghf = (randn((B, C, N), g), randn((B, C, N), g)) if "hf" in opts else None
    return t, gy, ghf


def _oracle(t, gy, ghf, gain, dtype=torch.float64):
    ins = {k: (v.to(dtype).clone().requires_grad_(True) if v is not None else None) for k, v in t.items()}
    out = oslru.selective_lru_op(
        ins["dnu"], ins["dth"], ins["a"], ins["om"], ins["Bre"], ins["Bim"], ins["Cre"],
        ins["Cim"], ins["x"], ins["D"], ins["g"], ins["s"], ins["h0r"], ins["h0i"],
        input_gain=gain, return_final_state=ghf is not None)
    if ghf is not None:
        y, hf = out
        loss = (y * gy.to(dtype)).sum() + (hf.real * ghf[0].to(dtype) + hf.imag * ghf[1].to(dtype)).sum()
    else:
        y = out
        loss = (y * gy.to(dtype)).sum()
    req = [k for k in NAMES if ins[k] is not None]
    grads = dict(zip(req, torch.autograd.grad(loss, [ins[k] for k in req])))
    return y.detach(), grads


def _gpu(t, gy, ghf, gain, chunk):
    from semambaxlinoss_b200.selective_lru import fused_selective_lru

    dev = cuda()
    ins = {k: (to32(v, dev).requires_grad_(True) if v is not None else None) for k, v in t.items()}
    y, hf_re, hf_im = fused_selective_lru(
        ins["dnu"], ins["dth"], ins["a"], ins["om"], ins["Bre"], ins["Bim"], ins["Cre"],
        ins["Cim"], ins["x"], ins["D"], ins["g"], ins["s"], ins["h0r"], ins["h0i"],
        block_t=chunk, want_final_state=ghf is not None, input_gain=gain)
    loss = (y * to32(gy, dev)).sum()
    if ghf is not None:
        loss = loss + (hf_re * to32(ghf[0], dev) + hf_im * to32(ghf[1], dev)).sum()
    loss.backward()
    return y.detach(), {k: v.grad for k, v in ins.items() if v is not None}


def _check(t, gy, ghf, gain, chunk):
    y_ref, g_ref = _oracle(t, gy, ghf, gain)
    y32, g32 = _oracle(t, gy, ghf, gain, dtype=torch.float32)
    y, grads = _gpu(t, gy, ghf, gain, chunk)
    assert_close(y, y_ref, floor_tol(rel_err(y32, y_ref)), "y")
    for k, ref in g_ref.items():
        assert_close(grads[k], ref, floor_tol(rel_err(g32[k], ref)), f"d{k}")


@pytest.mark.parametrize("gain", ["gamma", "mamba", "zoh"])
@pytest.mark.parametrize("B,T,C,N,chunk", [(2, 19, 3, 4, 16), (2, 40, 5, 4, 16), (3, 16, 4, 8, 16),
                                           (1, 33, 2, 4, 8)])
def test_fused_op_matches_oracle_reference_shapes(B, T, C, N, chunk, gain):
    t, gy, ghf = _inputs(B, T, C, N, B + T + C + N, ())
    _check(t, gy, ghf, gain, chunk)


@pytest.mark.parametrize("gain", ["gamma", "mamba", "zoh"])
@pytest.mark.parametrize("opts", [("env",), ("detune",), ("h0", "hf"), ("env", "detune", "h0", "hf")])
def test_fused_op_options(gain, opts):
    t, gy, ghf = _inputs(2, 23, 6, 8, 77, opts)
    _check(t, gy, ghf, gain, 8)


@pytest.mark.parametrize("B,T,C,N,chunk", [
    (2, 21, 40, 16, 8),     # NG = 4, two channel blocks in one cluster
    (1, 9, 7, 13, 4),       # N not a multiple of 4
    (2, 12, 20, 32, 12),    # N = 32 (NG = 8)
    (1, 17, 300, 16, 16),   # 10 channel blocks: two clusters, cross-cluster sum
    (2, 1, 5, 4, 4),        # single step
    (2, 70, 24, 16, 48),    # chunk of three staged tiles (pass 1 forwards, pass 2 backwards)
    (1, 45, 9, 8, 20),      # chunk of a full and a partial tile, ragged last chunk
])
def test_fused_op_edge_shapes(B, T, C, N, chunk):
    t, gy, ghf = _inputs(B, T, C, N, 1000 + C + N, ("env", "detune", "h0", "hf"))
    _check(t, gy, ghf, "gamma", chunk)


@pytest.mark.parametrize("gain", ["gamma", "mamba", "zoh"])
@pytest.mark.parametrize("B,T,C,N,chunk", [(2, 19, 3, 4, 16), (3, 70, 40, 16, 32), (1, 9, 7, 13, 4)])
def test_real_op_matches_oracle(B, T, C, N, chunk, gain):
    from semambaxlinoss_b200.selective_lru import fused_selective_lru_real

    g = gen(B * 31 + T + C + N)
    dnu = F.softplus(randn((B, T, C), g, mean=-1.0))
    a = torch.exp(torch.rand(C, N, generator=g, dtype=torch.float64) * 2.7)
    Bt, Ct = randn((B, T, N), g, scale=0.25), randn((B, T, N), g, scale=0.25)
    x, D, h0 = randn((B, T, C), g), randn(C, g), randn((B, C, N), g)
    gy, ghf = randn((B, T, C), g), randn((B, C, N), g)

    def run_oracle(dtype):
        ins = [v.to(dtype).clone().requires_grad_(True) for v in (dnu, a, Bt, Ct, x, D, h0)]
        y, hf = oslru.selective_lru_real_op(*ins[:6], input_gain=gain, h0=ins[6], return_final_state=True)
        loss = (y * gy.to(dtype)).sum() + (hf * ghf.to(dtype)).sum()
        return y.detach(), torch.autograd.grad(loss, ins)

    y_ref, g_ref = run_oracle(torch.float64)
    y32, g32 = run_oracle(torch.float32)
    dev = cuda()
    ins = [to32(v, dev).requires_grad_(True) for v in (dnu, a, Bt, Ct, x, D, h0)]
    y, hf = fused_selective_lru_real(*ins[:6], input_gain=gain, h0=ins[6], block_t=chunk,
                                     want_final_state=True)
    ((y * to32(gy, dev)).sum() + (hf * to32(ghf, dev)).sum()).backward()
    assert_close(y, y_ref, floor_tol(rel_err(y32, y_ref)), "y")
    for name, a_, r, r32 in zip(("dnu", "a", "B", "C", "x", "D", "h0"), ins, g_ref, g32):
        assert_close(a_.grad, r, floor_tol(rel_err(r32, r)), f"d{name}")


def _module_from_golden(rec, chunk):
    from semambaxlinoss_b200.selective_lru import SelectiveLRU

    cfg = dict(rec["config"])
    m = SelectiveLRU(chunk_size=chunk, **cfg)
    m.load_state_dict({k: v.float() for k, v in rec["state_dict"].items()})
    return m.to(cuda())


@pytest.mark.parametrize("chunk", [4, 16])
def test_module_matches_golden(golden, chunk):
    """SelectiveLRU with the reference's parameters reproduces the reference's float64
    outputs, final state and every gradient (all gains and options)."""
    dev = cuda()
    for name, rec in golden("selective_lru").items():
        m = _module_from_golden(rec, chunk)
        fk = rec["forward_kwargs"]
        x = to32(rec["x"], dev).requires_grad_(True)
        h0 = rec.get("h_init")
        out = m(x, h_init=None if h0 is None else h0.to(torch.complex64).to(dev),
                rate_scale=fk.get("rate_scale"), return_final_state=fk.get("return_final_state", False))
        if isinstance(out, tuple):
            y, hf = out
            ghf = rec["grad_hf"].to(torch.complex64).to(dev)
            loss = (y * to32(rec["grad_y"], dev)).sum() + (hf.real * ghf.real + hf.imag * ghf.imag).sum()
            assert_close(hf, rec["hf"], FP32_TOL, f"{name} hf")
        else:
            y = out
            loss = (y * to32(rec["grad_y"], dev)).sum()
        loss.backward()
        assert_close(y, rec["y"], FP32_TOL, f"{name} y")
        assert_close(x.grad, rec["grad_x"], FP32_TOL, f"{name} dx")
        for n, p in m.named_parameters():
            assert_close(p.grad, rec["param_grads"][n], FP32_TOL, f"{name} d{n}")


@pytest.mark.parametrize("gain", ["gamma", "mamba", "zoh"])
def test_module_properties(gain):
    from semambaxlinoss_b200.selective_lru import SelectiveLRU

    torch.manual_seed(0)
    m = SelectiveLRU(d_model=8, d_state=4, input_gain=gain).to(cuda()).eval()
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
    xg = torch.randn(3, 40, 8, device="cuda", requires_grad=True)
    outs = []
    for _ in range(2):
        m.zero_grad()
        xg.grad = None
        m(xg).square().sum().backward()
        outs.append([xg.grad.clone()] + [p.grad.clone() for p in m.parameters()])
    for a_, b_ in zip(*outs):
        assert torch.equal(a_, b_), "backward is not bitwise deterministic"


def test_full_size_real_scan_properties():
    """The real scan at 404 x 321, C = 256, N = 16 with the mamba gain: a sequence slice agrees
    with the float64 oracle and forward + backward are bitwise deterministic."""
    from semambaxlinoss_b200.selective_lru import fused_selective_lru_real

    dev = cuda()
    S, L, C, N = 404, 321, 256, 16
    g = gen(0)
    x = randn((S, L, C), g, dtype=torch.float32)
    dnu = F.softplus(randn((S, L, C), g, dtype=torch.float32, scale=0.5, mean=-2.0))
    a = torch.exp(torch.log(torch.rand(C, N, generator=g) * 15 + 1))
    Bt = randn((S, L, N), g, dtype=torch.float32, scale=0.25)
    Ct = randn((S, L, N), g, dtype=torch.float32, scale=0.25)
    D = randn(C, g, dtype=torch.float32)
    gy = randn((S, L, C), g, dtype=torch.float32)
    res = []
    for _ in range(2):
        ins = [v.to(dev).requires_grad_(True) for v in (dnu, a, Bt, Ct, x, D)]
        y, _ = fused_selective_lru_real(*ins, input_gain="mamba")
        y.backward(gy.to(dev))
        res.append([y.detach()] + [v.grad for v in ins])
    for a_, b_ in zip(*res):
        assert torch.equal(a_, b_)
    sl = [0, 201, 403]
    ins = [v.double().clone().requires_grad_(True) for v in (dnu[sl], a, Bt[sl], Ct[sl], x[sl], D)]
    y_ref = oslru.selective_lru_real_op(*ins, input_gain="mamba")
    y_ref.backward(gy[sl].double())
    assert_close(res[0][0][sl], y_ref, FP32_TOL, "y slice")
    for name, i in (("dnu", 1), ("B", 3), ("C", 4), ("x", 5)):
        assert_close(res[0][i][sl], ins[i - 1].grad, FP32_TOL, f"d{name} slice")


def test_full_size_complex_gamma_scan_slices():
    """The generator's time-axis scan at its full shape: complex selective-LRU with the
    gamma gain over 1600 sequences x 321 steps, C = 256 channels, N = 16 modes
    (x ~ N(0,1), delta_nu = softplus(N(-2, 0.5)), delta_theta ~ N(0, 0.1^2),
    a ~ U(1, 16), omega ~ N(0, 1), B, C ~ N(0, 1/16) per part, D ~ N(0,1)). The upstream
    gradient is zero outside four sequences, so every gradient, the parameter sums
    included, comes from those sequences alone and is checked against the float64
    oracle run on them (fp32 tolerance, raised to twice the fp32 oracle's own error where
    that is larger); the other sequences' channel gradients must be exactly zero."""
    from semambaxlinoss_b200.selective_lru import fused_selective_lru

    dev = cuda()
    S, L, C, N = 1600, 321, 256, 16
    gd = torch.Generator(device=dev).manual_seed(7)

    def rn(*shape, scale=1.0, mean=0.0):
        return torch.randn(*shape, generator=gd, device=dev) * scale + mean

    t = {
        "dnu": F.softplus(rn(S, L, C, scale=0.5, mean=-2.0)),
        "dth": rn(S, L, C, scale=0.1),
        "a": torch.rand(C, N, generator=gd, device=dev) * 15.0 + 1.0,
        "om": rn(C, N),
        "Bre": rn(S, L, N, scale=0.25), "Bim": rn(S, L, N, scale=0.25),
        "Cre": rn(S, L, N, scale=0.25), "Cim": rn(S, L, N, scale=0.25),
        "x": rn(S, L, C), "D": rn(C),
    }
    sl = [0, 533, 1066, S - 1]
    mask = torch.zeros(S, 1, 1, device=dev)
    mask[sl] = 1.0
    gy = rn(S, L, C) * mask
    ins = {k: v.clone().requires_grad_(True) for k, v in t.items()}
    y, _, _ = fused_selective_lru(ins["dnu"], ins["dth"], ins["a"], ins["om"], ins["Bre"], ins["Bim"],
                                  ins["Cre"], ins["Cim"], ins["x"], ins["D"], input_gain="gamma")
    y.backward(gy)
    rest = torch.ones(S, dtype=torch.bool, device=dev)
    rest[sl] = False
    for k in ("dnu", "dth", "x", "Bre", "Bim", "Cre", "Cim"):
        assert ins[k].grad[rest].abs().max().item() == 0.0, k
    per_seq = ("dnu", "dth", "Bre", "Bim", "Cre", "Cim", "x")
    sub = {k: (v[sl] if k in per_seq else v).detach().cpu() for k, v in t.items()}
    sub.update(g=None, s=None, h0r=None, h0i=None)
    y_ref, g_ref = _oracle(sub, gy[sl].cpu(), None, "gamma")
    y32, g32 = _oracle(sub, gy[sl].cpu(), None, "gamma", dtype=torch.float32)
    assert_close(y[sl], y_ref, floor_tol(rel_err(y32, y_ref)), "y slice")
    for k, ref in g_ref.items():
        got = ins[k].grad[sl] if k in per_seq else ins[k].grad
        assert_close(got, ref, floor_tol(rel_err(g32[k], ref)), f"d{k}")


@pytest.mark.parametrize("gain", ["gamma", "mamba"])
def test_streamed_layer_matches_one_piece(gain):
    """SelectiveLRU.stream_chunk: the sequence run as 32-step pieces that carry the state
    (h_init / return_final_state) gives the unsplit layer's output, final state and every
    gradient (only the projection GEMMs' row blocking differs)."""
    from semambaxlinoss_b200.selective_lru import SelectiveLRU

    torch.manual_seed(3)
    m = SelectiveLRU(d_model=64, d_state=16, input_gain=gain, envelope_readout=True).to(cuda())
    with torch.no_grad():
        for p_ in m.parameters():
            p_.add_(0.05 * torch.randn_like(p_))
    x = torch.randn(3, 101, 64, device="cuda")
    gy = torch.randn(3, 101, 64, device="cuda")
    h0 = torch.randn(3, 64, 16, dtype=torch.complex64, device="cuda")
    outs = []
    for K in (None, 32):
        m.stream_chunk = K
        m.zero_grad(set_to_none=True)
        xx = x.clone().requires_grad_(True)
        hh = h0.clone().requires_grad_(True)
        y, hf = m(xx, h_init=hh, return_final_state=True)
        ((y * gy).sum() + hf.real.sum() - hf.imag.sum()).backward()
        outs.append([y.detach(), hf.detach(), xx.grad, hh.grad] + [p_.grad.clone() for p_ in m.parameters()])
    m.stream_chunk = None
    for i, (a_, b_) in enumerate(zip(*outs)):
        assert_close(b_, a_, 1e-5, f"tensor {i}")
