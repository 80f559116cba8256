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
from semambaxlinoss_b200 import _lib
from tests.parity import BF16_TOL, FP32_TOL, assert_close, crandn, cuda, floor_tol, gen, randn, rel_err, to32

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


_LAYER_CASES = [
    (dict(in_features=16, state_dim=16, n_heads=2, rank=2, input_gain="gamma"), 2, 70),
    (dict(in_features=24, state_dim=15, n_heads=3, rank=0, input_gain="zoh", mode_detune=True,
          rate_scale=1.5), 2, 33),
    (dict(in_features=16, state_dim=32, n_heads=2, rank=4, input_gain="mamba", envelope_readout=True), 1, 40),
    (dict(in_features=8, state_dim=8, n_heads=1, rank=1, input_gain="none", envelope_readout=True,
          mode_detune=True, n_real_modes=2), 3, 5),
    (dict(in_features=64, state_dim=32, n_heads=2, rank=0, input_gain="zoh", envelope_readout=True,
          mode_detune=True), 2, 37),
    (dict(in_features=64, state_dim=32, n_heads=2, rank=4, input_gain="mamba", envelope_readout=True), 1, 50),
    (dict(in_features=256, state_dim=128, n_heads=8, rank=4, input_gain="gamma"), 2, 37),
]


def _layer_case(cfg, B, T, seed, scale=0.3):
    from semambaxlinoss_b200.selective_lru import SelectiveLRUMIMO

    torch.manual_seed(seed)
    m = SelectiveLRUMIMO(**cfg)
    g = gen(seed)
    with torch.no_grad():
        for p in m.parameters():
            p.add_(scale * torch.randn(p.shape, generator=g, dtype=torch.float32))
    x = randn((B, T, cfg["in_features"]), g, scale=0.5)
    gy = randn((B, T, cfg["in_features"]), g)
    return m, x, gy


def _layer_oracle(m, cfg, x, gy, dtype):
    names = [n for n, _ in m.named_parameters()]
    params = {k: v.detach().to(dtype).clone().requires_grad_(True) for k, v in m.state_dict().items()}
    xx = x.to(dtype).clone().requires_grad_(True)
    y = oslru.selective_lru_mimo_forward(params, xx, dict(cfg, rate_scale=m.rate_scale))
    grads = torch.autograd.grad((y * gy.to(dtype)).sum(), [xx] + [params[n] for n in names],
                                allow_unused=True)
    out = {"y": y.detach(), "dx": grads[0]}
    for n, g_ in zip(names, grads[1:]):
        out["d" + n] = torch.zeros_like(params[n]) if g_ is None else g_
    return out


def _layer_gpu(m, x, gy, dtype):
    dev = cuda()
    m = m.to(dev)
    m.zero_grad(set_to_none=True)
    xx = x.to(dtype).to(dev).requires_grad_(True)
    y = m(xx)
    y.backward(gy.float().to(dev))
    out = {"y": y.detach(), "dx": xx.grad}
    for n, p in m.named_parameters():
        out["d" + n] = p.grad if p.grad is not None else torch.zeros_like(p)
    return out


@pytest.mark.parametrize("case", range(len(_LAYER_CASES)))
def test_fused_layer_matches_oracle(case):
    """The fused layer (token projections incl. the static drive -> poles, gain, scan,
    readout, envelope, rank feedthrough) against the float64 oracle: output, input
    gradient and every parameter gradient, for every gain, rank 0-4, detune, envelope,
    rate scale, Nh not a power of two and ragged 32-token chunks."""
    cfg, B, T = _LAYER_CASES[case]
    m, x, gy = _layer_case(cfg, B, T, 40 + case)
    ref = _layer_oracle(m, cfg, x, gy, torch.float64)
    r32 = _layer_oracle(m, cfg, x, gy, torch.float32)
    out = _layer_gpu(m, x, gy, torch.float32)
    for k in ref:
        assert_close(out[k], ref[k], floor_tol(rel_err(r32[k], ref[k])), k)


def _bf16_workload_layer(seed, omega_std=None):
    """The 8-head x 32, state 128, rank 4 layer with the MIMO workload's distributions
    (projection weights N(0, 1/256) held at bf16 values, so that x ~ N(0, 1/4) gives
    b_t, c_t ~ N(0, 1/4); dt_nu bias -2; B, C, D ~ N(0, 1/4)). ``omega_std`` replaces the
    default omega (up to pi / dt_min) by N(0, omega_std^2)."""
    from semambaxlinoss_b200.selective_lru import SelectiveLRUMIMO

    cfg = dict(in_features=256, state_dim=128, n_heads=8, rank=4, input_gain="gamma")
    torch.manual_seed(seed)
    m = SelectiveLRUMIMO(**cfg)
    g = gen(seed + 1)
    with torch.no_grad():
        for lin in (m.dt_nu_proj, m.dt_theta_proj, m.b_dir, m.c_read, m.b_coef, m.c_coef):
            lin.weight.copy_((torch.randn(lin.weight.shape, generator=g) / 16.0).bfloat16().float())
        m.dt_nu_proj.bias.fill_(-2.0)
        for p_ in (m.B, m.C, m.D):
            p_.copy_(torch.randn(p_.shape, generator=g) * 0.5)
        if omega_std is not None:
            m.omega.copy_(torch.randn(m.omega.shape, generator=g) * omega_std)
    return m, cfg


def _bf16_layer_reference(m, cfg, x, gy, proj):
    """Float64 oracle of the bf16 layer given its projection rows ``proj`` (float64,
    without the dt biases; the layer adds those in fp32): output, input gradient and
    every parameter gradient, the projection weights' through the projection rows."""
    names = [n for n, _ in m.named_parameters()]
    W, b = m._projection()
    proj = proj.clone()
    H, r, Nh, Fd = cfg["n_heads"], cfg["rank"], cfg["state_dim"] // cfg["n_heads"], cfg["in_features"]
    proj[..., :2 * H] += b.detach().double().cpu()
    params = {k: v.detach().double().cpu().clone().requires_grad_(True) for k, v in m.state_dict().items()}
    x64 = x.double().cpu().clone().requires_grad_(True)
    proj64 = proj.requires_grad_(True)
    y = oslru.selective_lru_mimo_from_projection(proj64, params, x64, dict(cfg, rate_scale=m.rate_scale))
    grads = torch.autograd.grad((y * gy.double().cpu()).sum(), [x64, proj64] + [params[n] for n in names],
                                allow_unused=True)
    dproj = grads[1]
    W64 = W.detach().double().cpu()
    ref = {"y": y.detach(), "dx": grads[0] + dproj @ W64}
    for n, g_ in zip(names, grads[2:]):
        ref["d" + n] = torch.zeros_like(params[n]) if g_ is None else g_
    # Projection weights / biases get their gradient through the projection rows.
    dW = dproj.reshape(-1, dproj.shape[-1]).t() @ x64.detach().reshape(-1, Fd)
    blocks = [("dt_nu_proj", H), ("dt_theta_proj", H), ("b_coef", H * r), ("b_dir", H * r * Nh),
              ("c_coef", H * r), ("c_read", 2 * H * r * Nh)]
    o = 0
    for name, rows in blocks:
        if rows == 0:  # rank 0: no rank projections
            continue
        ref[f"d{name}.weight"] = dW[o:o + rows]
        if name.startswith("dt_"):
            ref[f"d{name}.bias"] = dproj[..., o:o + rows].sum((0, 1))
        o += rows
    # The static input map B is the block-diagonal drive block of the projection weight.
    Fh = Fd // H
    ref["dB"] = torch.stack([dW[o + h * 2 * Nh:o + (h + 1) * 2 * Nh, h * Fh:(h + 1) * Fh]
                             .reshape(Nh, 2, Fh).permute(0, 2, 1) for h in range(H)])
    return ref


def test_fused_layer_bf16_inputs():
    """bf16 input on the 8-head x 32, state 128, rank 4 layer with the workload's
    distributions and the layer's default omega: the projections and the kernel's operand
    reads are bf16, state and accumulation fp32. Checked against the float64 oracle given
    the same bf16 projection rows the GPU produced (the default omega, up to pi / dt_min,
    makes the pole phase far more sensitive to a one-ulp difference in the bf16 rounding
    of delta_nu than the 2e-2 bound, so this case isolates the layer kernels): output,
    input gradient and every parameter gradient within the bf16-input tolerance.
    test_bf16_layer_full_size_slices covers the projection GEMM with independently
    computed rows."""
    import torch.nn.functional as F

    m, cfg = _bf16_workload_layer(11)
    g = gen(12)
    x = randn((2, 45, 256), g, scale=0.5).to(torch.bfloat16)
    gy = randn((2, 45, 256), g)
    out = _layer_gpu(m, x, gy, torch.bfloat16)
    dev = cuda()
    with torch.no_grad():
        W, _ = m._projection()
        proj = F.linear(x.to(dev), W.to(torch.bfloat16)).double().cpu()
    ref = _bf16_layer_reference(m, cfg, x, gy, proj)
    for k in ref:
        assert_close(out[k], ref[k], BF16_TOL, k)
    assert _lib.tc_timeouts() == 0


@pytest.mark.parametrize("extra", [dict(rank=0), dict(rank=4, mode_detune=True), dict(rank=0, mode_detune=True),
                                   dict(rank=4, envelope_readout=True)])
def test_bf16_layer_variants(extra):
    """The bf16 16-mode x 32-channel layer beyond rank 4: rank 0, mode detune and the
    envelope readout (the tensor-core kernels serve every case but the envelope, which
    runs the CUDA-core kernels), 2 x 83 tokens (a partial 64-token tile and chunk),
    against the float64 oracle on the GPU's own projection rows, within the bf16-input
    tolerance."""
    _check_bf16_variant(extra, 83)


@pytest.mark.parametrize("T", [5, 16, 64, 65])
def test_bf16_layer_chunk_and_tile_edges(T):
    """The tensor-core kernels (rank 4) at sequence lengths on the edges of their 16-token
    chunks and 64-token tiles: one partial chunk (the dC sums then come from a single MMA
    pair that starts the accumulation), exactly one chunk, exactly one tile, one token
    past a tile."""
    _check_bf16_variant(dict(rank=4), T)


def _check_bf16_variant(extra, T):
    import torch.nn.functional as F

    from semambaxlinoss_b200.selective_lru import SelectiveLRUMIMO

    cfg = dict(in_features=256, state_dim=128, n_heads=8, input_gain="gamma", **extra)
    torch.manual_seed(31)
    m = SelectiveLRUMIMO(**cfg)
    g = gen(32)
    with torch.no_grad():
        for p_ in m.parameters():
            p_.add_((0.05 * torch.randn(p_.shape, generator=g)).to(p_.dtype))
        m.dt_nu_proj.bias.fill_(-2.0)
        m.omega.copy_(torch.randn(m.omega.shape, generator=g) * 3.0)
        if extra.get("envelope_readout"):
            m.env_gain.copy_(torch.randn(m.env_gain.shape, generator=g) * 0.1)
    x = randn((2, T, 256), g, scale=0.5).to(torch.bfloat16)
    gy = randn((2, T, 256), g)
    out = _layer_gpu(m, x, gy, torch.bfloat16)
    with torch.no_grad():
        W, _ = m._projection()
        proj = F.linear(x.to(cuda()), W.to(torch.bfloat16)).double().cpu()
    ref = _bf16_layer_reference(m, cfg, x, gy, proj)
    for k in ref:
        assert_close(out[k], ref[k], BF16_TOL, k)
    assert _lib.tc_timeouts() == 0


@pytest.mark.parametrize("S,L", [(404, 321), (1284, 101)])
def test_bf16_layer_full_size_slices(S, L):
    """The MIMO workload layer (256 features = 8 heads x 32, state 128, rank 4, bf16 input,
    fp32 state) at its full pass shapes, time 404 x 321 and frequency 1284 x 101. The
    upstream gradient is zero outside four sequences (first, two inner, last), so every
    gradient, the parameter sums included, comes from those sequences alone and can be
    checked against the float64 oracle run on them; the oracle's projection rows are
    computed on the CPU from the same bf16 x and bf16 weights and rounded to bf16, as the
    layer's bf16 GEMM rounds its output. Omega is drawn N(0, 3^2): the layer's default
    (up to pi / dt_min) makes a one-ulp difference in the bf16 rounding of delta_nu (the
    GPU GEMM accumulates in a different order) turn the pole phase by radians, in the
    reference under bf16 autocast as much as here."""
    m, cfg = _bf16_workload_layer(21, omega_std=3.0)
    dev = cuda()
    gd = torch.Generator(device=dev).manual_seed(S)
    x = (torch.randn(S, L, 256, generator=gd, device=dev) * 0.5).to(torch.bfloat16)
    sl = [0, S // 3, (2 * S) // 3 + 1, S - 1]
    mask = torch.zeros(S, 1, 1, device=dev)
    mask[sl] = 1.0
    gy = torch.randn(S, L, 256, generator=gd, device=dev) * mask
    out = _layer_gpu(m, x, gy, torch.bfloat16)
    # Sequences outside the slice got a zero upstream gradient: their input gradient is zero.
    rest = torch.ones(S, dtype=torch.bool)
    rest[sl] = False
    assert out["dx"][rest.to(dev)].abs().max().item() == 0.0
    xs = x[sl].cpu()
    W, _ = m._projection()
    proj = (xs.double() @ W.detach().to(torch.bfloat16).double().cpu().t()).to(torch.bfloat16).double()
    ref = _bf16_layer_reference(m, cfg, xs, gy[sl].cpu(), proj)
    for k in ref:
        got = out[k][sl] if k in ("y", "dx") else out[k]
        assert_close(got, ref[k], BF16_TOL, k)
    assert _lib.tc_timeouts() == 0


def test_fused_layer_deterministic():
    cfg, B, T = _LAYER_CASES[0]
    m, x, gy = _layer_case(cfg, B, T, 5)
    a = _layer_gpu(m, x, gy, torch.float32)
    a = {k: v.clone() for k, v in a.items()}
    b = _layer_gpu(m, x, gy, torch.float32)
    for k in a:
        assert torch.equal(a[k], b[k]), k
