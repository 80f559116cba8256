"""The SelectiveLRU step projections (semx_step_proj) on the GPU against the reference's
expressions in float64 (models/selective_lru/selective_lru.py:216-220:
delta_nu = rate_scale * softplus(dt_nu_up(dnu_r)), delta_theta = dt_theta_up(dth_r)),
forward and every gradient: z read in place from strided projection rows, fp32 and bf16
rows, ranks 1 / 4 / 8, channel counts of one and several 128-channel tiles and not a
multiple of 4, row counts that do not fill a row block, a missing upstream gradient,
empty inputs; and the layer using the GEMM formulation for ranks above 8."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from tests.parity import BF16_TOL, FP32_TOL, assert_close, cuda, gen, randn

pytestmark = pytest.mark.gpu


def _reference(zn, zt, Wn, bn, Wt, bt, scale):
    return scale * F.softplus(zn @ Wn.t() + bn), zt @ Wt.t() + bt


@pytest.mark.parametrize("rows,C,r", [(300, 256, 4), (1000, 300, 8), (37, 7, 1), (513, 100, 3), (5, 129, 2)])
@pytest.mark.parametrize("bf16", [False, True])
def test_step_projections_match_reference(rows, C, r, bf16):
    from semambaxlinoss_b200.selective_lru.selective_lru import _StepProjections

    g = gen(rows + C + r)
    width = 2 * r + 24
    proj = randn((rows, width), g, scale=1.5)
    if bf16:
        proj = proj.to(torch.bfloat16).double()  # the values the kernel reads
    Wn, Wt = randn((C, r), g, scale=0.5), randn((C, r), g, scale=0.5)
    bn, bt = randn(C, g, mean=-1.0), randn(C, g)
    gn, gt = randn((rows, C), g), randn((rows, C), g)
    scale = 0.75

    ins = [proj.clone().requires_grad_(True)] + [t.clone().requires_grad_(True) for t in (Wn, bn, Wt, bt)]
    ref_nu, ref_th = _reference(ins[0][:, :r], ins[0][:, r:2 * r], *ins[1:], scale)
    ref_grads = torch.autograd.grad((ref_nu * gn).sum() + (ref_th * gt).sum(), ins)

    dev = cuda()
    dt = torch.bfloat16 if bf16 else torch.float32
    p = proj.to(dt).to(dev).requires_grad_(True)
    params = [t.float().to(dev).requires_grad_(True) for t in (Wn, bn, Wt, bt)]
    dnu, dth = _StepProjections.apply(p[:, :r], p[:, r:2 * r], *params, scale)
    assert dnu.dtype == torch.float32 and dnu.shape == (rows, C)
    ((dnu * gn.float().to(dev)).sum() + (dth * gt.float().to(dev)).sum()).backward()
    assert_close(dnu, ref_nu, FP32_TOL, "delta_nu")
    assert_close(dth, ref_th, FP32_TOL, "delta_theta")
    assert p.grad.dtype == dt
    assert_close(p.grad, ref_grads[0], BF16_TOL if bf16 else FP32_TOL, "dz")
    assert torch.equal(p.grad[:, 2 * r:], torch.zeros_like(p.grad[:, 2 * r:]))
    for name, got, ref in zip(["dW_nu", "db_nu", "dW_th", "db_th"], [t.grad for t in params], ref_grads[1:]):
        assert_close(got, ref, FP32_TOL, name)
    # Fixed reduction order: the same call again gives the same bits.
    grads1 = [p.grad.clone()] + [t.grad.clone() for t in params]
    p.grad = None
    for t in params:
        t.grad = None
    dnu, dth = _StepProjections.apply(p[:, :r], p[:, r:2 * r], *params, scale)
    ((dnu * gn.float().to(dev)).sum() + (dth * gt.float().to(dev)).sum()).backward()
    for a, b in zip(grads1, [p.grad] + [t.grad for t in params]):
        assert torch.equal(a, b)


def test_step_projections_one_gradient_and_empty():
    from semambaxlinoss_b200.selective_lru.selective_lru import _StepProjections

    dev = cuda()
    g = gen(11)
    C, r = 64, 4
    proj = randn((3, 17, 2 * r + 8), g).float().to(dev).requires_grad_(True)
    params = [randn(s, g).float().to(dev).requires_grad_(True) for s in ((C, r), (C,), (C, r), (C,))]
    dnu, dth = _StepProjections.apply(proj[..., :r], proj[..., r:2 * r], *params, 1.0)
    assert dnu.shape == (3, 17, C)
    dth.sum().backward()  # no gradient reaches delta_nu
    assert torch.equal(params[0].grad, torch.zeros_like(params[0].grad))
    assert torch.equal(params[1].grad, torch.zeros_like(params[1].grad))
    assert torch.equal(proj.grad[..., :r], torch.zeros_like(proj.grad[..., :r]))
    assert params[3].grad.abs().sum() > 0
    for t in params:
        t.grad = None
    empty = torch.zeros(0, 2 * r, device=dev, requires_grad=True)
    dnu, dth = _StepProjections.apply(empty[:, :r], empty[:, r:], *params, 1.0)
    (dnu.sum() + dth.sum()).backward()
    assert dnu.shape == (0, C) and torch.equal(params[2].grad, torch.zeros_like(params[2].grad))


def test_layer_with_rank_above_the_fused_kernels():
    """d_model 576 gives dt_rank 9: the layer keeps the GEMM formulation and matches the
    fused-rank path's formula."""
    from semambaxlinoss_b200.selective_lru import SelectiveLRU

    torch.manual_seed(0)
    m = SelectiveLRU(d_model=576, d_state=4).to(cuda())
    assert m.dt_rank == 9
    x = torch.randn(2, 9, 576, device="cuda", requires_grad=True)
    y = m(x)
    y.square().sum().backward()
    assert torch.isfinite(y).all() and torch.isfinite(x.grad).all()
