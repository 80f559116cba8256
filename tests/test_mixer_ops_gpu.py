"""The mixer's channels-last convolution + SiLU and SiLU gate kernels on the GPU, inside
MambaStyleMixer (with an identity scan layer, so the surround is isolated), against a
float64 restatement of the reference formulation (models/mixer.py:82-99: in_proj, chunk,
padded depthwise Conv1d over transposed u, SiLU, gate, out_proj): output and every
gradient, causal and centred padding, widths 1-5, channel counts that are not a multiple
of 4, sequences shorter than the kernel, fp32 and bf16 autocast."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from tests.parity import BF16_TOL, FP32_TOL, assert_close, cuda, gen, randn

pytestmark = pytest.mark.gpu


def _reference(params, x, d_conv, causal):
    xz = x @ params["in_proj.weight"].t()
    u, z = xz.chunk(2, dim=-1)
    pad = (d_conv - 1, 0) if causal else ((d_conv - 1) // 2, d_conv - 1 - (d_conv - 1) // 2)
    C = u.shape[-1]
    u = F.conv1d(F.pad(u.transpose(1, 2), pad), params["conv.weight"], params["conv.bias"], groups=C)
    u = F.silu(u.transpose(1, 2))
    y = u * F.silu(z)  # identity scan layer
    return y @ params["out_proj.weight"].t()


CASES = [(2, 37, 12, 2, 4, True), (3, 5, 5, 3, 3, False), (1, 9, 8, 2, 1, True), (2, 1, 4, 4, 4, True),
         (2, 3, 6, 2, 5, False), (2, 64, 64, 4, 4, True)]


@pytest.mark.parametrize("B,L,F_,expand,d_conv,causal", CASES)
@pytest.mark.parametrize("bf16", [False, True])
def test_mixer_surround_matches_reference(B, L, F_, expand, d_conv, causal, bf16):
    from semambaxlinoss_b200.mixer import MambaStyleMixer

    torch.manual_seed(B * 100 + L + F_ + d_conv)
    m = MambaStyleMixer(F_, torch.nn.Identity(), expand=expand, d_conv=d_conv, causal_conv=causal)
    g = gen(7 + L)
    x = randn((B, L, F_), g)
    gy = randn((B, L, F_), g)
    names = [n for n, _ in m.named_parameters()]
    params = {n: p.detach().double().clone().requires_grad_(True) for n, p in m.named_parameters()}
    xr = x.clone().requires_grad_(True)
    yr = _reference(params, xr, d_conv, causal)
    ref = [yr.detach()] + list(torch.autograd.grad((yr * gy).sum(), [xr] + [params[n] for n in names]))
    dev = cuda()
    m = m.to(dev)
    xd = x.float().to(dev).requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=bf16):
        y = m(xd)
    (y.float() * gy.float().to(dev)).sum().backward()
    out = [y.detach()] + [xd.grad] + [p.grad for _, p in m.named_parameters()]
    tol = BF16_TOL if bf16 else FP32_TOL
    for name, o, r in zip(["y", "dx"] + ["d" + n for n in names], out, ref):
        assert_close(o, r, tol, name)
