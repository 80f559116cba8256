"""Pins the oracle to the reference: the oracle restatement, run on the committed golden
inputs and parameters, must reproduce the reference's own float64 outputs and gradients
(tests/golden/make_golden.py ran the reference to produce them)."""
from __future__ import annotations

import pytest
import torch

from oracle import blocks as oblk
from oracle import linoss as olin
from oracle import selective_lru as oslru

TOL = 1e-10  # both sides are float64 evaluations of the same expressions


def _rel(a, b):
    a = torch.as_tensor(a)
    b = torch.as_tensor(b)
    den = b.abs().max().item()
    return (a - b).abs().max().item() / (den if den > 0 else 1.0)


def _module_case(rec, forward_fn):
    params = {k: v.clone().requires_grad_(True) for k, v in rec["state_dict"].items()}
    x = rec["x"].clone().requires_grad_(True)
    out = forward_fn(params, x)
    if isinstance(out, tuple):
        y, hf = out
        ghf = rec["grad_hf"]
        loss = (y * rec["grad_y"]).sum() + (hf.real * ghf.real + hf.imag * ghf.imag).sum()
        assert _rel(hf.detach(), rec["hf"]) < TOL
    else:
        y = out
        loss = (y * rec["grad_y"]).sum()
    assert _rel(y.detach(), rec["y"]) < TOL
    names = list(params)
    grads = torch.autograd.grad(loss, [x] + [params[n] for n in names], allow_unused=True)
    assert _rel(grads[0], rec["grad_x"]) < TOL
    for n, g in zip(names, grads[1:]):
        ref = rec["param_grads"][n]
        g = torch.zeros_like(ref) if g is None else g
        assert _rel(g, ref) < TOL, n


def test_linoss_layers_match_reference(golden):
    cases = golden("linoss")
    n = 0
    for name, rec in cases.items():
        if name == "linoss_recurrence":
            continue
        cfg = rec["config"]
        _module_case(
            rec,
            lambda p, x: olin.linoss_forward(
                p, x, cfg["discretization"], cfg["damping"], cfg["a_from_g"]
            ),
        )
        n += 1
    assert n == 8


def test_linoss_recurrence_matches_reference(golden):
    rec = golden("linoss")["linoss_recurrence"]
    ins = [t.clone().requires_grad_(True) for t in (*rec["M"], rec["F1"], rec["F2"])]
    y2 = olin.linoss_recurrence(*ins)
    assert _rel(y2.detach(), rec["Y2"]) < TOL
    gy = rec["grad_Y2"]
    loss = (y2.real * gy.real + y2.imag * gy.imag).sum()
    for g, r in zip(torch.autograd.grad(loss, ins), rec["grads"]):
        assert _rel(g, r) < TOL


@pytest.mark.parametrize("idx", range(6))
def test_selective_lru_layers_match_reference(golden, idx):
    cases = golden("selective_lru")
    name = sorted(cases)[idx]
    rec = cases[name]
    cfg = dict(rec["config"])
    fk = rec["forward_kwargs"]

    def fwd(p, x):
        return oslru.selective_lru_forward(
            p, x, cfg, h_init=rec.get("h_init"), rate_scale=fk.get("rate_scale"),
            return_final_state=fk.get("return_final_state", False),
        )

    _module_case(rec, fwd)


@pytest.mark.parametrize("idx", range(5))
def test_mimo_layers_match_reference(golden, idx):
    cases = golden("mimo")
    name = sorted(cases)[idx]
    rec = cases[name]
    cfg = dict(rec["config"])
    _module_case(rec, lambda p, x: oslru.selective_lru_mimo_forward(p, x, cfg))


@pytest.mark.parametrize("idx", range(5))
def test_mimo_drive_columns_match_reference(golden, idx):
    """The layer kernels' input contract: projection rows that carry the static drive
    B x as extra columns give the reference's outputs and gradients (B's gradient then
    flows through those columns)."""
    cases = golden("mimo")
    name = sorted(cases)[idx]
    rec = cases[name]
    cfg = dict(rec["config"])

    def fwd(p, x):
        proj = oslru.mimo_projection(p, x, cfg, drive=True)
        return oslru.selective_lru_mimo_from_projection(proj, p, x, cfg)

    _module_case(rec, fwd)


def test_selective_recurrence_matches_reference(golden):
    rec = golden("recurrence")["selective_recurrence"]
    ins = [t.clone().requires_grad_(True) for t in (rec["lam"], rec["Bu"], rec["h0"])]
    h = oslru.selective_recurrence(*ins)
    assert _rel(h.detach(), rec["h"]) < TOL
    gh = rec["grad_h"]
    loss = (h.real * gh.real + h.imag * gh.imag).sum()
    for g, r in zip(torch.autograd.grad(loss, ins), rec["grads"]):
        assert _rel(g, r) < TOL


def test_real_special_case_equals_complex_op():
    """The real form is the complex op with omega = dtheta = B_im = C_im = 0."""
    g = torch.Generator().manual_seed(3)
    B, T, C, N = 2, 11, 5, 4
    dnu = torch.nn.functional.softplus(torch.randn(B, T, C, generator=g, dtype=torch.float64))
    a = torch.exp(torch.rand(C, N, generator=g, dtype=torch.float64) * 2.7)
    Bt = torch.randn(B, T, N, generator=g, dtype=torch.float64)
    Ct = torch.randn(B, T, N, generator=g, dtype=torch.float64)
    x = torch.randn(B, T, C, generator=g, dtype=torch.float64)
    D = torch.randn(C, generator=g, dtype=torch.float64)
    y = oslru.selective_lru_real_op(dnu, a, Bt, Ct, x, D, "mamba")
    # direct real recurrence
    lam = torch.exp(-dnu.unsqueeze(-1) * a)
    u = (dnu * x).unsqueeze(-1) * Bt.unsqueeze(-2)
    h = torch.zeros(B, C, N, dtype=torch.float64)
    ys = []
    for t in range(T):
        h = lam[:, t] * h + u[:, t]
        ys.append((h * Ct[:, t].unsqueeze(-2)).sum(-1) + D * x[:, t])
    assert _rel(y, torch.stack(ys, 1)) < 1e-12


@pytest.mark.parametrize("idx", range(4))
def test_mixer_matches_reference(golden, idx):
    cases = golden("mixer")
    rec = cases[sorted(cases)[idx]]
    cfg = rec["config"]
    _module_case(rec, lambda p, x: oblk.mixer_forward(p, x, cfg["kind"], cfg["ssm"], cfg["d_conv"], cfg["causal"]))


def _branch(sp):
    return sp["kind"], sp["ssm"], dict(bidirectional=sp["bidirectional"])


@pytest.mark.parametrize("name", ["mamba_block_0_selective_lru", "mamba_block_1_linoss"])
def test_mamba_blocks_match_reference(golden, name):
    """MambaBlock (models/mamba_block.py:344-396 of the reference, run on the mamba_ssm
    stand-in): the bidirectional branch flips, the residual stream and the concatenation."""
    rec = golden("blocks")[name]
    kind, scfg, kw = _branch(rec["oracle_spec"])
    _module_case(rec, lambda p, x: oblk.mamba_block_forward(p, x, kind, scfg, **kw))


@pytest.mark.parametrize("idx", [0, 1])
def test_tf_blocks_match_reference(golden, idx):
    """TFMambaBlock (models/mamba_block.py:419-508 of the reference): time blocks over the
    (batch x bins) sequences, frequency blocks over the (batch x frames) sequences, the
    channel projections (transposed conv or linear) and both residual adds."""
    rec = golden("blocks")[f"tf_block_{idx}"]
    sp = rec["oracle_spec"]
    _module_case(rec, lambda p, x: oblk.tf_block_forward(p, x, _branch(sp["time"]), _branch(sp["freq"]),
                                                          use_transpose=sp["use_transpose"]))
