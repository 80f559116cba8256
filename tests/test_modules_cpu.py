"""Host-side checks of the drop-in layers (no GPU): parameter names, shapes and order
match the reference's state dicts (golden fixtures), constructor validation matches the
reference, the block factory's behaviour, and that no layer silently runs on the CPU."""
from __future__ import annotations

import pytest
import torch

from semambaxlinoss_b200.linoss import LinOSS
from semambaxlinoss_b200.mamba_block import TFMambaBlock, _build_mixer_cls, _layer_spec_matches
from semambaxlinoss_b200.selective_lru import SelectiveLRU, SelectiveLRUMIMO


def _same_layout(module, state_dict):
    ours = module.state_dict()
    assert list(ours) == list(state_dict)
    for k, v in state_dict.items():
        assert ours[k].shape == v.shape, k


def test_linoss_state_dicts_match_reference(golden):
    for name, rec in golden("linoss").items():
        if name == "linoss_recurrence":
            continue
        c = rec["config"]
        _same_layout(LinOSS(c["in_features"], c["state_dim"], c["discretization"], c["damping"],
                            a_from_g=c["a_from_g"]), rec["state_dict"])


def test_selective_lru_state_dicts_match_reference(golden):
    for rec in golden("selective_lru").values():
        _same_layout(SelectiveLRU(**rec["config"]), rec["state_dict"])


def test_mimo_state_dicts_match_reference(golden):
    for rec in golden("mimo").values():
        _same_layout(SelectiveLRUMIMO(**rec["config"]), rec["state_dict"])


def test_tags_and_defaults():
    m = SelectiveLRU(d_model=16, d_state=8, envelope_readout=True, mode_detune=True)
    assert m.dt_rank == 1
    assert m.dt_nu_up.bias._no_reinit and m.dt_theta_up.bias._no_reinit
    for p in (m.A_log, m.omega, m.D, m.env_gain, m.detune_gain):
        assert p._no_weight_decay
    # Baseline delta_nu = softplus(bias) lies in [dt_min, dt_max] at init.
    dt = torch.nn.functional.softplus(m.dt_nu_up.bias)
    assert (dt >= 1e-3 - 1e-6).all() and (dt <= 0.1 + 1e-6).all()
    mm = SelectiveLRUMIMO(in_features=8, state_dim=16, n_heads=2, rank=2)
    assert mm.c_out.shape == (4, 4)


def test_constructor_validation():
    with pytest.raises(ValueError):
        SelectiveLRU(8, 4, input_gain="bogus")
    with pytest.raises(ValueError):
        SelectiveLRU(8, 4, n_real_modes=5)
    with pytest.raises(ValueError):
        SelectiveLRUMIMO(8, 16, n_heads=3)
    with pytest.raises(ValueError):
        SelectiveLRUMIMO(8, 16, input_gain="bogus")
    with pytest.raises(NotImplementedError):
        LinOSS(8, discretization="IM", damping=True)
    with pytest.raises(NotImplementedError):
        LinOSS(8, discretization="ZOH")


def test_no_cpu_fallback():
    """The layers run only on the CUDA path: CPU tensors raise like the reference's GPU
    operators, instead of silently taking a CPU route."""
    x = torch.randn(2, 5, 8)
    for layer in (SelectiveLRU(8, 4), SelectiveLRUMIMO(8, 16), LinOSS(8, 16)):
        with pytest.raises(RuntimeError):
            layer(x)


def test_factory_and_tf_block_structure():
    cfg = {"model_cfg": {"hid_feature": 8,
                         "time_mixer": {"ssm": "selective_lru", "d_state": 4, "d_conv": 4, "expand": 2},
                         "freq_mixer": {"ssm": "linoss", "d_state": 6, "d_conv": 4, "expand": 2}}}
    m = TFMambaBlock(cfg)
    names = [n for n, _ in m.named_parameters()]
    assert "time_mamba.forward_blocks.0.mixer.ssm.A_log" in names
    assert "time_mamba.backward_blocks.0.norm.weight" in names
    assert "freq_mamba.forward_blocks.0.mixer.ssm.steps" in names
    assert "tlinear.weight" in names and "flinear.bias" in names
    for kind in ("mamba", "mamba2", "s5", "selective_linoss"):
        with pytest.raises(NotImplementedError):
            _build_mixer_cls(8, {"ssm": kind, "d_state": 4, "d_conv": 4, "expand": 2})
    with pytest.raises(ValueError):
        _build_mixer_cls(8, {"ssm": "nope", "d_state": 4, "d_conv": 4, "expand": 2})


def test_layer_spec_matches():
    assert _layer_spec_matches([-1], 3, 4)
    assert _layer_spec_matches(["1-2"], 2, 4)
    assert not _layer_spec_matches(["1-2", 0], 3, 4)


def test_mimo_drive_weight_layout():
    """drive_weight(B) holds B block-diagonally: F.linear(x, drive_weight(B)) is the static
    drive sum_f B[h, n, f, c] x[h Fh + f] at column h 2Nh + 2n + c, and the projection of
    SelectiveLRUMIMO is proj_width() columns wide with the drive block last."""
    from semambaxlinoss_b200.selective_lru import drive_weight, proj_width

    g = torch.Generator().manual_seed(3)
    H, Nh, Fh = 3, 5, 4
    B = torch.randn(H, Nh, Fh, 2, generator=g, dtype=torch.float64)
    x = torch.randn(2, 7, H * Fh, generator=g, dtype=torch.float64)
    bx = torch.nn.functional.linear(x, drive_weight(B))
    want = torch.einsum("hnfc,bthf->bthnc", B, x.view(2, 7, H, Fh)).reshape(2, 7, 2 * H * Nh)
    assert torch.allclose(bx, want, rtol=0, atol=1e-12)
    m = SelectiveLRUMIMO(24, 16, n_heads=2, rank=3)
    W, b = m._projection()
    assert W.shape == (proj_width(2, 8, 3), 24) and b.shape == (2 * 2,)
    assert torch.equal(W[-2 * 16:], drive_weight(m.B.detach()))


def test_step_projection_matches_linear():
    """The rank-r step projections (one GEMM with the bias as a row of the weight) give
    nn.Linear's value and gradients, on the non-contiguous split the layer feeds them,
    and stay fp32 under bf16 autocast (the scan reads fp32)."""
    from semambaxlinoss_b200.selective_lru.selective_lru import _step_projection

    torch.manual_seed(0)
    lin = torch.nn.Linear(4, 32)
    rows = torch.randn(3, 11, 20)
    z_ref = rows[..., 2:6].clone().requires_grad_(True)
    z = rows[..., 2:6].detach().requires_grad_(True)
    ref = lin(z_ref)
    g = torch.randn_like(ref)
    (ref * g).sum().backward()
    w_ref, b_ref = lin.weight.grad.clone(), lin.bias.grad.clone()
    lin.zero_grad()
    out = _step_projection(lin, z)
    (out * g).sum().backward()
    assert out.shape == ref.shape and out.dtype == torch.float32
    torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(z.grad, z_ref.grad, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(lin.weight.grad, w_ref, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(lin.bias.grad, b_ref, rtol=1e-5, atol=1e-6)
    with torch.autocast(device_type="cpu", dtype=torch.bfloat16):
        assert _step_projection(lin, z.detach().to(torch.bfloat16)).dtype == torch.float32
