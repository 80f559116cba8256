"""The callers around the scans on the GPU: MambaStyleMixer against the reference's own
mixer outputs (golden), and TFMambaBlock (bidirectional time + frequency blocks with the
restated pre-norm Block / RMSNorm) against the float64 oracle, forward and every
gradient; plus a bf16-autocast run of a TF-block."""
from __future__ import annotations

import pytest
import torch

from oracle import blocks as oblk
from tests.parity import FP32_TOL, assert_close, cuda, floor_tol, rel_err, to32

pytestmark = pytest.mark.gpu


def _mixer_from_golden(rec):
    from semambaxlinoss_b200.linoss import LinOSS
    from semambaxlinoss_b200.mixer import MambaStyleMixer
    from semambaxlinoss_b200.selective_lru import SelectiveLRU

    cfg = rec["config"]
    inner = cfg["in_features"] * cfg["expand"]
    if cfg["kind"] == "selective_lru":
        ssm = SelectiveLRU(d_model=inner, chunk_size=4, **cfg["ssm"])
    else:
        ssm = LinOSS(in_features=inner, chunk_size=8, **cfg["ssm"])
    m = MambaStyleMixer(cfg["in_features"], ssm, expand=cfg["expand"], d_conv=cfg["d_conv"],
                        causal_conv=cfg["causal"])
    m.load_state_dict({k: v.float() for k, v in rec["state_dict"].items()})
    return m.to(cuda())


def test_mixer_matches_golden(golden):
    dev = cuda()
    for name, rec in golden("mixer").items():
        m = _mixer_from_golden(rec)
        x = to32(rec["x"], dev).requires_grad_(True)
        y = m(x)
        (y * to32(rec["grad_y"], dev)).sum().backward()
        assert_close(y, rec["y"], FP32_TOL, f"{name} y")
        assert_close(x.grad, rec["grad_x"], FP32_TOL, f"{name} dx")
        for n, p in m.named_parameters():
            assert_close(p.grad, rec["param_grads"][n], FP32_TOL, f"{name} d{n}")


def _tf_cfg(bidirectional=True, use_transpose=True):
    time_mixer = dict(ssm="selective_lru", d_state=4, d_conv=4, expand=2, bidirectional=bidirectional,
                      ssm_params=dict(dt_rank=2, n_real_modes=1, chunk_size=8))
    freq_mixer = dict(ssm="linoss", d_state=6, d_conv=4, expand=2, bidirectional=True,
                      ssm_params=dict(discretization="IMEX", damping=True))
    return {"model_cfg": dict(hid_feature=8, use_transpose=use_transpose, time_mixer=time_mixer,
                              freq_mixer=freq_mixer)}


def _oracle_specs(m, cfg):
    tm, fm = cfg["model_cfg"]["time_mixer"], cfg["model_cfg"]["freq_mixer"]
    ts = m.time_mamba.forward_blocks[0].mixer.ssm
    t_cfg = dict(dt_rank=ts.dt_rank, d_state=ts.d_state, input_gain=ts.input_gain)
    f_cfg = dict(discretization="IMEX", damping=True, a_from_g=True)
    return (("selective_lru", t_cfg, dict(bidirectional=tm.get("bidirectional", True))),
            ("linoss", f_cfg, dict(bidirectional=fm.get("bidirectional", True))))


@pytest.mark.parametrize("bidirectional,use_transpose", [(True, True), (False, False)])
def test_tf_block_matches_oracle(bidirectional, use_transpose):
    from semambaxlinoss_b200.mamba_block import TFMambaBlock

    torch.manual_seed(0)
    cfg = _tf_cfg(bidirectional, use_transpose)
    m = TFMambaBlock(cfg)
    with torch.no_grad():
        for p in m.parameters():
            p.add_(0.05 * torch.randn_like(p))
    g = torch.Generator().manual_seed(1)
    x = torch.randn(2, 8, 10, 6, generator=g, dtype=torch.float64)
    gy = torch.randn(2, 8, 10, 6, generator=g, dtype=torch.float64)
    specs = _oracle_specs(m, cfg)

    def oracle(dtype):
        params = {k: v.detach().to(dtype).clone().requires_grad_(True) for k, v in m.state_dict().items()}
        xo = x.to(dtype).clone().requires_grad_(True)
        y = oblk.tf_block_forward(params, xo, *specs, use_transpose=use_transpose)
        names = list(params)
        grads = torch.autograd.grad((y * gy.to(dtype)).sum(), [xo] + [params[n] for n in names], allow_unused=True)
        return y.detach(), dict(zip(["x"] + names, grads))

    y_ref, g_ref = oracle(torch.float64)
    y32, g32 = oracle(torch.float32)
    dev = cuda()
    m = m.to(dev)
    xg = to32(x, dev).requires_grad_(True)
    y = m(xg)
    (y * to32(gy, dev)).sum().backward()
    assert_close(y, y_ref, floor_tol(rel_err(y32, y_ref)), "y")
    assert_close(xg.grad, g_ref["x"], floor_tol(rel_err(g32["x"], g_ref["x"])), "dx")
    for n, p in m.named_parameters():
        ref = g_ref[n]
        assert ref is not None, n
        assert_close(p.grad, ref, floor_tol(rel_err(g32[n], ref)), f"d{n}")


@pytest.mark.parametrize("name", ["mamba_block_0_selective_lru", "mamba_block_1_linoss", "tf_block_0", "tf_block_1"])
def test_blocks_match_golden(golden, name):
    """MambaBlock and TFMambaBlock with the state dicts of the reference's own blocks (run
    on the mamba_ssm stand-in by tests/golden/make_golden.py) against the reference's
    float64 outputs and gradients; each tensor within the fp32 tolerance, floored at twice
    the error of the float32 oracle (as for the oracle comparison above)."""
    from semambaxlinoss_b200.mamba_block import MambaBlock, TFMambaBlock

    rec = golden("blocks")[name]
    sp = rec["oracle_spec"]

    def branch(b):
        return b["kind"], b["ssm"], dict(bidirectional=b["bidirectional"])

    if name.startswith("tf"):
        m = TFMambaBlock(rec["config"])

        def fwd(p, x):
            return oblk.tf_block_forward(p, x, branch(sp["time"]), branch(sp["freq"]), use_transpose=sp["use_transpose"])
    else:
        m = MambaBlock(rec["x"].shape[-1], rec["config"])

        def fwd(p, x):
            return oblk.mamba_block_forward(p, x, *branch(sp)[:2], **branch(sp)[2])
    m.load_state_dict({k: v.float() for k, v in rec["state_dict"].items()})
    # The float32 oracle's distance from the reference sets the floor of each tolerance.
    p32 = {k: v.float().clone().requires_grad_(True) for k, v in rec["state_dict"].items()}
    x32 = rec["x"].float().clone().requires_grad_(True)
    y32 = fwd(p32, x32)
    names = list(p32)
    g32 = torch.autograd.grad((y32 * rec["grad_y"].float()).sum(), [x32] + [p32[n] for n in names],
                              allow_unused=True)
    g32 = dict(zip(["x"] + names, g32))
    dev = cuda()
    m = m.to(dev)
    x = to32(rec["x"], dev).requires_grad_(True)
    y = m(x)
    (y * to32(rec["grad_y"], dev)).sum().backward()
    assert_close(y, rec["y"], floor_tol(rel_err(y32.detach(), rec["y"])), f"{name} y")
    assert_close(x.grad, rec["grad_x"], floor_tol(rel_err(g32["x"], rec["grad_x"])), f"{name} dx")
    for n, p in m.named_parameters():
        ref = rec["param_grads"][n]
        got32 = g32[n] if g32[n] is not None else torch.zeros_like(ref)
        assert_close(p.grad, ref, floor_tol(rel_err(got32, ref)), f"{name} d{n}")


def test_tf_block_bf16_autocast():
    """bf16 autocast around fp32 scans: finite, and close to the fp32 block."""
    from semambaxlinoss_b200.mamba_block import TFMambaBlock

    torch.manual_seed(0)
    cfg = _tf_cfg()
    m = TFMambaBlock(cfg).to(cuda())
    x = torch.randn(2, 8, 12, 7, device="cuda", requires_grad=True)
    y32 = m(x)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y16 = m(x)
    y16.float().square().sum().backward()
    assert torch.isfinite(y16).all() and torch.isfinite(x.grad).all()
    assert rel_err(y16.float(), y32) < 5e-2


@pytest.mark.parametrize("n,d,dtype", [(300, 64, torch.float32), (129, 48, torch.float32),
                                       (7, 1, torch.float32), (40, 1024, torch.float32),
                                       (513, 64, torch.bfloat16), (65, 200, torch.bfloat16)])
def test_rms_norm_kernels_match_oracle(n, d, dtype):
    """semx_rms_norm forward and backward (output, dx, dweight) against the float64
    restatement oracle/blocks.py:rms_norm, for widths that are not multiples of the warp,
    row counts that are not multiples of the 128-row thread block, and bf16 operands (the
    kernel computes in fp32 and rounds its outputs to bf16)."""
    from semambaxlinoss_b200.mamba_block import RMSNorm
    from tests.parity import BF16_TOL

    dev = cuda()
    g = torch.Generator().manual_seed(n * 7 + d)
    x = (torch.randn(2, n, d, generator=g) * 2.0).to(dtype)
    w = torch.randn(d, generator=g)
    gy = torch.randn(2, n, d, generator=g).to(dtype)
    m = RMSNorm(d, eps=1e-5).to(dev)
    with torch.no_grad():
        m.weight.copy_(w)
    xx = x.to(dev).requires_grad_(True)
    y = m(xx)
    assert y.dtype == dtype
    y.backward(gy.to(dev))
    ref = {}
    for dt in (torch.float64, torch.float32):
        xr = x.to(dt).requires_grad_(True)
        wr = w.to(dt).requires_grad_(True)
        yr = oblk.rms_norm(xr, wr, 1e-5)
        yr.backward(gy.to(dt))
        ref[dt] = {"y": yr.detach(), "dx": xr.grad, "dweight": wr.grad}
    # Base tolerance, raised to twice the fp32 restatement's own error (at d = 1 the
    # gradient is all cancellation: dx = w dy eps / (x^2 + eps)^(3/2)).
    base = FP32_TOL if dtype == torch.float32 else BF16_TOL
    out = {"y": y, "dx": xx.grad, "dweight": m.weight.grad}
    for k in out:
        r64 = ref[torch.float64][k]
        assert_close(out[k], r64, floor_tol(rel_err(ref[torch.float32][k], r64), base), k)
    # Fixed reduction order: a second run gives the same bits.
    dw1 = m.weight.grad.clone()
    m.weight.grad = None
    m(xx).backward(gy.to(dev))
    assert torch.equal(dw1, m.weight.grad)


def test_rms_norm_rejects_cpu_and_empty_rows():
    from semambaxlinoss_b200.mamba_block import RMSNorm

    with pytest.raises(RuntimeError):
        RMSNorm(8)(torch.randn(3, 8))
    m = RMSNorm(8).to(cuda())
    x = torch.zeros(0, 8, device=cuda(), requires_grad=True)
    y = m(x)
    y.sum().backward()
    assert y.shape == (0, 8) and torch.equal(m.weight.grad, torch.zeros_like(m.weight))
