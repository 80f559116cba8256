"""Generates the golden fixtures in this folder by running the reference implementation.

Runs on a machine that has the reference checkout: set SEMX_REFERENCE to its root
directory (the script refuses to run without it). Nothing else reads the reference: the committed ``*.pt`` fixtures
carry seeded inputs, parameters and the reference's float64 outputs and gradients, and
``tests/test_oracle_golden.py`` checks the oracle restatement against them.

What runs (all on CPU, float64, through the reference's own modules and functions):
* models/linoss/linoss.py          LinOSS (all variants) and _linoss_recurrence
* models/selective_lru/selective_lru.py  SelectiveLRU (every gain / option),
  SelectiveLRUMIMO (every gain / option, rank > 0) and _selective_recurrence
* models/mixer.py                  MambaStyleMixer around SelectiveLRU and LinOSS
* models/mamba_block.py            MambaBlock and TFMambaBlock (selective-LRU time mixers,
  LinOSS frequency mixers), with the third-party mamba_ssm package it imports replaced by
  the stand-in in mamba_ssm_standin/ (Block, RMSNorm restated from their documented
  behaviour): the fixtures pin the reference's own block code above those two pieces

Usage: SEMX_REFERENCE=<reference checkout> python tests/golden/make_golden.py
"""
from __future__ import annotations

import importlib.util
import os
import sys
import types
from pathlib import Path

import torch

OUT = Path(__file__).resolve().parent
REF = Path(os.environ["SEMX_REFERENCE"]) if "SEMX_REFERENCE" in os.environ else None


def _import_reference():
    if REF is None or not (REF / "models").is_dir():
        raise SystemExit("set SEMX_REFERENCE to the root of the reference checkout")
    sys.path.insert(0, str(REF))
    from models.selective_lru.selective_lru import (  # noqa: E402
        SelectiveLRU,
        SelectiveLRUMIMO,
        _selective_recurrence,
    )

    # models/linoss/__init__.py imports a module that does not exist in the reference,
    # so the layer file is loaded by path.
    spec = importlib.util.spec_from_file_location("ref_linoss", REF / "models/linoss/linoss.py")
    lin = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(lin)
    from models.mixer import MambaStyleMixer  # noqa: E402

    return SelectiveLRU, SelectiveLRUMIMO, _selective_recurrence, lin, MambaStyleMixer


def _import_reference_blocks():
    """The reference's models/mamba_block.py, on the mamba_ssm stand-in. Its
    ``from models.linoss import ...`` goes through models/linoss/__init__.py, which imports
    a module the reference does not contain, so ``models.linoss`` is registered from the
    layer file with a placeholder for the selective LinOSS variant (not used here)."""
    sys.path.insert(0, str(OUT / "mamba_ssm_standin"))
    sys.path.insert(0, str(OUT.parent.parent))  # the stand-in's _init_weights restatement
    import models  # noqa: F401,E402

    spec = importlib.util.spec_from_file_location("models.linoss.linoss", REF / "models/linoss/linoss.py")
    lin = importlib.util.module_from_spec(spec)
    sys.modules["models.linoss.linoss"] = lin
    spec.loader.exec_module(lin)
    pkg = types.ModuleType("models.linoss")
    pkg.__path__ = [str(REF / "models/linoss")]
    pkg.LinOSS = lin.LinOSS

    class SelectiveLinOSSIM:  # the module the reference's package file names is absent
        def __init__(self, *args, **kwargs):
            raise NotImplementedError

    pkg.SelectiveLinOSSIM = SelectiveLinOSSIM
    sys.modules["models.linoss"] = pkg
    from models.mamba_block import MambaBlock, TFMambaBlock  # noqa: E402

    return MambaBlock, TFMambaBlock


def _run_module(module, x, fwd_kwargs, seed):
    """Forward + backward of a float64 module; returns outputs and all gradients."""
    x = x.clone().requires_grad_(True)
    out = module(x, **fwd_kwargs)
    g = torch.Generator().manual_seed(seed + 1)
    if isinstance(out, tuple):
        y, hf = out
        gy = torch.randn(y.shape, generator=g, dtype=y.dtype)
        ghf = torch.randn(hf.shape, generator=g, dtype=torch.float64)
        ghf = torch.complex(ghf, torch.randn(hf.shape, generator=g, dtype=torch.float64))
        loss = (y * gy).sum() + (hf.real * ghf.real + hf.imag * ghf.imag).sum()
        extra = {"hf": hf.detach(), "grad_hf": ghf}
    else:
        y = out
        gy = torch.randn(y.shape, generator=g, dtype=y.dtype)
        loss = (y * gy).sum()
        extra = {}
    params = [p for _, p in module.named_parameters()]
    grads = torch.autograd.grad(loss, [x] + params, allow_unused=True)
    rec = {
        "x": x.detach(),
        "y": y.detach(),
        "grad_y": gy,
        "grad_x": grads[0],
        "state_dict": {k: v.detach().clone() for k, v in module.state_dict().items()},
        "param_grads": {
            n: (g_ if g_ is not None else torch.zeros_like(p))
            for (n, p), g_ in zip(module.named_parameters(), grads[1:])
        },
        "forward_kwargs": {k: v for k, v in fwd_kwargs.items() if not torch.is_tensor(v)},
    }
    if "h_init" in fwd_kwargs:
        rec["h_init"] = fwd_kwargs["h_init"]
    rec.update(extra)
    return rec


def _perturb(module, seed, scale=0.5):
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for _, p in module.named_parameters():
            p.add_(scale * torch.randn(p.shape, generator=g, dtype=p.dtype))


def linoss_cases(lin):
    cases = {}
    variants = [
        ("IMEX", True, True),
        ("IMEX", True, False),
        ("IMEX", False, True),
        ("IM", False, True),
    ]
    for disc, damp, afg in variants:
        for (H, P, S, L) in [(4, 16, 3, 17), (6, 20, 2, 37)]:
            torch.manual_seed(1000 + H + P + L)
            m = lin.LinOSS(in_features=H, state_dim=P, discretization=disc, damping=damp,
                           a_from_g=afg).double()
            # Spread parameters over every constraint branch (relu zero, clamp bands).
            _perturb(m, seed=7 + P + L, scale=0.7)
            g = torch.Generator().manual_seed(11 + P + L)
            x = torch.randn(S, L, H, generator=g, dtype=torch.float64)
            rec = _run_module(m, x, {}, seed=S * 100 + L)
            rec["config"] = dict(in_features=H, state_dim=P, discretization=disc,
                                 damping=damp, a_from_g=afg)
            cases[f"linoss_{disc}_{'damped' if damp else 'undamped'}_afg{int(afg)}_{S}x{L}"] = rec
    # The bare recurrence with a given transition (the generic op).
    g = torch.Generator().manual_seed(5)
    S, L, P = 3, 29, 16
    M = [0.3 * torch.randn(P, generator=g, dtype=torch.float64) + d for d in (0.9, 0, 0, 0.9)]
    F1 = torch.complex(torch.randn(S, L, P, generator=g, dtype=torch.float64),
                       torch.randn(S, L, P, generator=g, dtype=torch.float64))
    F2 = torch.complex(torch.randn(S, L, P, generator=g, dtype=torch.float64),
                       torch.randn(S, L, P, generator=g, dtype=torch.float64))
    ins = [t.clone().requires_grad_(True) for t in (*M, F1, F2)]
    y2 = lin._linoss_recurrence(*ins)
    gy = torch.complex(torch.randn(S, L, P, generator=g, dtype=torch.float64),
                       torch.randn(S, L, P, generator=g, dtype=torch.float64))
    loss = (y2.real * gy.real + y2.imag * gy.imag).sum()
    grads = torch.autograd.grad(loss, ins)
    cases["linoss_recurrence"] = {
        "M": [t.detach() for t in M], "F1": F1, "F2": F2, "Y2": y2.detach(), "grad_Y2": gy,
        "grads": list(grads),
    }
    return cases


def selective_lru_cases(SelectiveLRU):
    cases = {}
    opts = [
        dict(input_gain="gamma"),
        dict(input_gain="mamba"),
        dict(input_gain="zoh"),
        dict(input_gain="gamma", envelope_readout=True, mode_detune=True, n_real_modes=1),
        dict(input_gain="zoh", mode_detune=True, rate_scale=1.5),
        dict(input_gain="mamba", envelope_readout=True),
    ]
    for i, o in enumerate(opts):
        torch.manual_seed(200 + i)
        m = SelectiveLRU(d_model=8, d_state=4, **o).double()
        _perturb(m, seed=300 + i, scale=0.3)
        g = torch.Generator().manual_seed(400 + i)
        x = torch.randn(2, 19, 8, generator=g, dtype=torch.float64)
        fwd = {}
        if i == 4:
            fwd["rate_scale"] = 0.75
        if i in (1, 3):
            h0 = torch.complex(torch.randn(2, 8, 4, generator=g, dtype=torch.float64),
                               torch.randn(2, 8, 4, generator=g, dtype=torch.float64))
            fwd.update(h_init=h0, return_final_state=True)
        rec = _run_module(m, x, fwd, seed=500 + i)
        rec["config"] = dict(d_model=8, d_state=4, dt_rank=m.dt_rank, **o)
        cases[f"selective_lru_{i}_{o['input_gain']}"] = rec
    return cases


def mimo_cases(SelectiveLRUMIMO):
    cases = {}
    opts = [
        dict(input_gain="gamma", rank=2),
        dict(input_gain="mamba", rank=0),
        dict(input_gain="zoh", rank=2, mode_detune=True),
        dict(input_gain="none", rank=1, envelope_readout=True),
        dict(input_gain="gamma", rank=2, envelope_readout=True, mode_detune=True,
             n_real_modes=2, rate_scale=1.25),
    ]
    for i, o in enumerate(opts):
        torch.manual_seed(600 + i)
        m = SelectiveLRUMIMO(in_features=8, state_dim=16, n_heads=2, **o).double()
        _perturb(m, seed=700 + i, scale=0.2)
        g = torch.Generator().manual_seed(800 + i)
        x = torch.randn(2, 15, 8, generator=g, dtype=torch.float64)
        rec = _run_module(m, x, {}, seed=900 + i)
        rec["config"] = dict(in_features=8, state_dim=16, n_heads=2, **o)
        cases[f"mimo_{i}_{o['input_gain']}"] = rec
    return cases


def recurrence_case(_selective_recurrence):
    g = torch.Generator().manual_seed(9)
    B, T, N = 3, 17, 16
    nu = torch.rand(B, T, N, generator=g, dtype=torch.float64) * 0.99
    theta = torch.randn(B, T, N, generator=g, dtype=torch.float64)
    Bu = torch.complex(torch.randn(B, T, N, generator=g, dtype=torch.float64),
                       torch.randn(B, T, N, generator=g, dtype=torch.float64))
    h0 = torch.complex(torch.randn(B, N, generator=g, dtype=torch.float64),
                       torch.randn(B, N, generator=g, dtype=torch.float64))
    lam = torch.polar(nu, theta)
    ins = [lam.clone().requires_grad_(True), Bu.clone().requires_grad_(True),
           h0.clone().requires_grad_(True)]
    h = _selective_recurrence(*ins)
    gh = torch.complex(torch.randn(B, T, N, generator=g, dtype=torch.float64),
                       torch.randn(B, T, N, generator=g, dtype=torch.float64))
    loss = (h.real * gh.real + h.imag * gh.imag).sum()
    grads = torch.autograd.grad(loss, ins)
    return {"selective_recurrence": {"lam": lam, "Bu": Bu, "h0": h0, "h": h.detach(),
                                     "grad_h": gh, "grads": list(grads)}}


def mixer_cases(MambaStyleMixer, SelectiveLRU, lin):
    cases = {}
    specs = [
        ("selective_lru", dict(d_state=4, input_gain="gamma"), True),
        ("selective_lru", dict(d_state=8, input_gain="zoh", mode_detune=True), False),
        ("linoss", dict(state_dim=6, discretization="IMEX", damping=True), True),
        ("linoss", dict(state_dim=6, discretization="IM", damping=False), True),
    ]
    for i, (kind, kw, causal) in enumerate(specs):
        torch.manual_seed(1100 + i)
        d, expand = 4, 2
        if kind == "selective_lru":
            ssm = SelectiveLRU(d_model=d * expand, **kw)
        else:
            ssm = lin.LinOSS(in_features=d * expand, **kw)
        m = MambaStyleMixer(d, ssm, expand=expand, d_conv=4, causal_conv=causal).double()
        _perturb(m, seed=1200 + i, scale=0.2)
        g = torch.Generator().manual_seed(1300 + i)
        x = torch.randn(2, 13, d, generator=g, dtype=torch.float64)
        rec = _run_module(m, x, {}, seed=1400 + i)
        cfg = dict(kw)
        if kind == "selective_lru":
            cfg["dt_rank"] = ssm.dt_rank
        rec["config"] = dict(kind=kind, ssm=cfg, in_features=d, expand=expand, d_conv=4, causal=causal)
        cases[f"mixer_{i}_{kind}"] = rec
    return cases


def _tf_cfg(bidirectional, use_transpose):
    time_mixer = dict(ssm="selective_lru", d_state=4, d_conv=4, expand=2, bidirectional=bidirectional,
                      ssm_params=dict(dt_rank=2, n_real_modes=1))
    freq_mixer = dict(ssm="linoss", d_state=6, d_conv=4, expand=2, bidirectional=True,
                      ssm_params=dict(discretization="IMEX", damping=True))
    return {"model_cfg": dict(hid_feature=8, use_transpose=use_transpose, time_mixer=time_mixer,
                              freq_mixer=freq_mixer)}


def _oracle_spec(block, cfg):
    """How oracle/blocks.py evaluates one MambaBlock of the fixture: the scan layer's kind,
    its configuration and the branch mode."""
    ssm = block.forward_blocks[0].mixer.ssm
    if cfg["ssm"] == "selective_lru":
        scfg = dict(dt_rank=ssm.dt_rank, d_state=ssm.d_state, input_gain=ssm.input_gain)
    else:
        p = cfg.get("ssm_params", {})
        scfg = dict(discretization=p.get("discretization", "IMEX"), damping=p.get("damping", True),
                    a_from_g=p.get("a_from_g", True))
    return dict(kind=cfg["ssm"], ssm=scfg, bidirectional=cfg.get("bidirectional", True))


def block_cases(MambaBlock, TFMambaBlock):
    cases = {}
    # A bidirectional selective-LRU block and a unidirectional LinOSS block on (S, L, C).
    specs = [
        dict(ssm="selective_lru", d_state=4, d_conv=4, expand=2, bidirectional=True,
             ssm_params=dict(dt_rank=2, input_gain="gamma")),
        dict(ssm="linoss", d_state=6, d_conv=4, expand=2, bidirectional=False,
             ssm_params=dict(discretization="IMEX", damping=True)),
    ]
    for i, cfg in enumerate(specs):
        torch.manual_seed(1500 + i)
        m = MambaBlock(8, cfg).double()
        _perturb(m, seed=1600 + i, scale=0.1)
        g = torch.Generator().manual_seed(1700 + i)
        x = torch.randn(3, 11, 8, generator=g, dtype=torch.float64)
        rec = _run_module(m, x, {}, seed=1800 + i)
        rec["config"] = cfg
        rec["oracle_spec"] = _oracle_spec(m, cfg)
        cases[f"mamba_block_{i}_{cfg['ssm']}"] = rec
    # TF-blocks on (b, c, t, f): bidirectional time branch with the transposed-conv
    # projections, and a unidirectional time branch with the linear projections.
    for i, (bi, tr) in enumerate([(True, True), (False, False)]):
        torch.manual_seed(1900 + i)
        cfg = _tf_cfg(bi, tr)
        m = TFMambaBlock(cfg).double()
        _perturb(m, seed=2000 + i, scale=0.05)
        g = torch.Generator().manual_seed(2100 + i)
        x = torch.randn(2, 8, 10, 6, generator=g, dtype=torch.float64)
        rec = _run_module(m, x, {}, seed=2200 + i)
        rec["config"] = cfg
        mc = cfg["model_cfg"]
        rec["oracle_spec"] = dict(time=_oracle_spec(m.time_mamba, mc["time_mixer"]),
                                  freq=_oracle_spec(m.freq_mamba, mc["freq_mixer"]),
                                  use_transpose=mc["use_transpose"])
        cases[f"tf_block_{i}"] = rec
    return cases


def main():
    SelectiveLRU, SelectiveLRUMIMO, _selective_recurrence, lin, Mixer = _import_reference()
    groups = {
        "linoss": linoss_cases(lin),
        "selective_lru": selective_lru_cases(SelectiveLRU),
        "mimo": mimo_cases(SelectiveLRUMIMO),
        "recurrence": recurrence_case(_selective_recurrence),
        "mixer": mixer_cases(Mixer, SelectiveLRU, lin),
    }
    groups["blocks"] = block_cases(*_import_reference_blocks())
    for name, cases in groups.items():
        path = OUT / f"{name}.pt"
        torch.save(cases, path)
        print(f"{path.name}: {len(cases)} cases, {path.stat().st_size / 1024:.1f} KiB")


if __name__ == "__main__":
    main()
