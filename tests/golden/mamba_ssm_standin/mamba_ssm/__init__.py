"""Stand-in for the third-party ``mamba_ssm`` package (state-spaces/mamba at the commit the
reference cites, 9127d1f47f367f5c9cc49c73ad73557089d02cb8), which the reference's
``models/mamba_block.py`` imports but the reference checkout does not ship.

Used only by ``tests/golden/make_golden.py``, so that the reference's own block code
(``create_block``, ``MambaBlock``, ``TFMambaBlock``: the residual handling, the flips of the
backward branch, the permutes between the time and frequency axes, the channel
projections) runs as written and produces golden vectors. The pieces it calls are
restated from the package's documented behaviour, in plain float64-capable torch:

* ``modules.block.Block``: pre-norm residual block without an MLP; with no incoming
  residual it returns (mixer(norm(x)), x).
* ``ops.triton.layer_norm.RMSNorm``: x * rsqrt(mean(x^2) + eps) * weight.
* ``models.mixer_seq_simple._init_weights``: this repository's restatement of the
  re-initialisation rules (the fixtures record the parameters they use, so the rules
  affect no comparison).

The Mamba / Mamba2 / Mamba3 mixers and the fused ``layer_norm_fn`` are placeholders that
raise: the blocks the fixtures build never reach them.
"""
