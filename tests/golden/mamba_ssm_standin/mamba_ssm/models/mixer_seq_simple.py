"""``_init_weights`` for the stand-in: the restatement in ``semambaxlinoss_b200.mamba_block``."""
from semambaxlinoss_b200.mamba_block import _init_weights  # noqa: F401
