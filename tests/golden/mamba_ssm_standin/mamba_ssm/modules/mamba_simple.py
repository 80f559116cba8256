"""Placeholder for ``mamba_ssm.modules.mamba_simple.Mamba`` (not used by the fixtures)."""


class Mamba:
    def __init__(self, *args, **kwargs):
        raise NotImplementedError("Mamba is not part of the mamba_ssm stand-in")
