"""Placeholder for ``mamba_ssm.modules.mamba2.Mamba2`` (not used by the fixtures)."""


class Mamba2:
    def __init__(self, *args, **kwargs):
        raise NotImplementedError("Mamba2 is not part of the mamba_ssm stand-in")
