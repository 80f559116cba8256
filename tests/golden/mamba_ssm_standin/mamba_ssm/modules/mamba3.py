"""Placeholder for ``mamba_ssm.modules.mamba3.Mamba3`` (not used by the fixtures)."""


class Mamba3:
    def __init__(self, *args, **kwargs):
        raise NotImplementedError("Mamba3 is not part of the mamba_ssm stand-in")
