"""Part of the mamba_ssm stand-in (see the package docstring)."""
