"""Pre-norm residual block (stand-in for ``mamba_ssm.modules.block.Block``)."""
from __future__ import annotations

from torch import nn


class Block(nn.Module):
    def __init__(self, dim, mixer_cls, mlp_cls, norm_cls=nn.LayerNorm, fused_add_norm=False,
                 residual_in_fp32=False):
        super().__init__()
        if fused_add_norm or mlp_cls is not nn.Identity:
            raise NotImplementedError("the stand-in Block has neither the fused add-norm nor an MLP")
        self.residual_in_fp32 = residual_in_fp32
        self.norm = norm_cls(dim)
        self.mixer = mixer_cls(dim)

    def forward(self, hidden_states, residual=None, inference_params=None, **mixer_kwargs):
        # The residual stream carries the block input (plus the incoming residual, if any);
        # the mixer sees its normalised form.
        residual = hidden_states if residual is None else hidden_states + residual
        normed = self.norm(residual.to(self.norm.weight.dtype))
        if self.residual_in_fp32:
            residual = residual.float()
        return self.mixer(normed, inference_params=inference_params, **mixer_kwargs), residual
