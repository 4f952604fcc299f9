"""Drop-in for HydraNet's ``kernels/expert_mlp.py`` exports on sm_100a.

The reference's ``ExpertMLPTriton.forward`` dequantises and multiplies in
torch (``kernels/expert_mlp.py:289-303``); here it runs the fused CUDA MLP.
``expert_mlp_int4`` keeps the reference's extra ``hidden_dim`` and
``intermediate_dim`` arguments (``kernels/expert_mlp.py:334-354``).
"""

from __future__ import annotations

import torch

from .. import ops


class ExpertMLPTriton:
    """Same constructor and ``forward`` arguments as ``kernels/expert_mlp.py:230-303``."""

    def __init__(self, hidden_dim: int, intermediate_dim: int, group_size: int = 128,
                 device: torch.device = torch.device("cuda")):
        self.hidden_dim = hidden_dim
        self.intermediate_dim = intermediate_dim
        self.group_size = group_size
        self.device = device

    def forward(self, x, gate_packed, gate_scales, up_packed, up_scales, down_packed, down_scales):
        assert x.shape[-1] == self.hidden_dim and gate_packed.shape[0] == self.intermediate_dim
        return ops.expert_mlp_int4(x, gate_packed, gate_scales, up_packed, up_scales, down_packed, down_scales,
                                   self.group_size)

    __call__ = forward


def expert_mlp_int4(x, gate_packed, gate_scales, up_packed, up_scales, down_packed, down_scales,
                    hidden_dim: int, intermediate_dim: int, group_size: int = 128) -> torch.Tensor:
    return ExpertMLPTriton(hidden_dim, intermediate_dim, group_size, x.device).forward(
        x, gate_packed, gate_scales, up_packed, up_scales, down_packed, down_scales)
