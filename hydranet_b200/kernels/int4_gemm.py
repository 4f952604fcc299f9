"""Drop-in for HydraNet's ``kernels/int4_gemm.py`` on sm_100a.

Same names, arguments and return shapes as the reference module
(``kernels/int4_gemm.py:124-254``); the Triton kernels are replaced by the
hand-written CUDA library.  ``expert_mlp_int4_fused`` is ONE fused two-phase
pass (gate+up+SiLU, then down) instead of the reference's four launches, and
no gate/up intermediate ever reaches HBM in the activation dtype.
"""

from __future__ import annotations

import torch

from .. import ops


def int4_linear(x: torch.Tensor, w_packed: torch.Tensor, w_scales: torch.Tensor,
                group_size: int = 128) -> torch.Tensor:
    """``out = x @ W.T`` with W INT4-packed; x [M, K] or [B, S, K]
    (``kernels/int4_gemm.py:124-172``)."""
    return ops.int4_linear(x, w_packed, w_scales, group_size)


def fused_silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` (``kernels/int4_gemm.py:196-208``)."""
    return ops.silu_mul(gate, up)


def expert_mlp_int4_fused(x: torch.Tensor, gate_packed: torch.Tensor, gate_scales: torch.Tensor,
                          up_packed: torch.Tensor, up_scales: torch.Tensor, down_packed: torch.Tensor,
                          down_scales: torch.Tensor, group_size: int = 128) -> torch.Tensor:
    """``down(silu(gate(x)) * up(x))`` (``kernels/int4_gemm.py:211-254``)."""
    return ops.expert_mlp_int4(x, gate_packed, gate_scales, up_packed, up_scales, down_packed, down_scales,
                               group_size)


__all__ = ["int4_linear", "fused_silu_mul", "expert_mlp_int4_fused"]
