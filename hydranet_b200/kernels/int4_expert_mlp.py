"""Drop-in for HydraNet's ``kernels/int4_expert_mlp.py`` on sm_100a.

Same public functions as the reference (``kernels/int4_expert_mlp.py:99-272``):
``int4_linear``, ``silu_mul``, ``expert_mlp_int4`` and
``expert_mlp_int4_from_slot`` (which reads the six buffers of a
``GpuExpertSlot``-shaped object).
"""

from __future__ import annotations

import torch

from .. import ops


def int4_linear(x: torch.Tensor, w_packed: torch.Tensor, w_scales: torch.Tensor,
                group_size: int = 128) -> torch.Tensor:
    """``kernels/int4_expert_mlp.py:99-156``."""
    return ops.int4_linear(x, w_packed, w_scales, group_size)


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``kernels/int4_expert_mlp.py:189-210`` (accepts 2-D or 3-D inputs)."""
    return ops.silu_mul(gate, up)


def expert_mlp_int4(x: torch.Tensor, gate_packed: torch.Tensor, gate_scales: torch.Tensor, up_packed: torch.Tensor,
                    up_scales: torch.Tensor, down_packed: torch.Tensor, down_scales: torch.Tensor,
                    group_size: int = 128) -> torch.Tensor:
    """``kernels/int4_expert_mlp.py:213-252``."""
    return ops.expert_mlp_int4(x, gate_packed, gate_scales, up_packed, up_scales, down_packed, down_scales,
                               group_size)


def expert_mlp_int4_from_slot(x: torch.Tensor, gpu_slot, group_size: int = 128) -> torch.Tensor:
    """Run the expert held by a ``GpuExpertSlot`` (``kernels/int4_expert_mlp.py:255-272``).

    Like the reference it does not wait on the slot's ``ready_event``; callers
    obtain slots through the cache, which waits (``cache/packed_expert_store.py:323-331``).
    """
    return ops.expert_mlp_int4(x, gpu_slot.gate_packed, gpu_slot.gate_scales, gpu_slot.up_packed,
                               gpu_slot.up_scales, gpu_slot.down_packed, gpu_slot.down_scales, group_size)


__all__ = ["int4_linear", "silu_mul", "expert_mlp_int4", "expert_mlp_int4_from_slot"]
