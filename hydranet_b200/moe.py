"""Grouped INT4 MoE layers: one router launch + two expert launches per layer.

``MoELayerInt4`` replaces the host-synchronising per-expert loops of
``MixtralMoELayer.forward`` (``model/mixtral.py:259-370``) and the routed part
of ``GLM4MoELayer.forward`` (``model/glm4.py:365-473``): routing, per-expert
token lists, the INT4 SwiGLU experts and the weighted top-k combine all run
on the device with no host synchronisation, so a decode step can be captured
in a CUDA graph.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from . import ops
from .packing import ExpertTable
from .router import GLM4SigmoidRouter, RouterOutput, TopKRouter


class SharedExpertMLP(nn.Module):
    """GLM-4.5's shared expert: a dense MLP every token runs
    (``GLM4DenseMLP``, ``model/glm4.py:220-235``; built with
    ``moe_intermediate_dim * num_shared_experts`` rows, ``:341-344``):
    ``down(silu(gate(x)) * up(x))`` with unquantised weights in the model
    dtype, so it runs as library GEMMs, as in the reference."""

    def __init__(self, hidden_dim: int, intermediate_dim: int):
        super().__init__()
        self.hidden_dim, self.intermediate_dim = hidden_dim, intermediate_dim
        self.gate_proj = nn.Linear(hidden_dim, intermediate_dim, bias=False)
        self.up_proj = nn.Linear(hidden_dim, intermediate_dim, bias=False)
        self.down_proj = nn.Linear(intermediate_dim, hidden_dim, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj(torch.nn.functional.silu(self.gate_proj(x)) * self.up_proj(x))


class MoELayerInt4(nn.Module):
    """Router + INT4 experts + combine (+ an optional shared expert).

    ``router`` is a ``TopKRouter`` (softmax, Mixtral) or ``GLM4SigmoidRouter``.
    ``forward(hidden [B, S, H] or [T, H]) -> same shape``; with
    ``return_routing=True`` it also returns (idx int64, weights, logits).
    With ``shared_expert`` (GLM-4.5) the output is
    ``shared_expert(x) + routed(x)`` as in ``GLM4MoELayer.forward``
    (``model/glm4.py:378,473``).
    """

    def __init__(self, router: nn.Module, experts: ExpertTable, shared_expert: Optional[nn.Module] = None):
        super().__init__()
        self.router = router
        self.experts = experts
        self.shared_expert = shared_expert
        self.num_experts = len(experts)
        if router.num_experts != self.num_experts:
            raise ValueError("router and expert table disagree on the number of experts")

    def _params(self, x: torch.Tensor, top_k: Optional[int]):
        if isinstance(self.router, TopKRouter):
            k = top_k if top_k is not None else self.router.experts_per_token
            bonus = self.router.bonus_vector(x.device)
            return self.router.params(k, bonus), bonus
        if isinstance(self.router, GLM4SigmoidRouter):
            return self.router.params(), None
        raise TypeError("unsupported router type")

    def forward(self, hidden_states: torch.Tensor, top_k: Optional[int] = None, return_routing: bool = False):
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1]).contiguous()
        params, bonus = self._params(x, top_k)
        out, idx, w, logits = ops.moe_layer(x, params, self.experts.device_table, self.experts.device_maps,
                                            self.num_experts,
                                            self.experts.intermediate_dim, want_routing=return_routing,
                                            keep_refs=(bonus,))
        if self.shared_expert is not None:
            out = self.shared_expert(x) + out
        out = out.view(shape)
        if return_routing:
            return out, RouterOutput(idx.long(), w.to(x.dtype), logits)
        return out


    def forward_phases(self, hidden_states: torch.Tensor, between=None, top_k: Optional[int] = None):
        """Same result as ``forward``, issued as the three separate launches
        (routing/staging/plan, gate+up, down+combine); ``between(phase)`` runs
        after phases 1 and 2 (timing events, overlapping communication)."""
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1]).contiguous()
        params, bonus = self._params(x, top_k)
        out = ops.moe_layer_phases(x, params, self.experts.device_table, self.experts.device_maps,
                                   self.num_experts, self.experts.intermediate_dim, between=between)
        del bonus
        if self.shared_expert is not None:
            out = self.shared_expert(x) + out
        return out.view(shape)


def moe_experts(x: torch.Tensor, topk_idx: torch.Tensor, topk_w: torch.Tensor, experts: ExpertTable,
                expected_assignments: int = 0) -> torch.Tensor:
    """Experts + weighted combine for externally routed tokens (x [T, H]);
    ``expected_assignments`` as in ``ops.moe_experts``."""
    return ops.moe_experts(x, topk_idx, topk_w, experts.device_table, experts.device_maps, len(experts),
                           experts.intermediate_dim, expected_assignments)
