"""Group-by-expert gather and scatter with the interface of HydraNet's
``GatheredTokens`` / ``GroupByExpertGatherer`` (``scheduler/continuous_batch.py:266-381``).

For callers that drive their own per-expert loop: ``gather`` returns one
``GatheredTokens`` per expert that has tokens, in ascending expert order, each
listing its (token, slot) assignments by token, then slot; ``scatter`` sums
``routing_weight * expert_output`` back into token order.

The reference builds one boolean mask per touched expert (a pass over the
routing and several launches per expert).  Here one stable sort of the
flattened routing by expert id puts every assignment in that same order at
once, and one host read of the per-expert counts cuts it into the list (the
reference reads its list of experts back to the host too).  ``scatter`` is one
``index_add_`` over all experts' weighted rows in list order, which adds each
output row's terms in the order the reference's per-expert calls add them.

To run the experts themselves, ``hydranet_b200.moe.moe_experts`` does the
gather, the INT4 expert MLPs and the weighted combine in one device pass with
no host read.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Tuple

import torch


@dataclass
class GatheredTokens:
    """The assignments of one expert (``scheduler/continuous_batch.py:265-278``)."""

    expert_idx: int
    layer_idx: int
    token_indices: torch.Tensor     # int64 [n]: token of each assignment
    hidden_states: torch.Tensor     # [n, hidden]: those tokens' rows
    routing_weights: torch.Tensor   # [n]: the assignment's routing weight

    @property
    def num_tokens(self) -> int:
        return self.token_indices.shape[0]


class GroupByExpertGatherer:
    """Gather tokens by expert, scatter expert outputs back
    (``scheduler/continuous_batch.py:281-381``)."""

    def __init__(self, device: torch.device = torch.device("cuda")):
        self.device = device

    def gather(self, hidden_states: torch.Tensor, expert_indices: torch.Tensor, expert_weights: torch.Tensor,
               layer_idx: int) -> List[GatheredTokens]:
        """hidden_states [T, H], expert_indices / expert_weights [T, k] ->
        one ``GatheredTokens`` per expert present, ascending expert id.  A
        token that picks an expert twice appears twice in its list."""
        top_k = expert_indices.shape[1]
        flat = expert_indices.reshape(-1)
        order = torch.sort(flat, stable=True).indices        # by expert; (token, slot) order kept
        experts, counts = torch.unique_consecutive(flat.index_select(0, order), return_counts=True)
        tok = torch.div(order, top_k, rounding_mode="floor")
        slot = order - tok * top_k
        rows = hidden_states.index_select(0, tok)
        wts = expert_weights[tok, slot]
        sizes = counts.tolist()                                # the one host read
        return [GatheredTokens(expert_idx=int(e), layer_idx=layer_idx, token_indices=t, hidden_states=h,
                               routing_weights=w)
                for e, t, h, w in zip(experts.tolist(), tok.split(sizes), rows.split(sizes), wts.split(sizes))]

    def scatter(self, gathered_outputs: List[Tuple[GatheredTokens, torch.Tensor]],
                output_shape: Tuple[int, int]) -> torch.Tensor:
        """Sum ``routing_weight * output`` of every gathered assignment into a
        zeroed [T, H] tensor of the first output's dtype (float16 when the
        list is empty)."""
        dtype = gathered_outputs[0][1].dtype if gathered_outputs else torch.float16
        output = torch.zeros(output_shape, device=self.device, dtype=dtype)
        if not gathered_outputs:
            return output
        index = torch.cat([g.token_indices for g, _ in gathered_outputs])
        rows = torch.cat([out * g.routing_weights.unsqueeze(-1) for g, out in gathered_outputs])
        output.index_add_(0, index, rows)
        return output


__all__ = ["GatheredTokens", "GroupByExpertGatherer"]
