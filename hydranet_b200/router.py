"""Routers with the reference's module interfaces, running on the CUDA library.

``TopKRouter`` mirrors ``model/router.py:28-200`` (Mixtral softmax top-k with
the optional cache-affinity bonus); ``GLM4SigmoidRouter`` mirrors
``model/glm4.py:238-309`` (sigmoid top-k), plus the GLM-4.5
``e_score_correction_bias`` that the reference loads but never applies
(``model/glm4_loader.py:164-167``): when set it biases the SELECTION only.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.nn as nn

from . import _lib, ops


@dataclass
class RouterOutput:
    """``model/router.py:20-25``."""
    expert_indices: torch.Tensor  # (batch, seq, top_k) int64
    expert_weights: torch.Tensor  # (batch, seq, top_k) hidden dtype
    router_logits: torch.Tensor   # (batch, seq, num_experts) float32


def _cfg(obj, name, default):
    return getattr(obj, name, default) if obj is not None else default


class TopKRouter(nn.Module):
    """Mixtral router: logits -> (affinity bonus) -> top-k -> softmax over the selected.

    Constructor accepts the reference's ``(config, cache_config, layer_idx)``
    (``model/router.py:38-67``) or plain keyword sizes.
    """

    def __init__(self, config=None, cache_config=None, layer_idx: int = 0, *, hidden_dim: Optional[int] = None,
                 num_experts: Optional[int] = None, experts_per_token: int = 2):
        super().__init__()
        self.config = config
        self.cache_config = cache_config
        self.layer_idx = layer_idx
        self.hidden_dim = hidden_dim or config.hidden_dim
        self.num_experts = num_experts or config.num_experts
        self.experts_per_token = _cfg(config, "experts_per_token", experts_per_token)
        self.gate = nn.Linear(self.hidden_dim, self.num_experts, bias=False)
        self.affinity_bonus = _cfg(cache_config, "affinity_bonus", 0.1)
        self.entropy_threshold = _cfg(cache_config, "affinity_entropy_threshold", 0.5)
        self.enable_affinity_bonus = _cfg(cache_config, "enable_affinity_bonus", False)
        self.register_buffer("usage_counts", torch.zeros(self.num_experts, dtype=torch.long), persistent=False)
        self._is_cached_fn: Optional[Callable[[int], bool]] = None
        self._bonus_buf: Optional[torch.Tensor] = None

    def set_cache_checker(self, fn: Callable[[int], bool]):
        self._is_cached_fn = fn

    def bonus_vector(self, device) -> Optional[torch.Tensor]:
        """Per-expert affinity bonus (``model/router.py:160-168``), or None when disabled.

        The bonus lives in one persistent device buffer, refreshed in place
        from the cache checker on every call outside CUDA-graph capture, so a
        captured layer reads the current cache state when it replays (refresh
        it with ``refresh_bonus`` before a replay)."""
        if not self.enable_affinity_bonus or self._is_cached_fn is None:
            return None
        if self._bonus_buf is None or self._bonus_buf.device != torch.device(device):
            self._bonus_buf = torch.zeros(self.num_experts, dtype=torch.float32, device=device)
        if not torch.cuda.is_current_stream_capturing():
            self.refresh_bonus()
        return self._bonus_buf

    def refresh_bonus(self):
        """Write the current per-expert bonus into the persistent buffer (host values, one small copy)."""
        if self._bonus_buf is None or self._is_cached_fn is None:
            return
        vals = [self.affinity_bonus if self._is_cached_fn(e) else 0.0 for e in range(self.num_experts)]
        self._bonus_buf.copy_(torch.tensor(vals, dtype=torch.float32))

    def params(self, top_k: int, bonus: Optional[torch.Tensor]) -> _lib.RouterParams:
        return ops.router_params(_lib.HN_ROUTER_SOFTMAX_TOPK, top_k, self.gate.weight, logits_in_act_dtype=True,
                                 affinity_bonus=bonus, entropy_threshold=self.entropy_threshold)

    def forward(self, hidden_states: torch.Tensor, top_k_override: Optional[int] = None,
                apply_affinity: bool = True) -> RouterOutput:
        b, s, h = hidden_states.shape
        top_k = top_k_override if top_k_override is not None else self.experts_per_token
        x = hidden_states.reshape(b * s, h)
        if self.gate.weight.dtype != x.dtype:
            raise TypeError("router gate weight must be in the model dtype (model/router.py:102)")
        bonus = self.bonus_vector(x.device) if apply_affinity else None
        idx, w, logits = ops.moe_route(x, self.params(top_k, bonus), self.num_experts, keep_refs=(bonus,))
        if not self.training:
            # scatter_add_, not torch.bincount: bincount reads its maximum back to the host
            flat = idx.reshape(-1).long()
            self.usage_counts.scatter_add_(0, flat, torch.ones_like(flat))
        return RouterOutput(idx.long().view(b, s, top_k), w.to(hidden_states.dtype).view(b, s, top_k),
                            logits.view(b, s, self.num_experts))

    def get_expert_priorities(self) -> torch.Tensor:
        return self.usage_counts.float()

    def get_top_experts(self, k: int) -> torch.Tensor:
        return torch.topk(self.usage_counts, k).indices

    def reset_usage(self):
        self.usage_counts.zero_()


class GLM4SigmoidRouter(nn.Module):
    """GLM-4.5 router (``model/glm4.py:238-309``) with an optional correction bias;
    group-limited selection when ``n_group > 1`` (``model/glm4.py:285-297``)."""

    def __init__(self, config=None, layer_idx: int = 0, *, hidden_dim: Optional[int] = None,
                 num_experts: Optional[int] = None, experts_per_token: int = 8, n_group: int = 1,
                 topk_group: int = 1):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.hidden_dim = hidden_dim or config.hidden_dim
        self.num_experts = num_experts or config.num_experts
        self.top_k = _cfg(config, "experts_per_token", experts_per_token)
        self.n_group = _cfg(config, "n_group", n_group)
        self.topk_group = _cfg(config, "topk_group", topk_group)
        self.norm_topk_prob = _cfg(config, "norm_topk_prob", True)
        self.routed_scaling_factor = _cfg(config, "routed_scaling_factor", 1.0)
        self.weight = nn.Parameter(torch.empty(self.num_experts, self.hidden_dim))
        nn.init.normal_(self.weight, std=0.02)
        self.e_score_correction_bias: Optional[torch.Tensor] = None

    def set_correction_bias(self, bias: Optional[torch.Tensor]):
        self.e_score_correction_bias = None if bias is None else bias.detach().float().contiguous()

    def params(self) -> _lib.RouterParams:
        return ops.router_params(_lib.HN_ROUTER_SIGMOID_TOPK, self.top_k, self.weight, logits_in_act_dtype=False,
                                 correction_bias=self.e_score_correction_bias, norm_topk_prob=self.norm_topk_prob,
                                 routed_scaling_factor=self.routed_scaling_factor, n_group=self.n_group,
                                 topk_group=self.topk_group)

    def forward(self, hidden_states: torch.Tensor):
        h = hidden_states.shape[-1]
        x = hidden_states.reshape(-1, h)
        idx, w, _ = ops.moe_route(x, self.params(), self.num_experts, want_logits=False)
        return idx.long(), w.to(hidden_states.dtype)
