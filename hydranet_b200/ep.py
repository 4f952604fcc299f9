"""Expert parallelism for the INT4 MoE layer over torch.distributed (NCCL on GPUs).

Experts are partitioned in contiguous blocks: rank ``r`` of ``W`` owns experts
``[r*E/W, (r+1)*E/W)`` (GLM-4.5-Air: 64/32/16 experts per GPU at 2/4/8).
Each rank routes its own tokens, then per layer:

1. ``all_to_all_single`` of per-destination assignment counts (int64), read
   back to size the exchange;
2. one variable-split ``all_to_all_single`` of byte rows, each the routed
   token's activations followed by its (local expert, routing weight) pair;
3. the rank's grouped kernel over what it received, with caller-supplied
   routing (``hn_moe_experts_int4``: each received row is one assignment,
   top-1 with its routing weight, so the kernel returns weight * MLP_e(x));
4. the mirror ``all_to_all_single`` of the weighted rows back to their source
   ranks, summed per token in float32 and cast to the activation dtype.

The reference runs experts one at a time in Python on one GPU
(``model/glm4.py:375-473``, ``model/mixtral.py:282-370``); the exchange is the
standard expert-parallel dispatch/combine.  One row is sent per (token, slot)
assignment, which keeps the combine order fixed (slot order), so results do
not depend on the number of ranks beyond fp32 summation of the k partial
outputs.

``local_fn`` computes step 3 and defaults to the CUDA grouped kernel; tests
on CPU ranks (gloo) pass a reference implementation to check the exchange
bookkeeping without a GPU.
"""

from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist


def expert_range(num_experts: int, rank: int, world: int) -> Tuple[int, int]:
    """[first, last) experts owned by ``rank`` (contiguous blocks)."""
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not split evenly over {world} ranks")
    per = num_experts // world
    return rank * per, (rank + 1) * per


def owner_of(expert: torch.Tensor, num_experts: int, world: int) -> torch.Tensor:
    return torch.div(expert, num_experts // world, rounding_mode="floor")


class DispatchPlan:
    """Host-free bookkeeping of one exchange (all tensors stay on the device).

    ``order``     assignment ids (t*k + slot) sorted by destination rank, stable;
    ``send``      rows sent to each rank; ``recv`` rows received from each rank.
    """

    def __init__(self, idx: torch.Tensor, num_experts: int, world: int, group=None):
        T, k = idx.shape
        dest = owner_of(idx.reshape(-1), num_experts, world)
        self.order = torch.sort(dest, stable=True).indices
        self.send = torch.bincount(dest, minlength=world).to(torch.int64)
        self.recv = torch.empty_like(self.send)
        dist.all_to_all_single(self.recv, self.send, group=group)
        # split sizes must be host ints for all_to_all_single: one device->host read
        self.send_splits, self.recv_splits = torch.stack([self.send, self.recv]).tolist()
        self.T, self.k = T, k


def exchange(t: torch.Tensor, plan: DispatchPlan, forward: bool, group=None) -> torch.Tensor:
    """Variable-split all-to-all of rows of ``t`` (dispatch if ``forward``, else combine)."""
    ins, outs = (plan.send_splits, plan.recv_splits) if forward else (plan.recv_splits, plan.send_splits)
    out = torch.empty((sum(outs),) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    dist.all_to_all_single(out, t.contiguous(), output_split_sizes=outs, input_split_sizes=ins, group=group)
    return out


def ep_moe_forward(x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, num_experts: int,
                   local_fn: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor],
                   group=None) -> torch.Tensor:
    """Expert-parallel dispatch -> local experts -> combine for this rank's tokens.

    x [T, H] (this rank's tokens), idx [T, k] global expert ids, w [T, k]
    routing weights.  ``local_fn(rows [n, H], local_expert [n], weight [n])``
    returns weight * MLP_e(row) for each received row (activation dtype).
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    T, H = x.shape
    k = idx.shape[1]
    first, _ = expert_range(num_experts, rank, world)
    plan = DispatchPlan(idx, num_experts, world, group)
    tok = torch.div(plan.order, k, rounding_mode="floor")
    # one byte row per assignment: the token's activations, then the local
    # expert id (int32) and the routing weight (float32), so the dispatch is a
    # single all-to-all
    rb = H * x.element_size()
    packed = torch.empty(tok.numel(), rb + 8, dtype=torch.uint8, device=x.device)
    packed[:, :rb] = x.index_select(0, tok).view(torch.uint8).view(-1, rb)
    packed[:, rb:rb + 4] = idx.reshape(-1).index_select(0, plan.order).to(torch.int32).view(-1, 1).view(torch.uint8)
    packed[:, rb + 4:] = w.reshape(-1).index_select(0, plan.order).to(torch.float32).view(-1, 1).view(torch.uint8)
    recv = exchange(packed, plan, True, group)
    r_rows = recv[:, :rb].contiguous().view(x.dtype).view(-1, H)
    local = recv[:, rb:rb + 4].contiguous().view(torch.int32).view(-1) - first  # global id -> this rank's
    r_w = recv[:, rb + 4:].contiguous().view(torch.float32).view(-1)
    y = local_fn(r_rows, local, r_w) if r_rows.shape[0] else r_rows.new_zeros((0, H))
    back = exchange(y, plan, False, group)
    out = torch.zeros(T, H, dtype=torch.float32, device=x.device)
    out.index_add_(0, tok, back.to(torch.float32))
    return out.to(x.dtype)


def cuda_local_fn(table):
    """Step 3 on the GPU: the grouped kernel over the received rows, each row one
    assignment (top-1 with its routing weight) into this rank's expert table."""
    from .moe import moe_experts

    def fn(rows: torch.Tensor, local_expert: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
        return moe_experts(rows, local_expert.view(-1, 1).to(torch.int32), weight.view(-1, 1), table)

    return fn


class ExpertParallelMoE(torch.nn.Module):
    """MoE layer with experts sharded over the ranks of ``group``.

    ``router`` is the full router (replicated on every rank); ``local_table``
    is the ``ExpertTable`` of this rank's experts, in global order."""

    def __init__(self, router: torch.nn.Module, local_table, num_experts: int, group=None,
                 local_fn: Optional[Callable] = None):
        super().__init__()
        self.router = router
        self.table = local_table
        self.num_experts = num_experts
        self.group = group
        world = dist.get_world_size(group)
        if local_table is not None and len(local_table) * world != num_experts:
            raise ValueError("local expert table size times world size must equal the number of experts")
        self.local_fn = local_fn if local_fn is not None else cuda_local_fn(local_table)

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1]).contiguous()
        out = self.router(x.view(1, *x.shape))  # routers take [batch, seq, hidden]
        idx, w = (out.expert_indices, out.expert_weights) if hasattr(out, "expert_indices") else out
        idx = idx.reshape(x.shape[0], -1)
        w = w.reshape(x.shape[0], -1)
        y = ep_moe_forward(x, idx, w, self.num_experts, self.local_fn, self.group)
        return y.view(shape)
