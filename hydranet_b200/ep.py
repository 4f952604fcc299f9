"""Expert parallelism for the INT4 MoE layer over torch.distributed (NCCL on GPUs).

Experts are partitioned in contiguous blocks: rank ``r`` of ``W`` owns experts
``[r*E/W, (r+1)*E/W)`` (GLM-4.5-Air: 64/32/16 experts per GPU at 2/4/8).
Each rank routes its own tokens, then per layer, all on the device (no
host synchronisation, so the host keeps queueing work):

1. the T*k assignments are grouped by owner rank and placed into a send
   buffer of W blocks of C = T*k fixed slots (any split of the assignments
   fits), one byte row per slot: the token's activations, its global expert
   id (int32, -1 in an unused slot) and its routing weight (float32);
2. one ``all_to_all_single`` with equal splits delivers block r to rank r;
3. the rank's grouped kernel runs over the W*C received rows with
   caller-supplied routing (``hn_moe_experts_int4``: top-1 per row with its
   routing weight, so it returns weight * MLP_e(x); rows whose id is -1 are
   skipped and cost no expert work);
4. the mirror ``all_to_all_single`` returns the rows to their source ranks,
   which sum the k rows of each token in slot order in float32 and cast to
   the activation dtype.

The reference runs experts one at a time in Python on one GPU
(``model/mixtral.py:282-370``, ``model/glm4.py:375-473``); the exchange is the
standard expert-parallel dispatch/combine.  One row is sent per (token, slot)
assignment and the combine order is the slot order, so results do not depend
on the number of ranks beyond fp32 summation of the k partial outputs.  The
fixed slots trade a few MB of padding per step (W*T*k rows, mostly empty) for
split sizes that never have to be read back to the host.

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


def ep_moe_forward(x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, num_experts: int,
                   local_fn: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor],
                   group=None) -> torch.Tensor:
    """Expert-parallel dispatch -> local experts -> combine for this rank's tokens.

    x [T, H] (this rank's tokens), idx [T, k] global expert ids, w [T, k]
    routing weights.  ``local_fn(rows [n, H], local_expert [n], weight [n])``
    returns weight * MLP_e(row) for each received row whose local expert is
    >= 0 (activation dtype); rows with local expert -1 are unused slots and
    their outputs are ignored.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    T, H = x.shape
    k = idx.shape[1]
    dev = x.device
    first, _ = expert_range(num_experts, rank, world)
    n = T * k
    C = n  # slots per destination block
    flat = idx.reshape(-1)
    dest = owner_of(flat, num_experts, world)
    order = torch.sort(dest, stable=True).indices  # assignments grouped by destination, slot order kept
    d_sorted = dest.index_select(0, order)
    # per-destination counts without torch.bincount (which reads its maximum back to the host)
    counts = torch.zeros(world, dtype=dest.dtype, device=dev).scatter_add_(0, dest, torch.ones_like(dest))
    starts = torch.cumsum(counts, 0) - counts
    row = d_sorted * C + (torch.arange(n, device=dev) - starts.index_select(0, d_sorted))
    tok = torch.div(order, k, rounding_mode="floor")
    rb = H * x.element_size()
    # send buffer: W blocks of C rows; unused rows carry expert id -1 (0xFF bytes)
    send = torch.zeros(world * C, rb + 8, dtype=torch.uint8, device=dev)
    send[:, rb:rb + 4] = 255
    packed = torch.empty(n, rb + 8, dtype=torch.uint8, device=dev)
    packed[:, :rb] = x.index_select(0, tok).view(torch.uint8).view(-1, rb)
    packed[:, rb:rb + 4] = flat.index_select(0, order).to(torch.int32).view(-1, 1).view(torch.uint8)
    packed[:, rb + 4:] = w.reshape(-1).index_select(0, order).to(torch.float32).view(-1, 1).view(torch.uint8)
    send.index_copy_(0, row, packed)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    r_rows = recv[:, :rb].contiguous().view(x.dtype).view(-1, H)
    g = recv[:, rb:rb + 4].contiguous().view(torch.int32).view(-1)
    local = torch.where(g >= 0, g - first, g)  # global id -> this rank's; -1 stays
    r_w = recv[:, rb + 4:].contiguous().view(torch.float32).view(-1)
    y = local_fn(r_rows, local, r_w)
    back = torch.empty_like(y)
    dist.all_to_all_single(back, y.contiguous(), group=group)
    out = torch.zeros(T, H, dtype=torch.float32, device=dev)
    out.index_add_(0, tok, back.index_select(0, row).to(torch.float32))
    return out.to(x.dtype)


def cuda_local_fn(table):
    """Step 3 on the GPU: the grouped kernel over the received rows, each row one
    assignment (top-1 with its routing weight) into this rank's expert table."""
    from .moe import moe_experts

    def fn(rows: torch.Tensor, local_expert: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
        # local expert -1 (an unused slot) is skipped by the kernel
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
