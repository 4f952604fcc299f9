"""Expert parallelism for the INT4 MoE layer over torch.distributed (NCCL on GPUs).

Experts are partitioned in contiguous blocks: rank ``r`` of ``W`` owns experts
``[r*E/W, (r+1)*E/W)`` (GLM-4.5-Air: 64/32/16 experts per GPU at 2/4/8).
Each rank routes its own T tokens, then per layer, all on the device (no
host synchronisation, so a step can be captured in a CUDA graph):

1. ``hn_ep_pack`` writes a send buffer of W blocks of T fixed rows: row t of
   block d carries token t -- its activations only when one of its top-k picks
   lives on rank d, so a token crosses to each rank at most once whatever its
   k -- and its top-k list as rank d's local expert ids (-1 for picks owned
   elsewhere) with the routing weights;
2. one ``all_to_all_single`` with equal splits delivers block d to rank d;
3. ``hn_ep_unpack`` lays the W*T received rows out for the grouped kernel,
   which runs them with caller-supplied top-k routing (``hn_moe_experts_int4``:
   each row's output is the weighted sum of its local picks; rows whose picks
   are all -1 are skipped and cost no expert work);
4. the mirror ``all_to_all_single`` returns each row to its source rank;
5. ``hn_ep_combine`` sums, per token and in rank order in fp32, the partial
   outputs of the ranks that held one of its picks.

The reference runs experts one at a time in Python on one GPU
(``model/mixtral.py:282-370``, ``model/glm4.py:375-473``) and lists expert
parallelism on its roadmap (``README.md:179``).  Per step each rank sends and
receives W*T rows of H*2 + 8k bytes: at GLM-4.5 decode (T = 32, k = 8, W = 8)
that is 2 MB each way, against 16 MB with one row per (token, slot).

For prefill-size batches ``ep_moe_forward_chunked`` runs the same steps on
micro-batches of the rank's tokens, so each grouped call sees W*chunk rows
(the size of a one-GPU call) and the exchanges of one micro-batch are queued
beside the experts of the next: NCCL works on its own stream, the dispatch
of micro-batch i+1 is issued before the experts of micro-batch i and the
return of micro-batch i before the experts of micro-batch i+1.

``local_fn`` computes step 3 and ``exchange`` steps 1, 3 and 5; both default
to the CUDA kernels.  Tests on CPU ranks (gloo) pass reference
implementations to check the exchange bookkeeping without a GPU.
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


class CudaExchange:
    """Steps 1, 3 and 5 on the device (``hn_ep_pack`` / ``hn_ep_unpack`` / ``hn_ep_combine``)."""

    @staticmethod
    def row_bytes(H: int, k: int) -> int:
        from . import _lib
        return int(_lib.load().hn_ep_row_bytes(H, k))

    def pack(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, num_experts: int, world: int) -> torch.Tensor:
        from . import _lib
        T, H = x.shape
        k = idx.shape[1]
        send = torch.empty(world * T, self.row_bytes(H, k), dtype=torch.uint8, device=x.device)
        _lib.check(_lib.load().hn_ep_pack(x.data_ptr(), _lib.dtype_code(x.dtype), T, H, k, idx.data_ptr(),
                                          w.data_ptr(), num_experts, world, send.data_ptr(),
                                          _lib.stream_ptr(x.device)))
        return send

    def unpack(self, recv: torch.Tensor, H: int, k: int, dtype: torch.dtype):
        from . import _lib
        rows = recv.shape[0]
        xr = torch.empty(rows, H, dtype=dtype, device=recv.device)
        ir = torch.empty(rows, k, dtype=torch.int32, device=recv.device)
        wr = torch.empty(rows, k, dtype=torch.float32, device=recv.device)
        _lib.check(_lib.load().hn_ep_unpack(recv.data_ptr(), _lib.dtype_code(dtype), rows, H, k, xr.data_ptr(),
                                            ir.data_ptr(), wr.data_ptr(), _lib.stream_ptr(recv.device)))
        return xr, ir, wr

    def combine(self, back: torch.Tensor, idx: torch.Tensor, num_experts: int, world: int) -> torch.Tensor:
        from . import _lib
        T, k = idx.shape
        H = back.shape[-1]
        out = torch.empty(T, H, dtype=back.dtype, device=back.device)
        _lib.check(_lib.load().hn_ep_combine(back.data_ptr(), _lib.dtype_code(back.dtype), T, H, k, idx.data_ptr(),
                                             num_experts, world, out.data_ptr(), _lib.stream_ptr(back.device)))
        return out


def ep_moe_forward(x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, num_experts: int,
                   local_fn: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor],
                   group=None, exchange=None) -> torch.Tensor:
    """Expert-parallel dispatch -> local experts -> combine for this rank's tokens.

    x [T, H] (this rank's tokens), idx int32 [T, k] global expert ids, w
    float32 [T, k] routing weights.  ``local_fn(rows [n, H], ids int32 [n, k],
    weights float32 [n, k])`` returns, per row, the weighted sum of the
    row's picks with id >= 0 (this rank's experts, local numbering); rows whose
    ids are all -1 are unused and their outputs are ignored.
    """
    ex = exchange if exchange is not None else CudaExchange()
    world = dist.get_world_size(group)
    T, H = x.shape
    k = idx.shape[1]
    send = ex.pack(x, idx, w, num_experts, world)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    rows, ids, wts = ex.unpack(recv, H, k, x.dtype)
    y = local_fn(rows, ids, wts)
    back = torch.empty_like(y)
    dist.all_to_all_single(back, y.contiguous(), group=group)
    return ex.combine(back.view(world, T, H), idx, num_experts, world)


def ep_moe_forward_chunked(x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, num_experts: int,
                           local_fn: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor],
                           chunk: int, group=None, exchange=None, reserve_sms: int = 16) -> torch.Tensor:
    """``ep_moe_forward`` over micro-batches of ``chunk`` tokens with the
    all-to-alls issued asynchronously (every rank must pass the same T and
    chunk: the ranks take the same collective steps in the same order).  On
    the GPU the grouped kernels leave ``reserve_sms`` SMs free meanwhile
    (``hn_set_sm_limit``) so that NCCL's all-to-all kernels can run beside
    them."""
    if chunk <= 0:
        raise ValueError("chunk must be positive")
    if x.is_cuda and reserve_sms > 0:
        from . import _lib
        lib = _lib.load()
        sms = torch.cuda.get_device_properties(x.device).multi_processor_count
        prev = lib.hn_set_sm_limit(max(1, sms - reserve_sms))
        try:
            return ep_moe_forward_chunked(x, idx, w, num_experts, local_fn, chunk, group, exchange, 0)
        finally:
            lib.hn_set_sm_limit(prev)
    ex = exchange if exchange is not None else CudaExchange()
    world = dist.get_world_size(group)
    T, H = x.shape
    k = idx.shape[1]
    out = torch.empty_like(x)

    def dispatch(s):
        e = min(s + chunk, T)
        send = ex.pack(x[s:e], idx[s:e], w[s:e], num_experts, world)
        recv = torch.empty_like(send)
        return s, e, send, recv, dist.all_to_all_single(recv, send, group=group, async_op=True)

    pending = dispatch(0) if T else None
    returns = []
    while pending is not None:
        s, e, send, recv, work = pending
        work.wait()  # the current stream waits for the delivered rows
        pending = dispatch(e) if e < T else None
        rows, ids, wts = ex.unpack(recv, H, k, x.dtype)
        y = local_fn(rows, ids, wts).contiguous()
        back = torch.empty_like(y)
        returns.append((s, e, y, back, dist.all_to_all_single(back, y, group=group, async_op=True)))
    for s, e, y, back, work in returns:
        work.wait()
        out[s:e] = ex.combine(back.view(world, e - s, H), idx[s:e], num_experts, world)
    return out


def cuda_local_fn(table, world: int = 1):
    """Step 3 on the GPU: the grouped kernel over the received rows with their
    top-k local ids and weights (-1 slots take no work; all -1 rows are
    skipped).  About 1/world of the slots are this rank's; the kernel's
    token-segment width is chosen for half that (``expected_assignments``):
    measured on one B200 at the GLM-4.5 2-, 4- and 8-rank decode shapes, the
    narrower segments of the mma.sync engine were as fast or up to 12 %
    faster than the widths the mean occupancy gives."""
    from .moe import moe_experts

    def fn(rows: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        expected = max(1, rows.shape[0] * ids.shape[1] // (2 * max(world, 1)))
        return moe_experts(rows, ids, weights, table, expected_assignments=expected)

    return fn


class ExpertParallelMoE(torch.nn.Module):
    """MoE layer with experts sharded over the ranks of ``group``.

    ``router`` is the full router (replicated on every rank: a ``TopKRouter``
    or ``GLM4SigmoidRouter``); ``local_table`` is the ``ExpertTable`` of this
    rank's experts, in global order; an optional ``shared_expert`` (GLM-4.5)
    is replicated and runs on the rank's own tokens.  With ``chunk_tokens``
    set, batches larger than it go through ``ep_moe_forward_chunked``."""

    def __init__(self, router: torch.nn.Module, local_table, num_experts: int, group=None,
                 local_fn: Optional[Callable] = None, top_k: Optional[int] = None,
                 shared_expert: Optional[torch.nn.Module] = None, chunk_tokens: Optional[int] = None):
        super().__init__()
        self.chunk_tokens = chunk_tokens
        self.router = router
        self.shared_expert = shared_expert
        self.table = local_table
        self.num_experts = num_experts
        self.group = group
        self.top_k = top_k
        world = dist.get_world_size(group)
        if local_table is not None and len(local_table) * world != num_experts:
            raise ValueError("local expert table size times world size must equal the number of experts")
        self.local_fn = local_fn if local_fn is not None else cuda_local_fn(local_table, world)

    def route(self, x: torch.Tensor):
        """int32 top-k ids and float32 weights of x [T, H] (one device routing launch)."""
        from . import ops
        from .router import GLM4SigmoidRouter, TopKRouter
        if isinstance(self.router, TopKRouter):
            k = self.top_k if self.top_k is not None else self.router.experts_per_token
            bonus = self.router.bonus_vector(x.device)
            params = self.router.params(k, bonus)
            keep = (bonus,)
        elif isinstance(self.router, GLM4SigmoidRouter):
            params, keep = self.router.params(), ()
        else:
            raise TypeError("unsupported router type")
        idx, w, _ = ops.moe_route(x, params, self.num_experts, keep_refs=keep, want_logits=False)
        return idx, w

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1]).contiguous()
        idx, w = self.route(x)
        if self.chunk_tokens and x.shape[0] > self.chunk_tokens:
            y = ep_moe_forward_chunked(x, idx, w, self.num_experts, self.local_fn, self.chunk_tokens, self.group)
        else:
            y = ep_moe_forward(x, idx, w, self.num_experts, self.local_fn, self.group)
        if self.shared_expert is not None:
            y = self.shared_expert(x) + y
        return y.view(shape)
