"""Tensor parallelism for the dense parts of GLM-4.5 around the MoE layers.

Expert parallelism (``ep.py``) shards the routed experts; the rest of a
GLM-4.5 layer -- attention (96 query / 8 KV heads), the dense FFN of layer 0,
the shared expert and the lm_head (``model/glm4.py:113-240,341-344,640-641``)
-- would otherwise be replicated on every GPU and cap the scaling of a whole
model step.  Here each of them is split over the ranks of a process group in
the standard Megatron layout, so one layer costs one all-reduce after the
attention and one after the MLP:

* ``ColumnParallelLinear``: rank r holds rows [r*N/W, (r+1)*N/W) of the
  weight (and bias) and produces that slice of the output;
* ``RowParallelLinear``: rank r holds columns [r*K/W, (r+1)*K/W), multiplies
  its slice of the input and the partial outputs are summed by one
  all-reduce (NCCL; NVLink SHARP in the switch where NCCL enables it);
* ``TPDenseMLP``: gate/up column-parallel, SiLU(gate)*up on the local slice,
  down row-parallel -- ``GLM4DenseMLP`` (shared expert, dense FFN);
* ``TPAttention``: Q/K/V column-parallel by heads (n_heads/W query heads and
  n_kv/W KV heads per rank; when W exceeds n_kv, each KV head is replicated
  on the W/n_kv ranks whose query heads use it), partial rotary embedding,
  grouped-query attention with the per-rank ``TPKVCache``, O row-parallel --
  ``GLM4Attention``;
* ``VocabParallelLMHead``: the vocabulary split over the ranks, logits
  all-gathered (or left sharded).

Every module is built from the full (reference-layout) module with
``from_module`` and computes what the full module computes.  Linears take
either float weights (cuBLAS through torch) or INT4 ``Int4Linear`` weights,
which run on this library's ``hn_int4_linear`` (row-parallel INT4 splits K
on 128-column group boundaries).
"""

from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F


def _world(group) -> Tuple[int, int]:
    return dist.get_world_size(group), dist.get_rank(group)


def _split(n: int, world: int, rank: int, what: str) -> Tuple[int, int]:
    if n % world:
        raise ValueError(f"{what} ({n}) does not split evenly over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


class _Int4Weight:
    """INT4 weight slice (packed [N, K/2] uint8, scales [N, K/128] fp16) run by ``hn_int4_linear``."""

    def __init__(self, packed: torch.Tensor, scales: torch.Tensor):
        self.packed = packed.contiguous()
        self.scales = scales.contiguous()

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        from .kernels.int4_gemm import int4_linear
        return int4_linear(x, self.packed, self.scales)


def _int4_parts(lin) -> Optional[Tuple[torch.Tensor, torch.Tensor]]:
    """(packed, scales) of an ``Int4Linear`` (this package's or the reference's), else None."""
    p = getattr(lin, "weight_packed", None)
    s = getattr(lin, "weight_scale", None)
    if p is None or s is None:
        return None
    if getattr(lin, "group_size", 128) != 128:
        raise ValueError("INT4 tensor parallelism needs group size 128")
    return p, s


class ColumnParallelLinear(nn.Module):
    """Output features split over the ranks; ``gather_output`` all-gathers them."""

    def __init__(self, weight, bias: Optional[torch.Tensor], out_features: int, group=None,
                 gather_output: bool = False):
        super().__init__()
        self.group = group
        self.out_features = out_features
        self.gather_output = gather_output
        self.int4 = isinstance(weight, _Int4Weight)
        if self.int4:
            self._w4 = weight
        else:
            self.weight = nn.Parameter(weight, requires_grad=False)
        self.bias = nn.Parameter(bias, requires_grad=False) if bias is not None else None

    @classmethod
    def from_linear(cls, lin: nn.Module, group=None, gather_output: bool = False) -> "ColumnParallelLinear":
        W, r = _world(group)
        parts = _int4_parts(lin)
        n = lin.out_features
        a, b = _split(n, W, r, "output features")
        bias = getattr(lin, "bias", None)
        bias = None if bias is None else bias.detach()[a:b].clone()
        if parts is not None:
            w = _Int4Weight(parts[0][a:b], parts[1][a:b])
        else:
            w = lin.weight.detach()[a:b].clone()
        return cls(w, bias, n, group, gather_output)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        y = self._w4(x2) if self.int4 else F.linear(x2, self.weight)
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        if self.gather_output:
            W, _ = _world(self.group)
            parts = [torch.empty_like(y) for _ in range(W)]
            dist.all_gather(parts, y.contiguous(), group=self.group)
            y = torch.cat(parts, dim=-1)
        return y.view(*shape[:-1], y.shape[-1])


class RowParallelLinear(nn.Module):
    """Input features split over the ranks; partial products summed by one all-reduce
    (the bias, if any, is added once, after the sum)."""

    def __init__(self, weight, bias: Optional[torch.Tensor], in_features: int, group=None,
                 input_is_parallel: bool = True, reduce: bool = True):
        super().__init__()
        self.group = group
        self.in_features = in_features
        self.input_is_parallel = input_is_parallel
        self.reduce = reduce
        self.int4 = isinstance(weight, _Int4Weight)
        if self.int4:
            self._w4 = weight
        else:
            self.weight = nn.Parameter(weight, requires_grad=False)
        self.bias = nn.Parameter(bias, requires_grad=False) if bias is not None else None

    @classmethod
    def from_linear(cls, lin: nn.Module, group=None, input_is_parallel: bool = True,
                    reduce: bool = True) -> "RowParallelLinear":
        W, r = _world(group)
        parts = _int4_parts(lin)
        k = lin.in_features
        a, b = _split(k, W, r, "input features")
        bias = getattr(lin, "bias", None)
        bias = None if bias is None else bias.detach().clone()
        if parts is not None:
            if a % 128 or b % 128:
                raise ValueError("row-parallel INT4 needs each rank's input slice on 128-column group boundaries")
            w = _Int4Weight(parts[0][:, a // 2:b // 2], parts[1][:, a // 128:b // 128])
        else:
            w = lin.weight.detach()[:, a:b].clone()
        return cls(w, bias, k, group, input_is_parallel, reduce)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self.input_is_parallel:
            W, r = _world(self.group)
            a, b = _split(x.shape[-1], W, r, "input features")
            x = x[..., a:b]
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        y = self._w4(x2) if self.int4 else F.linear(x2, self.weight)
        if self.reduce:
            dist.all_reduce(y, group=self.group)
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y.view(*shape[:-1], y.shape[-1])


class TPDenseMLP(nn.Module):
    """``GLM4DenseMLP`` (``model/glm4.py:226-240``) split over the ranks: one all-reduce."""

    def __init__(self, gate: ColumnParallelLinear, up: ColumnParallelLinear, down: RowParallelLinear):
        super().__init__()
        self.gate_proj, self.up_proj, self.down_proj = gate, up, down

    @classmethod
    def from_module(cls, mlp: nn.Module, group=None) -> "TPDenseMLP":
        return cls(ColumnParallelLinear.from_linear(mlp.gate_proj, group),
                   ColumnParallelLinear.from_linear(mlp.up_proj, group),
                   RowParallelLinear.from_linear(mlp.down_proj, group))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class TPKVCache:
    """Per-rank key/value cache of the rank's KV heads, preallocated
    [batch, local kv heads, max_seq_len, head_dim] per layer; the interface of
    the reference's ``SimpleKVCache`` (``cache/kv_cache.py``: ``update``,
    ``get``, ``set_len``, ``advance``, ``cur_len``)."""

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, max_seq_len: int = 2048,
                 batch_size: int = 1, device=None, dtype=torch.bfloat16):
        self.num_layers, self.num_kv_heads, self.head_dim = num_layers, num_kv_heads, head_dim
        self.max_seq_len, self.batch_size = max_seq_len, batch_size
        self.cur_len = 0
        shape = (batch_size, num_kv_heads, max_seq_len, head_dim)
        self.k_cache: List[torch.Tensor] = [torch.zeros(shape, device=device, dtype=dtype) for _ in range(num_layers)]
        self.v_cache: List[torch.Tensor] = [torch.zeros(shape, device=device, dtype=dtype) for _ in range(num_layers)]

    def update(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor, start_pos: int) -> None:
        s = k.shape[2]
        if start_pos + s > self.max_seq_len:
            raise ValueError(f"KV cache overflow: {start_pos + s} > {self.max_seq_len}")
        self.k_cache[layer_idx][:, :, start_pos:start_pos + s] = k.to(self.k_cache[layer_idx].dtype)
        self.v_cache[layer_idx][:, :, start_pos:start_pos + s] = v.to(self.v_cache[layer_idx].dtype)

    def get(self, layer_idx: int, total_len: Optional[int] = None):
        n = self.cur_len if total_len is None else total_len
        return self.k_cache[layer_idx][:, :, :n], self.v_cache[layer_idx][:, :, :n]

    def set_len(self, length: int) -> None:
        self.cur_len = length

    def advance(self, n: int = 1) -> None:
        self.cur_len += n


def _rope_tables(head_dim: int, partial: float, base: float, max_pos: int, device):
    rd = int(head_dim * partial)
    inv = 1.0 / (base ** (torch.arange(0, rd, 2, device=device, dtype=torch.float32) / rd))
    f = torch.outer(torch.arange(max_pos, device=device, dtype=torch.float32), inv)
    emb = torch.cat([f, f], dim=-1)
    return emb.cos(), emb.sin(), rd


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


class TPAttention(nn.Module):
    """``GLM4Attention`` (``model/glm4.py:113-223``) split by heads over the ranks.

    Rank r runs query heads [r*n_heads/W, (r+1)*n_heads/W) and the KV heads
    they read; only the O projection's partial sums cross ranks (one
    all-reduce)."""

    def __init__(self, q: ColumnParallelLinear, k: ColumnParallelLinear, v: ColumnParallelLinear,
                 o: RowParallelLinear, n_heads: int, n_kv: int, head_dim: int, layer_idx: int,
                 partial_rotary_factor: float, rope_theta: float, max_position_embeddings: int, group=None):
        super().__init__()
        W, _ = _world(group)
        self.q_proj, self.k_proj, self.v_proj, self.o_proj = q, k, v, o
        self.layer_idx = layer_idx
        self.head_dim = head_dim
        self.n_heads_local = n_heads // W
        self.n_kv_local = max(1, n_kv // W)
        self.groups = self.n_heads_local // self.n_kv_local
        self.partial = partial_rotary_factor
        self.theta = rope_theta
        self.max_pos = max_position_embeddings
        self._rope = None

    @classmethod
    def from_module(cls, attn: nn.Module, group=None) -> "TPAttention":
        W, r = _world(group)
        nh, nkv, hd = attn.num_heads, attn.num_kv_heads, attn.head_dim
        if nh % W:
            raise ValueError(f"{nh} query heads do not split over {W} ranks")
        if not (nkv % W == 0 or W % nkv == 0):
            raise ValueError(f"{nkv} KV heads neither split over nor evenly replicate onto {W} ranks")
        q = ColumnParallelLinear.from_linear(attn.q_proj, group)
        if nkv % W == 0:
            k = ColumnParallelLinear.from_linear(attn.k_proj, group)
            v = ColumnParallelLinear.from_linear(attn.v_proj, group)
        else:
            # each rank's query heads read one KV head: rank r keeps head r // (W / nkv)
            h = r // (W // nkv)
            k = cls._head_slice(attn.k_proj, h, hd, group)
            v = cls._head_slice(attn.v_proj, h, hd, group)
        o = RowParallelLinear.from_linear(attn.o_proj, group)
        rot = getattr(attn, "rotary_emb", None)
        cfg = getattr(attn, "config", None)
        partial = getattr(rot, "partial_rotary_factor", getattr(cfg, "partial_rotary_factor", 0.5))
        base = getattr(rot, "base", getattr(cfg, "rope_theta", 1e6))
        max_pos = getattr(rot, "max_position_embeddings", getattr(cfg, "max_position_embeddings", 131072))
        return cls(q, k, v, o, nh, nkv, hd, getattr(attn, "layer_idx", 0), partial, base, max_pos, group)

    @staticmethod
    def _head_slice(lin: nn.Module, h: int, hd: int, group) -> ColumnParallelLinear:
        if _int4_parts(lin) is not None:
            p, s = _int4_parts(lin)
            w = _Int4Weight(p[h * hd:(h + 1) * hd], s[h * hd:(h + 1) * hd])
        else:
            w = lin.weight.detach()[h * hd:(h + 1) * hd].clone()
        b = getattr(lin, "bias", None)
        b = None if b is None else b.detach()[h * hd:(h + 1) * hd].clone()
        return ColumnParallelLinear(w, b, lin.out_features, group)

    def _cos_sin(self, position_ids: torch.Tensor, dtype):
        if self._rope is None or self._rope[0].device != position_ids.device:
            self._rope = _rope_tables(self.head_dim, self.partial, self.theta, self.max_pos, position_ids.device)
        cos, sin, rd = self._rope
        return cos[position_ids].to(dtype).unsqueeze(1), sin[position_ids].to(dtype).unsqueeze(1), rd

    def forward(self, hidden_states: torch.Tensor, position_ids: torch.Tensor,
                attention_mask: Optional[torch.Tensor] = None, kv_cache: Optional[TPKVCache] = None) -> torch.Tensor:
        B, S, _ = hidden_states.shape
        q = self.q_proj(hidden_states).view(B, S, self.n_heads_local, self.head_dim).transpose(1, 2)
        k = self.k_proj(hidden_states).view(B, S, self.n_kv_local, self.head_dim).transpose(1, 2)
        v = self.v_proj(hidden_states).view(B, S, self.n_kv_local, self.head_dim).transpose(1, 2)
        cos, sin, rd = self._cos_sin(position_ids, v.dtype)
        q = torch.cat([q[..., :rd] * cos + _rotate_half(q[..., :rd]) * sin, q[..., rd:]], dim=-1)
        k = torch.cat([k[..., :rd] * cos + _rotate_half(k[..., :rd]) * sin, k[..., rd:]], dim=-1)
        if kv_cache is not None:
            start = int(position_ids[0, 0].item())
            kv_cache.update(self.layer_idx, k, v, start)
            k, v = kv_cache.get(self.layer_idx, start + S)
        if self.groups > 1:
            k = k.repeat_interleave(self.groups, dim=1)
            v = v.repeat_interleave(self.groups, dim=1)
        o = F.scaled_dot_product_attention(q, k.to(q.dtype), v.to(q.dtype), attn_mask=attention_mask,
                                           is_causal=S > 1 and attention_mask is None)
        o = o.transpose(1, 2).reshape(B, S, self.n_heads_local * self.head_dim)
        return self.o_proj(o)


class VocabParallelLMHead(nn.Module):
    """``lm_head`` with the vocabulary split over the ranks (``model/glm4.py:641,717``)."""

    def __init__(self, inner: ColumnParallelLinear):
        super().__init__()
        self.inner = inner

    @classmethod
    def from_linear(cls, lin: nn.Module, group=None, gather_output: bool = True) -> "VocabParallelLMHead":
        return cls(ColumnParallelLinear.from_linear(lin, group, gather_output=gather_output))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.inner(x)


__all__ = ["ColumnParallelLinear", "RowParallelLinear", "TPDenseMLP", "TPAttention", "TPKVCache",
           "VocabParallelLMHead"]
