"""numpy restatement of HydraNet's INT4 MoE path (test oracle, CPU only).

Reference files are cited by their path inside the HydraNet project.

Conventions shared with the reference
-------------------------------------
* A weight matrix ``W[out, in]`` is quantised per (row, group of ``group_size``
  consecutive ``in`` elements): ``scale = absmax / 7`` (clamped to 1e-10),
  ``q = round_half_even(W / scale).clip(-8, 7) + 8`` stored as a nibble,
  two nibbles per byte with the EVEN ``in`` index in the LOW nibble
  (``preprocess/pack_weights.py:133-181``).  Scales are stored as float16.
* Dequantisation is ``(nibble - 8) * scale`` computed in float16
  (``preprocess/pack_weights.py:230-268``).
* The expert MLP is ``down(silu(gate(x)) * up(x))``
  (``kernels/int4_gemm.py:211-254``); the oracle evaluates it the way the
  reference's dequant mode does (``model/mixtral.py:355-362``): dequantise to
  float16, upcast to float32, float32 matmuls.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

# ----------------------------------------------------------------------------
# Packing (offline format)
# ----------------------------------------------------------------------------


def quantize_tensor(w: np.ndarray, group_size: int = 128):
    """Symmetric INT4 group quantisation.

    Follows ``ExpertWeightPacker.quantize_tensor``
    (``preprocess/pack_weights.py:133-181``).  Arithmetic happens in the input
    dtype (float32 or float16), exactly as the reference's torch ops do: the
    absmax, the ``/ 7.0``, the ``clamp(min=1e-10)`` and the ``w / scale``
    division are all evaluated in ``w.dtype``.

    Returns ``(packed uint8 [out, in/2], scales float16 [out, in/group_size])``.
    """
    if w.ndim != 2:
        raise ValueError("quantize_tensor expects a 2-D [out, in] matrix")
    out_f, in_f = w.shape
    if in_f % group_size != 0:
        raise ValueError(f"in_features {in_f} must be divisible by group_size {group_size}")
    dt = w.dtype
    if dt not in (np.float32, np.float16):
        raise TypeError(f"unsupported weight dtype {dt}")
    g = w.reshape(out_f, in_f // group_size, group_size)
    absmax = np.abs(g).max(axis=-1, keepdims=True)            # :156
    scales = (absmax / dt.type(7.0)).astype(dt)               # :157
    # :158  clamp(min=1e-10) in the tensor dtype (1e-10 rounds to 0 in fp16)
    scales = np.maximum(scales, dt.type(1e-10)).astype(dt)
    with np.errstate(divide="ignore", invalid="ignore"):
        qf = np.rint((g / scales).astype(dt))                  # :161 round half-even
    qf = np.clip(qf, -8, 7)
    # :162 (+8).to(uint8); NaN (only for all-zero fp16 groups) casts like torch
    q = np.where(np.isnan(qf), 0, qf + 8).astype(np.uint8).reshape(out_f, in_f)
    even = q[:, 0::2]
    odd = q[:, 1::2]
    packed = ((odd << 4) | even).astype(np.uint8)              # :177-179
    return np.ascontiguousarray(packed), np.ascontiguousarray(
        scales.reshape(out_f, in_f // group_size).astype(np.float16))  # :181


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    """Raw nibbles 0..15 as uint8 [out, in]: low nibble = even column.

    Mirrors the unpack in ``preprocess/pack_weights.py:248-259``.
    """
    out_f, half = packed.shape
    q = np.empty((out_f, half * 2), dtype=np.uint8)
    q[:, 0::2] = packed & 0x0F
    q[:, 1::2] = (packed >> 4) & 0x0F
    return q


def dequantize_tensor(packed: np.ndarray, scales: np.ndarray, group_size: int = 128) -> np.ndarray:
    """float16 dequantisation ``(nibble - 8) * scale``.

    Follows ``ExpertWeightPacker.dequantize_tensor``
    (``preprocess/pack_weights.py:230-268``) and
    ``GpuExpertSlot._dequant_tensor`` (``cache/packed_expert_store.py:287-315``).
    """
    q = unpack_int4(packed).astype(np.float32) - np.float32(8)
    out_f, in_f = q.shape
    qg = q.reshape(out_f, in_f // group_size, group_size)
    # (n - 8) * scale is exact in float32 (a 4-bit integer times an fp16), so
    # rounding the float32 product to fp16 equals the reference's fp16 multiply
    return (qg * scales.astype(np.float32)[:, :, None]).astype(np.float16).reshape(out_f, in_f)


def int4linear_quantize_ref(w: np.ndarray, group_size: int = 128):
    """Quantiser of the non-expert ``Int4Linear`` (``kernels/int4_linear.py:69-103``).

    Differs from the expert packer: the group absmax is clamped to 1e-8 first
    (``:90``), the stored scale is ``absmax / 7`` cast to float16 (``:92``), and
    the integer is ``round_half_even(w / absmax * 7)`` (``:95``), two roundings
    in ``w.dtype``.  Same nibble order (even column in the low nibble, ``:103``).
    float32 and float16 inputs; an all-zero float16 group is left undefined,
    as in the reference (0/0 cast to int8).
    """
    out_f, in_f = w.shape
    if in_f % group_size != 0:
        raise ValueError(f"in_features {in_f} must be divisible by group_size {group_size}")
    dt = w.dtype
    if dt not in (np.float32, np.float16):
        raise TypeError(f"unsupported weight dtype {dt}")
    g = w.reshape(out_f, in_f // group_size, group_size)
    absmax = np.maximum(np.abs(g).max(axis=-1, keepdims=True), dt.type(1e-8)).astype(dt)
    scales = (absmax / dt.type(7.0)).astype(dt).astype(np.float16)[:, :, 0]
    ratio = (g / absmax).astype(dt)
    q = np.clip(np.rint((ratio * dt.type(7.0)).astype(dt)), -8, 7).astype(np.int8)
    u = (q.astype(np.int16) + 8).astype(np.uint8).reshape(out_f, in_f)
    packed = ((u[:, 1::2] << 4) | u[:, 0::2]).astype(np.uint8)
    return np.ascontiguousarray(packed), np.ascontiguousarray(scales)


@dataclass
class BlobLayout:
    """Byte offsets of the six tensors inside one expert blob.

    Same layout as ``BlobLayout.from_dims`` (``cache/packed_expert_store.py:77-108``):
    gate_packed, gate_scales, up_packed, up_scales, down_packed, down_scales.
    """
    gate_packed_offset: int
    gate_packed_size: int
    gate_scales_offset: int
    gate_scales_size: int
    up_packed_offset: int
    up_packed_size: int
    up_scales_offset: int
    up_scales_size: int
    down_packed_offset: int
    down_packed_size: int
    down_scales_offset: int
    down_scales_size: int

    @classmethod
    def from_dims(cls, hidden_dim: int, intermediate_dim: int, group_size: int) -> "BlobLayout":
        gp = intermediate_dim * (hidden_dim // 2)
        gs = intermediate_dim * (hidden_dim // group_size) * 2
        dp = hidden_dim * (intermediate_dim // 2)
        ds = hidden_dim * (intermediate_dim // group_size) * 2
        o = 0
        vals = []
        for size in (gp, gs, gp, gs, dp, ds):
            vals += [o, size]
            o += size
        return cls(*vals)

    @property
    def total_size(self) -> int:
        return self.down_scales_offset + self.down_scales_size


def expert_blob(gp, gs, up, us, dp, ds) -> bytes:
    """Concatenate one expert's six tensors in blob order (``preprocess/pack_glm4.py:102-119``)."""
    return b"".join(np.ascontiguousarray(a).tobytes() for a in (gp, gs, up, us, dp, ds))


# ----------------------------------------------------------------------------
# Expert MLP (dequant-then-matmul, float32 accumulate)
# ----------------------------------------------------------------------------


def silu(v: np.ndarray) -> np.ndarray:
    v = v.astype(np.float32)
    return v / (np.float32(1.0) + np.exp(-v))


def int4_linear_ref(x: np.ndarray, packed: np.ndarray, scales: np.ndarray, group_size: int = 128) -> np.ndarray:
    """``x @ deq(W).T`` in float32 (``kernels/int4_gemm.py:124-172`` semantics)."""
    w = dequantize_tensor(packed, scales, group_size).astype(np.float32)
    return x.astype(np.float32) @ w.T


def silu_mul_ref(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """``silu(gate) * up`` in float32 (``kernels/int4_gemm.py:175-208``)."""
    return silu(gate) * up.astype(np.float32)


def expert_mlp_ref(x, gp, gs, up, us, dp, ds, group_size: int = 128) -> np.ndarray:
    """``down(silu(gate(x)) * up(x))`` in float32.

    Same math as ``expert_mlp_int4_fused`` (``kernels/int4_gemm.py:211-254``),
    evaluated like the reference dequant mode (``model/mixtral.py:355-362``).
    """
    g = int4_linear_ref(x, gp, gs, group_size)
    u = int4_linear_ref(x, up, us, group_size)
    h = silu_mul_ref(g, u)
    return int4_linear_ref(h, dp, ds, group_size)


@dataclass
class DequantExpert:
    """float32 dequantised expert weights (what the reference registers in dequant mode)."""
    gate: np.ndarray
    up: np.ndarray
    down: np.ndarray

    @classmethod
    def from_packed(cls, gp, gs, up, us, dp, ds, group_size: int = 128) -> "DequantExpert":
        return cls(dequantize_tensor(gp, gs, group_size).astype(np.float32),
                   dequantize_tensor(up, us, group_size).astype(np.float32),
                   dequantize_tensor(dp, ds, group_size).astype(np.float32))

    def __call__(self, x: np.ndarray) -> np.ndarray:
        x = x.astype(np.float32)
        return (silu(x @ self.gate.T) * (x @ self.up.T)) @ self.down.T


# ----------------------------------------------------------------------------
# Routers
# ----------------------------------------------------------------------------


def round_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 (nearest-even) and return it as float32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    r = ((u + rounding) >> 16) << 16
    nan = np.isnan(a)
    out = r.astype(np.uint32).view(np.float32).copy()
    out[nan] = np.nan
    return out


def cast_act(a: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to the activation dtype ("f32", "f16", "bf16"); returns float32."""
    if dtype == "f32":
        return a.astype(np.float32)
    if dtype == "f16":
        return a.astype(np.float32).astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        return round_to_bf16(a)
    raise ValueError(dtype)


def topk_desc(scores: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest scores per row, ties broken toward the lower index."""
    order = np.argsort(-scores, axis=-1, kind="stable")
    return order[..., :k]


def softmax_topk_router_ref(h: np.ndarray, gate_w: np.ndarray, top_k: int, act_dtype: str = "f32",
                            affinity_bonus: np.ndarray | None = None,
                            entropy_threshold: float = 0.5):
    """Mixtral softmax top-k router.

    Follows ``TopKRouter.forward`` (``model/router.py:73-130``):
    logits = gate(h) in the model dtype then ``.float()`` (:102); optional
    cache-affinity bonus (:104-106, ``_apply_affinity_bonus`` :132-175) given
    here as a per-expert bonus vector (0.1 for cached experts) applied only to
    tokens whose normalised routing entropy exceeds ``entropy_threshold``;
    top-k on logits (:109), softmax over the selected logits (:114),
    renormalise (:117), cast to the activation dtype (:120).

    Returns (indices int64 [T, k], weights float32 [T, k] already rounded to
    ``act_dtype``, logits float32 [T, E]).
    """
    h2 = h.reshape(-1, h.shape[-1]).astype(np.float32)
    logits = cast_act(h2 @ gate_w.astype(np.float32).T, act_dtype)
    if affinity_bonus is not None:
        p = np.exp(logits - logits.max(-1, keepdims=True))
        p = p / p.sum(-1, keepdims=True)
        ent = -(p * np.log(p + np.float32(1e-10))).sum(-1)
        gate_on = (ent / np.float32(math.log(logits.shape[-1])) > entropy_threshold).astype(np.float32)
        logits = logits + gate_on[:, None] * affinity_bonus.astype(np.float32)[None, :]
    idx = topk_desc(logits, top_k)
    sel = np.take_along_axis(logits, idx, -1)
    e = np.exp(sel - sel.max(-1, keepdims=True))
    w = e / e.sum(-1, keepdims=True)
    w = w / w.sum(-1, keepdims=True)
    return idx.astype(np.int64), cast_act(w, act_dtype), logits


def sigmoid_topk_router_ref(h: np.ndarray, router_w: np.ndarray, top_k: int, act_dtype: str = "f32",
                            correction_bias: np.ndarray | None = None, norm_topk_prob: bool = True,
                            routed_scaling_factor: float = 1.0, n_group: int = 1, topk_group: int = 0):
    """GLM-4.5 sigmoid top-k router.

    Follows ``GLM4SigmoidRouter.forward`` (``model/glm4.py:261-309``): float32
    logits (:279), sigmoid (:282), top-k (:300), normalise with ``+1e-9``
    (:303-304), scale (:307), cast (:309).  With ``n_group > 1`` and
    ``topk_group > 0`` the group mask (:285-297): groups of E / n_group
    experts scored by their best score, the ``topk_group`` best kept, the
    other experts' scores multiplied by 0 before the top-k.

    ``correction_bias`` (an extension: the reference loads
    ``e_score_correction_bias`` but never applies it,
    ``model/glm4_loader.py:164-167``) is added to the sigmoid scores for the
    SELECTION only; the weights come from the unbiased scores.  With
    ``correction_bias=None`` this is exactly the reference.
    """
    h2 = h.reshape(-1, h.shape[-1]).astype(np.float32)
    logits = h2 @ router_w.astype(np.float32).T
    scores = (np.float32(1.0) / (np.float32(1.0) + np.exp(-logits))).astype(np.float32)
    sel_scores = scores if correction_bias is None else scores + correction_bias.astype(np.float32)[None, :]
    if n_group > 1 and topk_group > 0:
        gs = sel_scores.shape[-1] // n_group
        gmax = sel_scores.reshape(-1, n_group, gs).max(-1)
        keep = np.zeros_like(gmax, dtype=bool)
        np.put_along_axis(keep, topk_desc(gmax, topk_group), True, -1)
        mask = np.repeat(keep, gs, axis=-1)
        sel_scores = np.where(mask, sel_scores, np.float32(0.0))
        scores = np.where(mask, scores, np.float32(0.0))
    idx = topk_desc(sel_scores, top_k)
    w = np.take_along_axis(scores, idx, -1)
    if norm_topk_prob:
        w = w / (w.sum(-1, keepdims=True) + np.float32(1e-9))
    w = w * np.float32(routed_scaling_factor)
    return idx.astype(np.int64), cast_act(w, act_dtype), logits


# ----------------------------------------------------------------------------
# MoE layer (dispatch + expert MLP + weighted combine)
# ----------------------------------------------------------------------------


def moe_combine_ref(x: np.ndarray, idx: np.ndarray, w: np.ndarray, experts) -> np.ndarray:
    """``out[t] = sum_k w[t,k] * MLP_{idx[t,k]}(x[t])`` in float32.

    Follows the per-expert dispatch loop of ``MixtralMoELayer.forward``
    (``model/mixtral.py:327-368``) and ``GLM4MoELayer.forward``
    (``model/glm4.py:421-466``): gather the tokens of one expert, run its MLP,
    scale by the routing weight and ``index_add_`` into the output.  The
    oracle accumulates in float32 (the reference accumulates in the
    activation dtype).  ``experts`` maps expert id -> callable([m, H]) -> [m, H].
    """
    x2 = x.reshape(-1, x.shape[-1]).astype(np.float32)
    out = np.zeros_like(x2)
    for e in np.unique(idx):
        tok, kpos = np.nonzero(idx == e)
        y = experts[int(e)](x2[tok])
        np.add.at(out, tok, y * w[tok, kpos][:, None].astype(np.float32))
    return out


def touched_experts(idx: np.ndarray) -> int:
    return int(np.unique(idx).size)
