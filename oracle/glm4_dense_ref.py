"""CPU restatement of GLM-4.5's dense layer parts (test infrastructure only).

The checker for ``hydranet_b200.tp``: numpy float64 versions of the
reference's ``GLM4Attention.forward`` (``model/glm4.py:113-223``: Q/K/V with
bias, partial rotary embedding on the first ``head_dim * partial_rotary_factor``
dims of each head (``model/glm4.py:40-110``), grouped-query attention, causal
softmax for a multi-token step, O without bias), ``GLM4DenseMLP.forward``
(``model/glm4.py:226-240``) and the ``lm_head`` projection
(``model/glm4.py:641,717``).  Pinned by ``tests/golden/glm4_dense.npz``,
recorded by running the reference's own modules (``make_golden.py``).
"""

from __future__ import annotations

import numpy as np


def silu(x):
    return x / (1.0 + np.exp(-x))


def dense_mlp_ref(x, gate_w, up_w, down_w):
    """``down(silu(gate(x)) * up(x))`` (``model/glm4.py:238-240``)."""
    x = np.asarray(x, np.float64)
    return (silu(x @ gate_w.T) * (x @ up_w.T)) @ down_w.T


def rope_cos_sin(positions, head_dim, partial_rotary_factor=0.5, base=1e6):
    """cos/sin tables of the partial rotary embedding (``model/glm4.py:40-83``):
    frequencies over the rotary dims, duplicated to the rotary width."""
    rd = int(head_dim * partial_rotary_factor)
    inv = 1.0 / (base ** (np.arange(0, rd, 2, dtype=np.float64) / rd))
    f = np.outer(np.asarray(positions, np.float64), inv)
    emb = np.concatenate([f, f], axis=-1)
    return np.cos(emb), np.sin(emb), rd


def _rotate_half(x):
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def apply_partial_rope(x, cos, sin, rd):
    """x [..., S, D]: the first rd dims rotated (``model/glm4.py:92-110``)."""
    xr, xp = x[..., :rd], x[..., rd:]
    return np.concatenate([xr * cos + _rotate_half(xr) * sin, xp], axis=-1)


def attention_ref(x, wq, bq, wk, bk, wv, bv, wo, n_heads, n_kv, head_dim, positions, past_k=None, past_v=None,
                  partial_rotary_factor=0.5, base=1e6):
    """x [S, H] of one sequence at ``positions``; optional cached keys/values
    [n_kv, P, D] of the earlier positions.  Returns (out [S, H], k_all, v_all)."""
    x = np.asarray(x, np.float64)
    S = x.shape[0]
    q = (x @ wq.T + (0 if bq is None else bq)).reshape(S, n_heads, head_dim).transpose(1, 0, 2)
    k = (x @ wk.T + (0 if bk is None else bk)).reshape(S, n_kv, head_dim).transpose(1, 0, 2)
    v = (x @ wv.T + (0 if bv is None else bv)).reshape(S, n_kv, head_dim).transpose(1, 0, 2)
    cos, sin, rd = rope_cos_sin(positions, head_dim, partial_rotary_factor, base)
    q = apply_partial_rope(q, cos, sin, rd)
    k = apply_partial_rope(k, cos, sin, rd)
    if past_k is not None:
        k = np.concatenate([past_k, k], axis=1)
        v = np.concatenate([past_v, v], axis=1)
    L = k.shape[1]
    rep = n_heads // n_kv
    kk = np.repeat(k, rep, axis=0)
    vv = np.repeat(v, rep, axis=0)
    s = q @ kk.transpose(0, 2, 1) / np.sqrt(head_dim)
    if S > 1:
        # SDPA's is_causal (``model/glm4.py:195-200``): query i sees keys 0..i
        # (the mask is aligned to the top left even when a cache makes L > S)
        mask = np.triu(np.ones((S, L), dtype=bool), k=1)
        s = np.where(mask[None], -np.inf, s)
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    o = (p @ vv).transpose(1, 0, 2).reshape(S, n_heads * head_dim)
    return o @ wo.T, k, v


def lm_head_ref(x, w):
    return np.asarray(x, np.float64) @ w.T
