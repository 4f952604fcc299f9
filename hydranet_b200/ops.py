"""Tensor-level wrappers of the C ABI (what the reference-shaped modules call).

Each function validates shapes the way the reference does (it raises
``AssertionError`` for the shape checks the reference asserts, e.g.
``kernels/int4_gemm.py:148-149``), allocates its output with the input's
dtype and device, and launches on the current CUDA stream.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check, load, ptr, stream_ptr

GROUP_SIZE = 128


def _act_dtype(x: torch.Tensor) -> int:
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError(f"activations must be float16 or bfloat16, got {x.dtype}")
    return _lib.dtype_code(x.dtype)


def quantize_int4(w: torch.Tensor, group_size: int = GROUP_SIZE):
    """GPU packer, bit-identical to ``ExpertWeightPacker.quantize_tensor``
    (``preprocess/pack_weights.py:133-181``).  Returns (packed u8, scales f16)."""
    _lib.require_cuda(w)
    assert w.dim() == 2, "quantize_int4 expects a 2-D [out, in] weight"
    out_f, in_f = w.shape
    assert in_f % group_size == 0, f"in_features {in_f} must be divisible by group_size {group_size}"
    w = w.contiguous()
    packed = torch.empty(out_f, in_f // 2, dtype=torch.uint8, device=w.device)
    scales = torch.empty(out_f, in_f // group_size, dtype=torch.float16, device=w.device)
    with torch.cuda.device(w.device):
        check(load().hn_quantize_int4(ptr(w), _lib.dtype_code(w.dtype), out_f, in_f, group_size, ptr(packed),
                                      ptr(scales), stream_ptr(w.device)))
    return packed, scales


def unpack_int4(packed: torch.Tensor) -> torch.Tensor:
    """Raw nibbles (0..15) as uint8 [out, in]; low nibble = even column."""
    _lib.require_cuda(packed)
    packed = packed.contiguous()
    out = torch.empty(packed.shape[0], packed.shape[1] * 2, dtype=torch.uint8, device=packed.device)
    with torch.cuda.device(packed.device):
        check(load().hn_unpack_int4(ptr(packed), packed.shape[0], packed.shape[1] * 2, ptr(out), stream_ptr(packed.device)))
    return out


def dequant_int4(packed: torch.Tensor, scales: torch.Tensor, group_size: int = GROUP_SIZE) -> torch.Tensor:
    """float16 ``(nibble - 8) * scale`` (``cache/packed_expert_store.py:287-315``)."""
    _lib.require_cuda(packed, scales)
    packed, scales = packed.contiguous(), scales.contiguous()
    rows, cols = packed.shape[0], packed.shape[1] * 2
    out = torch.empty(rows, cols, dtype=torch.float16, device=packed.device)
    with torch.cuda.device(packed.device):
        check(load().hn_dequant_int4(ptr(packed), ptr(scales), rows, cols, group_size, ptr(out), stream_ptr(packed.device)))
    return out


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` with fp32 math (``kernels/int4_gemm.py:175-208``)."""
    assert gate.shape == up.shape
    _lib.require_cuda(gate, up)
    gate, up = gate.contiguous(), up.contiguous()
    out = torch.empty_like(gate)
    with torch.cuda.device(gate.device):
        check(load().hn_silu_mul(ptr(gate), ptr(up), ptr(out), gate.numel(), _act_dtype(gate), stream_ptr(gate.device)))
    return out


def int4_linear(x: torch.Tensor, w_packed: torch.Tensor, w_scales: torch.Tensor,
                group_size: int = GROUP_SIZE) -> torch.Tensor:
    """``x @ W.T`` with INT4 W (``kernels/int4_gemm.py:124-172``)."""
    orig_shape = x.shape
    if x.dim() == 3:
        x = x.reshape(-1, x.shape[-1])
    M, K = x.shape
    N = w_packed.shape[0]
    assert w_packed.shape[1] == K // 2, f"w_packed shape {tuple(w_packed.shape)} vs K={K}"
    assert tuple(w_scales.shape) == (N, K // group_size), \
        f"w_scales shape {tuple(w_scales.shape)} vs ({N}, {K // group_size})"
    _lib.require_cuda(x, w_packed, w_scales)
    if x.stride(-1) != 1:
        x = x.contiguous()
    w_packed, w_scales = w_packed.contiguous(), w_scales.contiguous()
    out = torch.empty((M, N), dtype=x.dtype, device=x.device)
    if M > 0:
        lib = load()
        need = lib.hn_int4_linear_workspace_size(M, N, K)
        ws = _lib.workspaces.get(need, x.device)
        with torch.cuda.device(x.device):
            check(lib.hn_int4_linear(ptr(x), x.stride(0), _act_dtype(x), M, K, ptr(w_packed), ptr(w_scales), N,
                                     group_size, ptr(out), N, ptr(ws), ws.numel(), stream_ptr(x.device)))
    if len(orig_shape) == 3:
        out = out.view(orig_shape[0], orig_shape[1], N)
    return out


def expert_mlp_int4(x, gate_packed, gate_scales, up_packed, up_scales, down_packed, down_scales,
                    group_size: int = GROUP_SIZE) -> torch.Tensor:
    """``down(silu(gate(x)) * up(x))`` in one fused pass (``kernels/int4_gemm.py:211-254``)."""
    orig_shape = x.shape
    if x.dim() == 3:
        x = x.reshape(-1, x.shape[-1])
    T, H = x.shape
    F = gate_packed.shape[0]
    assert tuple(gate_packed.shape) == (F, H // 2) and tuple(up_packed.shape) == (F, H // 2), "gate/up shape"
    assert tuple(down_packed.shape) == (H, F // 2), "down shape"
    assert tuple(gate_scales.shape) == (F, H // group_size) and tuple(up_scales.shape) == (F, H // group_size)
    assert tuple(down_scales.shape) == (H, F // group_size)
    _lib.require_cuda(x, gate_packed, gate_scales, up_packed, up_scales, down_packed, down_scales)
    x = x.contiguous()
    out = torch.empty((T, H), dtype=x.dtype, device=x.device)
    if T > 0:
        lib = load()
        need = lib.hn_expert_mlp_workspace_size(T, H, F)
        ws = _lib.workspaces.get(need, x.device)
        t = [a.contiguous() for a in (gate_packed, gate_scales, up_packed, up_scales, down_packed, down_scales)]
        with torch.cuda.device(x.device):
            check(lib.hn_expert_mlp_int4(ptr(x), _act_dtype(x), T, H, F, *[ptr(a) for a in t], group_size, ptr(out),
                                         ptr(ws), ws.numel(), stream_ptr(x.device)))
    return out.view(orig_shape) if len(orig_shape) == 3 else out


def router_params(kind: int, top_k: int, weight: torch.Tensor, logits_in_act_dtype: bool,
                  affinity_bonus: torch.Tensor | None = None, entropy_threshold: float = 0.5,
                  correction_bias: torch.Tensor | None = None, norm_topk_prob: bool = True,
                  routed_scaling_factor: float = 1.0, n_group: int = 1, topk_group: int = 0) -> _lib.RouterParams:
    return _lib.RouterParams(kind, top_k, weight.data_ptr(), _lib.dtype_code(weight.dtype), int(logits_in_act_dtype),
                             ptr(affinity_bonus), entropy_threshold, ptr(correction_bias), int(norm_topk_prob),
                             routed_scaling_factor, int(n_group), int(topk_group))


def moe_route(x: torch.Tensor, params: _lib.RouterParams, num_experts: int, keep_refs=(), want_logits: bool = True):
    """Router only. Returns (idx int32 [T,k], w float32 [T,k], logits float32 [T,E] or None)."""
    T, H = x.shape
    k = params.top_k
    idx = torch.empty(T, k, dtype=torch.int32, device=x.device)
    w = torch.empty(T, k, dtype=torch.float32, device=x.device)
    logits = torch.empty(T, num_experts, dtype=torch.float32, device=x.device) if want_logits else None
    lib = load()
    need = lib.hn_moe_workspace_size(T, H, 128, num_experts, k)
    ws = _lib.workspaces.get(need, x.device)
    with torch.cuda.device(x.device):
        check(lib.hn_moe_route(ptr(x), _act_dtype(x), T, H, num_experts, ctypes.byref(params), ptr(idx), ptr(w),
                               ptr(logits), ptr(ws), ws.numel(), stream_ptr(x.device)))
    del keep_refs
    return idx, w, logits


def moe_layer(x: torch.Tensor, params: _lib.RouterParams, expert_table: torch.Tensor, expert_maps: torch.Tensor,
              num_experts: int, ffn: int, want_routing: bool = False, keep_refs=()):
    """Router + experts + combine for one MoE layer. ``expert_table`` is a device
    int64 tensor [E, 6] of pointers and ``expert_maps`` the device copy of their
    TMA descriptors (``ExpertTable.device_table`` / ``ExpertTable.device_maps``)."""
    T, H = x.shape
    k = params.top_k
    out = torch.empty_like(x)
    idx = w = logits = None
    if want_routing:
        idx = torch.empty(T, k, dtype=torch.int32, device=x.device)
        w = torch.empty(T, k, dtype=torch.float32, device=x.device)
        logits = torch.empty(T, num_experts, dtype=torch.float32, device=x.device)
    lib = load()
    need = lib.hn_moe_workspace_size(T, H, ffn, num_experts, k)
    ws = _lib.workspaces.get(need, x.device)
    with torch.cuda.device(x.device):
        check(lib.hn_moe_layer_int4(ptr(x), _act_dtype(x), T, H, ffn, num_experts, ctypes.byref(params),
                                    expert_table.data_ptr(), expert_maps.data_ptr(), ptr(out), ptr(idx), ptr(w),
                                    ptr(logits), ptr(ws), ws.numel(),
                                    stream_ptr(x.device)))
    del keep_refs
    return out, idx, w, logits


def moe_layer_phases(x: torch.Tensor, params: _lib.RouterParams, expert_table: torch.Tensor,
                     expert_maps: torch.Tensor, num_experts: int, ffn: int, between=None):
    """``moe_layer`` as its three launches (prep, gate/up, down+combine) on the
    current stream.  ``between(phase)``, if given, is called after each of the
    first two launches (to record events or issue other work); the result is
    identical to ``moe_layer``."""
    T, H = x.shape
    k = params.top_k
    out = torch.empty_like(x)
    lib = load()
    need = lib.hn_moe_workspace_size(T, H, ffn, num_experts, k)
    ws = _lib.workspaces.get(need, x.device)
    with torch.cuda.device(x.device):
        for phase in (1, 2, 3):
            check(lib.hn_moe_layer_int4_phase(phase, ptr(x), _act_dtype(x), T, H, ffn, num_experts,
                                              ctypes.byref(params), expert_table.data_ptr(),
                                              expert_maps.data_ptr(), ptr(out), None, None, None, ptr(ws),
                                              ws.numel(), stream_ptr(x.device)))
            if between is not None and phase < 3:
                between(phase)
    return out


def moe_experts(x: torch.Tensor, topk_idx: torch.Tensor, topk_w: torch.Tensor, expert_table: torch.Tensor,
                expert_maps: torch.Tensor, num_experts: int, ffn: int, expected_assignments: int = 0) -> torch.Tensor:
    """Experts + combine with caller-supplied routing (int32 idx, float32 weights).
    ``expected_assignments``: the caller's estimate of the slots that hold an
    expert when most are -1 (expert-parallel rows); it picks the segment width."""
    T, H = x.shape
    k = topk_idx.shape[1]
    out = torch.empty_like(x)
    if T == 0:
        return out
    topk_idx = topk_idx.to(torch.int32).contiguous()
    topk_w = topk_w.to(torch.float32).contiguous()
    lib = load()
    need = lib.hn_moe_experts_workspace_size_expected(T, H, ffn, num_experts, k, expected_assignments)
    ws = _lib.workspaces.get(need, x.device)
    with torch.cuda.device(x.device):
        check(lib.hn_moe_experts_int4_expected(ptr(x), _act_dtype(x), T, H, ffn, num_experts, k, ptr(topk_idx),
                                               ptr(topk_w), expert_table.data_ptr(), expert_maps.data_ptr(), ptr(out),
                                               int(expected_assignments), ptr(ws), ws.numel(), stream_ptr(x.device)))
    return out
