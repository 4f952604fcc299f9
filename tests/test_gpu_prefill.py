"""GPU parity of the prefill-size paths: token segments of 64 and 128 per MMA
(the engine picks them from the mean assignments per expert, T*K/E) and the
multi-CTA dispatch planner used when T*K exceeds what the prep kernel plans
in shared memory (4096 routing entries).

Same contract as the decode tests: router indices exact (near-ties of the
oracle's own scores reported), outputs rel-L2 <= 1e-2 with a tighter bound,
and bitwise repeatability (the plan's order is fixed: by token, then slot).
"""

import numpy as np
import pytest
import torch

from hydranet_b200 import _lib, synth
from hydranet_b200.kernels import int4_gemm as k_gemm
from hydranet_b200.moe import MoELayerInt4, moe_experts
from hydranet_b200.router import GLM4SigmoidRouter, TopKRouter
from oracle import int4_ref as R
from tests.gpu_util import act, host_moe, oracle_experts, rel_l2, to_np32

pytestmark = pytest.mark.gpu

TOL = 1e-2
TIGHT = 6e-3


def _check_indices(idx, ref_idx, ref_scores, k, ulp_rel):
    mism = np.nonzero(np.any(np.sort(idx, 1) != np.sort(ref_idx, 1), axis=1))[0]
    for t in mism:
        s = np.sort(ref_scores[t])[::-1]
        assert s[k - 1] - s[k] <= 2 * ulp_rel * abs(s[k - 1]) + 1e-30, f"token {t}: index mismatch"
    return len(mism)


@pytest.mark.parametrize("T,E,k,H,F,bias", [
    (1280, 16, 4, 1024, 512, False),  # T*K = 5120 > 4096: plan kernel; 320 per expert: N = 128
    (1280, 16, 4, 1024, 512, True),   # the same with a selection-only correction bias (GLM-4.5)
    (2200, 64, 2, 512, 256, False),   # plan kernel; ~69 per expert: N = 64
    (1280, 32, 2, 512, 384, False),   # prep-kernel plan; 80 per expert: N = 64
])
def test_prefill_sigmoid_layer(lib, T, E, k, H, F, bias):
    shape = synth.MoEShape(H, F, E, k)
    table, packed = host_moe(shape, 500 + E)
    x = torch.randn(T, H, generator=torch.Generator("cuda").manual_seed(T), device="cuda").to(torch.bfloat16)
    r = GLM4SigmoidRouter(hidden_dim=H, num_experts=E, experts_per_token=k).cuda()
    cb = torch.from_numpy(synth.host_correction_bias(9, E)).cuda() if bias else None
    if bias:
        r.set_correction_bias(cb)
    layer = MoELayerInt4(r, table)
    out, ro = layer(x, return_routing=True)
    xi, wi = to_np32(x), to_np32(r.weight)
    cbn = None if cb is None else to_np32(cb)
    idx, w, logits = R.sigmoid_topk_router_ref(xi, wi, k, "bf16", correction_bias=cbn)
    sel = 1 / (1 + np.exp(-logits)) + (0 if cbn is None else cbn[None, :])
    n_tie = _check_indices(ro.expert_indices.cpu().numpy(), idx, sel, k, 2 ** -22)
    assert n_tie == 0
    ref = R.moe_combine_ref(xi, idx, w, oracle_experts(packed))
    err = rel_l2(to_np32(out), ref)
    assert err <= TOL and err <= TIGHT, err
    assert torch.equal(layer(x), out)  # same plan order, same bits


def test_prefill_softmax_layer_plan_kernel(lib):
    """Mixtral-style router at a prefill size (T*K = 6000): plan kernel, N = 128."""
    H, F, E, k, T = 512, 512, 8, 2, 3000
    shape = synth.MoEShape(H, F, E, k)
    table, packed = host_moe(shape, 77)
    rw = (torch.randn(E, H, generator=torch.Generator("cuda").manual_seed(7), device="cuda") * 0.02)
    rw = rw.to(torch.bfloat16)
    r = TopKRouter(hidden_dim=H, num_experts=E, experts_per_token=k).cuda().to(torch.bfloat16)
    with torch.no_grad():
        r.gate.weight.copy_(rw)
    layer = MoELayerInt4(r, table)
    x = torch.randn(T, H, generator=torch.Generator("cuda").manual_seed(8), device="cuda").to(torch.bfloat16)
    out, ro = layer(x, return_routing=True)
    xi, wi = to_np32(x), to_np32(rw)
    idx, w, logits = R.softmax_topk_router_ref(xi, wi, k, "bf16")
    n_tie = _check_indices(ro.expert_indices.cpu().numpy(), idx, logits, k, 2 ** -8)
    use_idx = ro.expert_indices.cpu().numpy() if n_tie else idx
    use_w = to_np32(ro.expert_weights) if n_tie else w
    ref = R.moe_combine_ref(xi, use_idx, use_w, oracle_experts(packed))
    err = rel_l2(to_np32(out), ref)
    assert err <= TOL and err <= TIGHT, err


@pytest.mark.parametrize("k", [3, 8])
def test_given_routing_plan_kernel_with_duplicates(lib, k):
    """Caller-supplied routing above the prep kernel's planning size, with
    duplicate picks (each counts, in slot order)."""
    H, F, E, T = 256, 256, 12, 1500
    shape = synth.MoEShape(H, F, E, k)
    table, packed = host_moe(shape, 90 + k)
    rng = np.random.default_rng(k)
    idx = rng.integers(0, E, size=(T, k)).astype(np.int32)
    w = rng.random((T, k)).astype(np.float32)
    x = act(rng.standard_normal((T, H), dtype=np.float32), "bf16")
    out = moe_experts(x, torch.from_numpy(idx).cuda(), torch.from_numpy(w).cuda(), table)
    ref = R.moe_combine_ref(to_np32(x), idx.astype(np.int64), w, oracle_experts(packed))
    assert rel_l2(to_np32(out), ref) <= TIGHT


@pytest.mark.parametrize("M,N,K", [(70, 512, 1024), (300, 384, 512), (1000, 256, 256)])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_int4_linear_wide_segments(lib, M, N, K, dtype):
    """int4_linear with more than 64 rows per call uses 64- or 128-token segments."""
    rng = np.random.default_rng(M)
    p, s = R.quantize_tensor(rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    xt = act(rng.standard_normal((M, K), dtype=np.float32), dtype)
    out = k_gemm.int4_linear(xt, torch.from_numpy(p).cuda(), torch.from_numpy(s).cuda())
    ref = R.int4_linear_ref(to_np32(xt), p, s)
    err = rel_l2(to_np32(out), ref)
    assert err <= TOL and err <= {"bf16": 5e-3, "f16": 1e-3}[dtype], err


@pytest.mark.parametrize("wdtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("T,E,H", [(512, 128, 1024), (300, 40, 512)])
def test_large_batch_router_logits_precision(lib, wdtype, T, E, H):
    """Router logits of a batch that takes the router GEMM (T >= 256): within
    a few times the error of a float32 matrix product of the same operands,
    measured against float64 (the split weight parts must add up exactly)."""
    from hydranet_b200 import ops
    g = torch.Generator("cuda").manual_seed(T + E)
    x = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
    wt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[wdtype]
    rw = (torch.randn(E, H, generator=g, device="cuda") * 0.02).to(wt)
    p = ops.router_params(_lib.HN_ROUTER_SIGMOID_TOPK, 4, rw, logits_in_act_dtype=False)
    _, _, logits = ops.moe_route(x, p, E)
    xi, wi = to_np32(x).astype(np.float64), to_np32(rw).astype(np.float64)
    ref = xi @ wi.T
    err = np.abs(logits.cpu().numpy().astype(np.float64) - ref).max()
    err32 = np.abs((to_np32(x) @ to_np32(rw).T).astype(np.float64) - ref).max()
    assert err <= 4 * err32 + 1e-6, (err, err32)
