"""GPU parity of the grouped MoE layer (router + dispatch + experts + combine).

Routing indices must match the oracle exactly; a mismatch is tolerated only
where the oracle's own top-k boundary is a near-tie (gap within one ulp of
the logit dtype), which the test reports.  Outputs: rel-L2 <= 1e-2 (north
star) and a tighter precision bound.
"""

import numpy as np
import pytest
import torch

from hydranet_b200 import _lib, ops, synth
from hydranet_b200.moe import MoELayerInt4, moe_experts
from hydranet_b200.router import GLM4SigmoidRouter, TopKRouter
from oracle import int4_ref as R
from tests.gpu_util import act, device_moe, host_moe, oracle_experts, rel_l2, to_np32

pytestmark = pytest.mark.gpu

TOL = 1e-2
TIGHT = 6e-3


def check_indices(idx, ref_idx, ref_scores, k, ulp_rel):
    mism = np.nonzero(np.any(np.sort(idx, 1) != np.sort(ref_idx, 1), axis=1))[0]
    for t in mism:
        s = np.sort(ref_scores[t])[::-1]
        gap = s[k - 1] - s[k]
        assert gap <= 2 * ulp_rel * abs(s[k - 1]) + 1e-30, f"token {t}: index mismatch with logit gap {gap}"
    return len(mism)


def mixtral_layer(table, rw, k, bonus=None):
    r = TopKRouter(hidden_dim=table.hidden_dim, num_experts=len(table), experts_per_token=k).cuda().to(torch.bfloat16)
    with torch.no_grad():
        r.gate.weight.copy_(rw)
    if bonus is not None:
        r.enable_affinity_bonus = True
        r.set_cache_checker(lambda e: bool(bonus[e] > 0))
    return MoELayerInt4(r, table)


def test_c1_golden_layer(lib, golden_dir):
    """Config 1 (H=512, F=1024, E=8, top-2) on the fixture's inputs."""
    g = dict(np.load(golden_dir / "c1_mixtral_layer.npz"))
    shape = synth.MoEShape(512, 1024, 8, 2)
    table, packed = host_moe(shape, 0)
    x = act(g["x"], "bf16")
    rw = torch.from_numpy(g["router_w"]).cuda().to(torch.bfloat16)
    layer = mixtral_layer(table, rw, 2)
    out, ro = layer(x.view(1, 4, 512), return_routing=True)
    xi, wi = to_np32(x), to_np32(rw)
    idx, w, logits = R.softmax_topk_router_ref(xi, wi, 2, "bf16")
    check_indices(ro.expert_indices.view(4, 2).cpu().numpy(), idx, logits, 2, 2 ** -8)
    ref = R.moe_combine_ref(xi, idx, w, oracle_experts(packed))
    err = rel_l2(to_np32(out.view(4, 512)), ref)
    assert err <= TOL and err <= TIGHT, err


@pytest.mark.parametrize("T", [1, 8, 32, 64])
def test_mixtral_shape_layer(lib, T):
    """Config 2: Mixtral-8x7B MoE layer decode (H=4096, F=14336, E=8, top-2), bf16."""
    shape = synth.MoEShape(4096, 14336, 8, 2)
    table, packed = _mixtral_full()
    x = torch.randn(T, 4096, generator=torch.Generator("cuda").manual_seed(T), device="cuda").to(torch.bfloat16)
    rw = (torch.randn(8, 4096, generator=torch.Generator("cuda").manual_seed(99), device="cuda") * 0.02)
    rw = rw.to(torch.bfloat16)
    layer = mixtral_layer(table, rw, 2)
    out, ro = layer(x, return_routing=True)
    xi, wi = to_np32(x), to_np32(rw)
    idx, w, logits = R.softmax_topk_router_ref(xi, wi, 2, "bf16")
    n_tie = check_indices(ro.expert_indices.cpu().numpy(), idx, logits, 2, 2 ** -8)
    use_idx = ro.expert_indices.cpu().numpy() if n_tie else idx
    use_w = to_np32(ro.expert_weights) if n_tie else w
    np.testing.assert_allclose(to_np32(ro.expert_weights), use_w, rtol=2 ** -7, atol=1e-6)
    ref = R.moe_combine_ref(xi, use_idx, use_w, _mixtral_oracle())
    err = rel_l2(to_np32(out), ref)
    assert err <= TOL and err <= TIGHT, err


_FULL = {}


def _mixtral_full():
    if "m" not in _FULL:
        _FULL["m"] = device_moe(synth.MoEShape(4096, 14336, 8, 2), 1234)
    return _FULL["m"]


def _mixtral_oracle():
    if "mo" not in _FULL:
        _FULL["mo"] = oracle_experts(_mixtral_full()[1])
    return _FULL["mo"]


@pytest.mark.parametrize("bias", [False, True])
def test_glm_shape_layer(lib, bias):
    """Config 4 layer: GLM-4.5-Air shape (H=4096, F=1408, E=128, sigmoid top-8), T=32 bf16."""
    shape = synth.MoEShape(4096, 1408, 128, 8)
    if "g" not in _FULL:
        _FULL["g"] = device_moe(shape, 4321)
    table, packed = _FULL["g"]
    T = 32
    x = torch.randn(T, 4096, generator=torch.Generator("cuda").manual_seed(5), device="cuda").to(torch.bfloat16)
    r = GLM4SigmoidRouter(hidden_dim=4096, num_experts=128, experts_per_token=8).cuda()
    cb = None
    if bias:
        cb = torch.from_numpy(synth.host_correction_bias(3, 128)).cuda()
        r.set_correction_bias(cb)
    layer = MoELayerInt4(r, table)
    out, ro = layer(x, return_routing=True)
    xi, wi = to_np32(x), to_np32(r.weight)
    idx, w, logits = R.sigmoid_topk_router_ref(xi, wi, 8, "bf16", correction_bias=None if cb is None else to_np32(cb))
    sel = 1 / (1 + np.exp(-logits)) + (0 if cb is None else to_np32(cb)[None, :])
    n_tie = check_indices(ro.expert_indices.cpu().numpy(), idx, sel, 8, 2 ** -22)
    assert n_tie == 0
    ref = R.moe_combine_ref(xi, idx, w, oracle_experts(packed, idx.ravel()))
    err = rel_l2(to_np32(out), ref)
    assert err <= TOL and err <= TIGHT, err
    # module interface of the router alone matches the layer's routing
    i2, w2 = r(x.view(1, T, 4096))
    assert torch.equal(i2, ro.expert_indices) and torch.equal(w2, ro.expert_weights)


@pytest.mark.parametrize("k", [1, 2, 3])
def test_given_routing_with_duplicates(lib, k):
    """Caller-supplied routing (expert-parallel shards use this); duplicate picks count twice,
    as the reference loop does (``model/mixtral.py:329-368``)."""
    shape = synth.MoEShape(512, 256, 6, k)
    table, packed = host_moe(shape, 11)
    T = 37
    rng = np.random.default_rng(0)
    idx = rng.integers(0, 6, size=(T, k)).astype(np.int32)
    w = rng.random((T, k)).astype(np.float32)
    x = act(rng.standard_normal((T, 512), dtype=np.float32), "bf16")
    out = moe_experts(x, torch.from_numpy(idx).cuda(), torch.from_numpy(w).cuda(), table)
    ref = R.moe_combine_ref(to_np32(x), idx.astype(np.int64), w, oracle_experts(packed))
    assert rel_l2(to_np32(out), ref) <= TIGHT


def test_affinity_bonus_routing(lib):
    """Cache-affinity bonus (``model/router.py:132-175``) on a near-uniform router."""
    shape = synth.MoEShape(512, 256, 8, 2)
    table, packed = host_moe(shape, 21)
    bonus = np.zeros(8, np.float32)
    bonus[[0, 3, 5]] = 0.1
    x = act(np.random.default_rng(1).standard_normal((16, 512), dtype=np.float32), "bf16")
    rw = torch.from_numpy(synth.host_normal(2, (8, 512), 0.002)).cuda().to(torch.bfloat16)
    layer = mixtral_layer(table, rw, 2, bonus=bonus)
    out, ro = layer(x, return_routing=True)
    idx, w, logits = R.softmax_topk_router_ref(to_np32(x), to_np32(rw), 2, "bf16", affinity_bonus=bonus)
    check_indices(ro.expert_indices.cpu().numpy(), idx, logits, 2, 2 ** -8)
    assert np.isin(ro.expert_indices.cpu().numpy(), [0, 3, 5]).mean() > 0.5
    ref = R.moe_combine_ref(to_np32(x), idx, w, oracle_experts(packed))
    assert rel_l2(to_np32(out), ref) <= TIGHT


def test_layer_repeatable_and_error_word_clean(lib):
    shape = synth.MoEShape(1024, 512, 16, 4)
    table, _ = host_moe(shape, 31)
    r = GLM4SigmoidRouter(hidden_dim=1024, num_experts=16, experts_per_token=4).cuda()
    layer = MoELayerInt4(r, table)
    x = torch.randn(50, 1024, device="cuda", dtype=torch.bfloat16)
    outs = [layer(x) for _ in range(3)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    for ws in _lib.workspaces.all():
        assert _lib.workspace_error(ws) == 0


def test_cuda_graph_capture(lib):
    """A decode layer has no host sync, so it can be captured and replayed."""
    shape = synth.MoEShape(1024, 512, 8, 2)
    table, _ = host_moe(shape, 41)
    rw = torch.randn(8, 1024, device="cuda", dtype=torch.bfloat16) * 0.02
    layer = mixtral_layer(table, rw, 2)
    x = torch.randn(8, 1024, device="cuda", dtype=torch.bfloat16)
    ref = layer(x)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        layer(x)  # allocate this stream's workspace outside capture
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            y = layer(x)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, ref)


def test_router_usage_counts_capturable(lib):
    """``usage_counts`` (``model/router.py:177-182``) counts every pick, and a
    router call has no host read, so it can be captured in a graph."""
    r = TopKRouter(hidden_dim=512, num_experts=8, experts_per_token=2).cuda().to(torch.bfloat16).eval()
    x = torch.randn(1, 40, 512, device="cuda", dtype=torch.bfloat16)
    ro = r(x)
    want = torch.bincount(ro.expert_indices.reshape(-1), minlength=8)
    assert torch.equal(r.usage_counts, want)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        r(x)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            r(x)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(r.usage_counts, 3 * want)  # first call, side-stream call, replay (capture runs nothing)


def test_phase_split_equals_one_call(lib):
    """hn_moe_layer_int4_phase 1, 2, 3 in order == one hn_moe_layer_int4 call, bit for bit."""
    shape = synth.MoEShape(1024, 768, 8, 2)
    table, _ = host_moe(shape, 61)
    rw = torch.randn(8, 1024, generator=torch.Generator("cuda").manual_seed(3), device="cuda") * 0.02
    layer = mixtral_layer(table, rw.to(torch.bfloat16), 2)
    x = torch.randn(24, 1024, generator=torch.Generator("cuda").manual_seed(4), device="cuda").to(torch.bfloat16)
    seen = []
    a = layer(x)
    b = layer.forward_phases(x, between=seen.append)
    assert seen == [1, 2]
    assert torch.equal(a, b)
    with pytest.raises(_lib.HydraNetError):
        _lib.check(_lib.load().hn_moe_layer_int4_phase(4, None, 2, 1, 1024, 768, 8, None, None, None, None, None,
                                                       None, None, None, 0, None))


def test_driver_smoke_entry(lib):
    """The driver's smoke() (one small layer on cuda:0 against the oracle) runs clean."""
    import __graft_entry__
    __graft_entry__.smoke()


@pytest.mark.parametrize("T,k,E,sparse", [(37, 2, 6, 0.0), (100, 1, 4, 0.0), (5000, 1, 4, 0.0), (12, 8, 16, 0.8),
                                          (256, 8, 16, 0.8)])
def test_given_routing_unused_slots(lib, T, k, E, sparse):
    """Index -1 marks an unused slot (the expert-parallel exchange rewrites
    the picks owned by other ranks as -1): tokens whose slots are all -1 are
    skipped, -1 next to real picks takes no work and adds nothing; the other
    tokens match the oracle.  Sizes cover both engines, the gathered and the
    assignment-ordered token paths and the multi-CTA planner (T*k > 4096);
    ``sparse`` blanks that share of the slots, as at eight ranks with top-8."""
    shape = synth.MoEShape(256, 256, E, k)
    table, packed = host_moe(shape, 70 + T)
    rng = np.random.default_rng(T)
    idx = rng.integers(0, E, size=(T, k)).astype(np.int32)
    w = rng.random((T, k)).astype(np.float32)
    skip = rng.random(T) < 0.4
    idx[skip] = -1
    if k > 1:
        part = (~skip) & (rng.random(T) < 0.3)
        idx[part, 0] = -1
    if sparse:
        blank = rng.random((T, k)) < sparse
        blank[:, 1] = False  # every token not skipped keeps at least one pick
        idx[blank] = -1
    x = act(rng.standard_normal((T, 256), dtype=np.float32), "bf16")
    out = moe_experts(x, torch.from_numpy(idx).cuda(), torch.from_numpy(w).cuda(), table)
    keep = ~skip
    ref_idx = np.where(idx < 0, 0, idx).astype(np.int64)
    ref_w = np.where(idx < 0, 0.0, w).astype(np.float32)
    ref = R.moe_combine_ref(to_np32(x)[keep], ref_idx[keep], ref_w[keep], oracle_experts(packed))
    assert rel_l2(to_np32(out)[keep], ref) <= TIGHT
    for ws in _lib.workspaces.all():
        assert _lib.workspace_error(ws) == 0


def test_glm_layer_with_shared_expert(lib):
    """``GLM4MoELayer.forward`` (``model/glm4.py:365-473``): shared_expert(x) +
    routed(x), the shared expert a dense bf16 MLP of moe_ffn rows
    (``:341-344``).  Oracle: the routed oracle plus the dense MLP in float32 on
    the same bf16 weights."""
    from hydranet_b200.moe import SharedExpertMLP
    shape = synth.MoEShape(4096, 1408, 128, 8)
    if "g" not in _FULL:
        _FULL["g"] = device_moe(shape, 4321)
    table, packed = _FULL["g"]
    torch.manual_seed(9)
    shared = SharedExpertMLP(4096, 1408)
    for lin in (shared.gate_proj, shared.up_proj, shared.down_proj):
        torch.nn.init.normal_(lin.weight, std=0.02)
    shared = shared.cuda().to(torch.bfloat16)
    r = GLM4SigmoidRouter(hidden_dim=4096, num_experts=128, experts_per_token=8).cuda()
    layer = MoELayerInt4(r, table, shared_expert=shared)
    x = torch.randn(2, 16, 4096, generator=torch.Generator("cuda").manual_seed(6), device="cuda").to(torch.bfloat16)
    with torch.no_grad():
        out, ro = layer(x, return_routing=True)
    assert out.shape == x.shape
    xi = to_np32(x.view(32, 4096))
    idx = ro.expert_indices.view(32, 8).cpu().numpy()
    w = to_np32(ro.expert_weights.view(32, 8))
    routed = R.moe_combine_ref(xi, idx, w, oracle_experts(packed, idx.ravel()))
    g, u, d = (to_np32(l.weight) for l in (shared.gate_proj, shared.up_proj, shared.down_proj))
    sh = (R.silu(xi @ g.T) * (xi @ u.T)) @ d.T
    err = rel_l2(to_np32(out.view(32, 4096)), routed + sh)
    assert err <= TOL and err <= TIGHT, err


@pytest.mark.parametrize("case", ["g4", "g8"])
def test_group_limited_router_matches_reference(lib, golden_dir, case):
    """Group-limited sigmoid routing on the device (``model/glm4.py:285-297``),
    on the reference fixture's router and inputs rounded to bf16 (the
    device router takes 16-bit activations), against the oracle pinned to
    that fixture."""
    d = dict(np.load(golden_dir / "glm_group_router.npz"))
    E, ng, kg, k, H, T = (int(v) for v in d[case + "/cfg"])
    r = GLM4SigmoidRouter(hidden_dim=H, num_experts=E, experts_per_token=k, n_group=ng, topk_group=kg).cuda()
    with torch.no_grad():
        r.weight.copy_(torch.from_numpy(d[case + "/w"]))
    x = torch.from_numpy(d[case + "/x"]).cuda().to(torch.bfloat16)
    idx, w, logits = ops.moe_route(x.view(T, H), r.params(), E)
    ridx, rw, _ = R.sigmoid_topk_router_ref(to_np32(x.view(T, H)), d[case + "/w"], k, "bf16", n_group=ng,
                                            topk_group=kg)
    np.testing.assert_array_equal(np.sort(idx.cpu().numpy(), 1), np.sort(ridx, 1))
    # weights are cast to the activation dtype: equal up to one bf16 step
    np.testing.assert_allclose(np.sort(w.cpu().numpy(), 1), np.sort(rw, 1), rtol=2 ** -7, atol=1e-6)


def test_group_limited_glm_layer(lib):
    """A routed layer with group-limited routing (4 groups of 8 experts, 2 kept,
    top-6), bf16, against the oracle."""
    H, F, E, k = 512, 256, 32, 6
    shape = synth.MoEShape(H, F, E, k)
    table, packed = host_moe(shape, 808)
    r = GLM4SigmoidRouter(hidden_dim=H, num_experts=E, experts_per_token=k, n_group=4, topk_group=2).cuda()
    layer = MoELayerInt4(r, table)
    x = torch.randn(24, H, generator=torch.Generator("cuda").manual_seed(6), device="cuda").to(torch.bfloat16)
    out, ro = layer(x, return_routing=True)
    xi = to_np32(x)
    idx, w, logits = R.sigmoid_topk_router_ref(xi, to_np32(r.weight), k, "bf16", n_group=4, topk_group=2)
    np.testing.assert_array_equal(np.sort(ro.expert_indices.cpu().numpy(), 1), np.sort(idx, 1))
    ref = R.moe_combine_ref(xi, idx, w, oracle_experts(packed))
    assert rel_l2(to_np32(out), ref) <= TIGHT
