"""The reference's own MoE layers, unchanged, running on this library's kernels.

``baseline/_ref`` holds the reference installed unmodified from its own
sources (pip, no dependencies).  The test imports it as the package
``hydranet`` and, before any of its model code runs, points
``hydranet.kernels`` and its submodules at ``hydranet_b200.kernels`` -- the
module aliasing of the integration guide.  ``MixtralMoELayer.forward``
(``model/mixtral.py:259-370``, top-2) and ``GLM4MoELayer.forward``
(``model/glm4.py:365-473``, shared expert + routed) then run with the
reference's own ``ExpertCacheManager`` in packed mode over a store written by
``hydranet_b200.packing.write_store`` (the reference's format, byte for byte):
each of their lazy ``from ..kernels.int4_gemm import expert_mlp_int4_fused``
calls lands in this library (counted), and the outputs match the oracle on
the routing the reference's own routers chose.  Skipped when the reference is
not installed in ``baseline/_ref``.
"""

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from hydranet_b200 import synth
from hydranet_b200.packing import write_store
from oracle import int4_ref as R
from tests.gpu_util import oracle_experts, rel_l2, to_np32

REF = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not (REF / "model" / "mixtral.py").exists(),
                                 reason="the reference is not installed in baseline/_ref")]

TIGHT = 6e-3


@pytest.fixture(scope="module")
def ref(tmp_path_factory):
    """The reference as package ``hydranet`` with its kernels aliased to ours;
    yields (hydranet package modules, call counter)."""
    root = tmp_path_factory.mktemp("refpkg")
    (root / "hydranet").symlink_to(REF, target_is_directory=True)
    import hydranet_b200.kernels as hk
    import hydranet_b200.kernels.expert_mlp  # noqa: F401
    import hydranet_b200.kernels.int4_expert_mlp  # noqa: F401
    import hydranet_b200.kernels.int4_gemm as ours
    import hydranet_b200.kernels.int4_linear  # noqa: F401
    calls = {"n": 0}
    real = ours.expert_mlp_int4_fused

    def counted(*args, **kw):
        calls["n"] += 1
        return real(*args, **kw)

    saved = {k: v for k, v in sys.modules.items() if k == "hydranet" or k.startswith("hydranet.")}
    sys.path.insert(0, str(root))
    try:
        import hydranet  # noqa: F401  (namespace package over baseline/_ref)
        sys.modules["hydranet.kernels"] = hk
        for name in ("int4_gemm", "int4_expert_mlp", "expert_mlp", "int4_linear"):
            sys.modules[f"hydranet.kernels.{name}"] = sys.modules[f"hydranet_b200.kernels.{name}"]
        ours.expert_mlp_int4_fused = counted
        from hydranet import config as rcfg
        from hydranet.cache.expert_cache import ExpertCacheManager
        from hydranet.cache.packed_expert_store import PackedExpertStore
        from hydranet.model.glm4 import GLM4MoELayer
        from hydranet.model.mixtral import MixtralMoELayer
        yield dict(cfg=rcfg, ExpertCacheManager=ExpertCacheManager, PackedExpertStore=PackedExpertStore,
                   MixtralMoELayer=MixtralMoELayer, GLM4MoELayer=GLM4MoELayer), calls
    finally:
        ours.expert_mlp_int4_fused = real
        sys.path.remove(str(root))
        for k in [k for k in sys.modules if k == "hydranet" or k.startswith("hydranet.")]:
            del sys.modules[k]
        sys.modules.update(saved)


def _store(tmp_path, H, F, E, seed):
    shape = synth.MoEShape(H, F, E, 2)
    experts, packed = {}, []
    for e in range(E):
        g, u, d = synth.host_expert_weights(seed, shape, e)
        t = (*R.quantize_tensor(g), *R.quantize_tensor(u), *R.quantize_tensor(d))
        experts[(0, e)] = t
        packed.append(list(t))
    write_store(tmp_path, experts, H, F, num_layers=1, num_experts=E)
    return tmp_path / "experts.idx", packed


def _cache(m, model_config, idx_path, E):
    cc = m["cfg"].ExpertCacheConfig(pinned_slots=0, hot_slots=E // 2, probation_slots=E - E // 2,
                                    enable_affinity_bonus=False, enable_dynamic_slots=False,
                                    max_slots_per_layer=E + 1)
    cm = m["ExpertCacheManager"](model_config=model_config, cache_config=cc, device=torch.device("cuda"),
                                 dtype=torch.float16)
    cm.set_packed_store(m["PackedExpertStore"](index_path=idx_path, device=torch.device("cuda")))
    return cc, cm


def test_reference_mixtral_layer_on_our_kernels(ref, tmp_path):
    m, calls = ref
    H, F, E = 512, 1024, 8
    idx_path, packed = _store(tmp_path, H, F, E, 7)
    mc = m["cfg"].MixtralConfig()
    mc.num_layers, mc.num_experts, mc.hidden_dim, mc.intermediate_dim = 1, E, H, F
    cc, cm = _cache(m, mc, idx_path, E)
    try:
        layer = m["MixtralMoELayer"](mc, cc, 0, cm).cuda().half()
        with torch.no_grad():
            layer.router.gate.weight.copy_(torch.from_numpy(synth.host_router_weight(7, synth.MoEShape(H, F, E, 2))))
        x = torch.from_numpy(synth.host_activations(3, 6, H)).view(1, 6, H).cuda().half()
        before = calls["n"]
        with torch.no_grad():
            out = layer(x, top_k=2)
            ro = layer.router(x, top_k_override=2)
        assert calls["n"] - before >= len(torch.unique(ro.expert_indices))  # every expert ran on our kernel
        idx = ro.expert_indices.view(6, 2).cpu().numpy()
        w = to_np32(ro.expert_weights.view(6, 2))
        want = R.moe_combine_ref(to_np32(x.view(6, H)), idx, w, oracle_experts(packed))
        assert rel_l2(to_np32(out.view(6, H)), want) <= TIGHT
    finally:
        cm.shutdown()


def test_reference_glm4_layer_on_our_kernels(ref, tmp_path):
    m, calls = ref
    H, F, E, K = 512, 256, 16, 4
    idx_path, packed = _store(tmp_path, H, F, E, 11)
    gc = m["cfg"].GLM4AirConfig()
    gc.num_layers, gc.num_experts, gc.hidden_dim = 1, E, H
    gc.moe_intermediate_dim, gc.intermediate_dim, gc.experts_per_token = F, F, K

    class CacheView:  # what ExpertCacheManager reads of a model config
        num_layers, num_experts = 1, E
        expert_size_bytes = 3 * H * F * 2

    cc, cm = _cache(m, CacheView(), idx_path, E)
    try:
        layer = m["GLM4MoELayer"](gc, 0, cm).cuda().half()
        torch.manual_seed(4)
        with torch.no_grad():
            for p in layer.parameters():
                p.copy_(torch.randn_like(p) * 0.02)
        x = torch.from_numpy(synth.host_activations(5, 7, H)).view(1, 7, H).cuda().half()
        before = calls["n"]
        with torch.no_grad():
            out = layer(x)
            idx, w = layer.router(x)
        assert calls["n"] - before >= len(torch.unique(idx))
        xi = to_np32(x.view(7, H))
        routed = R.moe_combine_ref(xi, idx.view(7, K).cpu().numpy(), to_np32(w.view(7, K)),
                                   oracle_experts(packed))
        se = layer.shared_expert
        g, u, d = (to_np32(lin.weight) for lin in (se.gate_proj, se.up_proj, se.down_proj))
        shared = (R.silu(xi @ g.T) * (xi @ u.T)) @ d.T
        assert rel_l2(to_np32(out.view(7, H)), routed + shared) <= TIGHT
    finally:
        cm.shutdown()
