"""Over-budget expert residency (``hydranet_b200.slot_cache``): more experts
than device slots, misses loaded by H2D copies from pinned host blobs read
from a v2.0 store, least-recently-used eviction, each layer's expert table
repointed at the slots -- and every layer output equal to the oracle on the
routing the device chose (``MixtralMoELayer.forward`` over the reference's
slot cache, ``model/mixtral.py:259-370``, ``cache/expert_cache.py:601-679``)."""

import numpy as np
import pytest
import torch

from hydranet_b200 import synth
from hydranet_b200.packing import write_store
from hydranet_b200.router import TopKRouter
from hydranet_b200.slot_cache import ExpertSource, SlotCache, SlotCachedMoELayer
from oracle import int4_ref as R
from tests.gpu_util import oracle_experts, rel_l2, to_np32

pytestmark = pytest.mark.gpu

H, F, E, L = 512, 1024, 8, 3


def _build(tmp_path, slots, bonus=False):
    shape = synth.MoEShape(H, F, E, 2)
    experts, packed = {}, {}
    for layer in range(L):
        for e in range(E):
            g, u, d = synth.host_expert_weights(50 + layer, shape, e)
            t = (*R.quantize_tensor(g), *R.quantize_tensor(u), *R.quantize_tensor(d))
            experts[(layer, e)] = t
            packed[(layer, e)] = list(t)
    write_store(tmp_path, experts, H, F, num_layers=L, num_experts=E)
    cache = SlotCache(H, F, L, E, slots, ExpertSource.from_store(tmp_path / "experts.idx"))
    layers = []
    for layer in range(L):
        r = TopKRouter(hidden_dim=H, num_experts=E, experts_per_token=2).cuda().to(torch.bfloat16)
        with torch.no_grad():
            r.gate.weight.copy_(torch.from_numpy(synth.host_normal(70 + layer, (E, H), 0.02)))
        r.enable_affinity_bonus = bonus
        layers.append(SlotCachedMoELayer(r, cache, layer))
    return cache, layers, packed


@pytest.mark.parametrize("bonus", [False, True])
def test_over_budget_layers_match_oracle(lib, tmp_path, bonus):
    cache, layers, packed = _build(tmp_path, slots=14, bonus=bonus)  # 24 experts, 14 slots
    from hydranet_b200 import ops
    for step in range(5):
        x = torch.randn(3, H, generator=torch.Generator("cuda").manual_seed(step), device="cuda").to(torch.bfloat16)
        for layer, mod in enumerate(layers):
            r = mod.router
            bvec = r.bonus_vector(x.device)  # the bonus the layer call will see (residency before its loads)
            idx, w, _ = ops.moe_route(x, r.params(2, bvec), E, keep_refs=(bvec,), want_logits=False)
            with torch.no_grad():
                out = mod(x)
            torch.cuda.synchronize()
            ii, ww = idx.cpu().numpy(), w.cpu().numpy()
            for e in np.unique(ii):
                assert cache.is_resident(layer, int(e))
            exps = oracle_experts([packed[(layer, e)] for e in range(E)], ii.ravel())
            ref = R.moe_combine_ref(to_np32(x), ii, ww, exps)
            assert rel_l2(to_np32(out), ref) <= 6e-3, (step, layer)
    s = cache.stats
    assert s.misses > 14 and s.evictions > 0 and s.hits > 0
    assert s.h2d_bytes == s.misses * cache.blob_bytes


def test_budget_smaller_than_one_call_is_refused(lib, tmp_path):
    cache, layers, _ = _build(tmp_path, slots=1)
    x = torch.randn(4, H, device="cuda").to(torch.bfloat16)
    with pytest.raises(RuntimeError, match="slot budget"):
        with torch.no_grad():
            for mod in layers:
                mod(x)
