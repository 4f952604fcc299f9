"""The two decode engines side by side on the same inputs.

Segments of at most 16 tokens per expert run on the register-dequant
mma.sync engine by default and on the tcgen05 engine when
``hn_set_decode_engine(HN_ENGINE_TCGEN05)`` selects it.  Both must match the
oracle (the reference's dequant-then-matmul path, fp32 accumulation) within
the tolerances of the other parity tests, agree with each other closely (they
differ only in where the group scale is applied: the tcgen05 engine rounds
(n - 8) * scale to float16 as the reference kernel does, the mma.sync engine
applies the scale in fp32 after each k-group), and repeat bit for bit.
"""

import contextlib

import numpy as np
import pytest
import torch

from hydranet_b200 import _lib, ops, synth
from hydranet_b200.moe import MoELayerInt4, moe_experts
from hydranet_b200.router import GLM4SigmoidRouter, TopKRouter
from oracle import int4_ref as R
from tests.gpu_util import act, device_moe, oracle_experts, rel_l2, to_np32

pytestmark = pytest.mark.gpu

TOL = 1e-2
TIGHT = {"bf16": 6e-3, "f16": 2e-3}
ENGINE_AGREE = 3e-3


@contextlib.contextmanager
def engine(which):
    lib = _lib.load()
    prev = lib.hn_set_decode_engine(which)
    try:
        yield
    finally:
        lib.hn_set_decode_engine(prev)


def both(fn, rows=None):
    """Outputs of the mma.sync engine (called twice: must repeat bit for bit)
    and of the tcgen05 engine; ``rows`` limits the comparison to the rows the
    call defines."""
    torch.cuda.synchronize()
    with engine(_lib.HN_ENGINE_AUTO):
        a = fn()
        a2 = fn()
    with engine(_lib.HN_ENGINE_TCGEN05):
        b = fn()
    torch.cuda.synchronize()
    if rows is not None:
        a, a2, b = a[rows], a2[rows], b[rows]
    assert torch.equal(a, a2), "mma.sync engine is not bitwise repeatable"
    return to_np32(a), to_np32(b)


@pytest.mark.parametrize("M,N,K", [(1, 256, 128), (5, 1000, 512), (16, 77, 1024), (9, 2048, 4096),
                                   (3, 300, 384), (8, 4096, 14336), (12, 512, 2048), (40, 512, 2048)])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_int4_linear_engines(lib, M, N, K, dtype):
    w = np.random.default_rng(N + K).standard_normal((N, K), dtype=np.float32) * np.float32(0.02)
    p, s = R.quantize_tensor(w)
    x = act(np.random.default_rng(M).standard_normal((M, K), dtype=np.float32), dtype)
    pt, st = torch.from_numpy(p).cuda(), torch.from_numpy(s).cuda()
    a, b = both(lambda: ops.int4_linear(x, pt, st))
    ref = R.int4_linear_ref(to_np32(x), p, s)
    assert rel_l2(a, ref) <= min(TOL, TIGHT[dtype])
    assert rel_l2(b, ref) <= min(TOL, TIGHT[dtype])
    assert rel_l2(a, b) <= ENGINE_AGREE


@pytest.mark.parametrize("T", [1, 7, 16, 33])
def test_expert_mlp_engines(lib, T):
    H, F = 1024, 2048
    table, packed = device_moe(synth.MoEShape(H, F, 1, 1), 77 + T)
    sl = table.slots[0]
    x = act(np.random.default_rng(T).standard_normal((T, H), dtype=np.float32), "bf16")
    a, b = both(lambda: ops.expert_mlp_int4(x, *sl.tensors()))
    ref = R.expert_mlp_ref(to_np32(x), *packed[0])
    assert rel_l2(a, ref) <= TIGHT["bf16"]
    assert rel_l2(b, ref) <= TIGHT["bf16"]
    assert rel_l2(a, b) <= ENGINE_AGREE


_TABLES = {}


def _table(key, shape, seed):
    if key not in _TABLES:
        _TABLES[key] = device_moe(shape, seed)
    return _TABLES[key]


@pytest.mark.parametrize("T", [1, 3, 8, 9, 16, 40])
def test_mixtral_layer_engines(lib, T):
    shape = synth.MoEShape(1024, 2048, 8, 2)
    table, packed = _table("m", shape, 31)
    r = TopKRouter(hidden_dim=1024, num_experts=8, experts_per_token=2).cuda().to(torch.bfloat16)
    with torch.no_grad():
        r.gate.weight.copy_(torch.randn(8, 1024, generator=torch.Generator("cuda").manual_seed(7), device="cuda") * 0.02)
    layer = MoELayerInt4(r, table)
    x = torch.randn(T, 1024, generator=torch.Generator("cuda").manual_seed(T), device="cuda").to(torch.bfloat16)
    with torch.no_grad():
        a, b = both(lambda: layer(x))
        _, ro = layer(x, return_routing=True)
    idx, w = ro.expert_indices.cpu().numpy(), to_np32(ro.expert_weights)
    ref = R.moe_combine_ref(to_np32(x), idx, w, oracle_experts(packed))
    assert rel_l2(a, ref) <= TIGHT["bf16"]
    assert rel_l2(b, ref) <= TIGHT["bf16"]
    assert rel_l2(a, b) <= ENGINE_AGREE


@pytest.mark.parametrize("T", [1, 8, 32, 64])
def test_glm_layer_engines(lib, T):
    """GLM-4.5-Air shape: 128 experts of F = 1408 (11 k-groups in the down phase), sigmoid top-8."""
    shape = synth.MoEShape(4096, 1408, 128, 8)
    table, packed = _table("g", shape, 4321)
    r = GLM4SigmoidRouter(hidden_dim=4096, num_experts=128, experts_per_token=8).cuda()
    r.set_correction_bias(torch.from_numpy(synth.host_correction_bias(3, 128)).cuda())
    layer = MoELayerInt4(r, table)
    x = torch.randn(T, 4096, generator=torch.Generator("cuda").manual_seed(50 + T), device="cuda").to(torch.bfloat16)
    with torch.no_grad():
        a, b = both(lambda: layer(x))
        _, ro = layer(x, return_routing=True)
    idx, w = ro.expert_indices.cpu().numpy(), to_np32(ro.expert_weights)
    ref = R.moe_combine_ref(to_np32(x), idx, w, oracle_experts(packed, idx.ravel()))
    assert rel_l2(a, ref) <= TIGHT["bf16"]
    assert rel_l2(b, ref) <= TIGHT["bf16"]
    assert rel_l2(a, b) <= ENGINE_AGREE


def test_given_routing_duplicates_and_unused_engines(lib):
    """Caller routing with a token that picks one expert twice, -1 slots and an all -1 token."""
    shape = synth.MoEShape(512, 1024, 8, 2)
    table, packed = _table("s", shape, 9)
    T = 6
    idx = torch.tensor([[3, 3], [0, 7], [-1, 5], [-1, -1], [2, 1], [6, 6]], dtype=torch.int32, device="cuda")
    w = torch.tensor([[0.25, 0.75], [0.5, 0.5], [0.0, 1.0], [0.0, 0.0], [0.9, 0.1], [0.5, 0.5]], device="cuda")
    x = act(np.random.default_rng(1).standard_normal((T, 512), dtype=np.float32), "bf16")
    keep = [0, 1, 2, 4, 5]  # token 3 has no picks: its row is unspecified
    a, b = both(lambda: moe_experts(x, idx, w, table), rows=keep)
    ii = idx.cpu().numpy()[keep]
    ww = w.cpu().numpy()[keep]
    ii = np.where(ii < 0, 0, ii)
    ref = R.moe_combine_ref(to_np32(x)[keep], ii, ww, oracle_experts(packed))
    assert rel_l2(a, ref) <= TIGHT["bf16"]
    assert rel_l2(b, ref) <= TIGHT["bf16"]


@pytest.mark.parametrize("T", [8, 64, 300])
def test_sm_limit_same_results(lib, T):
    """Grids sized for fewer SMs (hn_set_sm_limit, as the expert-parallel
    prefill does to leave room for NCCL) compute the same layer."""
    shape = synth.MoEShape(1024, 2048, 8, 2)
    table, packed = _table("m", shape, 31)
    r = TopKRouter(hidden_dim=1024, num_experts=8, experts_per_token=2).cuda().to(torch.bfloat16)
    with torch.no_grad():
        r.gate.weight.copy_(torch.randn(8, 1024, generator=torch.Generator("cuda").manual_seed(7), device="cuda") * 0.02)
    layer = MoELayerInt4(r, table)
    x = torch.randn(T, 1024, generator=torch.Generator("cuda").manual_seed(T), device="cuda").to(torch.bfloat16)
    lib_ = _lib.load()
    with torch.no_grad():
        a = layer(x)
        prev = lib_.hn_set_sm_limit(100)
        try:
            b = layer(x)
        finally:
            lib_.hn_set_sm_limit(prev)
    assert rel_l2(to_np32(a), to_np32(b)) <= ENGINE_AGREE
