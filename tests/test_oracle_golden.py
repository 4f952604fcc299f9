"""The numpy oracle reproduces the reference's own outputs (CPU, no GPU).

Fixtures were produced by ``tests/golden/make_golden.py`` running HydraNet's
packer (``preprocess/pack_weights.py:133-268``), routers
(``model/router.py:73-130``, ``model/glm4.py:261-309``) and MoE layers in
dequant mode (``model/mixtral.py:259-370``, ``model/glm4.py:365-473``).
Integer outputs must match bit for bit; float32 outputs within 1e-5 relative
(the only difference is BLAS summation order).
"""

import hashlib

import numpy as np
import pytest

from oracle import int4_ref as R
from hydranet_b200 import synth


def load(golden_dir, name):
    return dict(np.load(golden_dir / name))


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("case", ["rand_f32", "rand_f16", "wide_f32", "edge_f32"])
def test_quantize_bit_exact(golden_dir, case):
    g = load(golden_dir, "pack_cases.npz")
    p, s = R.quantize_tensor(g[case + "/w"])
    np.testing.assert_array_equal(p, g[case + "/packed"])
    np.testing.assert_array_equal(s.view(np.uint16), g[case + "/scales"].view(np.uint16))


@pytest.mark.parametrize("case", ["rand_f32", "rand_f16", "wide_f32", "edge_f32"])
def test_dequantize_bit_exact(golden_dir, case):
    g = load(golden_dir, "pack_cases.npz")
    d = R.dequantize_tensor(g[case + "/packed"], g[case + "/scales"])
    np.testing.assert_array_equal(d.view(np.uint16), g[case + "/dequant"].view(np.uint16))


def test_quant_error_bounds(golden_dir):
    """Reference bound: max abs err < 0.1, mean < 0.01 (``tests/test_int4_pack.py:64-66``)."""
    w = synth.host_normal(42, (512, 256), 0.1).astype(np.float16)
    p, s = R.quantize_tensor(w)
    d = R.dequantize_tensor(p, s)
    err = np.abs(d.astype(np.float32) - w.astype(np.float32))
    assert err.max() < 0.1 and err.mean() < 0.01


def test_blob_layout_matches_reference_sizes():
    """Same checks as the reference's ``tests/test_int4_pack.py:179-230``."""
    lay = R.BlobLayout.from_dims(4096, 14336, 128)
    assert lay.gate_packed_size == 14336 * 2048
    assert lay.gate_scales_offset == lay.gate_packed_size
    assert lay.total_size == 90_832_896
    assert R.BlobLayout.from_dims(4096, 1408, 128).total_size == 8_921_088
    assert R.BlobLayout.from_dims(512, 1024, 128).total_size == 811_008


def _experts(dims, seed):
    H, F, E, K, G = (int(v) for v in dims[:5])
    shape = synth.MoEShape(H, F, E, K, G)
    packed, hashes = [], []
    for e in range(E):
        g, u, d = synth.host_expert_weights(seed, shape, e)
        t = [*R.quantize_tensor(g, G), *R.quantize_tensor(u, G), *R.quantize_tensor(d, G)]
        h = hashlib.sha256()
        for a in t:
            h.update(np.ascontiguousarray(a).tobytes())
        packed.append(t)
        hashes.append(h.hexdigest())
    return shape, packed, hashes


@pytest.mark.parametrize("name", ["c1_mixtral_layer.npz", "c1_mixtral_layer_affinity.npz",
                                  "c2_small_mixtral_layer.npz"])
def test_mixtral_layer(golden_dir, name):
    g = load(golden_dir, name)
    dims = g["dims"]
    seed, T = int(dims[6]), int(dims[5])
    shape, packed, hashes = _experts(dims, seed)
    # packer parity, bit-exact over every expert blob
    assert hashes == list(g["expert_sha256"])
    x = synth.host_activations(seed, T, shape.hidden)
    np.testing.assert_array_equal(x, g["x"])
    bonus = None
    if g["affinity_cached"].size:
        bonus = np.zeros(shape.experts, np.float32)
        bonus[g["affinity_cached"]] = 0.1
    idx, w, logits = R.softmax_topk_router_ref(x, g["router_w"], shape.top_k, "f32", affinity_bonus=bonus)
    np.testing.assert_array_equal(idx, g["idx"])
    np.testing.assert_allclose(logits, g["logits"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(w, g["weights"], rtol=1e-5, atol=1e-7)
    experts = {e: R.DequantExpert.from_packed(*t) for e, t in enumerate(packed)}
    out = R.moe_combine_ref(x, idx, w, experts)
    assert rel_l2(out, g["out"]) < 1e-5


def test_glm_layer(golden_dir):
    g = load(golden_dir, "glm_small_layer.npz")
    dims = g["dims"]
    seed, T = int(dims[6]), int(dims[5])
    shape, packed, hashes = _experts(dims, seed)
    assert hashes == list(g["expert_sha256"])
    x = synth.host_activations(seed, T, shape.hidden)
    idx, w, _ = R.sigmoid_topk_router_ref(x, g["router_w"], shape.top_k, "f32")
    np.testing.assert_array_equal(idx, g["idx"])
    np.testing.assert_allclose(w, g["weights"], rtol=1e-5, atol=1e-7)
    experts = {e: R.DequantExpert.from_packed(*t) for e, t in enumerate(packed)}
    out = R.moe_combine_ref(x, idx, w, experts)
    assert rel_l2(out, g["out"]) < 1e-5


def test_mixtral_router_bf16(golden_dir):
    """bf16 model: logits come out of a bf16 Linear (``model/router.py:102``)."""
    g = load(golden_dir, "mixtral_router_bf16.npz")
    H, E, K, T, seed = (int(v) for v in g["dims"])
    shape = synth.MoEShape(H, 128, E, K)
    x = R.round_to_bf16(synth.host_activations(seed, T, H))
    rw = R.round_to_bf16(synth.host_router_weight(seed, shape))
    idx, w, logits = R.softmax_topk_router_ref(x, rw, K, "bf16")
    # logits may differ by one bf16 ulp where the float32 sum lands near a rounding boundary
    ulp = np.abs(g["logits"]) * 2.0 ** -7 + 1e-30
    assert np.all(np.abs(logits - g["logits"]) <= ulp)
    mism = np.nonzero(np.any(idx != g["idx"], axis=1))[0]
    for t in mism:  # only tolerated on a near-tie of the reference's own logits
        s = np.sort(g["logits"][t])[::-1]
        assert s[K - 1] - s[K] <= 2 * ulp[t].max()
    assert len(mism) <= max(1, T // 32)


@pytest.mark.parametrize("name,dtype", [("glm_router_f32.npz", "f32"), ("glm_router_bf16.npz", "bf16")])
def test_glm_router_full_width(golden_dir, name, dtype):
    g = load(golden_dir, name)
    H, E, K, T, seed = (int(v) for v in g["dims"])
    shape = synth.MoEShape(H, 128, E, K)
    x = synth.host_activations(seed, T, H)
    if dtype == "bf16":
        x = R.round_to_bf16(x)
    idx, w, _ = R.sigmoid_topk_router_ref(x, synth.host_router_weight(seed, shape), K, dtype)
    np.testing.assert_array_equal(idx, g["idx"])
    np.testing.assert_allclose(w, g["weights"], rtol=1e-2 if dtype == "bf16" else 1e-5, atol=1e-6)


def test_glm_group_limited_router_golden(golden_dir):
    """Group-limited sigmoid routing (``model/glm4.py:285-297``) against the reference's own router."""
    d = dict(np.load(golden_dir / "glm_group_router.npz"))
    for n in ("g4", "g8"):
        E, ng, kg, k, H, T = (int(v) for v in d[n + "/cfg"])
        idx, w, _ = R.sigmoid_topk_router_ref(d[n + "/x"][0], d[n + "/w"], k, "f32", n_group=ng, topk_group=kg)
        np.testing.assert_array_equal(np.sort(idx, 1), np.sort(d[n + "/idx"], 1))
        np.testing.assert_allclose(np.sort(w, 1), np.sort(d[n + "/wt"], 1), rtol=1e-6, atol=1e-7)
        # the mask matters here: the plain top-k would pick other experts
        plain, _, _ = R.sigmoid_topk_router_ref(d[n + "/x"][0], d[n + "/w"], k, "f32")
        assert (np.sort(plain, 1) != np.sort(idx, 1)).any()
