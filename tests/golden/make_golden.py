#!/usr/bin/env python3
"""Generate the golden fixtures in this directory by running the REFERENCE.

This script imports HydraNet itself (read-only) and records what the
reference computes on seeded synthetic inputs: its packer, its dequantiser,
the non-expert ``Int4Linear`` quantiser, its group-by-expert gatherer, a
packed store written by its own test helper, its two routers and its MoE
layers in dequant mode.  The fixtures pin the numpy oracle under ``oracle/``; the GPU box never runs this script (the
reference is not there), it only reads the committed ``.npz`` files.

Usage (from the repository root)::

    python tests/golden/make_golden.py --reference <path to the hydranet checkout>

The reference checkout is exposed to Python as a package named ``hydranet``
through a symlink in a temporary directory.

Large weights are not stored: they are regenerated from their seed with
numpy's PCG64 stream (``hydranet_b200/synth.py``) and pinned by the SHA-256 of
the packed expert blobs the reference packer produced.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from hydranet_b200 import synth  # noqa: E402


def import_reference(ref: Path):
    tmp = Path(tempfile.mkdtemp(prefix="hnref_"))
    os.symlink(ref, tmp / "hydranet")
    sys.path.insert(0, str(tmp))
    import torch  # noqa: F401
    import hydranet  # noqa: F401
    return hydranet


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


# ---------------------------------------------------------------------------
# 1. Packer / dequantiser known answers
# ---------------------------------------------------------------------------

def pack_cases(torch, ExpertWeightPacker, QuantConfig):
    packer = ExpertWeightPacker(QuantConfig(group_size=128))
    cases = {}

    def add(name, w):
        t = torch.from_numpy(w.copy())
        p, s = packer.quantize_tensor(t)
        d = packer.dequantize_tensor(p, s, w.shape[0], w.shape[1])
        cases[name + "/w"] = w
        cases[name + "/packed"] = p.numpy()
        cases[name + "/scales"] = s.numpy()
        cases[name + "/dequant"] = d.numpy()

    add("rand_f32", synth.host_normal(11, (64, 256), 0.1))
    add("rand_f16", synth.host_normal(12, (32, 512), 0.1).astype(np.float16))
    add("wide_f32", synth.host_normal(13, (16, 1024), 0.02))
    # Edge rows: an all-zero group, exact half-way values (ties round to even),
    # a dominant outlier, very large and very small magnitudes, all-negative.
    e = synth.host_normal(14, (8, 256), 1.0)
    e[0, :128] = 0.0
    e[1, :128] = np.float32(7.0) * (np.arange(128, dtype=np.float32) % 15 - 7) / np.float32(7.0)
    e[1, 0] = 7.0  # absmax 7 -> scale 1: entries are integers; add exact halves below
    e[1, 1:15] = np.array([0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 3.5, -3.5, 4.5, -4.5, 5.5, -5.5, 6.5, -6.5],
                          dtype=np.float32)
    e[2, 128:] *= 1e-3
    e[2, 130] = 50.0
    e[3] *= 1e4
    e[4] *= 1e-30
    e[5] = -np.abs(e[5])
    add("edge_f32", e.astype(np.float32))
    return cases


def int4linear_cases(torch, Int4Linear):
    """The non-expert ``Int4Linear`` quantiser (``kernels/int4_linear.py:69-103``)
    and ``from_float``'s group-size choice (``:121-131``)."""
    cases = {}

    def add(name, w, gs):
        p, s = Int4Linear.quantize_weight(torch.from_numpy(w.copy()), gs)
        cases[name + "/w"] = w
        cases[name + "/packed"] = p.numpy()
        cases[name + "/scales"] = s.numpy()
        cases[name + "/group_size"] = np.int64(gs)

    add("rand_f32", synth.host_normal(21, (32, 512), 0.02), 128)
    add("rand_f16", synth.host_normal(22, (48, 256), 0.05).astype(np.float16), 128)
    add("g64_f32", synth.host_normal(23, (16, 192), 0.1), 64)
    e = synth.host_normal(24, (6, 256), 1.0)
    e[0, :128] = 0.0                                    # all-zero group: absmax clamps to 1e-8
    e[1, :128] = np.float32(3.5) * (np.arange(128, dtype=np.float32) % 3 - 1)  # w/absmax*7 = -7, 0, 7
    e[1, 128:142] = np.array([0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 3.5, -3.5, 4.5, -4.5, 5.5, -5.5, 6.5, -6.5],
                             dtype=np.float32)
    e[1, 142] = 7.0                                     # absmax 7: halves above are exact ties
    e[2] *= 1e4
    e[3] *= 1e-20
    e[4] = -np.abs(e[4])
    add("edge_f32", e.astype(np.float32), 128)
    for n_in in (256, 192, 96):
        m = Int4Linear.from_float(torch.nn.Linear(n_in, 8), group_size=128)
        cases[f"from_float_group/{n_in}"] = np.int64(m.group_size)
    return cases


def gatherer_cases(torch, GroupByExpertGatherer):
    """The reference's group-by-expert gather and scatter
    (``scheduler/continuous_batch.py:281-381``) on CPU tensors.  Each expert's
    output is a fixed function of its gathered rows, ``rows * (e + 1) - e``."""
    cases = {}

    def add(name, T, k, E, H, dtype, dup=False):
        rng = np.random.default_rng(T * 31 + k)
        idx = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int64)
        if dup:
            idx[::3, 1] = idx[::3, 0]                     # some tokens pick an expert twice
        idx[:, :][idx == 2] = 3                            # expert 2 unused
        hid = rng.standard_normal((T, H)).astype(np.float32)
        w = rng.random((T, k)).astype(np.float32)
        g = GroupByExpertGatherer(device=torch.device("cpu"))
        tdt = getattr(torch, dtype)
        got = g.gather(torch.from_numpy(hid).to(tdt), torch.from_numpy(idx), torch.from_numpy(w).to(tdt), 5)
        outs = [(x, x.hidden_states * (x.expert_idx + 1) - x.expert_idx) for x in got]
        y = g.scatter(outs, (T, H))
        cases[name + "/hidden"] = hid
        cases[name + "/idx"] = idx
        cases[name + "/w"] = w
        cases[name + "/dtype"] = np.array(dtype)
        cases[name + "/experts"] = np.array([x.expert_idx for x in got], dtype=np.int64)
        cases[name + "/counts"] = np.array([x.num_tokens for x in got], dtype=np.int64)
        cases[name + "/layer"] = np.array([x.layer_idx for x in got], dtype=np.int64)
        cases[name + "/tokens"] = torch.cat([x.token_indices for x in got]).numpy()
        cases[name + "/weights"] = torch.cat([x.routing_weights for x in got]).float().numpy()
        cases[name + "/rows"] = torch.cat([x.hidden_states for x in got]).float().numpy()
        cases[name + "/scatter"] = y.float().numpy()
        cases[name + "/scatter_dtype"] = np.array(str(y.dtype))

    add("f32", 37, 3, 8, 16, "float32")
    add("f32_dup", 25, 4, 6, 8, "float32", dup=True)
    add("f16", 19, 2, 8, 8, "float16")
    return cases


def scheduler_trace(torch):
    """The scripted scheduler session of ``scheduler_script.py`` run on the
    reference's ``scheduler/continuous_batch.py``."""
    sys.path.insert(0, str(HERE))
    import scheduler_script
    from hydranet.scheduler import continuous_batch
    return {"lines": np.array(scheduler_script.run(continuous_batch, torch))}


def glm4_dense_cases(torch):
    """The reference's ``GLM4Attention`` (prefill of 5 positions, then one
    decode position through its ``SimpleKVCache``), ``GLM4DenseMLP`` and an
    lm_head-shaped linear, float32 on CPU, at a small GLM-4.5 layout (8 query
    / 2 KV heads, head_dim 32, partial rotary 0.5, attention bias)."""
    from hydranet.config import GLM4AirConfig
    from hydranet.model.glm4 import GLM4Attention, GLM4DenseMLP
    from hydranet.cache.kv_cache import SimpleKVCache
    cfg = GLM4AirConfig()
    cfg.hidden_dim, cfg.num_attention_heads, cfg.num_kv_heads, cfg.head_dim = 256, 8, 2, 32
    cfg.intermediate_dim, cfg.max_position_embeddings = 192, 64
    torch.manual_seed(0)
    attn = GLM4Attention(cfg, 0).float()
    mlp = GLM4DenseMLP(cfg).float()
    out = {}
    with torch.no_grad():
        for name, mod in (("attn", attn), ("mlp", mlp)):
            for pn, p in mod.named_parameters():
                v = torch.from_numpy(synth.host_normal(sum(pn.encode()) + 31, tuple(p.shape), 0.05))
                p.copy_(v)
                out[f"{name}/{pn}"] = v.numpy()
        x = torch.from_numpy(synth.host_normal(5, (1, 6, 256), 1.0))
        out["x"] = x.numpy()
        cache = SimpleKVCache(num_layers=1, num_kv_heads=2, head_dim=32, max_seq_len=16, device=torch.device("cpu"),
                              dtype=torch.float32)
        out["attn_prefill"] = attn(x[:, :5], torch.arange(5).view(1, 5), kv_cache=cache).numpy()
        cache.set_len(5)
        out["attn_decode"] = attn(x[:, 5:6], torch.tensor([[5]]), kv_cache=cache).numpy()
        out["attn_nocache"] = attn(x, torch.arange(6).view(1, 6)).numpy()
        out["mlp"] = mlp(x).numpy()
        lm = torch.nn.Linear(256, 96, bias=False).float()
        lm.weight.copy_(torch.from_numpy(synth.host_normal(77, (96, 256), 0.05)))
        out["lm_w"] = lm.weight.numpy()
        out["lm"] = lm(x).numpy()
    return out


def glm_group_router_cases(torch):
    """The reference's ``GLM4SigmoidRouter`` with group-limited selection
    (``model/glm4.py:285-297``): 32 experts in 4 groups, 2 groups kept, top-6,
    and 64 experts in 8 groups, 3 kept, top-8; float32 on CPU."""
    from hydranet.config import GLM4AirConfig
    from hydranet.model.glm4 import GLM4SigmoidRouter
    out = {}
    for name, (E, ng, kg, k, H, T) in {"g4": (32, 4, 2, 6, 256, 40), "g8": (64, 8, 3, 8, 512, 33)}.items():
        cfg = GLM4AirConfig()
        cfg.num_experts, cfg.hidden_dim, cfg.experts_per_token = E, H, k
        cfg.n_group, cfg.topk_group = ng, kg
        r = GLM4SigmoidRouter(cfg, 0).float()
        w = synth.host_normal(60 + E, (E, H), 0.05)
        x = synth.host_normal(70 + E, (1, T, H), 1.0)
        with torch.no_grad():
            r.weight.copy_(torch.from_numpy(w))
            idx, wt = r(torch.from_numpy(x))
        out.update({f"{name}/w": w, f"{name}/x": x, f"{name}/idx": idx.numpy(), f"{name}/wt": wt.numpy(),
                    f"{name}/cfg": np.array([E, ng, kg, k, H, T])})
    return out


def store_case(ref: Path):
    """A packed store written by the reference's own test helper
    (``tests/test_int4_loader.py:28-119``: 2 layers x 2 experts, H 256, F 512,
    weights from ``torch.manual_seed(42)``): its index JSON and the SHA-256 of
    its ``experts.bin`` (the bytes themselves are regenerated by the test)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("ref_test_int4_loader", ref / "tests" / "test_int4_loader.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    out = Path(tempfile.mkdtemp(prefix="hnstore_"))
    mod.create_synthetic_packed_store(out, num_layers=2, num_experts=2, hidden_dim=256, intermediate_dim=512)
    data = (out / "experts.bin").read_bytes()
    return {"idx_json": np.array((out / "experts.idx").read_text()),
            "bin_sha256": np.array(hashlib.sha256(data).hexdigest()),
            "bin_size": np.int64(len(data))}


# ---------------------------------------------------------------------------
# 2. MoE layers through the reference (dequant mode, float32)
# ---------------------------------------------------------------------------

def packed_experts(torch, packer, base_seed, shape):
    """Pack every expert with the REFERENCE packer; return numpy tensors + blob hashes."""
    out, hashes = [], []
    for e in range(shape.experts):
        g, u, d = synth.host_expert_weights(base_seed, shape, e)
        pe = packer.pack_expert(0, e, {"gate_proj": torch.from_numpy(g), "up_proj": torch.from_numpy(u),
                                       "down_proj": torch.from_numpy(d)})
        t = [pe.gate_proj_packed.numpy(), pe.gate_proj_scales.numpy(), pe.up_proj_packed.numpy(),
             pe.up_proj_scales.numpy(), pe.down_proj_packed.numpy(), pe.down_proj_scales.numpy()]
        out.append(t)
        hashes.append(sha(*t))
    return out, hashes


def dequant_weights(torch, packer, t, shape):
    H, F = shape.hidden, shape.ffn
    gp, gs, up, us, dp, ds = [torch.from_numpy(a) for a in t]
    return {"gate_proj": packer.dequantize_tensor(gp, gs, F, H).float(),
            "up_proj": packer.dequantize_tensor(up, us, F, H).float(),
            "down_proj": packer.dequantize_tensor(dp, ds, H, F).float()}


def mixtral_layer(ref, torch, base_seed, shape, tokens, affinity_cached=None):
    from hydranet.config import MixtralConfig, ExpertCacheConfig
    from hydranet.cache.expert_cache import ExpertCacheManager
    from hydranet.model.mixtral import MixtralMoELayer
    from hydranet.preprocess.pack_weights import ExpertWeightPacker, QuantConfig

    cfg = MixtralConfig()
    cfg.hidden_dim, cfg.intermediate_dim = shape.hidden, shape.ffn
    cfg.num_experts, cfg.experts_per_token, cfg.num_layers = shape.experts, shape.top_k, 1
    cc = ExpertCacheConfig(pinned_slots=shape.experts, hot_slots=0, probation_slots=0,
                           enable_affinity_bonus=affinity_cached is not None)
    mgr = ExpertCacheManager(cfg, cc, device=torch.device("cpu"), dtype=torch.float32)
    packer = ExpertWeightPacker(QuantConfig(group_size=shape.group_size))
    experts, hashes = packed_experts(torch, packer, base_seed, shape)
    for e, t in enumerate(experts):
        mgr.register_expert(0, e, dequant_weights(torch, packer, t, shape))
    layer = MixtralMoELayer(cfg, cc, 0, mgr)
    rw = synth.host_router_weight(base_seed, shape)
    layer.router.gate.weight.data.copy_(torch.from_numpy(rw))
    if affinity_cached is not None:
        layer.router.set_cache_checker(lambda i: i in affinity_cached)
    x = synth.host_activations(base_seed, tokens, shape.hidden)
    with torch.no_grad():
        h = torch.from_numpy(x).view(1, tokens, shape.hidden)
        ro = layer.router(h, top_k_override=shape.top_k)
        layer.router.reset_usage()
        out = layer(h, top_k=shape.top_k)
    mgr.shutdown()
    return {
        "x": x, "router_w": rw, "expert_sha256": np.array(hashes),
        "idx": ro.expert_indices.view(tokens, -1).numpy(),
        "weights": ro.expert_weights.view(tokens, -1).float().numpy(),
        "logits": ro.router_logits.view(tokens, -1).numpy(),
        "out": out.view(tokens, -1).numpy(),
        "dims": np.array([shape.hidden, shape.ffn, shape.experts, shape.top_k, shape.group_size, tokens, base_seed]),
        "affinity_cached": np.array(sorted(affinity_cached) if affinity_cached else [], dtype=np.int64),
    }


def glm_layer(ref, torch, base_seed, shape, tokens):
    """Routed part of GLM4MoELayer (shared expert zeroed so the output is the routed sum)."""
    from hydranet.config import GLM4AirConfig, ExpertCacheConfig
    from hydranet.cache.expert_cache import ExpertCacheManager
    from hydranet.model.glm4 import GLM4MoELayer
    from hydranet.preprocess.pack_weights import ExpertWeightPacker, QuantConfig
    from dataclasses import dataclass

    cfg = GLM4AirConfig()
    cfg.hidden_dim, cfg.moe_intermediate_dim = shape.hidden, shape.ffn
    cfg.num_experts, cfg.experts_per_token = shape.experts, shape.top_k

    @dataclass
    class Adapter:
        num_layers: int
        num_experts: int
        expert_size_bytes: int

    cc = ExpertCacheConfig(pinned_slots=shape.experts, hot_slots=0, probation_slots=0)
    mgr = ExpertCacheManager(Adapter(1, shape.experts, 3 * shape.hidden * shape.ffn * 2), cc,
                             device=torch.device("cpu"), dtype=torch.float32)
    packer = ExpertWeightPacker(QuantConfig(group_size=shape.group_size))
    experts, hashes = packed_experts(torch, packer, base_seed, shape)
    for e, t in enumerate(experts):
        mgr.register_expert(0, e, dequant_weights(torch, packer, t, shape))
    layer = GLM4MoELayer(cfg, 0, mgr)
    rw = synth.host_router_weight(base_seed, shape)
    with torch.no_grad():
        layer.router.weight.copy_(torch.from_numpy(rw))
        for p in layer.shared_expert.parameters():
            p.zero_()
    x = synth.host_activations(base_seed, tokens, shape.hidden)
    with torch.no_grad():
        h = torch.from_numpy(x).view(1, tokens, shape.hidden)
        idx, w = layer.router(h)
        out = layer(h)
    mgr.shutdown()
    return {
        "x": x, "router_w": rw, "expert_sha256": np.array(hashes),
        "idx": idx.numpy(), "weights": w.float().numpy(), "out": out.view(tokens, -1).numpy(),
        "dims": np.array([shape.hidden, shape.ffn, shape.experts, shape.top_k, shape.group_size, tokens, base_seed]),
    }


# ---------------------------------------------------------------------------
# 3. Routers at full model width, including bf16 activations
# ---------------------------------------------------------------------------

def mixtral_router_bf16(torch, base_seed, shape, tokens):
    from hydranet.config import MixtralConfig, ExpertCacheConfig
    from hydranet.model.router import TopKRouter
    cfg = MixtralConfig()
    cfg.hidden_dim, cfg.num_experts = shape.hidden, shape.experts
    r = TopKRouter(cfg, ExpertCacheConfig(enable_affinity_bonus=False), 0).to(torch.bfloat16)
    rw = synth.host_router_weight(base_seed, shape)
    x = synth.host_activations(base_seed, tokens, shape.hidden)
    with torch.no_grad():
        r.gate.weight.copy_(torch.from_numpy(rw).to(torch.bfloat16))
        o = r(torch.from_numpy(x).to(torch.bfloat16).view(1, tokens, -1), top_k_override=shape.top_k)
    return {"idx": o.expert_indices.view(tokens, -1).numpy(),
            "weights": o.expert_weights.view(tokens, -1).float().numpy(),
            "logits": o.router_logits.view(tokens, -1).numpy(),
            "dims": np.array([shape.hidden, shape.experts, shape.top_k, tokens, base_seed])}


def glm_router(torch, base_seed, shape, tokens, dtype):
    from hydranet.config import GLM4AirConfig
    from hydranet.model.glm4 import GLM4SigmoidRouter
    cfg = GLM4AirConfig()
    cfg.hidden_dim, cfg.num_experts, cfg.experts_per_token = shape.hidden, shape.experts, shape.top_k
    r = GLM4SigmoidRouter(cfg, 0)
    rw = synth.host_router_weight(base_seed, shape)
    x = synth.host_activations(base_seed, tokens, shape.hidden)
    tdt = {"f32": torch.float32, "bf16": torch.bfloat16}[dtype]
    with torch.no_grad():
        r.weight.copy_(torch.from_numpy(rw))
        idx, w = r(torch.from_numpy(x).to(tdt).view(1, tokens, -1))
    return {"idx": idx.numpy(), "weights": w.float().numpy(),
            "dims": np.array([shape.hidden, shape.experts, shape.top_k, tokens, base_seed])}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--only", default=None, help="write only this fixture (file stem)")
    args = ap.parse_args()
    ref = import_reference(args.reference.resolve())
    import torch
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    from hydranet.kernels.int4_linear import Int4Linear
    from hydranet.scheduler.continuous_batch import GroupByExpertGatherer
    light = {"int4linear_quant": lambda: int4linear_cases(torch, Int4Linear),
             "gatherer": lambda: gatherer_cases(torch, GroupByExpertGatherer),
             "reference_store": lambda: store_case(args.reference.resolve()),
             "scheduler_trace": lambda: scheduler_trace(torch),
             "glm4_dense": lambda: glm4_dense_cases(torch),
             "glm_group_router": lambda: glm_group_router_cases(torch)}
    for stem, make in light.items():
        if args.only in (None, stem):
            np.savez_compressed(HERE / f"{stem}.npz", **make())
    if args.only in light:
        return
    from hydranet.preprocess.pack_weights import ExpertWeightPacker, QuantConfig

    np.savez_compressed(HERE / "pack_cases.npz", **pack_cases(torch, ExpertWeightPacker, QuantConfig))

    c1 = synth.MoEShape(hidden=512, ffn=1024, experts=8, top_k=2)
    np.savez_compressed(HERE / "c1_mixtral_layer.npz", **mixtral_layer(ref, torch, 0, c1, 4))
    np.savez_compressed(HERE / "c1_mixtral_layer_affinity.npz",
                        **mixtral_layer(ref, torch, 0, c1, 4, affinity_cached={0, 3, 5}))
    c2s = synth.MoEShape(hidden=1024, ffn=2048, experts=8, top_k=2)
    np.savez_compressed(HERE / "c2_small_mixtral_layer.npz", **mixtral_layer(ref, torch, 2, c2s, 16))
    g = synth.MoEShape(hidden=512, ffn=256, experts=16, top_k=4)
    np.savez_compressed(HERE / "glm_small_layer.npz", **glm_layer(ref, torch, 4, g, 8))

    mix_full = synth.MoEShape(hidden=4096, ffn=14336, experts=8, top_k=2)
    np.savez_compressed(HERE / "mixtral_router_bf16.npz", **mixtral_router_bf16(torch, 5, mix_full, 64))
    glm_full = synth.MoEShape(hidden=4096, ffn=1408, experts=128, top_k=8)
    np.savez_compressed(HERE / "glm_router_f32.npz", **glm_router(torch, 6, glm_full, 32, "f32"))
    np.savez_compressed(HERE / "glm_router_bf16.npz", **glm_router(torch, 7, glm_full, 32, "bf16"))
    for f in sorted(HERE.glob("*.npz")):
        print(f"{f.name}: {f.stat().st_size} bytes")


if __name__ == "__main__":
    main()
