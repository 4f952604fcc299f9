"""Tensor parallelism of GLM-4.5's dense parts on CPU ranks (gloo, world
sizes 2 and 4): every rank's output equals the oracle's restatement of the
reference modules (``oracle/glm4_dense_ref.py``, pinned to outputs recorded
from the reference's own ``GLM4Attention`` / ``GLM4DenseMLP``), for prefill,
a decode step through the per-rank KV cache, the dense MLP and the
vocabulary-parallel lm_head.  World size 4 with 2 KV heads replicates each KV
head on two ranks."""

import os
import socket
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import glm4_dense_ref as G

GOLDEN = Path(__file__).resolve().parent / "golden" / "glm4_dense.npz"


def test_oracle_matches_reference_outputs():
    d = dict(np.load(GOLDEN))
    x = d["x"][0]
    a = lambda n: d["attn/" + n]  # noqa: E731
    args = (a("q_proj.weight"), a("q_proj.bias"), a("k_proj.weight"), a("k_proj.bias"), a("v_proj.weight"),
            a("v_proj.bias"), a("o_proj.weight"), 8, 2, 32)
    o, k, v = G.attention_ref(x[:5], *args, np.arange(5))
    np.testing.assert_allclose(o, d["attn_prefill"][0], atol=2e-6)
    o2, _, _ = G.attention_ref(x[5:6], *args, np.arange(5, 6), past_k=k, past_v=v)
    np.testing.assert_allclose(o2, d["attn_decode"][0], atol=2e-6)
    m = lambda n: d["mlp/" + n]  # noqa: E731
    np.testing.assert_allclose(G.dense_mlp_ref(x, m("gate_proj.weight"), m("up_proj.weight"), m("down_proj.weight")),
                               d["mlp"][0], atol=2e-6)
    np.testing.assert_allclose(G.lm_head_ref(x, d["lm_w"]), d["lm"][0], atol=2e-6)


class _Cfg:
    partial_rotary_factor, rope_theta, max_position_embeddings = 0.5, 1e6, 64


def full_modules(d):
    """Reference-layout float32 modules holding the fixture's weights."""
    attn = torch.nn.Module()
    attn.num_heads, attn.num_kv_heads, attn.head_dim, attn.layer_idx, attn.config = 8, 2, 32, 0, _Cfg()
    for n, (o, i, b) in {"q_proj": (256, 256, True), "k_proj": (64, 256, True), "v_proj": (64, 256, True),
                         "o_proj": (256, 256, False)}.items():
        lin = torch.nn.Linear(i, o, bias=b)
        with torch.no_grad():
            lin.weight.copy_(torch.from_numpy(d[f"attn/{n}.weight"]))
            if b:
                lin.bias.copy_(torch.from_numpy(d[f"attn/{n}.bias"]))
        setattr(attn, n, lin)
    mlp = torch.nn.Module()
    for n, (o, i) in {"gate_proj": (192, 256), "up_proj": (192, 256), "down_proj": (256, 192)}.items():
        lin = torch.nn.Linear(i, o, bias=False)
        with torch.no_grad():
            lin.weight.copy_(torch.from_numpy(d[f"mlp/{n}.weight"]))
        setattr(mlp, n, lin)
    lm = torch.nn.Linear(256, 96, bias=False)
    with torch.no_grad():
        lm.weight.copy_(torch.from_numpy(d["lm_w"]))
    return attn, mlp, lm


def worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from hydranet_b200.tp import TPAttention, TPDenseMLP, TPKVCache, VocabParallelLMHead
        d = dict(np.load(GOLDEN))
        attn, mlp, lm = full_modules(d)
        tpa, tpm, tpl = TPAttention.from_module(attn), TPDenseMLP.from_module(mlp), VocabParallelLMHead.from_linear(lm)
        x = torch.from_numpy(d["x"])
        cache = TPKVCache(1, tpa.n_kv_local, 32, max_seq_len=16, device="cpu", dtype=torch.float32)
        with torch.no_grad():
            pre = tpa(x[:, :5], torch.arange(5).view(1, 5), kv_cache=cache)
            cache.set_len(5)
            dec = tpa(x[:, 5:6], torch.tensor([[5]]), kv_cache=cache)
            full = tpa(x, torch.arange(6).view(1, 6))
            y = tpm(x)
            logits = tpl(x)
        errs = {
            "prefill": np.abs(pre.numpy() - d["attn_prefill"]).max(),
            "decode": np.abs(dec.numpy() - d["attn_decode"]).max(),
            "nocache": np.abs(full.numpy() - d["attn_nocache"]).max(),
            "mlp": np.abs(y.numpy() - d["mlp"]).max(),
            "lm": np.abs(logits.numpy() - d["lm"]).max(),
        }
        results[rank] = {k: float(v) for k, v in errs.items()}
    finally:
        dist.destroy_process_group()


def run(world):
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    procs = [ctx.Process(target=worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    return [results[r] for r in range(world)]


@pytest.mark.parametrize("world", [2, 4])
def test_tp_dense_parts_match_reference(world):
    for errs in run(world):
        for k, v in errs.items():
            assert v < 1e-5, (world, k, v)


def test_tp_refuses_uneven_splits():
    from hydranet_b200 import tp
    with pytest.raises(ValueError):
        tp._split(10, 4, 0, "features")
