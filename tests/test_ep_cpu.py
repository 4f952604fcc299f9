"""Expert-parallel dispatch/combine bookkeeping on CPU ranks (gloo, world sizes 2 and 4; Mixtral and GLM-4.5 routing).

Each rank routes its own tokens with the oracle router, exchanges rows with
``hydranet_b200.ep.ep_moe_forward`` (one row per token and destination rank,
the token's picks rewritten as that rank's local ids) and runs its share of
the experts with a test-only local function built from the oracle; the pack,
unpack and combine steps use the torch reference of the CUDA kernels
(``tests/ep_ref.py``).  The result must equal the single-process oracle layer
(``model/mixtral.py:282-370`` semantics) on that rank's tokens.  No GPU is
involved.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hydranet_b200 import synth
from oracle import int4_ref as R
from tests.ep_ref import TorchExchange

H, F, E, K = 256, 256, 8, 3
GLM = dict(E=16, K=8, router="sigmoid")  # GLM-4.5 layout at a small size


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def experts_oracle(n_exp=E, k=K):
    shape = synth.MoEShape(H, F, n_exp, k)
    out = {}
    for e in range(n_exp):
        g, u, d = synth.host_expert_weights(7, shape, e)
        out[e] = R.DequantExpert.from_packed(*R.quantize_tensor(g), *R.quantize_tensor(u), *R.quantize_tensor(d))
    return out


def worker(rank, world, port, T, force_idx, results, n_exp=E, k=K, router="softmax", chunk=None):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from hydranet_b200.ep import ep_moe_forward, ep_moe_forward_chunked, expert_range
        experts = experts_oracle(n_exp, k)
        first, last = expert_range(n_exp, rank, world)
        x = synth.host_activations(100 + rank, T, H)
        rw = synth.host_normal(5, (n_exp, H), 0.02)
        if router == "sigmoid":
            idx, w, _ = R.sigmoid_topk_router_ref(x, rw, k, "f32", correction_bias=synth.host_correction_bias(3, n_exp))
        else:
            idx, w, _ = R.softmax_topk_router_ref(x, rw, k, "f32")
        if force_idx is not None:
            idx = force_idx[rank].copy()
        def local_fn(rows, ids, weight):
            rr = rows.numpy().astype(np.float32)
            out = np.zeros_like(rr)
            for i in range(rr.shape[0]):
                for j in range(ids.shape[1]):
                    if int(ids[i, j]) < 0:
                        continue  # a pick owned by another rank (or an unused row)
                    e = first + int(ids[i, j])
                    assert first <= e < last
                    out[i] += float(weight[i, j]) * experts[e](rr[i:i + 1])[0]
            return torch.from_numpy(out)
        args = (torch.from_numpy(x), torch.from_numpy(idx.astype(np.int32)), torch.from_numpy(w), n_exp, local_fn)
        if chunk is None:
            y = ep_moe_forward(*args, exchange=TorchExchange())
        else:
            y = ep_moe_forward_chunked(*args, chunk, exchange=TorchExchange())
        ref = R.moe_combine_ref(x, idx, w, experts)
        err = float(np.abs(y.numpy() - ref).max() / max(np.abs(ref).max(), 1e-30))
        results[rank] = err
    finally:
        dist.destroy_process_group()


def run(world, T, force_idx=None, **layout):
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, T, force_idx, results),
                         kwargs={"n_exp": layout.get("E", E), "k": layout.get("K", K),
                                 "router": layout.get("router", "softmax"), "chunk": layout.get("chunk")})
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    return [results[r] for r in range(world)]


def test_ep_matches_single_process_oracle():
    errs = run(2, 9)
    assert max(errs) < 1e-5, errs


def test_ep_uneven_and_empty_splits_and_duplicates():
    # rank 0 sends everything to rank 1's experts (nothing to itself), picks an
    # expert twice; rank 1 keeps everything local
    f0 = np.array([[5, 5, 7], [6, 4, 5], [7, 7, 7]], dtype=np.int64)
    f1 = np.array([[0, 1, 2], [3, 3, 0], [1, 2, 3]], dtype=np.int64)
    errs = run(2, 3, force_idx={0: f0, 1: f1})
    assert max(errs) < 1e-5, errs


def test_ep_four_ranks():
    """Four ranks, two experts each (the layout of the 4-GPU bench run);
    token counts differ per rank only through routing, as in the bench."""
    errs = run(4, 6)
    assert max(errs) < 1e-5, errs


def test_ep_glm_layout_four_ranks():
    """Sigmoid top-8 with a correction bias over 16 experts, 4 experts per
    rank: every token reaches several ranks, some more than once."""
    errs = run(4, 5, **GLM)
    assert max(errs) < 1e-5, errs


def test_ep_chunked_micro_batches():
    """Prefill-size path: 11 tokens per rank in micro-batches of 4 (the last
    one ragged), asynchronous all-to-alls, GLM routing over 2 ranks."""
    errs = run(2, 11, chunk=4, **GLM)
    assert max(errs) < 1e-5, errs


def test_expert_range_partition():
    from hydranet_b200.ep import expert_range
    assert [expert_range(128, r, 8) for r in range(8)][3] == (48, 64)
    with pytest.raises(ValueError):
        expert_range(10, 0, 4)
