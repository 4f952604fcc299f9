"""Group-by-expert gather/scatter (``scheduler/continuous_batch.py:266-381``)
against fixtures recorded from the reference's own ``GroupByExpertGatherer``
(``tests/golden/make_golden.py``): the same experts in the same order, the
same (token, weight, row) lists, and a bit-identical scatter on CPU, including
tokens that pick an expert twice and an expert no token picks.
"""

import numpy as np
import pytest
import torch

from hydranet_b200.gather import GatheredTokens, GroupByExpertGatherer


@pytest.fixture(scope="module")
def golden(golden_dir):
    z = np.load(golden_dir / "gatherer.npz")
    return {k: z[k] for k in z.files}


@pytest.mark.parametrize("case", ["f32", "f32_dup", "f16"])
def test_gather_scatter_match_reference(golden, case):
    g = {k.split("/", 1)[1]: v for k, v in golden.items() if k.startswith(case + "/")}
    dt = getattr(torch, str(g["dtype"]))
    T, H = g["hidden"].shape
    hid = torch.from_numpy(g["hidden"]).to(dt)
    w = torch.from_numpy(g["w"]).to(dt)
    gat = GroupByExpertGatherer(device=torch.device("cpu"))
    got = gat.gather(hid, torch.from_numpy(g["idx"]), w, 5)
    assert all(isinstance(x, GatheredTokens) for x in got)
    assert [x.expert_idx for x in got] == g["experts"].tolist()
    assert 2 not in g["experts"].tolist()
    assert [x.num_tokens for x in got] == g["counts"].tolist()
    assert [x.layer_idx for x in got] == g["layer"].tolist()
    assert all(x.token_indices.dtype == torch.int64 for x in got)
    assert np.array_equal(torch.cat([x.token_indices for x in got]).numpy(), g["tokens"])
    assert np.array_equal(torch.cat([x.routing_weights for x in got]).float().numpy(), g["weights"])
    assert np.array_equal(torch.cat([x.hidden_states for x in got]).float().numpy(), g["rows"])
    outs = [(x, x.hidden_states * (x.expert_idx + 1) - x.expert_idx) for x in got]
    y = gat.scatter(outs, (T, H))
    assert str(y.dtype) == str(g["scatter_dtype"])
    assert np.array_equal(y.float().numpy(), g["scatter"])


def test_duplicate_picks_listed_twice(golden):
    idx = golden["f32_dup/idx"]
    dup_tokens = [t for t in range(idx.shape[0]) if len(set(idx[t].tolist())) < idx.shape[1]]
    assert dup_tokens
    gat = GroupByExpertGatherer(device=torch.device("cpu"))
    got = gat.gather(torch.from_numpy(golden["f32_dup/hidden"]), torch.from_numpy(idx),
                     torch.from_numpy(golden["f32_dup/w"]), 0)
    t = dup_tokens[0]
    e = int(idx[t, 0])
    lst = next(x for x in got if x.expert_idx == e).token_indices.tolist()
    assert lst.count(t) == list(idx[t]).count(e)


def test_scatter_of_nothing():
    y = GroupByExpertGatherer(device=torch.device("cpu")).scatter([], (4, 8))
    assert y.dtype == torch.float16 and y.shape == (4, 8) and not y.any()
