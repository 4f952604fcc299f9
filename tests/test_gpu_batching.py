"""Continuous batching on the GPU: requests at different stages share each
step's grouped-kernel call (chunked prefill beside decode tokens), and every
request's outputs match the oracle layer on that request's own inputs."""

import numpy as np
import pytest
import torch

from hydranet_b200 import batching, synth
from oracle import int4_ref as R
from tests.gpu_util import host_moe, oracle_experts, rel_l2, to_np32
from tests.test_gpu_moe import check_indices, mixtral_layer

pytestmark = pytest.mark.gpu


class Counted(torch.nn.Module):
    def __init__(self, inner):
        super().__init__()
        self.inner, self.calls = inner, 0

    def forward(self, x):
        self.calls += 1
        return self.inner(x)


def test_mixed_prefill_decode_batches_match_oracle(lib):
    H, F, E, K = 512, 1024, 8, 2
    shape = synth.MoEShape(H, F, E, K)
    table, packed = host_moe(shape, 3)
    rw = (torch.randn(E, H, generator=torch.Generator("cuda").manual_seed(8), device="cuda") * 0.02).to(torch.bfloat16)
    layer = Counted(mixtral_layer(table, rw, K))
    b = batching.ContinuousBatcher(max_batch_size=4, max_queue_size=16)
    g = torch.Generator().manual_seed(2)
    reqs = []
    for i, (L, m) in enumerate([(37, 3), (5, 6), (1, 2), (64, 1), (20, 4), (9, 0)]):
        r = batching.Request(f"q{i}", torch.arange(L), max_tokens=m)
        r.prompt_hidden = torch.randn(L, H, generator=g).to(torch.bfloat16)
        reqs.append(r)
        assert b.submit(r)
    run = batching.MoEBatchRunner([layer], b, H, prefill_chunk=16, keep_inputs=True)
    steps = run.run()
    assert layer.calls == steps
    assert any(rec.prefill_rows and rec.decode_rows for rec in run.records)
    assert all(r.state == batching.RequestState.COMPLETED for r in reqs)
    experts = oracle_experts(packed)
    wi = to_np32(rw)
    for r in reqs:
        x = torch.stack(r.inputs).cuda()
        assert x.shape[0] == r.prompt_hidden.shape[0] + r.max_tokens
        with torch.no_grad():
            _, ro = layer.inner(x, return_routing=True)
        xi = to_np32(x)
        idx, w, logits = R.softmax_topk_router_ref(xi, wi, K, "bf16")
        n_tie = check_indices(ro.expert_indices.cpu().numpy(), idx, logits, K, 2 ** -8)
        use_idx = ro.expert_indices.cpu().numpy() if n_tie else idx
        use_w = to_np32(ro.expert_weights) if n_tie else w
        ref = R.moe_combine_ref(xi, use_idx, use_w, experts)
        got = to_np32(torch.stack(r.outputs))
        assert rel_l2(got, ref) <= 6e-3, r.request_id
