"""Continuous batching on CPU: the scheduler's behaviour against a trace
recorded from the reference (``scheduler/continuous_batch.py``, fixture made
by ``tests/golden/make_golden.py``), and the runner's bookkeeping -- chunked
prefill, decode positions fed back, one call per layer per step over the
mixed batch -- with a token-wise test layer on CPU tensors."""

from pathlib import Path

import numpy as np
import pytest
import torch

from hydranet_b200 import batching
from tests.golden import scheduler_script

GOLDEN = Path(__file__).resolve().parent / "golden" / "scheduler_trace.npz"


def test_scheduler_trace_matches_reference():
    want = [str(x) for x in np.load(GOLDEN)["lines"]]
    got = scheduler_script.run(batching, torch)
    assert got == want


class CountingLayer(torch.nn.Module):
    """Token-wise stand-in for an MoE layer: y = tanh(x @ W) + x, counting calls."""

    def __init__(self, H, seed):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.W = torch.randn(H, H, generator=g) / H ** 0.5
        self.calls, self.rows = 0, []

    def forward(self, x):
        self.calls += 1
        self.rows.append(x.shape[0])
        return (torch.tanh(x.float() @ self.W) + x.float()).to(x.dtype)


def make_requests(H, specs, seed=0):
    g = torch.Generator().manual_seed(seed)
    reqs = []
    for i, (L, m) in enumerate(specs):
        r = batching.Request(f"q{i}", torch.arange(L), max_tokens=m)
        r.prompt_hidden = torch.randn(L, H, generator=g).to(torch.float32)
        reqs.append(r)
    return reqs


def test_runner_chunked_prefill_and_decode_cpu():
    H = 16
    layers = [CountingLayer(H, 1), CountingLayer(H, 2)]
    b = batching.ContinuousBatcher(max_batch_size=3, max_queue_size=8)
    reqs = make_requests(H, [(5, 3), (11, 2), (1, 4), (7, 0)])
    for r in reqs:
        assert b.submit(r)
    run = batching.MoEBatchRunner(layers, b, H, prefill_chunk=4, device="cpu", dtype=torch.float32,
                                  keep_inputs=True)
    steps = run.run()
    assert steps == len(run.records) and steps > 0
    assert all(r.state == batching.RequestState.COMPLETED for r in reqs)
    # one call per layer per step, over all rows of the step
    for layer in layers:
        assert layer.calls == steps
        assert layer.rows == [rec.rows for rec in run.records]
    # some step mixed prefill chunks and decode tokens of different requests
    assert any(rec.prefill_rows and rec.decode_rows for rec in run.records)
    assert max(rec.rows for rec in run.records) <= 3 * 4
    for r in reqs:
        L = r.prompt_hidden.shape[0]
        assert len(r.outputs) == L + r.max_tokens and len(r.generated_ids) == r.max_tokens
        # the inputs are the prompt, then each output fed back
        assert torch.equal(torch.stack(r.inputs[:L]), r.prompt_hidden)
        for j in range(L, L + r.max_tokens):
            assert torch.equal(r.inputs[j], batching.rms_feedback(r.outputs[j - 1]))
        # token-wise layers: the batch composition does not change a row's result
        x = torch.stack(r.inputs)
        for layer in layers:
            x = layer(x)
        assert torch.allclose(torch.stack(r.outputs), x, atol=1e-5, rtol=1e-5)
    # positions of each request are contiguous and in order across steps
    for r in reqs:
        pos = [(first, m) for rec in run.records for rid, first, m in rec.parts if rid == r.request_id]
        nxt = 0
        for first, m in pos:
            assert first == nxt
            nxt += m


def test_runner_refuses_bad_chunk_and_empty_prompt():
    b = batching.ContinuousBatcher()
    with pytest.raises(ValueError):
        batching.MoEBatchRunner([], b, 8, prefill_chunk=0, device="cpu")
    r = batching.Request("e", torch.arange(0), max_tokens=1)
    r.prompt_hidden = torch.zeros(0, 8)
    b.submit(r)
    run = batching.MoEBatchRunner([], b, 8, device="cpu", dtype=torch.float32)
    with pytest.raises(ValueError):
        run.step()
