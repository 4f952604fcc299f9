"""Expert-parallel exchange kernels on one GPU, with W ranks emulated in one process.

Each emulated rank routes its own 32 tokens (GLM-4.5-Air layer: 128 experts,
sigmoid top-8 with correction bias); ``hn_ep_pack`` builds its send buffer,
the all-to-all is a block transpose between the emulated ranks' buffers,
``hn_ep_unpack`` and the grouped kernel run each rank's 128/W experts, the
mirror transpose returns the rows and ``hn_ep_combine`` sums them.  Every
rank's output must match the single-GPU layer holding all 128 experts; the
packed bytes must equal the torch reference of the exchange
(``tests/ep_ref.py``) wherever the contract defines them.
"""

import numpy as np
import pytest
import torch

from hydranet_b200 import synth
from hydranet_b200.ep import CudaExchange, cuda_local_fn
from hydranet_b200.moe import MoELayerInt4
from hydranet_b200.packing import ExpertTable
from hydranet_b200.router import GLM4SigmoidRouter
from tests.ep_ref import TorchExchange
from tests.gpu_util import rel_l2, to_np32

pytestmark = pytest.mark.gpu

H, F, E, K, T = 4096, 1408, 128, 8, 32
_STATE = {}


def _setup():
    if "s" not in _STATE:
        dev = torch.device("cuda")
        slots = synth.device_experts(21, synth.MoEShape(H, F, E, K), dev)
        router = GLM4SigmoidRouter(hidden_dim=H, num_experts=E, experts_per_token=K).to(dev)
        router.set_correction_bias(torch.from_numpy(synth.host_correction_bias(3, E)).to(dev))
        _STATE["s"] = (slots, router, MoELayerInt4(router, ExpertTable(slots)))
    return _STATE["s"]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_emulated_ranks_match_single_gpu_layer(lib, world):
    from hydranet_b200 import ops
    slots, router, full = _setup()
    per = E // world
    ex = CudaExchange()
    xs, idxs, ws, sends = [], [], [], []
    for r in range(world):
        x = torch.randn(T, H, generator=torch.Generator("cuda").manual_seed(100 + r), device="cuda").to(torch.bfloat16)
        idx, w, _ = ops.moe_route(x, router.params(), E, want_logits=False)
        xs.append(x), idxs.append(idx), ws.append(w), sends.append(ex.pack(x, idx, w, E, world))
    # the all-to-all: rank d receives block d of every rank's send buffer, in rank order
    recvs = [torch.cat([sends[r][d * T:(d + 1) * T] for r in range(world)]) for d in range(world)]
    ys = []
    for d in range(world):
        rows, ids, wts = ex.unpack(recvs[d], H, K, torch.bfloat16)
        # the local call is told that about 1/world of the slots are this rank's
        ys.append(cuda_local_fn(ExpertTable(slots[d * per:(d + 1) * per]), world)(rows, ids, wts))
    for r in range(world):
        back = torch.stack([ys[d][r * T:(r + 1) * T] for d in range(world)])
        out = ex.combine(back, idxs[r], E, world)
        with torch.no_grad():
            ref = full(xs[r])
        err = rel_l2(to_np32(out), to_np32(ref))
        assert err <= 1e-2, (r, err)
        # the bytes the contract defines match the torch reference of the exchange
        tref = TorchExchange().pack(xs[r].cpu(), idxs[r].cpu(), ws[r].cpu(), E, world).view(world, T, -1)
        got = sends[r].cpu().view(world, T, -1)
        xb = H * 2
        assert torch.equal(got[:, :, xb:xb + 8 * K], tref[:, :, xb:xb + 8 * K])
        used = (tref[:, :, xb:xb + 4 * K].contiguous().view(torch.int32) >= 0).any(-1)
        assert torch.equal(got[:, :, :xb][used], tref[:, :, :xb][used])
