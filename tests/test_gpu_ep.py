"""Expert parallelism on 2 GPUs over NCCL (skipped with fewer GPUs).

Runs as two child processes so a failing rank cannot leave the pytest process
holding a communicator; NVLS is off (peer traffic only) and the process
group has a short timeout.  Each rank's output must match the single-GPU
grouped layer computed with all experts on that rank's tokens.
"""

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parent.parent

CHILD = r'''
import os, sys, torch, torch.distributed as dist
from datetime import timedelta
sys.path.insert(0, os.environ["REPO"])
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dev = torch.device("cuda", rank)
dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=60))
from hydranet_b200 import synth
from hydranet_b200.packing import ExpertTable
from hydranet_b200.router import GLM4SigmoidRouter
from hydranet_b200.moe import MoELayerInt4
from hydranet_b200.ep import ExpertParallelMoE
H, F, E, K, T = 1024, 256, 16, 4, 24
shape = synth.MoEShape(H, F, E, K)
slots = synth.device_experts(7, shape, dev)           # every rank builds all experts (same seed)
per = E // world
router = GLM4SigmoidRouter(hidden_dim=H, num_experts=E, experts_per_token=K).to(dev)
with torch.no_grad():
    router.weight.copy_(torch.randn(E, H, generator=torch.Generator(dev).manual_seed(3), device=dev) * 0.02)
ep = ExpertParallelMoE(router, ExpertTable(slots[rank * per:(rank + 1) * per]), E)
full = MoELayerInt4(router, ExpertTable(slots))
x = torch.randn(T, H, generator=torch.Generator(dev).manual_seed(11 + rank), device=dev).to(torch.bfloat16)
# micro-batched path (prefill): 40 tokens in chunks of 16, the last one ragged
ep_mb = ExpertParallelMoE(router, ExpertTable(slots[rank * per:(rank + 1) * per]), E, chunk_tokens=16)
x2 = torch.randn(40, H, generator=torch.Generator(dev).manual_seed(21 + rank), device=dev).to(torch.bfloat16)
with torch.no_grad():
    y = ep(x)
    ref = full(x)
    y2 = ep_mb(x2)
    ref2 = full(x2)
err = ((y.float() - ref.float()).norm() / ref.float().norm()).item()
err2 = ((y2.float() - ref2.float()).norm() / ref2.float().norm()).item()
dist.destroy_process_group()
print(f"rank {rank} rel_l2 {err:.3e} chunked {err2:.3e}")
sys.exit(0 if max(err, err2) < 1e-2 else 3)
'''


def test_ep_two_gpus_matches_single_gpu_layer():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    env = dict(os.environ, REPO=str(REPO), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE="2",
               NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, "-c", CHILD], env=dict(env, RANK=str(r), LOCAL_RANK=str(r)),
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True) for r in range(2)]
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=240)
        except subprocess.TimeoutExpired:
            p.kill()
            out, _ = p.communicate()
        outs.append(out)
    for p, out in zip(procs, outs):
        assert p.returncode == 0, out[-2000:]
