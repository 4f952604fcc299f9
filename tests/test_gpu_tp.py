"""Tensor parallelism on the GPU.

* INT4 shards (``Int4Linear`` weights split by rows for column-parallel and
  by 128-column groups for row-parallel) run on ``hn_int4_linear`` and add up
  to the full layer, on one GPU with the ranks emulated;
* on 2 GPUs over NCCL (child processes, NVLS off, short process-group
  timeout; skipped with fewer GPUs): attention and the dense MLP split by
  ``TPAttention`` / ``TPDenseMLP`` match the full modules."""

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from hydranet_b200 import tp
from hydranet_b200.kernels.int4_linear import Int4Linear

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parent.parent


@pytest.mark.parametrize("world", [2, 4])
def test_int4_shards_add_up(lib, monkeypatch, world):
    g = torch.Generator().manual_seed(world)
    full = torch.nn.Linear(1024, 512, bias=False)
    with torch.no_grad():
        full.weight.copy_(torch.randn(512, 1024, generator=g) * 0.02)
    q = Int4Linear.from_float(full, group_size=128).cuda()
    x = torch.randn(6, 1024, generator=g).cuda().to(torch.float16)
    want = q(x).float()
    cols, rows = [], torch.zeros_like(want)
    for r in range(world):
        monkeypatch.setattr(tp, "_world", lambda group, r=r: (world, r))
        c = tp.ColumnParallelLinear.from_linear(q)
        cols.append(c(x).float())
        rp = tp.RowParallelLinear.from_linear(q, input_is_parallel=False, reduce=False)
        rows += rp(x).float()
    # row slices and K slices: the same products, summed in another order
    assert ((torch.cat(cols, dim=-1) - want).norm() / want.norm()).item() < 1e-3
    assert ((rows - want).norm() / want.norm()).item() < 2e-3


CHILD = r'''
import os, sys, torch, torch.distributed as dist
from datetime import timedelta
sys.path.insert(0, os.environ["REPO"])
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dev = torch.device("cuda", rank)
dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=60))
from hydranet_b200.tp import TPAttention, TPDenseMLP
torch.manual_seed(0)
H, NH, NKV, HD, FF = 1024, 16, 2, 64, 2048
class Cfg: partial_rotary_factor, rope_theta, max_position_embeddings = 0.5, 1e6, 256
attn = torch.nn.Module()
attn.num_heads, attn.num_kv_heads, attn.head_dim, attn.layer_idx, attn.config = NH, NKV, HD, 0, Cfg()
attn.q_proj = torch.nn.Linear(H, NH * HD, bias=True)
attn.k_proj = torch.nn.Linear(H, NKV * HD, bias=True)
attn.v_proj = torch.nn.Linear(H, NKV * HD, bias=True)
attn.o_proj = torch.nn.Linear(NH * HD, H, bias=False)
mlp = torch.nn.Module()
mlp.gate_proj, mlp.up_proj, mlp.down_proj = (torch.nn.Linear(H, FF, bias=False), torch.nn.Linear(H, FF, bias=False),
                                             torch.nn.Linear(FF, H, bias=False))
for m in (attn, mlp):
    for p in m.parameters():
        torch.nn.init.normal_(p, std=0.02)
    m.to(dev, torch.bfloat16)
x = torch.randn(2, 40, H, generator=torch.Generator().manual_seed(3)).to(dev, torch.bfloat16)
pos = torch.arange(40, device=dev).view(1, 40).expand(2, 40)
tpa, tpm = TPAttention.from_module(attn), TPDenseMLP.from_module(mlp)
# the full modules, computed the reference's way on every rank
def full_attention(x):
    B, S, _ = x.shape
    q = attn.q_proj(x).view(B, S, NH, HD).transpose(1, 2)
    k = attn.k_proj(x).view(B, S, NKV, HD).transpose(1, 2)
    v = attn.v_proj(x).view(B, S, NKV, HD).transpose(1, 2)
    rd = HD // 2
    inv = 1.0 / (1e6 ** (torch.arange(0, rd, 2, device=dev).float() / rd))
    f = torch.outer(torch.arange(256, device=dev).float(), inv)
    emb = torch.cat([f, f], -1)
    cos, sin = emb.cos()[pos].to(v.dtype).unsqueeze(1), emb.sin()[pos].to(v.dtype).unsqueeze(1)
    rot = lambda t: torch.cat([-t[..., rd // 2:], t[..., :rd // 2]], -1)
    q = torch.cat([q[..., :rd] * cos + rot(q[..., :rd]) * sin, q[..., rd:]], -1)
    k = torch.cat([k[..., :rd] * cos + rot(k[..., :rd]) * sin, k[..., rd:]], -1)
    k, v = k.repeat_interleave(NH // NKV, 1), v.repeat_interleave(NH // NKV, 1)
    o = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
    return attn.o_proj(o.transpose(1, 2).reshape(B, S, NH * HD))
with torch.no_grad():
    ya, wa = tpa(x, pos).float(), full_attention(x).float()
    ym = tpm(x).float()
    wm = mlp.down_proj(torch.nn.functional.silu(mlp.gate_proj(x)) * mlp.up_proj(x)).float()
ea = ((ya - wa).norm() / wa.norm()).item()
em = ((ym - wm).norm() / wm.norm()).item()
dist.destroy_process_group()
print(f"rank {rank} attention {ea:.3e} mlp {em:.3e}")
sys.exit(0 if max(ea, em) < 2e-2 else 3)
'''


def test_tp_two_gpus_match_full_modules():
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
