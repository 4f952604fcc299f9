"""GPU parity of the drop-in kernels against the numpy oracle.

Contract (north star): rel-L2 <= 1e-2 against the reference's
dequant-then-matmul path with float32 accumulation.  A tighter bound is also
asserted: weights enter the MMA as the float16 (n - 8) * scale the reference
dequantiser produces, tokens as float16 and products accumulate in fp32, so
the sizeable errors are the roundings of the activations to float16 and of
the result to the activation dtype (and, in the MLP, of the SiLU*up
intermediate, kept as float16).
"""

import numpy as np
import pytest
import torch

from hydranet_b200 import ops
from hydranet_b200.kernels import expert_mlp as k_em
from hydranet_b200.kernels import int4_expert_mlp as k_v1
from hydranet_b200.kernels import int4_gemm as k_gemm
from hydranet_b200.packing import ExpertSlot
from oracle import int4_ref as R
from tests.gpu_util import act, rel_l2, to_np32

pytestmark = pytest.mark.gpu

TOL = 1e-2
TIGHT = {"bf16": 5e-3, "f16": 1e-3}


def packed_weight(seed, n, k):
    w = np.random.default_rng(seed).standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
    return R.quantize_tensor(w)


@pytest.mark.parametrize("M,N,K", [(1, 256, 128), (3, 384, 256), (8, 512, 512), (17, 1024, 512),
                                   (33, 512, 1024), (5, 200, 512), (64, 4096, 4096), (130, 256, 256),
                                   (2, 14336, 4096)])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_int4_linear(lib, M, N, K, dtype):
    p, s = packed_weight(M * 7 + N, N, K)
    x = np.random.default_rng(M).standard_normal((M, K), dtype=np.float32)
    xt = act(x, dtype)
    out = k_gemm.int4_linear(xt, torch.from_numpy(p).cuda(), torch.from_numpy(s).cuda())
    assert out.shape == (M, N) and out.dtype == xt.dtype
    ref = R.int4_linear_ref(to_np32(xt), p, s)
    err = rel_l2(to_np32(out), ref)
    assert err <= TOL and err <= TIGHT[dtype], err


def test_int4_linear_3d_and_strided(lib):
    p, s = packed_weight(1, 384, 512)
    x = torch.randn(2, 3, 1024, device="cuda", dtype=torch.bfloat16)[..., :512]   # row stride 1024
    out = k_v1.int4_linear(x, torch.from_numpy(p).cuda(), torch.from_numpy(s).cuda())
    assert out.shape == (2, 3, 384)
    ref = R.int4_linear_ref(to_np32(x.reshape(6, 512)), p, s)
    assert rel_l2(to_np32(out.reshape(6, 384)), ref) <= TIGHT["bf16"]


@pytest.mark.parametrize("dtype,bias", [("f16", True), ("f16", False), ("bf16", True)])
def test_int4linear_module(lib, dtype, bias):
    """``Int4Linear.from_float`` and its forward (``kernels/int4_linear.py:105-168``):
    the engine's output plus the float16 bias, with the reference's type
    promotion (a bf16 input plus the float16 bias gives float32)."""
    from hydranet_b200.kernels import Int4Linear
    torch.manual_seed(3)
    lin = torch.nn.Linear(1024, 384, bias=bias)
    m = Int4Linear.from_float(lin, device=torch.device("cuda"))
    p, s = R.int4linear_quantize_ref(lin.weight.detach().numpy())
    assert np.array_equal(m.weight_packed.cpu().numpy(), p)
    x = act(np.random.default_rng(4).standard_normal((14, 1024), dtype=np.float32), dtype).view(2, 7, 1024)
    y = m(x)
    want_dtype = x.dtype if (not bias or dtype == "f16") else torch.float32
    assert y.shape == (2, 7, 384) and y.dtype == want_dtype
    ref = R.int4_linear_ref(to_np32(x.reshape(14, 1024)), p, s)
    if bias:
        ref = ref + lin.bias.detach().numpy().astype(np.float16).astype(np.float32)
    assert rel_l2(to_np32(y.reshape(14, 384)), ref) <= TIGHT[dtype]


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_silu_mul(lib, dtype):
    g = act(np.random.default_rng(0).standard_normal((7, 1000), dtype=np.float32) * 3, dtype)
    u = act(np.random.default_rng(1).standard_normal((7, 1000), dtype=np.float32), dtype)
    out = k_gemm.fused_silu_mul(g, u)
    ref = R.silu_mul_ref(to_np32(g), to_np32(u))
    assert rel_l2(to_np32(out), ref) <= TIGHT[dtype]
    out2 = k_v1.silu_mul(g.view(1, 7, 1000), u.view(1, 7, 1000))
    assert torch.equal(out2.view(7, 1000), out)


def make_expert(seed, H, F):
    t = []
    for i, shape in enumerate(((F, H), (F, H), (H, F))):
        t += list(packed_weight(seed * 3 + i, *shape))
    return t


@pytest.mark.parametrize("T,H,F", [(1, 512, 1024), (4, 512, 1024), (9, 1024, 2048), (40, 256, 512),
                                   (64, 4096, 1408), (2, 4096, 14336), (100, 512, 256)])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_expert_mlp_fused(lib, T, H, F, dtype):
    t = make_expert(T + H + F, H, F)
    x = act(np.random.default_rng(T).standard_normal((T, H), dtype=np.float32), dtype)
    dev = [torch.from_numpy(a).cuda() for a in t]
    out = k_gemm.expert_mlp_int4_fused(x, *dev, group_size=128)
    ref = R.expert_mlp_ref(to_np32(x), *t)
    err = rel_l2(to_np32(out), ref)
    assert err <= TOL and err <= 2 * TIGHT[dtype], err


def test_expert_mlp_entry_points_agree(lib):
    H, F, T = 512, 1024, 6
    t = make_expert(5, H, F)
    slot = ExpertSlot(H, F, 128, "cuda")
    for dst, src in zip(slot.tensors(), t):
        dst.copy_(torch.from_numpy(src))
    x = torch.randn(1, T, H, device="cuda", dtype=torch.bfloat16)
    a = k_gemm.expert_mlp_int4_fused(x, *slot.tensors())
    b = k_v1.expert_mlp_int4_from_slot(x, slot)
    c = k_em.expert_mlp_int4(x.view(T, H), *slot.tensors(), hidden_dim=H, intermediate_dim=F)
    assert a.shape == (1, T, H)
    assert torch.equal(a, b) and torch.equal(a.view(T, H), c)
    ref = R.expert_mlp_ref(to_np32(x.view(T, H)), *t)
    assert rel_l2(to_np32(c), ref) <= 2 * TIGHT["bf16"]


def test_repeatable_bitwise(lib):
    """Counters reset by the kernels: repeated calls give identical bits."""
    H, F, T = 1024, 2048, 24
    dev = [torch.from_numpy(a).cuda() for a in make_expert(9, H, F)]
    x = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    outs = [ops.expert_mlp_int4(x, *dev) for _ in range(4)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


def test_workspace_only_head_must_be_zero(lib):
    """Only the first 512 bytes of a workspace must start at zero: the rest may
    hold anything another call of another shape left there."""
    M, N, K = 40, 1024, 2048
    p, s = packed_weight(3, N, K)
    x = act(np.random.default_rng(4).standard_normal((M, K), dtype=np.float32), "bf16")
    need = lib.hn_int4_linear_workspace_size(M, N, K)
    ws = torch.full((need + 4096,), 0xFF, dtype=torch.uint8, device="cuda")
    ws[:512] = 0
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    pd, sd = torch.from_numpy(p).cuda(), torch.from_numpy(s).cuda()
    from hydranet_b200._lib import check, ptr, stream_ptr
    for _ in range(2):
        check(lib.hn_int4_linear(ptr(x), K, 2, M, K, ptr(pd), ptr(sd), N, 128, ptr(out), N, ptr(ws), ws.numel(),
                                 stream_ptr(x.device)))
        ref = R.int4_linear_ref(to_np32(x), p, s)
        assert rel_l2(to_np32(out), ref) <= TIGHT["bf16"]
        ws[512:].fill_(0xFF)  # as if a call of another shape had used the rest
    assert _lib_error(ws) == 0


def _lib_error(ws):
    from hydranet_b200 import _lib
    return _lib.workspace_error(ws)


@pytest.mark.parametrize("M,N,K", [(64, 4096, 14336), (64, 14336, 4096), (32, 14336, 4096)])
def test_long_k_runs_bitwise_repeatable(lib, M, N, K):
    """Mixtral-size projections: every CTA streams long runs of k-groups through
    the weight ring; each call must give the same bits and match the oracle.
    The L2 is flushed before each call so weights stream from HBM."""
    p, s = packed_weight(17, N, K)
    x = act(np.random.default_rng(5).standard_normal((M, K), dtype=np.float32), "bf16")
    pd, sd = torch.from_numpy(p).cuda(), torch.from_numpy(s).cuda()
    scrub = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    outs = []
    for _ in range(6):
        scrub.add_(1)
        outs.append(k_gemm.int4_linear(x, pd, sd))
    ref = R.int4_linear_ref(to_np32(x), p, s)
    for o in outs:
        assert torch.equal(o, outs[0])
    assert rel_l2(to_np32(outs[0]), ref) <= TIGHT["bf16"]
