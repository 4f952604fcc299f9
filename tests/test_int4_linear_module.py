"""The non-expert ``Int4Linear`` module (``kernels/int4_linear.py``) on CPU.

The quantiser is pinned bit for bit to fixtures made by running the
reference's own ``Int4Linear.quantize_weight`` (``tests/golden/make_golden.py``),
both for the oracle's numpy restatement and for the module's torch version.
The forward's wiring (engine call, then the float16 bias) is checked with
the engine call replaced by the oracle; the engine itself is covered by the
GPU tests.
"""

import numpy as np
import pytest
import torch
import torch.nn as nn

from hydranet_b200.kernels import int4_linear as mod
from hydranet_b200.kernels import Int4Linear, convert_model_to_int4, estimate_int4_memory
from oracle import int4_ref as R


@pytest.fixture(scope="module")
def golden(golden_dir):
    z = np.load(golden_dir / "int4linear_quant.npz")
    return {k: z[k] for k in z.files}


def _cases(golden):
    return sorted({k.split("/")[0] for k in golden if not k.startswith("from_float")})


def test_oracle_quantiser_matches_reference(golden):
    names = _cases(golden)
    assert {"rand_f32", "rand_f16", "g64_f32", "edge_f32"} <= set(names)
    for n in names:
        p, s = R.int4linear_quantize_ref(golden[n + "/w"], int(golden[n + "/group_size"]))
        assert np.array_equal(p, golden[n + "/packed"]), n
        assert np.array_equal(s.view(np.uint16), golden[n + "/scales"].view(np.uint16)), n


def test_module_quantiser_matches_reference(golden):
    for n in _cases(golden):
        p, s = Int4Linear.quantize_weight(torch.from_numpy(golden[n + "/w"]), int(golden[n + "/group_size"]))
        assert p.dtype == torch.uint8 and s.dtype == torch.float16
        assert np.array_equal(p.numpy(), golden[n + "/packed"]), n
        assert np.array_equal(s.numpy().view(np.uint16), golden[n + "/scales"].view(np.uint16)), n


def test_differs_from_expert_packer(golden):
    """The two quantisers are different functions: on float16 weights their
    roundings disagree on some entries of the fixture (in float32 they
    happen to agree there), so neither can stand in for the other."""
    w = golden["rand_f16/w"]
    p_lin, _ = R.int4linear_quantize_ref(w)
    p_exp, _ = R.quantize_tensor(w)
    assert np.array_equal(p_lin, golden["rand_f16/packed"])
    assert not np.array_equal(p_lin, p_exp)


def test_from_float_group_size_and_bias(golden):
    for key in [k for k in golden if k.startswith("from_float_group/")]:
        n_in = int(key.split("/")[1])
        m = Int4Linear.from_float(nn.Linear(n_in, 8), group_size=128)
        assert m.group_size == int(golden[key]), key
    with pytest.raises(ValueError):
        Int4Linear.from_float(nn.Linear(40, 8))
    lin = nn.Linear(256, 24)
    m = Int4Linear.from_float(lin)
    assert m.weight_packed.shape == (24, 128) and m.weight_scale.shape == (24, 2)
    assert m.bias.dtype == torch.float16
    assert torch.equal(m.bias.data, lin.bias.data.to(torch.float16))
    p, s = R.int4linear_quantize_ref(lin.weight.data.numpy())
    assert np.array_equal(m.weight_packed.numpy(), p)
    assert Int4Linear.from_float(nn.Linear(256, 4, bias=False)).bias is None
    assert "dtype=int4, group_size=128" in repr(m)


def test_constructor_checks():
    with pytest.raises(AssertionError):
        Int4Linear(200, 8)            # not a multiple of the group size
    m = Int4Linear(256, 8, bias=False)
    assert m.bias is None and m.weight_scale.dtype == torch.float16
    assert {n for n, _ in m.named_buffers()} == {"weight_packed", "weight_scale"}


def test_forward_wiring(monkeypatch):
    """Engine result + float16 bias, with the reference's type promotion."""
    def engine(x, packed, scales, group_size):
        y = R.int4_linear_ref(x.float().numpy(), packed.numpy(), scales.numpy(), group_size)
        return torch.from_numpy(y).to(x.dtype)
    monkeypatch.setattr(mod, "int4_linear", engine)
    lin = nn.Linear(256, 32)
    m = Int4Linear.from_float(lin)
    x = torch.randn(5, 256, dtype=torch.float16)
    y = m(x)
    p, s = R.int4linear_quantize_ref(lin.weight.data.numpy())
    ref = torch.from_numpy(R.int4_linear_ref(x.float().numpy(), p, s)).to(torch.float16) + m.bias
    assert y.dtype == torch.float16 and torch.equal(y, ref)


def test_forward_refuses_cpu_tensors():
    m = Int4Linear.from_float(nn.Linear(256, 16))
    with pytest.raises(ValueError, match="CUDA"):
        m(torch.randn(2, 256, dtype=torch.float16))


def test_convert_model_to_int4(capsys):
    model = nn.Sequential()
    model.add_module("q_proj", nn.Linear(256, 64))
    model.add_module("odd", nn.Linear(255, 8))
    model.add_module("g64", nn.Linear(192, 8))         # would need group size 64
    model.add_module("lm_head", nn.Linear(256, 100))
    model.add_module("act", nn.SiLU())
    convert_model_to_int4(model, skip_layers=["lm_head"])
    assert isinstance(model.q_proj, Int4Linear)
    assert isinstance(model.odd, nn.Linear) and isinstance(model.g64, nn.Linear)
    assert isinstance(model.lm_head, nn.Linear)
    out = capsys.readouterr().out
    assert "Converted 1 layers to INT4, skipped 3" in out


def test_estimate_int4_memory():
    model = nn.Sequential(nn.Linear(256, 64), nn.Linear(64, 10, bias=False))
    est = estimate_int4_memory(model)
    fp16 = 2 * (256 * 64 + 64 + 64 * 10)
    int4 = (256 * 64 // 2 + 64 * 2 * 2) + 2 * 64 + (64 * 10 // 2 + 10 * 1 * 2)
    assert est["fp16_mb"] == fp16 / 1e6 and est["int4_mb"] == int4 / 1e6
    assert est["savings_mb"] == (fp16 - int4) / 1e6
