"""GPU packer / unpacker / dequantiser are bit-exact against the reference's
golden outputs (``preprocess/pack_weights.py:133-268``)."""

import numpy as np
import pytest
import torch

from hydranet_b200 import ops, synth
from oracle import int4_ref as R

pytestmark = pytest.mark.gpu

CASES = ["rand_f32", "rand_f16", "wide_f32", "edge_f32"]


@pytest.fixture(scope="module")
def golden(golden_dir):
    return dict(np.load(golden_dir / "pack_cases.npz"))


@pytest.mark.parametrize("case", CASES)
def test_quantize_matches_reference(lib, golden, case):
    w = torch.from_numpy(golden[case + "/w"]).cuda()
    p, s = ops.quantize_int4(w)
    np.testing.assert_array_equal(p.cpu().numpy(), golden[case + "/packed"])
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint16), golden[case + "/scales"].view(np.uint16))


@pytest.mark.parametrize("case", CASES)
def test_dequant_matches_reference(lib, golden, case):
    p = torch.from_numpy(golden[case + "/packed"]).cuda()
    s = torch.from_numpy(golden[case + "/scales"]).cuda()
    d = ops.dequant_int4(p, s)
    np.testing.assert_array_equal(d.cpu().numpy().view(np.uint16), golden[case + "/dequant"].view(np.uint16))


@pytest.mark.parametrize("case", CASES)
def test_unpack_bit_exact(lib, golden, case):
    p = torch.from_numpy(golden[case + "/packed"]).cuda()
    np.testing.assert_array_equal(ops.unpack_int4(p).cpu().numpy(), R.unpack_int4(golden[case + "/packed"]))


def test_fp16_zero_group_and_large_matrix(lib):
    """All-zero fp16 group (0/0 in the reference -> nibble 0) and a Mixtral-width matrix."""
    w = synth.host_normal(3, (512, 4096), 0.02)
    w[7, :128] = 0.0
    for arr in (w, w.astype(np.float16)):
        p, s = ops.quantize_int4(torch.from_numpy(arr).cuda())
        rp, rs = R.quantize_tensor(arr)
        np.testing.assert_array_equal(p.cpu().numpy(), rp)
        np.testing.assert_array_equal(s.cpu().numpy().view(np.uint16), rs.view(np.uint16))


def test_roundtrip_error_bounds(lib):
    """Reference bound: max |err| < 0.1, mean < 0.01 (``tests/test_int4_pack.py:64-66``)."""
    torch.manual_seed(42)  # the reference test's own input (tests/test_int4_pack.py:33-35)
    w = (torch.randn(512, 256, dtype=torch.float16) * 0.1).cuda()
    p, s = ops.quantize_int4(w)
    err = (ops.dequant_int4(p, s).float() - w.float()).abs()
    assert err.max().item() < 0.1 and err.mean().item() < 0.01
