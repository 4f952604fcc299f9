"""Allocation-free ``hn_int4_linear_static`` against the workspace entry point.

The file name makes pytest collect it last, so it runs both alone and after
every other GPU test.  Each case calls the static entry point twice in a row
through the C ABI and compares both results with ``hn_int4_linear`` (through
``kernels.int4_gemm.int4_linear``) and with the oracle.
"""

import ctypes

import numpy as np
import pytest
import torch

from hydranet_b200 import _lib
from hydranet_b200.kernels import int4_gemm as k_gemm
from oracle import int4_ref as R
from tests.gpu_util import act, rel_l2, to_np32

pytestmark = pytest.mark.gpu

TIGHT = {"bf16": 5e-3, "f16": 1e-3}   # same precision bound as the workspace entry point
STATIC_BYTES = 16 << 20               # HN_INT4_LINEAR_STATIC_SCRATCH_BYTES


def call_static(lib, x, p, s, n):
    m, k = x.shape
    out = torch.empty(m, n, device=x.device, dtype=x.dtype)
    _lib.check(lib.hn_int4_linear_static(x.data_ptr(), x.stride(0), _lib.dtype_code(x.dtype), m, k, p.data_ptr(),
                                         s.data_ptr(), n, 128, out.data_ptr(), n, _lib.stream_ptr(x.device)))
    return out


def weights(seed, n, k):
    w = np.random.default_rng(seed).standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
    p, s = R.quantize_tensor(w)
    return p, s, torch.from_numpy(p).cuda(), torch.from_numpy(s).cuda()


@pytest.mark.parametrize("M,N,K,dtype", [(1, 14336, 4096, "bf16"), (17, 1024, 512, "f16"),
                                         (64, 4096, 14336, "bf16"), (40, 2048, 1024, "bf16"),
                                         (80, 2048, 1024, "bf16"), (300, 1024, 512, "f16")])
def test_static_matches_workspace_entry_point(lib, M, N, K, dtype):
    p, s, pd, sd = weights(M + N + K, N, K)
    x = act(np.random.default_rng(M).standard_normal((M, K), dtype=np.float32), dtype)
    expect = k_gemm.int4_linear(x, pd, sd)
    ref = R.int4_linear_ref(to_np32(x), p, s)
    for _ in range(2):
        got = call_static(lib, x, pd, sd, N)
        torch.cuda.synchronize()
        assert rel_l2(to_np32(got), to_np32(expect)) <= TIGHT[dtype]
        assert rel_l2(to_np32(got), ref) <= TIGHT[dtype]


def test_static_refuses_shapes_beyond_its_scratch(lib):
    M, N, K = 4096, 4096, 14336
    assert lib.hn_int4_linear_static_scratch_size(M, N, K) > STATIC_BYTES
    # the shapes the matching test accepts fit by the same rule
    for m, n, k in [(1, 14336, 4096), (64, 4096, 14336), (80, 2048, 1024), (300, 1024, 512)]:
        assert 0 < lib.hn_int4_linear_static_scratch_size(m, n, k) <= STATIC_BYTES
    x = torch.zeros(M, K, device="cuda", dtype=torch.bfloat16)
    pd = torch.zeros(N, K // 2, device="cuda", dtype=torch.uint8)
    sd = torch.zeros(N, K // 128, device="cuda", dtype=torch.float16)
    with pytest.raises(_lib.HydraNetError) as e:
        call_static(lib, x, pd, sd, N)
    assert e.value.code == _lib.HN_ERR_WORKSPACE
    assert "hn_int4_linear with a workspace" in str(e.value)


def test_static_error_word_is_reported_and_cleared(lib):
    """The array's error word is reachable: the bounded-wait self-test run on
    the static array (workspace NULL) sets it, hn_int4_linear_static_error
    reports it and clears it, and the next static call is correct."""
    code = ctypes.c_int(-1)
    stream = _lib.stream_ptr(torch.device("cuda"))
    _lib.check(lib.hn_int4_linear_static_error(ctypes.byref(code), stream))
    assert code.value == 0
    _lib.check(lib.hn_selftest_wait_timeout(None, 0, 1, stream))
    torch.cuda.synchronize()
    _lib.check(lib.hn_int4_linear_static_error(ctypes.byref(code), stream))
    assert code.value == 1                      # DEV_ERR_WAIT_TIMEOUT, seen through the static entry's query
    _lib.check(lib.hn_int4_linear_static_error(ctypes.byref(code), stream))
    assert code.value == 0                      # read and cleared
    p, s, pd, sd = weights(5, 512, 1024)
    x = act(np.random.default_rng(6).standard_normal((3, 1024), dtype=np.float32), "bf16")
    got = call_static(lib, x, pd, sd, 512)
    torch.cuda.synchronize()
    assert rel_l2(to_np32(got), R.int4_linear_ref(to_np32(x), p, s)) <= TIGHT["bf16"]
