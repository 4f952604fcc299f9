"""Failure detection on the device, without a fault: a bounded wait whose
partner never arrives gives up after its limit (2 s), records the timeout in
the workspace's error word and lets the launch end.  The host reads the
status with ``hn_workspace_error`` (which clears it), and the context keeps
running kernels afterwards.
"""

import time

import numpy as np
import pytest
import torch

from hydranet_b200 import _lib
from hydranet_b200.kernels import int4_gemm as k_gemm
from oracle import int4_ref as R
from tests.gpu_util import act, rel_l2, to_np32

pytestmark = pytest.mark.gpu

DEV_ERR_WAIT_TIMEOUT = 1


@pytest.mark.parametrize("mode", [0, 1])
def test_wait_runs_out_and_reports(lib, mode):
    ws = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _lib.check(lib.hn_selftest_wait_timeout(ws.data_ptr(), ws.numel(), mode, _lib.stream_ptr(ws.device)))
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert 1.5 < elapsed < 60, elapsed           # gave up at the limit, not at once and not never
    assert _lib.workspace_error(ws) == DEV_ERR_WAIT_TIMEOUT
    assert _lib.workspace_error(ws) == 0          # read and cleared
    # the context is intact: an ordinary call still runs and is correct
    w = np.random.default_rng(1).standard_normal((256, 512), dtype=np.float32) * np.float32(0.02)
    p, s = R.quantize_tensor(w)
    x = act(np.random.default_rng(2).standard_normal((4, 512), dtype=np.float32), "bf16")
    out = k_gemm.int4_linear(x, torch.from_numpy(p).cuda(), torch.from_numpy(s).cuda())
    assert rel_l2(to_np32(out), R.int4_linear_ref(to_np32(x), p, s)) <= 5e-3


def test_selftest_rejects_bad_arguments(lib):
    ws = torch.zeros(256, dtype=torch.uint8, device="cuda")
    assert lib.hn_selftest_wait_timeout(ws.data_ptr(), ws.numel(), 0, _lib.stream_ptr(ws.device)) \
        == _lib.HN_ERR_INVALID
    assert lib.hn_selftest_wait_timeout(ws.data_ptr(), 4096, 2, _lib.stream_ptr(ws.device)) == _lib.HN_ERR_INVALID
