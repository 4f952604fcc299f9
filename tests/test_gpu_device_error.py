"""A device-side error reaches the Python caller without a synchronising read.

The bounded-wait self-test runs on the workspace the library's ops use on
this stream; its timeout is recorded in the workspace's error word and
copied to the pinned host word the workspace names (bytes 8..15).  The next
op on that stream raises ``DeviceError`` (the earlier call's results are
invalid) and clears both words; the op after that runs and is correct.
"""

import numpy as np
import pytest
import torch

from hydranet_b200 import _lib
from hydranet_b200.kernels import int4_gemm as k_gemm
from oracle import int4_ref as R
from tests.gpu_util import act, rel_l2, to_np32

pytestmark = pytest.mark.gpu


def test_wait_timeout_surfaces_as_device_error(lib):
    w = np.random.default_rng(1).standard_normal((256, 512), dtype=np.float32) * np.float32(0.02)
    p, s = R.quantize_tensor(w)
    pd, sd = torch.from_numpy(p).cuda(), torch.from_numpy(s).cuda()
    x = act(np.random.default_rng(2).standard_normal((4, 512), dtype=np.float32), "bf16")
    ref = R.int4_linear_ref(to_np32(x), p, s)
    k_gemm.int4_linear(x, pd, sd)  # makes the stream's workspace (and its host word)
    ws = _lib.workspaces.get(1, x.device)
    _lib.check(lib.hn_selftest_wait_timeout(ws.data_ptr(), ws.numel(), 1, _lib.stream_ptr(x.device)))
    torch.cuda.synchronize()
    with pytest.raises(_lib.DeviceError) as e:
        k_gemm.int4_linear(x, pd, sd)
    assert e.value.code == 1 and "timed out" in str(e.value)
    out = k_gemm.int4_linear(x, pd, sd)  # the words were cleared: the next call runs
    torch.cuda.synchronize()
    assert _lib.workspace_error(ws) == 0
    assert rel_l2(to_np32(out), ref) <= 5e-3
