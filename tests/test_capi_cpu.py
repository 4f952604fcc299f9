"""C-ABI library and host-side logic, without a GPU.

* the library loads and exports every entry point ``include/hydranet_b200.h`` declares;
* the ctypes table in ``hydranet_b200/_lib.py`` binds exactly those;
* workspace-size queries behave; ops refuse CPU tensors (no CPU fallback);
* the workspace cache refuses to allocate during CUDA-graph capture;
* the packed-format helpers agree with the reference layout.
"""

import re
from pathlib import Path

import numpy as np
import pytest
import torch

from hydranet_b200 import _lib, ops
from hydranet_b200.packing import BlobLayout, ExpertSlot, ExpertTable, load_store, write_store
from oracle import int4_ref as R

HEADER = Path(__file__).resolve().parent.parent / "include" / "hydranet_b200.h"


def declared():
    return sorted(set(re.findall(r"HN_API\s+[\w\s\*]+?\b(hn_\w+)\s*\(", HEADER.read_text())))


def test_header_declares_entry_points():
    names = declared()
    assert "hn_moe_layer_int4" in names and "hn_int4_linear" in names and len(names) >= 16


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared():
        assert hasattr(lib, name), name


def test_ctypes_table_matches_header():
    assert sorted(_lib.SIGNATURES) == declared()


def test_abi_and_sizes_without_gpu():
    lib = _lib.load()
    assert lib.hn_abi_version() == 3
    a = lib.hn_moe_workspace_size(1, 4096, 14336, 8, 2)
    b = lib.hn_moe_workspace_size(64, 4096, 14336, 8, 2)
    assert 0 < a < b
    assert lib.hn_moe_workspace_size(0, 4096, 14336, 8, 2) == 0
    assert lib.hn_expert_mlp_workspace_size(4, 512, 1024) > 0
    assert lib.hn_int4_linear_workspace_size(1, 4096, 4096) > 0


def test_invalid_arguments_are_rejected_before_any_launch():
    lib = _lib.load()
    with pytest.raises(_lib.HydraNetError) as e:
        _lib.check(lib.hn_quantize_int4(None, 0, 4, 100, 128, None, None, None))
    assert e.value.code == _lib.HN_ERR_INVALID
    # group size other than 128 is reported as unsupported, not silently mis-computed
    with pytest.raises(_lib.HydraNetError) as e:
        _lib.check(lib.hn_quantize_int4(16, 0, 4, 256, 64, 16, 16, None))
    assert e.value.code == _lib.HN_ERR_UNSUPPORTED
    with pytest.raises(_lib.HydraNetError) as e:
        _lib.check(lib.hn_expert_mlp_int4(16, 2, 4, 100, 256, 16, 16, 16, 16, 16, 16, 128, 16, 256, 1 << 20, None))
    assert e.value.code == _lib.HN_ERR_INVALID


def test_ops_refuse_cpu_tensors():
    x = torch.zeros(2, 256, dtype=torch.bfloat16)
    p = torch.zeros(128, 128, dtype=torch.uint8)
    s = torch.zeros(128, 2, dtype=torch.float16)
    with pytest.raises(ValueError):
        ops.int4_linear(x, p, s)


def test_reference_shape_asserts():
    x = torch.zeros(2, 256, dtype=torch.bfloat16)
    with pytest.raises(AssertionError):
        ops.int4_linear(x, torch.zeros(128, 64, dtype=torch.uint8), torch.zeros(128, 2, dtype=torch.float16))


@pytest.mark.parametrize("H,F", [(4096, 14336), (4096, 1408), (512, 1024), (256, 512)])
def test_blob_layout_matches_oracle(H, F):
    a = BlobLayout.from_dims(H, F, 128)
    b = R.BlobLayout.from_dims(H, F, 128)
    assert a.__dict__ == b.__dict__
    assert a.total_size == b.total_size


def test_store_roundtrip_on_host(tmp_path):
    H, F = 256, 512
    rng = np.random.default_rng(0)
    experts = {}
    for e in range(3):
        t = []
        for shape in ((F, H), (F, H), (H, F)):
            t += list(R.quantize_tensor(rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)))
        experts[(0, e)] = tuple(t)
    write_store(tmp_path, experts, H, F, num_layers=1, num_experts=3)
    table = load_store(tmp_path / "experts.idx", 0, device="cpu")
    assert len(table) == 3
    for e, slot in enumerate(table.slots):
        np.testing.assert_array_equal(slot.gate_packed.numpy(), experts[(0, e)][0])
        np.testing.assert_array_equal(slot.down_scales.numpy(), experts[(0, e)][5])
    assert table.device_table.shape == (3, 6)
    assert int(table.device_table[1, 0]) == table.slots[1].gate_packed.data_ptr()


def test_corrupt_store_is_rejected(tmp_path):
    H, F = 256, 512
    p = R.quantize_tensor(np.zeros((F, H), np.float32))
    d = R.quantize_tensor(np.zeros((H, F), np.float32))
    write_store(tmp_path, {(0, 0): (*p, *p, *d)}, H, F)
    (tmp_path / "experts.bin").write_bytes((tmp_path / "experts.bin").read_bytes()[:-10])
    with pytest.raises(ValueError):
        load_store(tmp_path / "experts.idx", 0, device="cpu")
    with pytest.raises(ValueError):
        load_store(tmp_path / "experts.idx", 5, device="cpu")


def test_expert_slot_views_are_aligned():
    s = ExpertSlot(4096, 1408, 128, device="cpu")
    for t in s.tensors():
        assert t.data_ptr() % 16 == 0
    ExpertTable([s, ExpertSlot(4096, 1408, 128, device="cpu")])


def test_workspace_not_made_during_graph_capture(monkeypatch):
    """A workspace allocated inside CUDA-graph capture would only be zeroed
    when the graph replays, so the cache refuses to make or grow one then."""
    ws = _lib._Workspaces()
    monkeypatch.setattr(_lib, "stream_ptr", lambda device=None: 1234)
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: True)
    with pytest.raises(RuntimeError, match="outside CUDA-graph capture"):
        ws.get(4096, torch.device("cuda:0"))
    assert ws.all() == []


def test_moe_layer_launch_count_query():
    """``hn_moe_layer_launches`` (host-only) at config 2 across the batch sizes
    where the library adds kernels, at the GLM prefill shape, and for sizes
    the layer rejects."""
    lib = _lib.load()
    want = {1: 3, 16: 3, 32: 3, 64: 4, 255: 4, 256: 5, 512: 5, 513: 6, 2048: 6, 2049: 7, 8192: 7}
    assert {T: lib.hn_moe_layer_launches(T, 4096, 14336, 8, 2) for T in want} == want
    # the engine choice does not change the count at decode sizes
    prev = lib.hn_set_decode_engine(_lib.HN_ENGINE_TCGEN05)
    try:
        assert lib.hn_moe_layer_launches(8, 4096, 14336, 8, 2) == 3
        assert lib.hn_moe_layer_launches(64, 4096, 14336, 8, 2) == 4
    finally:
        lib.hn_set_decode_engine(prev)
    assert lib.hn_set_decode_engine(7) == -1
    assert lib.hn_moe_layer_launches(8192, 4096, 1408, 128, 8) == 7
    assert lib.hn_moe_layer_launches(32, 4096, 1408, 128, 8) == 4  # + the router GEMV (128 x 4096 router)
    assert lib.hn_moe_layer_launches(0, 4096, 14336, 8, 2) == 0
    assert lib.hn_moe_layer_launches(4, 64, 14336, 8, 2) == 0


def test_sm_limit_setter():
    lib = _lib.load()
    prev = lib.hn_set_sm_limit(100)
    try:
        assert lib.hn_set_sm_limit(90) == 100
        assert lib.hn_set_sm_limit(-3) == -1
    finally:
        lib.hn_set_sm_limit(prev)
