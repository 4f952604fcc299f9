"""The packed store format (``cache/packed_expert_store.py:77-108``, index
format 2.0) against a store written by the reference's own test helper
(``tests/test_int4_loader.py:28-119``), recorded as its index JSON and the
SHA-256 of its ``experts.bin`` by ``tests/golden/make_golden.py``.

The same seeded float16 weights, packed by the oracle (itself pinned bit for
bit to the reference packer) and written by ``write_store``, must give the same
bytes; ``load_store`` must read the reference's index and hand back exactly the
packed tensors of each expert.
"""

import hashlib
import json

import numpy as np
import torch

from hydranet_b200.packing import load_store, write_store
from oracle import int4_ref as R

H, F, LAYERS, EXPERTS = 256, 512, 2, 2


def _reference_weights():
    """The helper's weights: ``torch.manual_seed(42)``, then per layer and expert
    gate [F, H], up [F, H], down [H, F] as ``randn(float16) * 0.02``."""
    torch.manual_seed(42)
    out = {}
    for layer in range(LAYERS):
        for e in range(EXPERTS):
            out[(layer, e)] = [(torch.randn(*shape, dtype=torch.float16) * 0.02).numpy()
                               for shape in ((F, H), (F, H), (H, F))]
    return out


def test_store_bytes_and_index_match_reference(golden_dir, tmp_path):
    g = np.load(golden_dir / "reference_store.npz")
    packed = {}
    for key, mats in _reference_weights().items():
        t = []
        for w in mats:
            t += list(R.quantize_tensor(w))
        packed[key] = tuple(t)
    write_store(tmp_path, packed, H, F, num_layers=LAYERS, num_experts=EXPERTS)
    data = (tmp_path / "experts.bin").read_bytes()
    assert len(data) == int(g["bin_size"])
    assert hashlib.sha256(data).hexdigest() == str(g["bin_sha256"])
    assert json.loads((tmp_path / "experts.idx").read_text()) == json.loads(str(g["idx_json"]))

    # the reference's own index file, next to the identical bytes
    (tmp_path / "experts.idx").write_text(str(g["idx_json"]))
    for layer in range(LAYERS):
        table = load_store(tmp_path / "experts.idx", layer, device="cpu")
        assert len(table) == EXPERTS
        for e, slot in enumerate(table.slots):
            for got, want in zip(slot.tensors(), packed[(layer, e)]):
                np.testing.assert_array_equal(got.numpy().view(want.dtype), want)
