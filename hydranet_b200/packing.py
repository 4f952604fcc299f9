"""The reference's packed expert format, on the GPU.

* ``BlobLayout`` -- byte offsets of the six tensors in one expert blob
  (``cache/packed_expert_store.py:77-108``).
* ``quantize_expert`` -- packs one expert's fp32/fp16 weights on the GPU,
  bit-identical to ``ExpertWeightPacker.pack_expert``
  (``preprocess/pack_weights.py:183-228``).
* ``ExpertSlot`` -- the ``GpuExpertSlot`` buffer set
  (``cache/packed_expert_store.py:111-172,323-331``).
* ``load_store`` / ``write_store`` -- ``experts.bin`` + ``experts.idx`` v2.0
  (``preprocess/pack_glm4.py:73-143``) read straight into device slots.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from . import ops


@dataclass
class BlobLayout:
    gate_packed_offset: int = 0
    gate_packed_size: int = 0
    gate_scales_offset: int = 0
    gate_scales_size: int = 0
    up_packed_offset: int = 0
    up_packed_size: int = 0
    up_scales_offset: int = 0
    up_scales_size: int = 0
    down_packed_offset: int = 0
    down_packed_size: int = 0
    down_scales_offset: int = 0
    down_scales_size: int = 0

    @classmethod
    def from_dims(cls, hidden_dim: int, intermediate_dim: int, group_size: int) -> "BlobLayout":
        l = cls()
        gp = intermediate_dim * (hidden_dim // 2)
        gs = intermediate_dim * (hidden_dim // group_size) * 2
        dp = hidden_dim * (intermediate_dim // 2)
        ds = hidden_dim * (intermediate_dim // group_size) * 2
        l.gate_packed_offset, l.gate_packed_size = 0, gp
        l.gate_scales_offset, l.gate_scales_size = gp, gs
        l.up_packed_offset, l.up_packed_size = gp + gs, gp
        l.up_scales_offset, l.up_scales_size = 2 * gp + gs, gs
        l.down_packed_offset, l.down_packed_size = 2 * (gp + gs), dp
        l.down_scales_offset, l.down_scales_size = 2 * (gp + gs) + dp, ds
        return l

    @property
    def total_size(self) -> int:
        return self.down_scales_offset + self.down_scales_size


class ExpertSlot:
    """Device buffers of one INT4 expert, same attributes as ``GpuExpertSlot``."""

    def __init__(self, hidden_dim: int, intermediate_dim: int, group_size: int = 128,
                 device: torch.device | str = "cuda", blob: Optional[torch.Tensor] = None):
        self.hidden_dim, self.intermediate_dim, self.group_size = hidden_dim, intermediate_dim, group_size
        self.device = torch.device(device)
        self.layer_idx: Optional[int] = None
        self.expert_idx: Optional[int] = None
        lay = BlobLayout.from_dims(hidden_dim, intermediate_dim, group_size)
        if blob is None:
            blob = torch.empty(lay.total_size, dtype=torch.uint8, device=self.device)
        assert blob.numel() == lay.total_size and blob.dtype == torch.uint8
        self.blob = blob
        H, F, g = hidden_dim, intermediate_dim, group_size

        def view(off, size, dtype, shape):
            return blob[off:off + size].view(dtype).view(shape)

        # every offset of the layout is a multiple of 2; packed buffers start 16-byte aligned
        # when (F*H/2 + F*H/64) is, which holds for every H, F multiple of 128
        self.gate_packed = view(lay.gate_packed_offset, lay.gate_packed_size, torch.uint8, (F, H // 2))
        self.gate_scales = view(lay.gate_scales_offset, lay.gate_scales_size, torch.float16, (F, H // g))
        self.up_packed = view(lay.up_packed_offset, lay.up_packed_size, torch.uint8, (F, H // 2))
        self.up_scales = view(lay.up_scales_offset, lay.up_scales_size, torch.float16, (F, H // g))
        self.down_packed = view(lay.down_packed_offset, lay.down_packed_size, torch.uint8, (H, F // 2))
        self.down_scales = view(lay.down_scales_offset, lay.down_scales_size, torch.float16, (H, F // g))
        self.ready_event = torch.cuda.Event() if self.device.type == "cuda" else None

    def tensors(self) -> Tuple[torch.Tensor, ...]:
        return (self.gate_packed, self.gate_scales, self.up_packed, self.up_scales, self.down_packed,
                self.down_scales)

    def wait_ready(self):
        """GPU-side wait for an async load (``cache/packed_expert_store.py:323-331``)."""
        if self.ready_event is not None:
            torch.cuda.current_stream().wait_event(self.ready_event)

    def size_bytes(self) -> int:
        return self.blob.numel()


def quantize_expert(gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor, group_size: int = 128,
                    slot: Optional[ExpertSlot] = None) -> ExpertSlot:
    """Pack one expert on the GPU into a (new) ``ExpertSlot``."""
    F, H = gate.shape
    if slot is None:
        slot = ExpertSlot(H, F, group_size, gate.device)
    for w, (p, s) in ((gate, (slot.gate_packed, slot.gate_scales)), (up, (slot.up_packed, slot.up_scales)),
                      (down, (slot.down_packed, slot.down_scales))):
        pk, sc = ops.quantize_int4(w, group_size)
        p.copy_(pk)
        s.copy_(sc)
    return slot


SLOT_TENSORS = ("gate_packed", "gate_scales", "up_packed", "up_scales", "down_packed", "down_scales")


class ExpertTable:
    """Device table of expert pointers (``hn_expert_ptrs`` rows) for the grouped ops.

    Accepts ``ExpertSlot`` objects or any object with the six ``GpuExpertSlot``
    buffer attributes (``cache/packed_expert_store.py:136-162``).  Holds references to the slots so their memory outlives the table.  Rebuild
    (``refresh``) after a slot is re-pointed; re-filling a slot in place needs
    no rebuild.
    """

    def __init__(self, slots: List[ExpertSlot]):
        if not slots:
            raise ValueError("empty expert table")
        self.slots = list(slots)
        self.hidden_dim = slots[0].hidden_dim
        self.intermediate_dim = slots[0].intermediate_dim
        self.group_size = slots[0].group_size
        for s in slots:
            if (s.hidden_dim, s.intermediate_dim, s.group_size) != (self.hidden_dim, self.intermediate_dim,
                                                                     self.group_size):
                raise ValueError("all experts of a table must share dims")
            for t in (getattr(s, n) for n in SLOT_TENSORS):
                if not t.is_contiguous() or t.data_ptr() % 16:
                    raise ValueError("expert buffers must be contiguous and 16-byte aligned")
        self.device = slots[0].gate_packed.device
        self.device_table = torch.empty(len(slots), 6, dtype=torch.int64, device=self.device)
        self.device_maps = None
        self.refresh()

    def refresh(self):
        """Re-publish the pointer table and the TMA descriptors (after a slot moved)."""
        rows = [[getattr(s, n).data_ptr() for n in SLOT_TENSORS] for s in self.slots]
        self.device_table.copy_(torch.tensor(rows, dtype=torch.int64))
        if self.device.type == "cuda":
            self.device_maps = self._encode_maps(rows)

    def _encode_maps(self, rows):
        import ctypes
        from . import _lib
        lib = _lib.load()
        per = lib.hn_expert_maps_bytes()
        E = len(rows)
        host_ptrs = (ctypes.c_uint64 * (6 * E))(*[p for r in rows for p in r])
        raw = ctypes.create_string_buffer(E * per + 64)
        aligned = (ctypes.addressof(raw) + 63) & ~63
        _lib.check(lib.hn_expert_maps_encode(ctypes.addressof(host_ptrs), E, self.hidden_dim, self.intermediate_dim,
                                             aligned))
        blob = ctypes.string_at(aligned, E * per)
        dev = torch.frombuffer(bytearray(blob), dtype=torch.uint8).to(self.device)
        assert dev.data_ptr() % 64 == 0
        return dev

    def __len__(self):
        return len(self.slots)


def write_store(out_dir: Path, experts: Dict[Tuple[int, int], Tuple[np.ndarray, ...]], hidden_dim: int,
                intermediate_dim: int, group_size: int = 128, num_layers: int = 1, num_experts: int = 1) -> None:
    """Write ``experts.bin`` + ``experts.idx`` (format 2.0) from packed numpy tensors."""
    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    lay = BlobLayout.from_dims(hidden_dim, intermediate_dim, group_size)
    index = {"format_version": "2.0",
             "quant_config": {"bits": 4, "group_size": group_size, "symmetric": True},
             "model_config": {"num_layers": num_layers, "num_experts": num_experts, "hidden_dim": hidden_dim,
                              "intermediate_dim": intermediate_dim},
             "experts": []}
    off = 0
    with open(out_dir / "experts.bin", "wb") as f:
        for (layer, e), t in sorted(experts.items()):
            blob = b"".join(np.ascontiguousarray(a).tobytes() for a in t)
            assert len(blob) == lay.total_size
            f.write(blob)
            index["experts"].append({"layer_idx": layer, "expert_idx": e, "offset": off, "size": lay.total_size})
            off += lay.total_size
    (out_dir / "experts.idx").write_text(json.dumps(index, indent=2))


def load_store(index_path: Path, layer_idx: int, device="cuda") -> ExpertTable:
    """Load every expert of one layer of a v2.0 store into device slots."""
    index_path = Path(index_path)
    idx = json.loads(index_path.read_text())
    if idx.get("format_version") != "2.0":
        raise ValueError(f"unsupported packed store format {idx.get('format_version')!r}")
    mc, qc = idx["model_config"], idx["quant_config"]
    H, F, g = mc["hidden_dim"], mc["intermediate_dim"], qc["group_size"]
    lay = BlobLayout.from_dims(H, F, g)
    entries = sorted((e for e in idx["experts"] if e["layer_idx"] == layer_idx), key=lambda e: e["expert_idx"])
    if not entries:
        raise ValueError(f"layer {layer_idx} not in index")
    # the table is indexed by expert id: the layer must list each of 0..E-1 exactly once
    ids = [e["expert_idx"] for e in entries]
    n_exp = mc.get("num_experts", len(ids))
    if ids != list(range(n_exp)):
        raise ValueError(f"layer {layer_idx} of the index lists experts {ids[:8]}{'...' if len(ids) > 8 else ''}, "
                         f"not each of 0..{n_exp - 1} once")
    data = np.memmap(index_path.parent / "experts.bin", dtype=np.uint8, mode="r")
    slots = []
    for e in entries:
        if e["size"] != lay.total_size or e["offset"] + e["size"] > data.size:
            raise ValueError(f"corrupt index entry for expert {e['expert_idx']}")
        host = torch.from_numpy(np.array(data[e["offset"]:e["offset"] + e["size"]]))
        slot = ExpertSlot(H, F, g, device)
        slot.blob.copy_(host)
        slot.layer_idx, slot.expert_idx = layer_idx, e["expert_idx"]
        slots.append(slot)
    return ExpertTable(slots)
