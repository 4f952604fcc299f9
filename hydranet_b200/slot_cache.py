"""Over-budget expert residency: a fixed pool of device slots fed from host memory.

The reference serves models whose experts do not all fit in VRAM through
per-layer slot caches (``ExpertCacheManager.get_int4_slot`` /
``prefetch_int4_slot``, ``cache/expert_cache.py:601-679,963-981``) filled by
async H2D copies through pinned staging (``PinnedStagingRing`` and
``load_to_gpu_slot``, ``cache/packed_expert_store.py:334-395,557-597``), one
``GpuExpertSlot`` of six tensors per slot.  Here:

* the slots are one device allocation of ``num_slots`` expert blobs in the
  store's byte layout, so a miss is ONE host-to-device copy of one blob, on a
  copy stream, from pinned host memory (``ExpertSource``);
* slot memory never moves, so each slot's three TMA descriptors are encoded
  once; a layer's expert table (``hn_expert_ptrs`` rows + descriptors) is
  rebuilt on the host from the slot numbers of its resident experts and
  uploaded as one small copy when residency changes;
* the residency decisions are the library's host-side table (``hn_slots_*``,
  C++): eviction picks, among the slots whose expert the current call does not
  need, the least frequently used one (policy "lfu", the default: a use
  count per (layer, expert) that halves every ``decay_every`` uses of the
  cache, ties to the least recent -- the frequency idea of the reference's
  sticky-LFU tiers, ``cache/expert_cache.py``) or the least recently used
  one (policy "lru"); the copy stream waits for the compute stream before
  overwriting a slot, and the compute stream waits for the copy before the
  experts run.

``SlotCachedMoELayer`` is the routed MoE layer over such a cache: the
router runs on the device, the selected experts reach the host (one read,
as the reference's ``.unique().tolist()``), misses are loaded, and the
grouped kernel runs with the routing as given.  Not CUDA-graph capturable
(the residency decision needs the routing on the host).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn as nn

from . import _lib
from .packing import SLOT_TENSORS, BlobLayout, ExpertSlot


class ExpertSource:
    """Host copies of expert blobs (``blob(layer, expert) -> uint8 tensor``),
    pinned so the H2D copy is asynchronous.  ``from_blobs`` keeps given blobs;
    ``from_store`` reads a v2.0 store (``experts.bin`` + ``experts.idx``) into
    pinned memory."""

    def __init__(self, fetch: Callable[[int, int], torch.Tensor]):
        self.fetch = fetch

    def blob(self, layer: int, expert: int) -> torch.Tensor:
        return self.fetch(layer, expert)

    @classmethod
    def from_blobs(cls, blobs: Dict[Tuple[int, int], torch.Tensor]) -> "ExpertSource":
        pinned = {k: (v if v.is_pinned() else v.pin_memory()) for k, v in blobs.items()}
        return cls(lambda layer, expert: pinned[(layer, expert)])

    @classmethod
    def from_store(cls, index_path) -> "ExpertSource":
        import json
        from pathlib import Path
        import numpy as np
        index_path = Path(index_path)
        idx = json.loads(index_path.read_text())
        data = np.memmap(index_path.parent / "experts.bin", dtype=np.uint8, mode="r")
        blobs = {}
        for e in idx["experts"]:
            t = torch.from_numpy(np.array(data[e["offset"]:e["offset"] + e["size"]])).pin_memory()
            blobs[(e["layer_idx"], e["expert_idx"])] = t
        return cls(lambda layer, expert: blobs[(layer, expert)])


@dataclass
class CacheStats:
    hits: int = 0
    misses: int = 0
    h2d_bytes: int = 0
    evictions: int = 0
    per_layer_misses: Dict[int, int] = field(default_factory=dict)

    @property
    def hit_rate(self) -> float:
        n = self.hits + self.misses
        return self.hits / n if n else 0.0


class Residency:
    """Which (layer, expert) lives in which of ``num_slots`` slots: the
    library's host-side residency table (``hn_slots_*``, C++), with a Python
    mirror of the placement for lookups.

    ``admit(layer, experts)`` makes the given experts resident, evicting by
    the policy among the slots the call does not need, and returns the
    loads to make as (slot, key) pairs and the evicted keys; it never evicts
    an expert of the same call and refuses a call that needs more experts
    than there are slots (nothing changes then)."""

    def __init__(self, num_slots: int, policy: str = "lfu", decay_every: int = 4096):
        if num_slots < 1:
            raise ValueError("need at least one slot")
        if policy not in ("lfu", "lru"):
            raise ValueError("policy must be 'lfu' or 'lru'")
        self.S = num_slots
        self.policy = policy
        self._lib = _lib.load()
        self._h = self._lib.hn_slots_create(num_slots, 0 if policy == "lfu" else 1, decay_every)
        if not self._h:
            raise ValueError("hn_slots_create refused the arguments")
        self._loads = (ctypes.c_int32 * (2 * num_slots))()
        self._evicted = (ctypes.c_int32 * (2 * num_slots))()
        self._n_ev = ctypes.c_int(0)
        self._st = (ctypes.c_int64 * 3)()
        self.where: Dict[Tuple[int, int], int] = {}
        self.stats = CacheStats()

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h:
            self._lib.hn_slots_destroy(h)

    def admit(self, layer: int, experts: Sequence[int]):
        """Returns (loads [(slot, key)], evicted keys)."""
        es = [int(e) for e in experts]
        arr = (ctypes.c_int32 * max(1, len(es)))(*es)
        nl = self._lib.hn_slots_admit(self._h, layer, arr, len(es), self._loads, self._evicted,
                                      ctypes.byref(self._n_ev))
        if nl < 0:
            raise RuntimeError(f"slot budget {self.S} is smaller than the experts one call needs "
                               f"({len({e for e in es if e >= 0})})")
        evicted = [(self._evicted[2 * i], self._evicted[2 * i + 1]) for i in range(self._n_ev.value)]
        loads = [(self._loads[2 * i], (layer, self._loads[2 * i + 1])) for i in range(nl)]
        for key in evicted:
            self.where.pop(key, None)
        for slot, key in loads:
            self.where[key] = slot
        self._lib.hn_slots_stats(self._h, self._st)
        self.stats.hits, self.stats.misses, self.stats.evictions = self._st[0], self._st[1], self._st[2]
        if nl:
            self.stats.per_layer_misses[layer] = self.stats.per_layer_misses.get(layer, 0) + nl
        return loads, evicted


class SlotCache:
    """``num_slots`` device slots shared by every layer (the reference's per-layer
    caches sum to a slot budget too, e.g. 126 for Mixtral on 16 GB)."""

    def __init__(self, hidden_dim: int, intermediate_dim: int, num_layers: int, num_experts: int,
                 num_slots: int, source: ExpertSource, device="cuda", group_size: int = 128,
                 policy: str = "lfu", decay_every: int = 4096):
        self.res = Residency(num_slots, policy, decay_every)
        self.H, self.F, self.L, self.E, self.S = hidden_dim, intermediate_dim, num_layers, num_experts, num_slots
        self.group_size = group_size
        self.device = torch.device(device)
        self.source = source
        self.layout = BlobLayout.from_dims(hidden_dim, intermediate_dim, group_size)
        self.blob_bytes = self.layout.total_size
        # one allocation; slot s = bytes [s*blob, (s+1)*blob) (blob sizes keep 16-byte alignment)
        self.pool = torch.empty(num_slots, self.blob_bytes, dtype=torch.uint8, device=self.device)
        self.slots = [ExpertSlot(hidden_dim, intermediate_dim, group_size, self.device, blob=self.pool[s])
                      for s in range(num_slots)]
        self.slot_ptrs = [[getattr(sl, n).data_ptr() for n in SLOT_TENSORS] for sl in self.slots]
        self.per_map = int(_lib.load().hn_expert_maps_bytes())
        self.slot_maps = self._encode(self.slot_ptrs)  # bytes: per slot, its three descriptors
        self.copy_stream = torch.cuda.Stream(self.device)
        self.loaded = [torch.cuda.Event() for _ in range(num_slots)]
        # per layer: device table [E, 6] int64 and descriptors [E * per_map], host row -> slot
        self.tables = [torch.zeros(num_experts, 6, dtype=torch.int64, device=self.device) for _ in range(num_layers)]
        self.maps = [torch.zeros(num_experts * self.per_map + 64, dtype=torch.uint8, device=self.device)
                     for _ in range(num_layers)]
        self.row_slot = [[-1] * num_experts for _ in range(num_layers)]

    @property
    def stats(self) -> CacheStats:
        return self.res.stats

    @property
    def where(self) -> Dict[Tuple[int, int], int]:
        return self.res.where

    def _encode(self, rows: Sequence[Sequence[int]]) -> bytes:
        lib = _lib.load()
        n = len(rows)
        host_ptrs = (ctypes.c_uint64 * (6 * n))(*[p for r in rows for p in r])
        raw = ctypes.create_string_buffer(n * self.per_map + 64)
        aligned = (ctypes.addressof(raw) + 63) & ~63
        _lib.check(lib.hn_expert_maps_encode(ctypes.addressof(host_ptrs), n, self.H, self.F, aligned))
        return ctypes.string_at(aligned, n * self.per_map)

    def is_resident(self, layer: int, expert: int) -> bool:
        return (layer, expert) in self.where

    def ensure(self, layer: int, experts: Sequence[int]) -> None:
        """Make every expert in ``experts`` (of ``layer``) resident and point the
        layer's table at their slots; the current stream waits for the loads."""
        compute = torch.cuda.current_stream(self.device)
        keep = {(layer, int(e)) for e in experts}
        loads, evicted = self.res.admit(layer, experts)
        for lyr, e in evicted:
            self.row_slot[lyr][e] = -1
        if loads:
            # nothing queued on the compute stream may still read a slot being overwritten
            self.copy_stream.wait_stream(compute)
            with torch.cuda.stream(self.copy_stream):
                for s, (lyr, e) in loads:
                    src = self.source.blob(lyr, e)
                    if src.numel() != self.blob_bytes:
                        raise ValueError(f"blob of layer {lyr} expert {e} has {src.numel()} bytes, "
                                         f"expected {self.blob_bytes}")
                    self.pool[s].copy_(src, non_blocking=True)
                    self.loaded[s].record(self.copy_stream)
                    self.stats.h2d_bytes += self.blob_bytes
            for s, _ in loads:
                compute.wait_event(self.loaded[s])
        self._publish(layer, keep)

    def _publish(self, layer: int, keep: set) -> None:
        rows = self.row_slot[layer]
        changed = False
        for (lyr, e) in keep:
            s = self.where[(lyr, e)]
            if rows[e] != s:
                rows[e] = s
                changed = True
        if not changed:
            return
        # rows of non-resident experts point at slot 0: the routing never selects them
        slots = [s if s >= 0 else 0 for s in rows]
        ptrs = torch.tensor([self.slot_ptrs[s] for s in slots], dtype=torch.int64)
        blob = b"".join(self.slot_maps[s * self.per_map:(s + 1) * self.per_map] for s in slots)
        maps = torch.frombuffer(bytearray(blob), dtype=torch.uint8)
        self.tables[layer].copy_(ptrs, non_blocking=False)
        dst = self._maps_view(layer)
        dst.copy_(maps, non_blocking=False)

    def _maps_view(self, layer: int) -> torch.Tensor:
        buf = self.maps[layer]
        off = (-buf.data_ptr()) % 64  # descriptors must be 64-byte aligned
        return buf[off:off + self.E * self.per_map]

    def table(self, layer: int) -> Tuple[torch.Tensor, torch.Tensor]:
        return self.tables[layer], self._maps_view(layer)


class SlotCachedMoELayer(nn.Module):
    """Routed MoE layer whose experts live in a ``SlotCache``
    (``MixtralMoELayer.forward`` over the reference's cache, ``model/mixtral.py:259-370``).

    With the router's affinity bonus enabled, the bonus follows this layer's
    residency (``router.set_cache_checker``), as in the reference."""

    def __init__(self, router: nn.Module, cache: SlotCache, layer_idx: int, top_k: Optional[int] = None):
        super().__init__()
        self.router = router
        self.cache = cache
        self.layer_idx = layer_idx
        self.top_k = top_k
        if hasattr(router, "set_cache_checker"):
            router.set_cache_checker(lambda e: cache.is_resident(layer_idx, e))

    def route(self, x: torch.Tensor):
        """int32 top-k ids and float32 weights of x on the device."""
        from . import ops
        from .router import GLM4SigmoidRouter, TopKRouter
        if isinstance(self.router, TopKRouter):
            k = self.top_k if self.top_k is not None else self.router.experts_per_token
            bonus = self.router.bonus_vector(x.device)
            idx, w, _ = ops.moe_route(x, self.router.params(k, bonus), self.cache.E, keep_refs=(bonus,),
                                      want_logits=False)
        elif isinstance(self.router, GLM4SigmoidRouter):
            idx, w, _ = ops.moe_route(x, self.router.params(), self.cache.E, want_logits=False)
        else:
            raise TypeError("unsupported router type")
        return idx, w

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        from . import ops
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1]).contiguous()
        idx, w = self.route(x)
        needed = torch.unique(idx).tolist()  # the one host read of the step
        self.cache.ensure(self.layer_idx, [e for e in needed if e >= 0])
        table, maps = self.cache.table(self.layer_idx)
        out = ops.moe_experts(x, idx, w, table, maps, self.cache.E, self.cache.F)
        return out.view(shape)
