"""Residency decisions of the over-budget slot cache on CPU (no device
memory involved): the eviction policies, the refusal of a call that needs
more experts than there are slots, and the hit rates of LFU and LRU on a
Zipf-skewed decode stream shaped like config 3 (32 layers x 8 experts,
126 slots, top-2)."""

import numpy as np
import pytest

from hydranet_b200.slot_cache import Residency


def test_lru_evicts_least_recent_and_keeps_the_call():
    r = Residency(3, policy="lru")
    assert [s for s, _ in r.admit(0, [0, 1, 2])[0]] == [0, 1, 2]
    r.admit(0, [0])                     # expert 1 is now the least recent
    loads, evicted = r.admit(0, [3])
    assert evicted == [(0, 1)] and loads == [(1, (0, 3))]
    loads, evicted = r.admit(0, [2, 4])  # 2 is needed: the victim is 0 (older than 3)
    assert (0, 2) not in evicted and evicted == [(0, 0)]
    assert r.stats.hits == 2 and r.stats.misses == 5


def test_lfu_evicts_least_frequent():
    r = Residency(2, policy="lfu")
    for _ in range(5):
        r.admit(1, [7])
    r.admit(1, [8])
    _, evicted = r.admit(1, [9])        # 8 was used once, 7 five times
    assert evicted == [(1, 8)]


def test_call_larger_than_the_budget_is_refused():
    r = Residency(4)
    with pytest.raises(RuntimeError):
        r.admit(0, [0, 1, 2, 3, 4])
    assert r.stats.misses == 0          # nothing was admitted


def _stream_hit_rate(policy, seed=3):
    rng = np.random.default_rng(seed)
    L, E, k = 32, 8, 2
    bias = [-1.1 * np.log(rng.permutation(E) + 1) for _ in range(L)]
    r = Residency(126, policy=policy)
    warm = None
    for tok in range(640):
        if tok == 128:
            warm = (r.stats.hits, r.stats.misses)
        for li in range(L):
            logits = rng.standard_normal(E) * 1.3 + bias[li]
            r.admit(li, np.argsort(-logits)[:k].tolist())
    h, m = r.stats.hits - warm[0], r.stats.misses - warm[1]
    return h / (h + m)


def test_lfu_beats_lru_on_a_zipf_stream():
    lfu, lru = _stream_hit_rate("lfu"), _stream_hit_rate("lru")
    assert lfu > lru + 0.05, (lfu, lru)


def test_native_table_lookup_and_refusal_through_the_c_abi():
    """The C ABI of the residency table directly: loads, lookups, duplicates
    and -1 ids, and a too-large call that changes nothing."""
    import ctypes
    from hydranet_b200 import _lib
    lib = _lib.load()
    h = lib.hn_slots_create(2, 1, 4096)  # LRU
    try:
        loads, ev, nev = (ctypes.c_int32 * 4)(), (ctypes.c_int32 * 4)(), ctypes.c_int(0)
        ids = (ctypes.c_int32 * 4)(5, -1, 5, 3)
        assert lib.hn_slots_admit(h, 2, ids, 4, loads, ev, ctypes.byref(nev)) == 2 and nev.value == 0
        assert list(loads) == [0, 3, 1, 5]          # ascending ids: 3 -> slot 0, 5 -> slot 1
        assert lib.hn_slots_lookup(h, 2, 5) == 1 and lib.hn_slots_lookup(h, 1, 5) == -1
        big = (ctypes.c_int32 * 3)(7, 8, 9)
        assert lib.hn_slots_admit(h, 2, big, 3, loads, ev, ctypes.byref(nev)) == -_lib.HN_ERR_WORKSPACE
        st = (ctypes.c_int64 * 3)()
        lib.hn_slots_stats(h, st)
        assert list(st) == [0, 2, 0]
        assert lib.hn_slots_create(0, 0, 1) is None
    finally:
        lib.hn_slots_destroy(h)
