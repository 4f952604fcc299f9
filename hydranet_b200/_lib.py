"""ctypes binding of ``libhydranet_b200.so`` (the C ABI in ``include/hydranet_b200.h``).

There is no fallback: if the library is missing or fails to load, every op
raises.  Tensors are passed as raw device pointers; kernels run on
``torch.cuda.current_stream()`` so the reference's stream ordering (slot
``ready_event`` waits, ``cache/packed_expert_store.py:323-331``) still holds.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libhydranet_b200.so"

HN_OK, HN_ERR_INVALID, HN_ERR_UNSUPPORTED, HN_ERR_CUDA, HN_ERR_WORKSPACE = range(5)
HN_DTYPE_F32, HN_DTYPE_F16, HN_DTYPE_BF16 = range(3)
HN_ROUTER_SOFTMAX_TOPK, HN_ROUTER_SIGMOID_TOPK = range(2)
HN_ENGINE_AUTO, HN_ENGINE_TCGEN05 = range(2)

c_void_p, c_int, c_int64, c_size_t, c_float = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_float


class ExpertPtrs(ctypes.Structure):
    """``hn_expert_ptrs``: device pointers of one expert's six packed tensors."""
    _fields_ = [("gate_packed", c_void_p), ("gate_scales", c_void_p), ("up_packed", c_void_p),
                ("up_scales", c_void_p), ("down_packed", c_void_p), ("down_scales", c_void_p)]


class RouterParams(ctypes.Structure):
    """``hn_router_params``."""
    _fields_ = [("kind", c_int), ("top_k", c_int), ("weight", c_void_p), ("weight_dtype", c_int),
                ("logits_in_act_dtype", c_int), ("affinity_bonus", c_void_p), ("entropy_threshold", c_float),
                ("correction_bias", c_void_p), ("norm_topk_prob", c_int), ("routed_scaling_factor", c_float),
                ("n_group", c_int), ("topk_group", c_int)]


# name -> (restype, argtypes)
SIGNATURES = {
    "hn_abi_version": (c_int, []),
    "hn_set_sm_limit": (c_int, [c_int]),
    "hn_slots_create": (c_void_p, [c_int, c_int, c_int64]),
    "hn_slots_destroy": (None, [c_void_p]),
    "hn_slots_admit": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "hn_slots_lookup": (c_int, [c_void_p, c_int, c_int]),
    "hn_slots_stats": (c_int, [c_void_p, c_void_p]),
    "hn_last_error": (ctypes.c_char_p, []),
    "hn_device_sm_count": (c_int, [c_int]),
    "hn_quantize_int4": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int, c_void_p, c_void_p, c_void_p]),
    "hn_unpack_int4": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p]),
    "hn_dequant_int4": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int, c_void_p, c_void_p]),
    "hn_silu_mul": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p]),
    "hn_int4_linear_workspace_size": (c_size_t, [c_int64, c_int64, c_int64]),
    "hn_int4_linear": (c_int, [c_void_p, c_int64, c_int, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int,
                               c_void_p, c_int64, c_void_p, c_size_t, c_void_p]),
    "hn_expert_mlp_workspace_size": (c_size_t, [c_int64, c_int64, c_int64]),
    "hn_expert_mlp_int4": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                                   c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_size_t, c_void_p]),
    "hn_moe_workspace_size": (c_size_t, [c_int64, c_int64, c_int64, c_int64, c_int]),
    "hn_moe_experts_workspace_size_expected": (c_size_t, [c_int64, c_int64, c_int64, c_int64, c_int, c_int64]),
    "hn_moe_experts_int4_expected": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int64, c_int64, c_int, c_void_p,
                                             c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_size_t,
                                             c_void_p]),
    "hn_moe_layer_launches": (c_int, [c_int64, c_int64, c_int64, c_int64, c_int]),
    "hn_expert_maps_bytes": (c_size_t, []),
    "hn_expert_maps_encode": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p]),
    "hn_moe_layer_int4": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int64, c_int64, ctypes.POINTER(RouterParams),
                                  c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
                                  c_void_p]),
    "hn_moe_layer_int4_phase": (c_int, [c_int, c_void_p, c_int, c_int64, c_int64, c_int64, c_int64,
                                        ctypes.POINTER(RouterParams), c_void_p, c_void_p, c_void_p, c_void_p,
                                        c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "hn_moe_experts_int4": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int64, c_int64, c_int, c_void_p, c_void_p,
                                    c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "hn_moe_route": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int64, ctypes.POINTER(RouterParams), c_void_p,
                             c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "hn_workspace_error": (c_int, [c_void_p, c_size_t, ctypes.POINTER(c_int), c_void_p]),
    "hn_int4_linear_static": (c_int, [c_void_p, c_int64, c_int, c_int64, c_int64, c_void_p, c_void_p, c_int64,
                                      c_int, c_void_p, c_int64, c_void_p]),
    "hn_selftest_wait_timeout": (c_int, [c_void_p, c_size_t, c_int, c_void_p]),
    "hn_set_decode_engine": (c_int, [c_int]),
    "hn_ep_row_bytes": (c_size_t, [c_int64, c_int]),
    "hn_ep_pack": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int, c_void_p, c_void_p, c_int64, c_int, c_void_p,
                           c_void_p]),
    "hn_ep_unpack": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "hn_ep_combine": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int, c_void_p, c_int64, c_int, c_void_p,
                              c_void_p]),
    "hn_int4_linear_static_scratch_size": (c_size_t, [c_int64, c_int64, c_int64]),
    "hn_int4_linear_static_error": (c_int, [ctypes.POINTER(c_int), c_void_p]),
}

_lib = None
_lock = threading.Lock()


class HydraNetError(RuntimeError):
    """A C-ABI call returned an error status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[hn status {code}] {msg}")
        self.code = code


def load():
    """Load the CUDA C-ABI library (raises if it is missing: there is no CPU fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m hydranet_b200.build` "
                                   "(nvcc, sm_100a). hydranet_b200 has no CPU fallback.")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            if lib.hn_abi_version() != 3:
                raise RuntimeError("libhydranet_b200.so ABI version mismatch")
            _lib = lib
    return _lib


def check(rc: int):
    if rc != HN_OK:
        msg = load().hn_last_error()
        raise HydraNetError(rc, msg.decode() if msg else "unknown error")


# --------------------------------------------------------------------------
# torch helpers (torch is imported lazily so the symbol checks run without it)
# --------------------------------------------------------------------------

def dtype_code(dt) -> int:
    import torch
    if dt == torch.bfloat16:
        return HN_DTYPE_BF16
    if dt == torch.float16:
        return HN_DTYPE_F16
    if dt == torch.float32:
        return HN_DTYPE_F32
    raise TypeError(f"unsupported dtype {dt}")


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device=None) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("hydranet_b200 ops take CUDA tensors (no CPU fallback)")


class DeviceError(HydraNetError):
    """A bounded device wait timed out, or caller-given routing named an
    expert outside the table, in an earlier call on this stream: the results
    of that call (and of calls issued before this one noticed) are invalid."""


class _Workspaces:
    """One zero-filled workspace per (device, stream), grown on demand.

    The library keeps a workspace's counter section zero between calls, so one
    buffer serves every call shape on its stream (see the header comment of
    ``include/hydranet_b200.h``).  Each workspace also names a pinned host
    word (bytes 8..15) into which the kernels copy any device error they
    record; ``get`` reads that word -- a plain host read, no synchronisation --
    and raises ``DeviceError`` for an error an earlier call left there.
    """

    def __init__(self):
        self._ws = {}
        self._mirror = {}
        self._lock = threading.Lock()

    def get(self, nbytes: int, device):
        import torch
        dev = torch.device(device)
        key = (dev.index if dev.index is not None else torch.cuda.current_device(), stream_ptr(dev))
        with self._lock:
            buf = self._ws.get(key)
            mirror = self._mirror.get(key)
            if mirror is not None and int(mirror[0]) != 0:
                code = int(mirror[0])
                mirror.zero_()
                buf[:4].zero_()  # the device word, cleared in stream order
                raise DeviceError(code, f"device error {code} ({DEVICE_ERRORS.get(code, 'unknown')}) recorded by "
                                        "an earlier call on this stream; its results are invalid")
            if buf is None or buf.numel() < nbytes:
                if torch.cuda.is_current_stream_capturing():
                    # a buffer made during capture is only zeroed when the graph
                    # replays, so eager calls would find its counters unset
                    raise RuntimeError(
                        f"hydranet_b200: the workspace of this stream needs {nbytes} bytes; make one call of "
                        "the same shape on this stream outside CUDA-graph capture before capturing")
                size = max(nbytes, 1 << 20)
                if buf is not None:
                    size = max(size, buf.numel() * 2)
                buf = torch.zeros(size, dtype=torch.uint8, device=dev)
                if mirror is None:
                    mirror = torch.zeros(1, dtype=torch.int32).pin_memory()
                    self._mirror[key] = mirror
                buf[8:16].view(torch.int64).fill_(mirror.data_ptr())
                self._ws[key] = buf
            return buf

    def all(self):
        return list(self._ws.values())

    def clear_mirror(self, ws):
        for key, buf in self._ws.items():
            if buf.data_ptr() == ws.data_ptr():
                self._mirror[key].zero_()


DEVICE_ERRORS = {1: "a bounded device wait timed out", 2: "a routing index outside [0, E)"}

workspaces = _Workspaces()


def workspace_error(ws) -> int:
    """Read and clear a workspace's device error word (synchronises its stream)."""
    code = c_int(0)
    check(load().hn_workspace_error(ws.data_ptr(), ws.numel(), ctypes.byref(code), stream_ptr(ws.device)))
    workspaces.clear_mirror(ws)
    return code.value
