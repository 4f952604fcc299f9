"""Shared helpers of the GPU parity tests (builds inputs, runs the oracle)."""

from __future__ import annotations

import numpy as np
import torch

from hydranet_b200 import synth
from hydranet_b200.packing import ExpertSlot, ExpertTable, quantize_expert
from oracle import int4_ref as R

DT = {"bf16": torch.bfloat16, "f16": torch.float16}


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def to_np32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def host_moe(shape: synth.MoEShape, seed: int, device="cuda"):
    """Host-generated experts packed by the ORACLE packer, uploaded into slots."""
    packed, slots = [], []
    for e in range(shape.experts):
        g, u, d = synth.host_expert_weights(seed, shape, e)
        t = [*R.quantize_tensor(g), *R.quantize_tensor(u), *R.quantize_tensor(d)]
        packed.append(t)
        s = ExpertSlot(shape.hidden, shape.ffn, 128, device)
        for dst, src in zip(s.tensors(), t):
            dst.copy_(torch.from_numpy(src).view(dst.dtype) if src.dtype == np.float16 else torch.from_numpy(src))
        slots.append(s)
    return ExpertTable(slots), packed


def device_moe(shape: synth.MoEShape, seed: int, device="cuda"):
    """Device-generated experts (torch CUDA RNG) packed by the GPU packer; host copies for the oracle."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    slots, packed = [], []
    H, F = shape.hidden, shape.ffn
    for e in range(shape.experts):
        g = torch.randn(F, H, generator=gen, device=device) * synth.WEIGHT_STD
        u = torch.randn(F, H, generator=gen, device=device) * synth.WEIGHT_STD
        d = torch.randn(H, F, generator=gen, device=device) * synth.WEIGHT_STD
        s = quantize_expert(g, u, d)
        slots.append(s)
        packed.append([t.cpu().numpy() for t in s.tensors()])
        del g, u, d
    return ExpertTable(slots), packed


def oracle_experts(packed, touched=None):
    """float32 dequantised oracle experts, built in threads (numpy releases the GIL)."""
    from concurrent.futures import ThreadPoolExecutor
    ids = list(range(len(packed))) if touched is None else sorted(set(int(e) for e in touched))
    with ThreadPoolExecutor(max_workers=8) as ex:
        built = list(ex.map(lambda e: R.DequantExpert.from_packed(*packed[e]), ids))
    return dict(zip(ids, built))


def act(x_np: np.ndarray, dtype: str, device="cuda") -> torch.Tensor:
    return torch.from_numpy(x_np).to(device=device, dtype=DT[dtype])
