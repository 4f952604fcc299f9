"""Seeded synthetic MoE workloads (no checkpoints or datasets exist offline).

Host generation uses numpy's PCG64 generator, whose float32 normal stream is
reproducible across machines for a given numpy version, so test fixtures can
store a seed instead of megabytes of weights.  Large workloads are generated
on the GPU instead (``device_moe_layer``), where only the seed matters.

Distributions follow the synthetic configurations the reference is measured
on: weights ~ N(0, 0.02) in float32 before INT4 packing (the reference's own
synthetic tests use the same scale, e.g. ``tests/test_synthetic_smoke.py:96-118``),
activations ~ N(0, 1).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

WEIGHT_STD = 0.02


def host_normal(seed: int, shape, std: float = 1.0) -> np.ndarray:
    """float32 N(0, std^2) samples from a seeded PCG64 stream."""
    a = np.random.default_rng(seed).standard_normal(shape, dtype=np.float32)
    if std != 1.0:
        a = a * np.float32(std)
    return a


@dataclass(frozen=True)
class MoEShape:
    hidden: int
    ffn: int
    experts: int
    top_k: int
    group_size: int = 128


def expert_seed(base: int, expert: int, which: int) -> int:
    """Seed of one projection (0 gate, 1 up, 2 down) of one expert."""
    return base * 1_000_003 + expert * 7 + which + 1


def host_expert_weights(base_seed: int, shape: MoEShape, expert: int):
    """float32 (gate [F,H], up [F,H], down [H,F]) of one expert, ~N(0, 0.02)."""
    H, F = shape.hidden, shape.ffn
    return (host_normal(expert_seed(base_seed, expert, 0), (F, H), WEIGHT_STD),
            host_normal(expert_seed(base_seed, expert, 1), (F, H), WEIGHT_STD),
            host_normal(expert_seed(base_seed, expert, 2), (H, F), WEIGHT_STD))


def host_router_weight(base_seed: int, shape: MoEShape) -> np.ndarray:
    return host_normal(base_seed * 1_000_003 + 999_983, (shape.experts, shape.hidden), WEIGHT_STD)


def host_activations(base_seed: int, tokens: int, hidden: int) -> np.ndarray:
    return host_normal(base_seed * 1_000_003 + 499_979, (tokens, hidden), 1.0)


def host_correction_bias(base_seed: int, experts: int, std: float = 0.1) -> np.ndarray:
    return host_normal(base_seed * 1_000_003 + 777_767, (experts,), std)


def device_experts(seed: int, shape: MoEShape, device="cuda"):
    """Experts generated on the GPU (seeded torch CUDA RNG, ~N(0, 0.02)) and packed
    there by the CUDA packer.  Returns a list of ``packing.ExpertSlot``."""
    import torch
    from .packing import quantize_expert
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    H, F = shape.hidden, shape.ffn
    slots = []
    for _ in range(shape.experts):
        g = torch.randn(F, H, generator=gen, device=device).mul_(WEIGHT_STD)
        u = torch.randn(F, H, generator=gen, device=device).mul_(WEIGHT_STD)
        d = torch.randn(H, F, generator=gen, device=device).mul_(WEIGHT_STD)
        slots.append(quantize_expert(g, u, d, shape.group_size))
        del g, u, d
    return slots
