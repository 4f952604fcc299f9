"""Drop-in for HydraNet's ``kernels/int4_linear.py`` on sm_100a: the INT4
``Int4Linear`` module for non-expert weights, ``convert_model_to_int4`` and
``estimate_int4_memory``.

The forward runs ``hn_int4_linear`` (the tcgen05 engine behind
``kernels.int4_gemm.int4_linear``) and then adds the float16 bias as the
reference does (``:164-168``).  The engine implements group size 128 only;
other group sizes raise from the library, and ``convert_model_to_int4``
leaves such layers in floating point (it reports them as skipped).

``quantize_weight`` keeps the reference's own arithmetic, which is not the
expert packer's: the group absmax is clamped to 1e-8, the integer is
``round_half_even(w / absmax * 7)`` with both operations rounded in the
weight dtype, and the stored scale is ``absmax / 7`` cast to float16
(``:69-103``).  It is offline conversion, so it runs as tensor operations on
whatever device the weight is on; the same steps in the same order are what
make the result bit-identical.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from .int4_gemm import int4_linear

SUPPORTED_GROUP_SIZE = 128


class Int4Linear(nn.Module):
    """``y = x @ W.T + b`` with W stored as INT4 nibbles and per-group float16
    scales (``kernels/int4_linear.py:18-175``).

    Buffers: ``weight_packed`` uint8 [out, in/2] (even column in the low
    nibble), ``weight_scale`` float16 [out, in/group_size]; ``bias`` a float16
    parameter or None.
    """

    def __init__(self, in_features: int, out_features: int, bias: bool = True, group_size: int = 128,
                 device: Optional[torch.device] = None):
        super().__init__()
        assert in_features % group_size == 0, \
            f"in_features ({in_features}) must be divisible by group_size ({group_size})"
        assert in_features % 2 == 0, f"in_features ({in_features}) must be even for INT4 packing"
        self.in_features = in_features
        self.out_features = out_features
        self.group_size = group_size
        self.register_buffer("weight_packed",
                             torch.zeros(out_features, in_features // 2, dtype=torch.uint8, device=device))
        self.register_buffer("weight_scale",
                             torch.ones(out_features, in_features // group_size, dtype=torch.float16,
                                        device=device))
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features, dtype=torch.float16, device=device))
        else:
            self.register_parameter("bias", None)

    @staticmethod
    def quantize_weight(weight: torch.Tensor, group_size: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
        """(packed uint8 [out, in/2], scale float16 [out, in/group_size]) of a
        float weight [out, in] (``kernels/int4_linear.py:69-103``)."""
        rows, cols = weight.shape
        assert cols % group_size == 0
        grp = weight.reshape(rows, cols // group_size, group_size)
        peak = grp.abs().amax(dim=-1, keepdim=True).clamp(min=1e-8)
        scale = (peak / 7.0).to(torch.float16).squeeze(-1)
        level = torch.round(grp / peak * 7.0).clamp(-8, 7).to(torch.int8)
        nib = (level + 8).to(torch.uint8).reshape(rows, cols)
        packed = nib[:, 0::2] | (nib[:, 1::2] << 4)
        return packed, scale

    @classmethod
    def from_float(cls, linear: nn.Linear, group_size: int = 128,
                   device: Optional[torch.device] = None) -> "Int4Linear":
        """Quantise an ``nn.Linear`` (``kernels/int4_linear.py:105-150``).  When
        ``in_features`` is not a multiple of ``group_size`` the group size
        falls back to 64, then 32, as in the reference."""
        device = device or linear.weight.device
        n_in = linear.in_features
        if n_in % group_size != 0:
            group_size = 64
            if n_in % group_size != 0:
                group_size = 32
                if n_in % group_size != 0:
                    raise ValueError(f"in_features ({n_in}) must be divisible by a power-of-2 group size")
        mod = cls(n_in, linear.out_features, bias=linear.bias is not None, group_size=group_size, device=device)
        packed, scale = cls.quantize_weight(linear.weight.data, group_size)
        mod.weight_packed.copy_(packed)
        mod.weight_scale.copy_(scale)
        if linear.bias is not None:
            mod.bias.data.copy_(linear.bias.data.to(torch.float16))
        return mod

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        out = int4_linear(x, self.weight_packed, self.weight_scale, self.group_size)
        if self.bias is not None:
            out = out + self.bias
        return out

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, dtype=int4, group_size={self.group_size}")


def convert_model_to_int4(model: nn.Module, skip_layers: Optional[list[str]] = None, group_size: int = 128,
                          device: Optional[torch.device] = None) -> nn.Module:
    """Replace the model's ``nn.Linear`` layers by ``Int4Linear`` in place
    (``kernels/int4_linear.py:178-236``): names containing a ``skip_layers``
    pattern are kept, odd ``in_features`` are kept, the group size halves
    until it divides ``in_features``.  Layers whose group size the sm_100a
    engine does not implement (anything but 128) are kept too."""
    skip_layers = skip_layers or []
    converted = skipped = 0
    for name, module in list(model.named_modules()):
        if any(pat in name for pat in skip_layers):
            skipped += 1
            continue
        if not isinstance(module, nn.Linear):
            continue
        if module.in_features % 2 != 0:
            print(f"  Skipping {name}: in_features ({module.in_features}) not even")
            skipped += 1
            continue
        gs = group_size
        while gs > 1 and module.in_features % gs != 0:
            gs //= 2
        if gs < 32:
            print(f"  Skipping {name}: no compatible group size for in_features={module.in_features}")
            skipped += 1
            continue
        if gs != SUPPORTED_GROUP_SIZE:
            print(f"  Skipping {name}: group size {gs} (the sm_100a kernels implement {SUPPORTED_GROUP_SIZE})")
            skipped += 1
            continue
        parent_name, _, attr = name.rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else model
        setattr(parent, attr, Int4Linear.from_float(module, group_size=gs, device=device))
        converted += 1
    print(f"  Converted {converted} layers to INT4, skipped {skipped}")
    return model


def estimate_int4_memory(model: nn.Module, group_size: int = 128) -> dict:
    """fp16 vs INT4 footprint of the model's parameters in MB
    (``kernels/int4_linear.py:239-269``): 2-D parameters as INT4 nibbles plus a
    float16 scale per group of each row, everything else as float16."""
    fp16_bytes = int4_bytes = 0
    for _, param in model.named_parameters():
        n = param.numel()
        fp16_bytes += 2 * n
        if param.dim() == 2:
            rows, cols = param.shape
            int4_bytes += n // 2 + rows * (-(-cols // group_size)) * 2
        else:
            int4_bytes += 2 * n
    return {"fp16_mb": fp16_bytes / 1e6, "int4_mb": int4_bytes / 1e6, "savings_mb": (fp16_bytes - int4_bytes) / 1e6}


__all__ = ["Int4Linear", "convert_model_to_int4", "estimate_int4_memory"]
