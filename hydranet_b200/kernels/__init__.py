"""sm_100a replacements for HydraNet's ``kernels`` package (INT4 expert path).

Exports the INT4 names of the reference's ``kernels/__init__.py:15-19``.
The INT8 / ``Int4Linear`` module helpers of that package are outside the
MoE hot path and are not provided.
"""

from .expert_mlp import ExpertMLPTriton, expert_mlp_int4
from .int4_gemm import int4_linear, expert_mlp_int4_fused, fused_silu_mul

__all__ = ["ExpertMLPTriton", "expert_mlp_int4", "int4_linear", "expert_mlp_int4_fused", "fused_silu_mul"]
