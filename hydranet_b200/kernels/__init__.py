"""sm_100a replacements for HydraNet's ``kernels`` package (INT4 paths).

Exports the INT4 names of the reference's ``kernels/__init__.py:15-19``:
the expert kernels and the non-expert ``Int4Linear`` module helpers.  The
INT8 module helpers of that package are outside the INT4 hot path and are
not provided.
"""

from .expert_mlp import ExpertMLPTriton, expert_mlp_int4
from .int4_gemm import int4_linear, expert_mlp_int4_fused, fused_silu_mul
from .int4_linear import Int4Linear, convert_model_to_int4, estimate_int4_memory

__all__ = ["ExpertMLPTriton", "expert_mlp_int4", "int4_linear", "expert_mlp_int4_fused", "fused_silu_mul",
           "Int4Linear", "convert_model_to_int4", "estimate_int4_memory"]
