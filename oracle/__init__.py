"""CPU oracle for the INT4 MoE hot path (TEST INFRASTRUCTURE ONLY).

This package restates, in numpy, the reference algorithm of HydraNet's INT4
mixture-of-experts path: the offline packer, the dequantise-then-matmul expert
MLP, the two routers and the weighted top-k combine.  Every function cites the
reference file:line it follows.

It is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import
it.  The product path (``hydranet_b200``) never imports this package and fails
loudly when its CUDA library is missing.

Parity is pinned: ``tests/golden/make_golden.py`` ran the reference itself
(packer, ``TopKRouter``, ``GLM4SigmoidRouter``, ``MixtralMoELayer``) on seeded
inputs and committed its outputs under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks this oracle against them.
"""
