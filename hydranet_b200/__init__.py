"""hydranet_b200: the INT4 mixture-of-experts hot path of HydraNet on B200 (sm_100a).

The compute lives in ``libhydranet_b200.so`` (C ABI: ``include/hydranet_b200.h``);
this package holds the host-side mirror of the reference's interfaces:

* ``hydranet_b200.kernels``  -- ``kernels/int4_gemm.py``, ``kernels/int4_expert_mlp.py``
  and ``kernels/expert_mlp.py`` drop-ins;
* ``hydranet_b200.router``   -- ``TopKRouter`` / ``GLM4SigmoidRouter``;
* ``hydranet_b200.moe``      -- one-launch-per-phase grouped MoE layer;
* ``hydranet_b200.packing``  -- the packed expert format on the GPU;
* ``hydranet_b200.ep``       -- expert parallelism over NCCL all-to-all.

There is no CPU fallback: ops raise if the CUDA library is missing.
"""

__version__ = "0.1.0"
