"""B200-native (sm_100a) MoE-layer hot path with dispatch's call surface.

``dispatch_b200.kernels`` mirrors ``dispatch.kernels`` (bsreecharanreddy/dispatch)
module by module; every op runs hand-written CUDA from ``libmoe_b200.so``
through its C ABI (``include/moe_b200.h``). There is no CPU or Triton fallback.
"""

__version__ = "0.1.0"
