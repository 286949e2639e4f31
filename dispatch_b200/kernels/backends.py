"""Backend name -> GroupedMatmul (mirror of the reference's
src/dispatch/kernels/backends.py:10-35). There is exactly one backend, the
tcgen05 kernels; no multi-backend dispatch happens inside this package."""

from __future__ import annotations

from dispatch_b200.kernels.moe_forward import GroupedMatmul
from dispatch_b200.kernels.quantization import QuantizedGroupedMatmul

BACKENDS = ("b200",)
QUANTIZED_BACKEND = "quantized"
QUANTIZED_BACKENDS = ("b200",)


def resolve_backend(name: str) -> GroupedMatmul:
    if name not in BACKENDS:
        raise ValueError(f"unknown backend {name!r}; expected one of {BACKENDS}")
    from dispatch_b200.kernels.grouped_gemm import grouped_matmul  # noqa: PLC0415

    return grouped_matmul


def resolve_quantized_backend() -> QuantizedGroupedMatmul:
    from dispatch_b200.kernels.grouped_gemm_int8 import grouped_matmul_int8  # noqa: PLC0415

    return grouped_matmul_int8
