"""Weight-only int8 quantisation (mirror of the reference's
src/dispatch/kernels/quantization.py). The quantiser runs as a CUDA kernel
(bit-exact with the reference's f32 arithmetic); the expert kernels consume
the int8 data plus per-output-channel scales (f32, or bf16 as the BASELINE int8
config asks) and apply the scale once after the K loop."""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass

import torch

from dispatch_b200 import _lib as L
from dispatch_b200.kernels.tile_schedule import TileSchedule

INT8_MAX = 127


@dataclass(frozen=True)
class QuantizedTensor:
    """An (E, N, K) weight tensor quantised to int8, one scale per expert per
    output channel (E, N) (reference quantization.py:23-28)."""

    data: torch.Tensor
    scale: torch.Tensor


def quantize_per_channel_int8(weight: torch.Tensor, *, scale_dtype: torch.dtype = torch.float32) -> QuantizedTensor:
    """scale = absmax/127 in f32 (1.0 for an all-zero channel), q =
    clamp(round_half_even(w / scale), -127, 127) (reference quantization.py:31-50).
    ``scale_dtype=torch.bfloat16`` stores the f32 scale rounded to bf16."""
    dev = L.require_cuda(weight, what="quantize_per_channel_int8")
    w = weight.detach().contiguous()
    if w.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        w = w.float()
    k = w.shape[-1]
    rows = w.numel() // max(k, 1)
    q = torch.empty(w.shape, dtype=torch.int8, device=dev)
    scale = torch.empty(w.shape[:-1], dtype=scale_dtype, device=dev)
    rc = L.lib().moe_quantize_int8(w.data_ptr(), L.dt(w), rows, k, q.data_ptr(), scale.data_ptr(), L.dt(scale),
                                   L.stream_ptr(dev))
    L.check(rc, "quantize_per_channel_int8")
    return QuantizedTensor(data=q, scale=scale)


def dequantize_int8(qtensor: QuantizedTensor) -> torch.Tensor:
    """q * scale in f32 (reference quantization.py:53-54); a test helper."""
    return qtensor.data.to(torch.float32) * qtensor.scale.float().unsqueeze(-1)


@dataclass(frozen=True)
class QuantizedStackedExpertWeights:
    gate: QuantizedTensor
    up: QuantizedTensor
    down: QuantizedTensor

    @property
    def num_experts(self) -> int:
        return int(self.gate.data.shape[0])


QuantizedGroupedMatmul = Callable[[torch.Tensor, QuantizedTensor, TileSchedule], torch.Tensor]


def quantize_stacked_weights(weights, *, scale_dtype: torch.dtype = torch.float32) -> QuantizedStackedExpertWeights:
    return QuantizedStackedExpertWeights(
        gate=quantize_per_channel_int8(weights.gate, scale_dtype=scale_dtype),
        up=quantize_per_channel_int8(weights.up, scale_dtype=scale_dtype),
        down=quantize_per_channel_int8(weights.down, scale_dtype=scale_dtype),
    )


def grouped_moe_routed_quantized(
    x: torch.Tensor,
    topk_idx: torch.Tensor,
    topk_weight: torch.Tensor,
    weights: QuantizedStackedExpertWeights,
    matmul: QuantizedGroupedMatmul | None = None,
    *,
    block_m: int = 16,
    shared=None,
) -> torch.Tensor:
    """Reference: quantization.py:92-107. Runs the fused int8 path (two tcgen05
    launches with in-smem dequantisation) whatever ``matmul`` is given."""
    from dispatch_b200.kernels.moe_forward import _routed_forward  # noqa: PLC0415

    _check_matmul(matmul)
    if block_m <= 0:
        raise ValueError(f"block_m must be positive, got {block_m}")
    return _routed_forward(x, topk_idx, topk_weight, weights, shared)


def _check_matmul(matmul) -> None:
    from dispatch_b200.kernels.grouped_gemm import grouped_matmul  # noqa: PLC0415
    from dispatch_b200.kernels.grouped_gemm_int8 import grouped_matmul_int8  # noqa: PLC0415

    if matmul is not None and matmul not in (grouped_matmul, grouped_matmul_int8):
        raise ValueError("the B200 layer path runs its own fused kernels; pass matmul=None or the b200 backend")


def stacked_weights_nbytes(weights) -> int:
    return sum(t.element_size() * t.nelement() for t in (weights.gate, weights.up, weights.down))


def quantized_stacked_weights_nbytes(weights: QuantizedStackedExpertWeights) -> int:
    total = 0
    for qt in (weights.gate, weights.up, weights.down):
        total += qt.data.element_size() * qt.data.nelement()
        total += qt.scale.element_size() * qt.scale.nelement()
    return total
