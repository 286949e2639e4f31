"""int8 weight-only grouped GEMM (replaces the reference's Triton
src/dispatch/kernels/grouped_gemm_int8.py): int8 weight tiles arrive by TMA,
are converted exactly to the activation type in shared memory by two
dequantiser warps, feed bf16/f16 tcgen05 MMAs, and the per-output-channel
scale multiplies the f32 accumulator in the epilogue."""

from __future__ import annotations

import torch

from dispatch_b200 import _lib as L
from dispatch_b200.kernels.quantization import QuantizedTensor
from dispatch_b200.kernels.tile_schedule import TileSchedule, device_offsets


def _validated_quantized_output(x: torch.Tensor, qweight: QuantizedTensor, schedule: TileSchedule) -> torch.Tensor:
    """Mirrors reference grouped_gemm_int8.py:179-196 (same error substrings);
    bf16 scales are accepted as well as f32."""
    if not (x.is_cuda and qweight.data.is_cuda and qweight.scale.is_cuda):
        raise ValueError("the B200 int8 grouped-GEMM kernel needs CUDA tensors")
    if qweight.data.dtype != torch.int8:
        raise ValueError(f"expected int8 weight data, got {qweight.data.dtype}")
    if qweight.scale.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError(f"expected float32 or bfloat16 scales, got {qweight.scale.dtype}")
    if qweight.scale.shape != qweight.data.shape[:2]:
        raise ValueError(f"scale shape {tuple(qweight.scale.shape)} does not match weight (E, N)")
    if x.shape[1] != qweight.data.shape[2]:
        raise ValueError(f"K mismatch: x has {x.shape[1]}, qweight has {qweight.data.shape[2]}")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"dtype mismatch: activations must be bf16/f16, got {x.dtype}")
    if schedule.block_m < 1:
        raise ValueError(f"schedule.block_m={schedule.block_m} must be positive")
    return torch.empty((x.shape[0], qweight.data.shape[1]), device=x.device, dtype=x.dtype)


def grouped_matmul_int8(x: torch.Tensor, qweight: QuantizedTensor, schedule: TileSchedule) -> torch.Tensor:
    out = _validated_quantized_output(x, qweight, schedule)
    if x.shape[0] == 0:
        return out
    dev = L.require_cuda(x, qweight.data, qweight.scale)
    x = x.contiguous()
    q = qweight.data.contiguous()
    s = qweight.scale.contiguous()
    offsets = device_offsets(schedule, dev)
    e, n, k = q.shape
    rc = L.lib().moe_grouped_gemm(
        x.data_ptr(), L.dt(x), x.shape[0], k, q.data_ptr(), L.DT_I8, s.data_ptr(), L.dt(s), e, n,
        offsets.data_ptr(), out.data_ptr(), n, L.status_word(dev).data_ptr(), L.stream_ptr(dev),
    )
    L.check(rc, "grouped_matmul_int8")
    return out
