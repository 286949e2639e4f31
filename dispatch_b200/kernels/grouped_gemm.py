"""The ``GroupedMatmul`` backend on tcgen05 tensor cores (replaces the
reference's Triton src/dispatch/kernels/grouped_gemm.py).

``grouped_matmul(x, expert_weight, schedule)`` computes
out[rows of e] = x[rows of e] @ expert_weight[e].T with f32 accumulation; only
``schedule.group_offsets`` is read. Tiles are 128 x 256 x 64 with TMA loads and
a TMEM accumulator, so ``block_m`` does not constrain the kernel."""

from __future__ import annotations

import torch

from dispatch_b200 import _lib as L
from dispatch_b200.kernels.tile_schedule import TileSchedule, device_offsets

MIN_BLOCK_M = 1
TILE_M, TILE_N, TILE_K = 128, 256, 64


def _validated_output(x: torch.Tensor, expert_weight: torch.Tensor, schedule: TileSchedule) -> torch.Tensor:
    """Mirrors reference grouped_gemm.py:248-263 (same error substrings)."""
    if not (x.is_cuda and expert_weight.is_cuda):
        raise ValueError("the B200 grouped-GEMM kernels need CUDA tensors")
    if x.dtype != expert_weight.dtype:
        raise ValueError(f"dtype mismatch: x is {x.dtype}, expert_weight is {expert_weight.dtype}")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"dtype mismatch: the tensor-core kernels take bf16/f16, got {x.dtype}")
    if x.shape[1] != expert_weight.shape[2]:
        raise ValueError(f"K mismatch: x has {x.shape[1]}, expert_weight has {expert_weight.shape[2]}")
    if schedule.block_m < MIN_BLOCK_M:
        raise ValueError(f"schedule.block_m={schedule.block_m} must be positive")
    if len(schedule.group_offsets) != expert_weight.shape[0] + 1:
        raise ValueError("schedule.group_offsets does not match the number of experts")
    if schedule.group_offsets[-1] != x.shape[0]:
        raise ValueError(f"schedule covers {schedule.group_offsets[-1]} rows, x has {x.shape[0]}")
    return torch.empty((x.shape[0], expert_weight.shape[1]), device=x.device, dtype=x.dtype)


def grouped_matmul(x: torch.Tensor, expert_weight: torch.Tensor, schedule: TileSchedule) -> torch.Tensor:
    out = _validated_output(x, expert_weight, schedule)
    if x.shape[0] == 0:
        return out
    dev = L.require_cuda(x, expert_weight)
    x = x.contiguous()
    w = expert_weight.contiguous()
    offsets = device_offsets(schedule, dev)
    e, n, k = w.shape
    rc = L.lib().moe_grouped_gemm(
        x.data_ptr(), L.dt(x), x.shape[0], k, w.data_ptr(), L.dt(w), None, 0, e, n, offsets.data_ptr(),
        out.data_ptr(), n, L.status_word(dev).data_ptr(), L.stream_ptr(dev),
    )
    L.check(rc, "grouped_matmul")
    return out


# The reference also exports a persistent variant; the tcgen05 kernel is
# always persistent (one CTA per SM walking the tile list).
grouped_matmul_persistent = grouped_matmul
