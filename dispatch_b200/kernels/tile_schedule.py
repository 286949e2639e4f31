"""Host-side tile schedule, kept for the ``GroupedMatmul`` contract.

Same semantics as the reference's ``build_tile_schedule``
(src/dispatch/kernels/tile_schedule.py:28-50): per-expert ``block_m``-row tiles
and the exclusive prefix sum ``group_offsets``. The B200 kernels only read
``group_offsets`` (on the device) and derive their own 128-row tiles in-kernel;
the fused layer path never builds this object and never synchronises.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class TileSchedule:
    block_m: int
    group_offsets: tuple[int, ...]  # host-side row offsets, len n_experts + 1
    tile_expert: torch.Tensor  # (num_tiles,) int32
    tile_row_start: torch.Tensor  # (num_tiles,) int32
    tile_valid_rows: torch.Tensor  # (num_tiles,) int32, each <= block_m

    @property
    def num_tiles(self) -> int:
        return int(self.tile_expert.shape[0])


def build_tile_schedule(group_sizes: torch.Tensor, block_m: int) -> TileSchedule:
    """Tensors land on group_sizes' device. Reads the sizes on the host, as the
    reference does; prefer the fused path, which keeps offsets on the device."""
    if block_m <= 0:
        raise ValueError(f"block_m must be positive, got {block_m}")
    sizes = [int(s) for s in group_sizes.tolist()]
    offsets = [0]
    te: list[int] = []
    ts: list[int] = []
    tv: list[int] = []
    for expert_id, size in enumerate(sizes):
        for local_start in range(0, size, block_m):
            te.append(expert_id)
            ts.append(offsets[-1] + local_start)
            tv.append(min(block_m, size - local_start))
        offsets.append(offsets[-1] + size)
    dev = group_sizes.device

    def i32(v: list[int]) -> torch.Tensor:
        return torch.tensor(v, dtype=torch.int32, device=dev)

    return TileSchedule(block_m, tuple(offsets), i32(te), i32(ts), i32(tv))


def device_offsets(schedule, device: torch.device) -> torch.Tensor:
    """``schedule.group_offsets`` as an int32 device tensor (accepts the
    reference's TileSchedule too: only ``group_offsets`` is read)."""
    cached = getattr(schedule, "_b200_offsets", None)
    if cached is not None and cached.device == device:
        return cached
    t = torch.tensor(schedule.group_offsets, dtype=torch.int32).to(device, non_blocking=True)
    try:
        object.__setattr__(schedule, "_b200_offsets", t)
    except (AttributeError, TypeError):
        pass
    return t
