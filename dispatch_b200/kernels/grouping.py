"""Token-to-expert grouping on the device (mirror of the reference's
src/dispatch/kernels/grouping.py).

``group_tokens_by_expert`` is a stable counting sort in two launches (no host
sync, no argsort); ``ungroup_and_combine`` is the deterministic weighted
combine (f32 sum in slot order, one rounding) instead of ``index_add_``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from dispatch_b200 import _lib as L


@dataclass(frozen=True)
class TokenGrouping:
    """Row i of the grouped layout is token sorted_token_idx[i], weighted by
    sorted_weight[i]; the first group_sizes[0] rows belong to expert 0, and so
    on (reference grouping.py:15-22). The extra fields keep the grouping on the
    device: ``offsets`` (E+1) int32, ``pos`` (T*k) int32 with
    pos[t*k+s] = grouped row of (token t, slot s), and the flat f32 weights."""

    sorted_token_idx: torch.Tensor  # (num_tokens * top_k,) int64
    sorted_weight: torch.Tensor  # (num_tokens * top_k,)
    group_sizes: torch.Tensor  # (n_routed_experts,) int64
    offsets: torch.Tensor
    pos: torch.Tensor
    flat_weight: torch.Tensor
    top_k: int


def _group(topk_idx: torch.Tensor, topk_weight: torch.Tensor | None, n_experts: int,
           x: torch.Tensor | None = None, xs_dtype: torch.dtype | None = None,
           want_sorted: bool = True):
    dev = L.require_cuda(topk_idx, topk_weight, x, what="token grouping")
    t, k = topk_idx.shape
    idx = topk_idx.contiguous()
    if idx.dtype not in (torch.int32, torch.int64):
        raise ValueError(f"topk_idx must be int32 or int64, got {idx.dtype}")
    w = None if topk_weight is None else topk_weight.contiguous().float()
    n = t * k
    counts = torch.empty(n_experts, dtype=torch.int32, device=dev)
    offsets = torch.empty(n_experts + 1, dtype=torch.int32, device=dev)
    pos = torch.empty(n, dtype=torch.int32, device=dev)
    sti = torch.empty(n, dtype=torch.int64, device=dev) if want_sorted else None
    sw = torch.empty(n, dtype=torch.float32, device=dev) if (want_sorted and w is not None) else None
    xs = None
    h = 0
    if x is not None:
        h = x.shape[1]
        xs = torch.empty(n, h, dtype=xs_dtype, device=dev)
    lib = L.lib()
    nbytes = lib.moe_group_workspace_bytes(t, k, n_experts)
    ws = L.workspace(dev, nbytes, "group")
    rc = lib.moe_group_tokens(
        idx.data_ptr(), L.dt(idx), L.ptr(w), t, k, n_experts, counts.data_ptr(), offsets.data_ptr(),
        pos.data_ptr(), L.ptr(sti), L.ptr(sw),
        L.ptr(x), L.dt(x) if x is not None else 0, h, L.ptr(xs), L.dt(xs_dtype) if xs is not None else 0,
        ws.data_ptr(), ws.numel(), L.status_word(dev).data_ptr(), L.stream_ptr(dev),
    )
    L.check(rc, "group_tokens_by_expert")
    return counts, offsets, pos, sti, sw, w, xs


def group_tokens_by_expert(
    topk_idx: torch.Tensor, topk_weight: torch.Tensor, n_routed_experts: int
) -> TokenGrouping:
    """Reference: src/dispatch/kernels/grouping.py:25-41."""
    if topk_idx.shape != topk_weight.shape:
        raise ValueError(
            f"topk_idx.shape {tuple(topk_idx.shape)} != topk_weight.shape {tuple(topk_weight.shape)}"
        )
    counts, offsets, pos, sti, sw, w, _ = _group(topk_idx, topk_weight, n_routed_experts)
    return TokenGrouping(
        sorted_token_idx=sti,
        sorted_weight=sw.to(topk_weight.dtype),
        group_sizes=counts.to(torch.int64),
        offsets=offsets,
        pos=pos,
        flat_weight=w.reshape(-1),
        top_k=topk_idx.shape[1],
    )


def combine(y: torch.Tensor, pos: torch.Tensor, flat_weight: torch.Tensor, num_tokens: int, top_k: int,
            y_shared: torch.Tensor | None = None, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """out[t] = sum_s w[t,s] * y[pos[t*k+s]] (+ y_shared[t]) in f32, slot order."""
    dev = L.require_cuda(y, pos, flat_weight, y_shared, what="ungroup_and_combine")
    h = y.shape[-1]
    out = torch.empty(num_tokens, h, dtype=out_dtype or y.dtype, device=dev)
    ys = None if y_shared is None else y_shared.contiguous()
    if ys is not None and ys.dtype != y.dtype:
        ys = ys.to(y.dtype)
    rc = L.lib().moe_combine(
        y.contiguous().data_ptr(), L.dt(y), pos.data_ptr(), flat_weight.contiguous().data_ptr(), num_tokens,
        top_k, h, L.ptr(ys), out.data_ptr(), L.dt(out), L.status_word(dev).data_ptr(), L.stream_ptr(dev),
    )
    L.check(rc, "ungroup_and_combine")
    return out


def ungroup_and_combine(
    grouped_output: torch.Tensor, grouping: TokenGrouping, num_tokens: int
) -> torch.Tensor:
    """Reference: src/dispatch/kernels/grouping.py:44-61."""
    if grouped_output.shape[0] != grouping.sorted_token_idx.shape[0]:
        raise ValueError(
            f"grouped_output has {grouped_output.shape[0]} rows, "
            f"grouping describes {grouping.sorted_token_idx.shape[0]}"
        )
    return combine(grouped_output, grouping.pos, grouping.flat_weight, num_tokens, grouping.top_k)
