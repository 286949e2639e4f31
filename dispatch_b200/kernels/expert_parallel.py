"""Expert parallelism over NCCL (mirror of the reference's
src/dispatch/kernels/expert_parallel.py, which drives DeepEP's V1 Buffer).

Experts are split contiguously across ranks (``assign_experts_to_ranks``, the
reference's and DeepEP's convention). One ``EPLayer`` call on a rank's T local
tokens:

1. route and group locally on the device: rows come out sorted by expert,
   which is also sorted by destination rank;
2. all-to-all of the per-expert row counts (E int32 per rank);
3. one host synchronisation to size the payload, then an all-to-all of the
   bf16 rows (NCCL send/recv over NVLink);
4. the expert FFN on the received rows, grouped by (source rank, local expert)
   with no regrouping copy, plus the shared expert on the local tokens -- one
   pair of tcgen05 launches;
5. the reverse all-to-all of the per-row expert outputs (unweighted);
6. the weighted combine on the source rank, in slot order.

Every per-row product is computed by the same kernels with the same tile
configuration as the 1-GPU layer, and the final sum order is the same, so the
output is byte-identical to the 1-GPU result. The exchange is written against
``torch.distributed`` collectives only; the compute steps are an injectable
``ops`` object so the orchestration is testable on CPU gloo ranks.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


def assign_experts_to_ranks(n_experts: int, n_ranks: int) -> torch.Tensor:
    """expert_id -> rank_id, contiguous blocks (reference expert_parallel.py:33-41)."""
    if n_experts <= 0 or n_ranks <= 0:
        raise ValueError(f"n_experts={n_experts} and n_ranks={n_ranks} must both be positive")
    if n_experts < n_ranks:
        raise ValueError(f"n_experts={n_experts} is fewer than n_ranks={n_ranks}")
    return torch.arange(n_experts) * n_ranks // n_experts


@dataclass
class Grouped:
    counts: torch.Tensor  # (E,) int32, rows per expert
    offsets: torch.Tensor  # (E+1,) int32
    pos: torch.Tensor  # (T*k,) int32
    xs: torch.Tensor  # (T*k, H) rows in expert order
    topk_weight: torch.Tensor  # (T, k) f32


@dataclass(frozen=True)
class Layout:
    """Host-side sizes of one exchange."""

    send_splits: list[int]  # rows to each destination rank
    recv_splits: list[int]  # rows from each source rank
    recv_offsets: list[int]  # (R*E_local + 1) prefix over (source rank, local expert) blocks


def exchange_layout(counts: torch.Tensor, world: int, group=None) -> tuple[Layout, torch.Tensor]:
    """All-to-all of per-expert counts, then the host-side split sizes.

    counts: (E,) int32 rows this rank sends to each expert (expert-major, so
    the block of destination rank r is experts [r*E/R, (r+1)*E/R)).
    Returns the layout and the received counts (R*E_local,) on counts' device.
    """
    e = counts.numel()
    if e % world:
        raise ValueError(f"{e} experts do not split evenly over {world} ranks")
    e_loc = e // world
    recv = torch.empty_like(counts)
    dist.all_to_all_single(recv, counts.contiguous(), group=group)
    host = torch.stack([counts, recv]).cpu()  # the one host synchronisation per call
    sent, got = host[0].view(world, e_loc), host[1].view(world, e_loc)
    send_splits = sent.sum(1).tolist()
    recv_splits = got.sum(1).tolist()
    off = [0]
    for c in got.reshape(-1).tolist():
        off.append(off[-1] + c)
    return Layout(send_splits, recv_splits, off), recv


def all_to_all_rows(out: torch.Tensor, inp: torch.Tensor, out_splits: list[int], in_splits: list[int],
                    group=None) -> None:
    dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits, group=group)


class B200Ops:
    """The compute steps on the B200 kernels (C ABI)."""

    def __init__(self, router_weight, local_weights, shared, router_cfg, e_score_bias=None):
        self.router_weight = router_weight
        self.weights = local_weights
        self.shared = shared
        self.cfg = router_cfg
        self.bias = e_score_bias
        self.n_local = local_weights.num_experts

    def route_and_group(self, x: torch.Tensor, n_experts: int) -> Grouped:
        from dispatch_b200.kernels.grouping import _group  # noqa: PLC0415
        from dispatch_b200.kernels.layer import route  # noqa: PLC0415

        idx, w = route(x, self.router_weight, self.cfg, e_score_bias=self.bias)
        counts, offsets, pos, _, _, wf, xs = _group(idx, w, n_experts, x=x, xs_dtype=x.dtype, want_sorted=False)
        return Grouped(counts, offsets, pos, xs, wf)

    def ffn(self, recv_x: torch.Tensor, recv_offsets: torch.Tensor, n_groups: int, x: torch.Tensor):
        import ctypes  # noqa: F401,PLC0415

        from dispatch_b200 import _lib as L  # noqa: PLC0415
        from dispatch_b200.kernels.quantization import QuantizedStackedExpertWeights  # noqa: PLC0415

        dev = x.device
        quant = isinstance(self.weights, QuantizedStackedExpertWeights)
        g, u, d = ((self.weights.gate.data, self.weights.up.data, self.weights.down.data) if quant
                   else (self.weights.gate, self.weights.up, self.weights.down))
        r, h = recv_x.shape
        i = g.shape[1]
        t = x.shape[0]
        sh = self.shared
        i_sh = 0 if sh is None else sh.gate.shape[0]
        y = torch.empty(r, h, dtype=x.dtype, device=dev)
        ys = torch.empty(t, h, dtype=x.dtype, device=dev) if sh is not None else None
        lib = L.lib()
        nbytes = lib.moe_ffn_workspace_bytes(r, i, t if sh is not None else 0, i_sh)
        ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
        sc = (self.weights.gate.scale, self.weights.up.scale, self.weights.down.scale) if quant else (None,) * 3
        rc = lib.moe_expert_ffn_grouped(
            3, recv_x.data_ptr() if r else None, L.dt(x), r, h, recv_offsets.data_ptr(), n_groups, self.n_local,
            None, 0, i,
            g.data_ptr(), u.data_ptr(), d.data_ptr(), L.DT_I8 if quant else L.dt(g),
            L.ptr(sc[0]), L.ptr(sc[1]), L.ptr(sc[2]), L.dt(sc[0]) if quant else 0,
            x.data_ptr() if sh is not None else None, t if sh is not None else 0, i_sh,
            L.ptr(None if sh is None else sh.gate), L.ptr(None if sh is None else sh.up),
            L.ptr(None if sh is None else sh.down),
            y.data_ptr() if r else None, L.ptr(ys), ws.data_ptr(), ws.numel(), L.status_word(dev).data_ptr(),
            L.stream_ptr(dev),
        )
        L.check(rc, "moe_expert_ffn_grouped")
        return y, ys

    def combine(self, y_back, grouped: Grouped, t: int, k: int, ys, out_dtype):
        from dispatch_b200.kernels.grouping import combine  # noqa: PLC0415

        return combine(y_back, grouped.pos, grouped.topk_weight.reshape(-1), t, k, ys, out_dtype=out_dtype)


class EPLayer:
    """Expert-parallel MoE layer for one rank (see the module docstring).

    ``weights`` may be the full stacked experts (this rank's slice is taken)
    or, with ``weights_are_local=True``, already this rank's E/R experts.
    """

    def __init__(self, router_weight, weights, shared, router_cfg, *, rank: int, world: int, group=None,
                 e_score_bias=None, n_experts: int | None = None, weights_are_local: bool = False, ops=None):
        self.rank, self.world, self.group = rank, world, group
        e = n_experts if n_experts is not None else (
            weights.num_experts * (world if weights_are_local else 1))
        if e % world:
            raise ValueError(f"{e} experts do not split evenly over {world} ranks")
        self.n_experts = e
        self.e_local = e // world
        if not weights_are_local and ops is None:
            weights = _slice_experts(weights, rank * self.e_local, (rank + 1) * self.e_local)
        self.ops = ops or B200Ops(router_weight, weights, shared, router_cfg, e_score_bias)
        self.top_k = router_cfg.top_k
        # launches of this library per call: route GEMM + select, group x2, FFN x2, combine
        self.launches_per_step = 7

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        t = x.shape[0]
        gr = self.ops.route_and_group(x, self.n_experts)
        layout, _ = exchange_layout(gr.counts, self.world, self.group)
        recv_rows = sum(layout.recv_splits)
        recv_x = x.new_empty(recv_rows, x.shape[1])
        all_to_all_rows(recv_x, gr.xs, layout.recv_splits, layout.send_splits, self.group)
        offs = torch.tensor(layout.recv_offsets, dtype=torch.int32)
        if x.is_cuda:
            offs = offs.pin_memory().to(x.device, non_blocking=True)
        y_recv, ys = self.ops.ffn(recv_x, offs, self.world * self.e_local, x)
        y_back = y_recv.new_empty(gr.xs.shape[0], y_recv.shape[1])
        all_to_all_rows(y_back, y_recv, layout.send_splits, layout.recv_splits, self.group)
        return self.ops.combine(y_back, gr, t, self.top_k, ys, x.dtype)


def _slice_experts(weights, lo: int, hi: int):
    from dispatch_b200.kernels.moe_forward import StackedExpertWeights  # noqa: PLC0415
    from dispatch_b200.kernels.quantization import (  # noqa: PLC0415
        QuantizedStackedExpertWeights,
        QuantizedTensor,
    )

    if isinstance(weights, QuantizedStackedExpertWeights):
        q = lambda t: QuantizedTensor(t.data[lo:hi], t.scale[lo:hi])  # noqa: E731
        return QuantizedStackedExpertWeights(q(weights.gate), q(weights.up), q(weights.down))
    return StackedExpertWeights(weights.gate[lo:hi], weights.up[lo:hi], weights.down[lo:hi])
