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


class NcclEPBuffer:
    """DeepEP V1 ``Buffer``-compatible dispatch/combine over NCCL, so callers
    written against DeepEP (the reference's ``make_ep_moe_infer``,
    expert_parallel.py:119-190) run unchanged on ``torch.distributed``.

    Semantics follow the reference's use of DeepEP: tokens go once to each
    rank that owns at least one of their experts; received top-k ids are
    local (0..E/R-1) or -1 for slots owned elsewhere; ``combine`` sums the
    per-rank partial outputs of each token -- here in rank order, in f32,
    with the deterministic combine kernel (one rounding), instead of DeepEP's
    unordered reduction.
    """

    def __init__(self, group=None, *, rank: int | None = None, world: int | None = None):
        self.group = group
        self.rank = dist.get_rank(group) if rank is None else rank
        self.world = dist.get_world_size(group) if world is None else world

    def get_dispatch_layout(self, topk_idx: torch.Tensor, num_experts: int):
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not split evenly over {self.world} ranks")
        e_loc = num_experts // self.world
        valid = topk_idx >= 0
        dest = torch.where(valid, topk_idx // e_loc, torch.full_like(topk_idx, -1))
        ranks = torch.arange(self.world, device=topk_idx.device)
        is_token_in_rank = (dest.unsqueeze(-1) == ranks).any(dim=1)
        num_tokens_per_rank = is_token_in_rank.sum(0).to(torch.int32)
        num_tokens_per_expert = torch.bincount(topk_idx[valid].reshape(-1), minlength=num_experts).to(torch.int32)
        return num_tokens_per_rank, None, num_tokens_per_expert, is_token_in_rank, None

    def dispatch(self, x, topk_idx=None, topk_weights=None, num_tokens_per_rank=None, num_tokens_per_rdma_rank=None,
                 is_token_in_rank=None, num_tokens_per_expert=None, **_unused):
        if topk_weights is not None and topk_weights.dtype != torch.float32:
            raise ValueError("topk_weights must be float32 (DeepEP V1 contract)")
        e = int(num_tokens_per_expert.numel())
        e_loc = e // self.world
        send_idx, send_x, send_topk, send_w, splits = [], [], [], [], []
        for r in range(self.world):
            tok = is_token_in_rank[:, r].nonzero(as_tuple=True)[0]
            local = topk_idx[tok] - r * e_loc
            owned = (topk_idx[tok] >= 0) & (local >= 0) & (local < e_loc)
            send_idx.append(tok)
            send_x.append(x[tok])
            send_topk.append(torch.where(owned, local, torch.full_like(local, -1)))
            send_w.append(topk_weights[tok] if topk_weights is not None else None)
            splits.append(int(tok.numel()))
        recv_splits = _exchange_splits(splits, x.device, self.group)
        n_recv = sum(recv_splits)
        recv_x = x.new_empty(n_recv, x.shape[1])
        all_to_all_rows(recv_x, torch.cat(send_x), recv_splits, splits, self.group)
        k = topk_idx.shape[1]
        recv_topk = topk_idx.new_empty(n_recv, k)
        all_to_all_rows(recv_topk, torch.cat(send_topk), recv_splits, splits, self.group)
        recv_w = None
        if topk_weights is not None:
            recv_w = topk_weights.new_empty(n_recv, k)
            all_to_all_rows(recv_w, torch.cat(send_w), recv_splits, splits, self.group)
        per_expert = torch.bincount(recv_topk[recv_topk >= 0].reshape(-1), minlength=e_loc).tolist()
        handle = {"send_idx": send_idx, "send_splits": splits, "recv_splits": recv_splits,
                  "num_tokens": x.shape[0]}
        return recv_x, recv_topk, recv_w, per_expert, handle, None

    def combine(self, x: torch.Tensor, handle, topk_weights=None, **_unused):
        splits, recv_splits = handle["send_splits"], handle["recv_splits"]
        back = x.new_empty(sum(splits), x.shape[1])
        all_to_all_rows(back, x.contiguous(), splits, recv_splits, self.group)
        t = handle["num_tokens"]
        # pos[token, rank] = row of that rank's partial in `back`, -1 if none
        pos = torch.full((t, self.world), -1, dtype=torch.int32, device=x.device)
        start = 0
        for r, idx in enumerate(handle["send_idx"]):
            pos[idx, r] = torch.arange(start, start + idx.numel(), dtype=torch.int32, device=x.device)
            start += idx.numel()
        if back.shape[0] == 0:
            return torch.zeros(t, x.shape[1], dtype=x.dtype, device=x.device), None, None
        return self._sum_partials(back, pos, t), None, None

    def _sum_partials(self, back: torch.Tensor, pos: torch.Tensor, t: int) -> torch.Tensor:
        """out[token] = sum over ranks r (in order) of back[pos[token, r]]: the
        combine kernel with unit weights (missing partials have pos -1)."""
        from dispatch_b200.kernels.grouping import combine  # noqa: PLC0415

        ones = (pos >= 0).to(torch.float32)
        return combine(back, pos.reshape(-1), ones.reshape(-1), t, self.world)


def _exchange_splits(splits: list[int], device, group=None) -> list[int]:
    world = len(splits)
    send = torch.tensor(splits, dtype=torch.int64, device=device)
    recv = torch.empty(world, dtype=torch.int64, device=device)
    dist.all_to_all_single(recv, send, group=group)
    return recv.tolist()


def local_expert_contribution(x, topk_idx, topk_weight, local_weights, matmul=None, local_expert_ids=None, *,
                              block_m: int = 16):
    """This rank's weighted output for received tokens (reference
    expert_parallel.py:44-86): slots whose expert is not local get weight 0;
    ids are remapped to 0..E_local-1 and -1 padding is ignored."""
    from dispatch_b200.kernels.moe_forward import grouped_moe_routed  # noqa: PLC0415

    n_local = local_weights.num_experts
    if local_expert_ids is None:
        local_expert_ids = torch.arange(n_local, device=topk_idx.device)
    local_expert_ids = local_expert_ids.to(topk_idx.device)
    is_local = torch.isin(topk_idx, local_expert_ids)
    span = max(int(local_expert_ids.max().item()), int(topk_idx.max().item()) if topk_idx.numel() else 0) + 1
    remap = torch.zeros(span, dtype=torch.int64, device=topk_idx.device)
    remap[local_expert_ids] = torch.arange(n_local, device=topk_idx.device)
    local_idx = remap[topk_idx.clamp(min=0)]
    local_w = torch.where(is_local, topk_weight, torch.zeros_like(topk_weight))
    if x.shape[0] == 0:
        return x.new_zeros(0, x.shape[1])
    return grouped_moe_routed(x, local_idx, local_w, local_weights, matmul, block_m=block_m)


def make_ep_moe_infer(local_weights, matmul, buffer, num_experts: int, *, block_m: int = 16):
    """The reference's DeepEP round trip (expert_parallel.py:119-190) on any
    Buffer-compatible transport (``NcclEPBuffer``)."""

    @torch.no_grad()
    def moe_infer(x, flat_expert_indices, flat_expert_weights):
        top_k = flat_expert_indices.numel() // x.shape[0]
        topk_idx = flat_expert_indices.view(-1, top_k)
        topk_weight = flat_expert_weights.view(-1, top_k).to(torch.float32)
        per_rank, per_rdma, per_expert, in_rank, _ = buffer.get_dispatch_layout(topk_idx, num_experts)
        recv_x, recv_idx, recv_w, _, handle, _ = buffer.dispatch(
            x, topk_idx=topk_idx, topk_weights=topk_weight, num_tokens_per_rank=per_rank,
            num_tokens_per_rdma_rank=per_rdma, is_token_in_rank=in_rank, num_tokens_per_expert=per_expert)
        local_out = local_expert_contribution(recv_x, recv_idx, recv_w.to(x.dtype), local_weights, matmul,
                                              block_m=block_m)
        combined, _, _ = buffer.combine(local_out, handle)
        return combined

    return moe_infer


def patch_moe_infer_ep(model: torch.nn.Module, matmul, buffer, rank: int, n_ranks: int, *, block_m: int = 16) -> int:
    """Each MoE layer's moe_infer computes only this rank's expert shard and
    exchanges the rest through ``buffer`` (reference expert_parallel.py:193-229)."""
    from dispatch_b200.kernels.integration import _iter_validated_moe_layers  # noqa: PLC0415
    from dispatch_b200.kernels.moe_forward import StackedExpertWeights, stack_expert_weights  # noqa: PLC0415

    model.eval()
    patched = 0
    for module, experts in _iter_validated_moe_layers(model):
        n_experts = len(experts)
        local = (assign_experts_to_ranks(n_experts, n_ranks) == rank).nonzero(as_tuple=True)[0]
        all_w = stack_expert_weights(experts)
        local_w = StackedExpertWeights(all_w.gate[local], all_w.up[local], all_w.down[local])
        module.moe_infer = make_ep_moe_infer(local_w, matmul, buffer, n_experts, block_m=block_m)  # type: ignore[assignment]
        patched += 1
    return patched


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
