"""The routed-expert half of the MoE layer (mirror of the reference's
src/dispatch/kernels/moe_forward.py).

``grouped_moe_routed`` keeps the reference's signature but runs the fused B200
path: device grouping + row gather, then the expert FFN as two tcgen05
launches (gate and up in one tile with SwiGLU in the epilogue, then down),
then the deterministic combine. ``matmul`` is accepted for signature
compatibility and must be None or the b200 backend."""

from __future__ import annotations

import itertools
from collections.abc import Callable, Iterable
from dataclasses import dataclass

import torch

from dispatch_b200 import _lib as L
from dispatch_b200.kernels.grouping import _group, combine
from dispatch_b200.kernels.tile_schedule import TileSchedule

GroupedMatmul = Callable[[torch.Tensor, torch.Tensor, TileSchedule], torch.Tensor]

CORRECTNESS_RTOL = 1.6e-2  # the reference's tolerance (moe_forward.py:23)


@dataclass(frozen=True)
class StackedExpertWeights:
    """Each projection's weights for every expert, as (n_experts, N, K)."""

    gate: torch.Tensor
    up: torch.Tensor
    down: torch.Tensor

    @property
    def num_experts(self) -> int:
        return int(self.gate.shape[0])


@dataclass(frozen=True)
class SharedExpertWeights:
    """The always-on shared expert: gate/up (I_s, H), down (H, I_s), in the
    activation dtype (it stays bf16 in the int8 configs, as in the reference)."""

    gate: torch.Tensor
    up: torch.Tensor
    down: torch.Tensor


def torch_grouped_matmul(x: torch.Tensor, expert_weight: torch.Tensor, schedule: TileSchedule) -> torch.Tensor:
    """The reference's eager contract (moe_forward.py:39-47), kept as a test
    helper for the GroupedMatmul surface; not used by any B200 op."""
    out = x.new_empty((x.shape[0], expert_weight.shape[1]))
    for expert_id, (start, end) in enumerate(itertools.pairwise(schedule.group_offsets)):
        if end > start:
            out[start:end] = x[start:end] @ expert_weight[expert_id].T
    return out


def stack_expert_weights(experts: Iterable[torch.nn.Module]) -> StackedExpertWeights:
    """Stacks each projection and re-points every expert's Linear at a view of
    it (reference moe_forward.py:50-58, 95-99)."""
    modules = list(experts)
    return StackedExpertWeights(
        gate=_stack_and_share([_linear(m, "gate_proj") for m in modules]),
        up=_stack_and_share([_linear(m, "up_proj") for m in modules]),
        down=_stack_and_share([_linear(m, "down_proj") for m in modules]),
    )


def shared_expert_weights(module: torch.nn.Module) -> SharedExpertWeights:
    return SharedExpertWeights(
        gate=_linear(module, "gate_proj").weight.detach(),
        up=_linear(module, "up_proj").weight.detach(),
        down=_linear(module, "down_proj").weight.detach(),
    )


def assert_matches_reference(actual: torch.Tensor, expected: torch.Tensor) -> None:
    """assert_close with atol scaled to the reference's magnitude (reference
    moe_forward.py:79-85)."""
    atol = CORRECTNESS_RTOL * float(expected.detach().abs().max())
    torch.testing.assert_close(actual.detach().float(), expected.detach().float(), rtol=CORRECTNESS_RTOL, atol=atol)


def _linear(module: torch.nn.Module, name: str) -> torch.nn.Linear:
    projection = getattr(module, name)
    if not isinstance(projection, torch.nn.Linear):
        raise TypeError(f"expected {name} to be nn.Linear, got {type(projection).__name__}")
    return projection


def _stack_and_share(linears: list[torch.nn.Linear]) -> torch.Tensor:
    stacked = torch.stack([linear.weight.detach() for linear in linears])
    for index, linear in enumerate(linears):
        linear.weight = torch.nn.Parameter(stacked[index], requires_grad=False)
    return stacked


# ---------------------------------------------------------------- fused path
def expert_ffn(xs: torch.Tensor, offsets: torch.Tensor, weights, shared: SharedExpertWeights | None = None,
               x_shared: torch.Tensor | None = None, *, gather_rows: torch.Tensor | None = None,
               n_rows: int | None = None) -> tuple[torch.Tensor, torch.Tensor | None]:
    """y = down(silu(gate(xs)) * up(xs)) per expert group, and the shared
    expert over x_shared, in two tcgen05 launches. ``weights`` is a
    StackedExpertWeights (bf16/f16) or a QuantizedStackedExpertWeights.
    With ``gather_rows`` (int64, n_rows entries) routed row r is row
    gather_rows[r] of ``xs``, fetched by the GEMM's TMA gather instead of a copy."""
    from dispatch_b200.kernels.quantization import QuantizedStackedExpertWeights  # noqa: PLC0415

    quant = isinstance(weights, QuantizedStackedExpertWeights)
    g, u, d = (weights.gate.data, weights.up.data, weights.down.data) if quant else (weights.gate, weights.up, weights.down)
    dev = L.require_cuda(xs, offsets, g, u, d, x_shared, gather_rows, what="the B200 expert FFN")
    act = xs.dtype
    if act not in (torch.bfloat16, torch.float16):
        raise ValueError(f"dtype mismatch: activations must be bf16/f16, got {act}")
    if not quant and not (g.dtype == u.dtype == d.dtype == act):
        raise ValueError(f"dtype mismatch: x is {act}, expert weights are {g.dtype}")
    h = xs.shape[1]
    if gather_rows is not None:
        if gather_rows.dtype != torch.int64:
            raise ValueError("gather_rows must be int64")
        r = int(n_rows if n_rows is not None else gather_rows.numel())
    else:
        r = xs.shape[0]
    e, i, _ = g.shape
    if g.shape[2] != h or d.shape[1] != h or d.shape[2] != i:
        raise ValueError(f"K mismatch: x has {h}, weights are gate {tuple(g.shape)} down {tuple(d.shape)}")
    y = torch.empty(r, h, dtype=act, device=dev)
    ys = None
    t_sh = 0
    i_sh = 0
    if shared is not None:
        if x_shared is None:
            raise ValueError("shared expert needs x_shared")
        if shared.gate.dtype != act or x_shared.dtype != act:
            raise ValueError(f"dtype mismatch: shared expert must be {act}")
        t_sh = x_shared.shape[0]
        i_sh = shared.gate.shape[0]
        ys = torch.empty(t_sh, h, dtype=act, device=dev)
    lib = L.lib()
    nbytes = lib.moe_ffn_workspace_bytes(r, i, t_sh, i_sh)
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
    sc = (weights.gate.scale, weights.up.scale, weights.down.scale) if quant else (None, None, None)
    rc = lib.moe_expert_ffn_grouped(
        3, xs.data_ptr(), L.dt(act), r, h, offsets.data_ptr(), e, e,
        L.ptr(gather_rows), xs.shape[0] if gather_rows is not None else 0, i,
        g.contiguous().data_ptr(), u.contiguous().data_ptr(), d.contiguous().data_ptr(),
        L.DT_I8 if quant else L.dt(act),
        L.ptr(sc[0]), L.ptr(sc[1]), L.ptr(sc[2]), L.dt(sc[0]) if quant else 0,
        L.ptr(x_shared), t_sh, i_sh,
        L.ptr(None if shared is None else shared.gate.contiguous()),
        L.ptr(None if shared is None else shared.up.contiguous()),
        L.ptr(None if shared is None else shared.down.contiguous()),
        y.data_ptr(), L.ptr(ys), ws.data_ptr(), ws.numel(), L.status_word(dev).data_ptr(), L.stream_ptr(dev),
    )
    L.check(rc, "expert_ffn")
    return y, ys


def act_dtype_for(x: torch.Tensor, weights) -> torch.dtype:
    """The tensor-core input type: the weights' type, or for int8 weights the
    activation type (bf16 when x is f32)."""
    gate = getattr(weights.gate, "data", weights.gate)
    if gate.dtype == torch.int8:
        return x.dtype if x.dtype in (torch.bfloat16, torch.float16) else torch.bfloat16
    return gate.dtype


def _routed_forward(x, topk_idx, topk_weight, weights, shared: SharedExpertWeights | None) -> torch.Tensor:
    if topk_idx.shape != topk_weight.shape:
        raise ValueError(
            f"topk_idx.shape {tuple(topk_idx.shape)} != topk_weight.shape {tuple(topk_weight.shape)}"
        )
    act = act_dtype_for(x, weights)
    if act not in (torch.bfloat16, torch.float16):
        raise ValueError(f"dtype mismatch: expert weights must be bf16/f16 (or int8), got {act}")
    if x.dtype not in (act, torch.float32):
        raise ValueError(f"dtype mismatch: x is {x.dtype}, expert weights are {act}")
    t, k = topk_idx.shape
    e = weights.num_experts
    x = x.contiguous()
    x_sh = None
    if shared is not None:
        x_sh = x if x.dtype == act else x.to(act)
    # the grouping kernel gathers the rows (a TMA gather inside the GEMM is
    # available through expert_ffn(gather_rows=...) but measured slower)
    _, offsets, pos, _, _, w, xs = _group(topk_idx, topk_weight, e, x=x, xs_dtype=act, want_sorted=False)
    y, ys = expert_ffn(xs, offsets, weights, shared, x_sh)
    return combine(y, pos, w.reshape(-1), t, k, ys, out_dtype=x.dtype)


def grouped_moe_routed(  # noqa: PLR0913 -- mirrors the reference signature
    x: torch.Tensor,
    topk_idx: torch.Tensor,
    topk_weight: torch.Tensor,
    weights: StackedExpertWeights,
    matmul: GroupedMatmul | None = None,
    *,
    block_m: int = 16,
    shared: SharedExpertWeights | None = None,
) -> torch.Tensor:
    """Reference: moe_forward.py:61-76. Output dtype = x.dtype; x may be f32
    with bf16 weights (computed in bf16, combined in f32)."""
    from dispatch_b200.kernels.quantization import _check_matmul  # noqa: PLC0415

    _check_matmul(matmul)
    if block_m <= 0:
        raise ValueError(f"block_m must be positive, got {block_m}")
    return _routed_forward(x, topk_idx, topk_weight, weights, shared)
