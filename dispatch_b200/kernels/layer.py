"""The whole MoE layer in one C-ABI call: router -> grouping + gather ->
expert FFN (routed + shared) -> combine, five launches, no host sync.

Mirrors ReferenceMoE.forward (src/dispatch/kernels/reference_moe.py:74-78)
and adds the routers the BASELINE configs need: renormalised softmax top-k
(``renormalize=True``) and the DeepSeek-V3 group-limited sigmoid router.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from dispatch_b200 import _lib as L
from dispatch_b200.kernels.moe_forward import SharedExpertWeights, StackedExpertWeights, act_dtype_for
from dispatch_b200.kernels.quantization import QuantizedStackedExpertWeights


@dataclass(frozen=True)
class RouterConfig:
    top_k: int
    mode: str = "softmax"  # "softmax" | "sigmoid_group"
    renormalize: bool = False
    n_group: int = 1
    topk_group: int = 1
    routed_scaling_factor: float = 1.0


@dataclass(frozen=True)
class LayerOutput:
    out: torch.Tensor
    topk_idx: torch.Tensor  # (T, k) int32
    topk_weight: torch.Tensor  # (T, k) f32
    group_sizes: torch.Tensor  # (E,) int32
    group_offsets: torch.Tensor  # (E+1,) int32


def moe_layer_forward(
    x: torch.Tensor,
    router_weight: torch.Tensor | None,
    weights: StackedExpertWeights | QuantizedStackedExpertWeights,
    router: RouterConfig,
    *,
    shared: SharedExpertWeights | None = None,
    e_score_bias: torch.Tensor | None = None,
    topk: tuple[torch.Tensor, torch.Tensor] | None = None,
    out_dtype: torch.dtype | None = None,
) -> LayerOutput:
    """x (T, H) bf16/f16 (or f32 with bf16 weights and no shared expert);
    router_weight (E, H) bf16/f32; ``topk`` = (idx int32 (T,k), w f32 (T,k))
    skips the router (the moe_infer contract)."""
    quant = isinstance(weights, QuantizedStackedExpertWeights)
    g = weights.gate.data if quant else weights.gate
    u = weights.up.data if quant else weights.up
    dn = weights.down.data if quant else weights.down
    dev = L.require_cuda(x, router_weight, g, u, dn, e_score_bias, what="moe_layer_forward")
    act = act_dtype_for(x, weights)
    t, h = x.shape
    e, i, _ = g.shape
    k = router.top_k
    x = x.contiguous()
    desc = L.MoeLayerDesc()
    desc.T, desc.H, desc.E, desc.I = t, h, e, i
    desc.I_shared = 0 if shared is None else shared.gate.shape[0]
    desc.k = k
    desc.act_dtype = L.dt(act)
    desc.x_dtype = L.dt(x)
    desc.out_dtype = L.dt(out_dtype or x.dtype)
    desc.w_dtype = L.DT_I8 if quant else L.dt(g)
    desc.scale_dtype = L.dt(weights.gate.scale) if quant else L.DT_F32
    desc.router_mode = L.ROUTER_SIGMOID_GROUP if router.mode == "sigmoid_group" else L.ROUTER_SOFTMAX
    desc.renorm = int(router.renormalize)
    desc.n_group = router.n_group
    desc.topk_group = router.topk_group
    desc.routed_scaling = router.routed_scaling_factor
    desc.router_w_dtype = L.dt(router_weight) if router_weight is not None else L.DT_BF16
    lib = L.lib()
    nbytes = lib.moe_layer_workspace_bytes(ctypes.byref(desc))
    ws = L.workspace(dev, nbytes, "layer")
    out = torch.empty(t, h, dtype=out_dtype or x.dtype, device=dev)
    if topk is not None:
        idx = topk[0].to(torch.int32).contiguous()
        wts = topk[1].to(torch.float32).contiguous()
        idx_in, w_in = idx, wts
    else:
        idx = torch.empty(t, k, dtype=torch.int32, device=dev)
        wts = torch.empty(t, k, dtype=torch.float32, device=dev)
        idx_in = w_in = None
    counts = torch.empty(e, dtype=torch.int32, device=dev)
    offsets = torch.empty(e + 1, dtype=torch.int32, device=dev)
    rw = None if router_weight is None else router_weight.contiguous()
    sc = (weights.gate.scale, weights.up.scale, weights.down.scale) if quant else (None, None, None)
    rc = lib.moe_layer_forward(
        ctypes.byref(desc), x.data_ptr(), L.ptr(rw), L.ptr(e_score_bias),
        L.ptr(idx_in), L.ptr(w_in),
        g.contiguous().data_ptr(), u.contiguous().data_ptr(), dn.contiguous().data_ptr(),
        L.ptr(sc[0]), L.ptr(sc[1]), L.ptr(sc[2]),
        L.ptr(None if shared is None else shared.gate), L.ptr(None if shared is None else shared.up),
        L.ptr(None if shared is None else shared.down),
        out.data_ptr(), None if topk is not None else idx.data_ptr(), None if topk is not None else wts.data_ptr(),
        counts.data_ptr(), offsets.data_ptr(), ws.data_ptr(), ws.numel(), L.status_word(dev).data_ptr(),
        L.stream_ptr(dev),
    )
    L.check(rc, "moe_layer_forward")
    return LayerOutput(out, idx, wts, counts, offsets)


def route(
    x: torch.Tensor | None,
    router_weight: torch.Tensor | None,
    router: RouterConfig,
    *,
    logits: torch.Tensor | None = None,
    e_score_bias: torch.Tensor | None = None,
    return_logits: bool = False,
):
    """Router only: (topk_idx int32 (T,k), topk_weight f32 (T,k)[, logits f32]).
    With ``logits`` given the selection runs on exactly those values (the
    parity boundary "same logits in -> same ids out"). Returned logits are the
    raw gate output x @ router_weight.T; in softmax mode ``e_score_bias`` is
    added to them before the selection."""
    ref = logits if logits is not None else x
    dev = L.require_cuda(ref, router_weight if logits is None else None, e_score_bias, what="route")
    if logits is not None:
        logits = logits.contiguous().float()
        t, e = logits.shape
        h = 0
    else:
        t, h = x.shape
        e = router_weight.shape[0]
        x = x.contiguous()
        router_weight = router_weight.contiguous()
    k = router.top_k
    idx = torch.empty(t, k, dtype=torch.int32, device=dev)
    w = torch.empty(t, k, dtype=torch.float32, device=dev)
    # the tensor-core logit GEMM writes here (needed whenever x is given)
    lg = torch.empty(t, e, dtype=torch.float32, device=dev) if (return_logits or logits is None) else None
    bias = None if e_score_bias is None else e_score_bias.contiguous().float()
    lib = L.lib()
    ws = None if logits is not None else L.workspace(dev, lib.moe_route_workspace_bytes(t, e), "route")
    rc = lib.moe_route(
        None if logits is not None else x.data_ptr(), 0 if logits is not None else L.dt(x),
        None if logits is not None else router_weight.data_ptr(), 0 if logits is not None else L.dt(router_weight),
        L.ptr(logits), t, h, e, k,
        L.ROUTER_SIGMOID_GROUP if router.mode == "sigmoid_group" else L.ROUTER_SOFTMAX,
        int(router.renormalize), L.ptr(bias), router.n_group, router.topk_group, router.routed_scaling_factor,
        idx.data_ptr(), w.data_ptr(), L.ptr(lg), L.ptr(ws), 0 if ws is None else ws.numel(),
        L.status_word(dev).data_ptr(), L.stream_ptr(dev),
    )
    L.check(rc, "route")
    return (idx, w, lg) if return_logits else (idx, w)


class CapturedLayer:
    """``moe_layer_forward`` for a fixed token count, captured once into a CUDA
    graph and replayed: one graph launch per step instead of seven kernel
    launches and their host-side argument encoding. Decode steps are short
    enough (tens of microseconds of device time) for that host work to be the
    bound; the kernels themselves are the same, so the output is the same bits
    as the eager call. ``__call__`` copies x into the graph's input buffer and
    returns the graph's output buffer (overwritten by the next call)."""

    def __init__(self, x_like: torch.Tensor, router_weight, weights, router: RouterConfig, *,
                 shared: SharedExpertWeights | None = None, e_score_bias: torch.Tensor | None = None,
                 out_dtype: torch.dtype | None = None):
        dev = L.require_cuda(x_like, what="CapturedLayer")
        self.x = torch.empty_like(x_like, memory_format=torch.contiguous_format)
        self.x.copy_(x_like)
        self._args = (router_weight, weights, router)
        self._kw = dict(shared=shared, e_score_bias=e_score_bias, out_dtype=out_dtype)
        self.stream = torch.cuda.Stream(dev)
        self.stream.wait_stream(torch.cuda.current_stream(dev))
        L.status_word(dev)
        with torch.cuda.stream(self.stream):
            # the warm-up call caches the workspace for this stream and does
            # the once-per-process kernel attribute set-up outside the capture
            moe_layer_forward(self.x, *self._args, **self._kw)
        self.stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.result = moe_layer_forward(self.x, *self._args, **self._kw)
        # the graph holds raw pointers into this stream's cached workspaces: keep them alive
        sid = self.stream.cuda_stream
        self._keep = [buf for (_, s, _), buf in L._workspaces.items() if s == sid]
        torch.cuda.current_stream(dev).wait_stream(self.stream)

    def replay(self) -> LayerOutput:
        self.graph.replay()
        return self.result

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape != self.x.shape or x.dtype != self.x.dtype:
            raise ValueError(f"captured for {tuple(self.x.shape)} {self.x.dtype}, got {tuple(x.shape)} {x.dtype}")
        self.x.copy_(x)
        self.graph.replay()
        return self.result.out


def run_host_batches(fn, inputs: list[torch.Tensor], outputs: list[torch.Tensor]) -> None:
    """``outputs[i][:] = fn(inputs[i])`` for host (pinned) batches, with the
    copies off the compute stream: batch i+1's host->device copy and batch
    i-1's device->host copy run on their own streams while ``fn`` computes
    batch i, so a stream of requests costs max(copy, compute) per batch
    instead of their sum. ``fn`` is any layer call (``moe_layer_forward(...).out``,
    a ``CapturedLayer``, an expert-parallel layer) that runs on the current
    stream; it may return a fresh tensor or the same buffer every call (a
    ``CapturedLayer`` does): each result is copied on the compute stream into
    one of two private device buffers, which the device->host copy reads, so
    the next batch never overwrites a result still being copied out. Returns
    with all work enqueued and the current stream ordered after the last copy;
    synchronise before reading ``outputs``."""
    if not inputs:
        return
    if len(inputs) != len(outputs):
        raise ValueError(f"{len(inputs)} inputs but {len(outputs)} outputs")
    dev = torch.device("cuda", torch.cuda.current_device())
    comp = torch.cuda.current_stream(dev)
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    slots = [torch.empty(inputs[0].shape, dtype=inputs[0].dtype, device=dev) for _ in range(2)]
    # The slots come from the compute stream's pool: the caching allocator may
    # hand back memory that kernels already queued there still read, so the
    # copy stream starts after everything queued on the compute stream so far.
    h2d.wait_stream(comp)
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    snaps: list[torch.Tensor | None] = [None, None]  # private copies of the results
    copied = [torch.cuda.Event() for _ in range(2)]  # device->host copy of a snapshot done
    for i, (xin, yout) in enumerate(zip(inputs, outputs)):
        s = i % 2
        if xin.shape != slots[s].shape or xin.dtype != slots[s].dtype:
            raise ValueError("all input batches must share one shape and dtype")
        with torch.cuda.stream(h2d):
            if i >= 2:
                h2d.wait_event(free[s])  # the layer has finished reading this slot
            slots[s].copy_(xin, non_blocking=True)
            ready[s].record(h2d)
        comp.wait_event(ready[s])
        out = fn(slots[s])
        free[s].record(comp)
        if snaps[s] is None:
            snaps[s] = torch.empty(out.shape, dtype=out.dtype, device=dev)
        elif snaps[s].shape != out.shape or snaps[s].dtype != out.dtype:
            raise ValueError("fn must return one shape and dtype for every batch")
        else:
            comp.wait_event(copied[s])  # batch i-2's result has left this snapshot
        snaps[s].copy_(out)
        d2h.wait_stream(comp)
        with torch.cuda.stream(d2h):
            yout.copy_(snaps[s], non_blocking=True)
            copied[s].record(d2h)
    comp.wait_stream(d2h)
    for t in slots:
        t.record_stream(h2d)
    for t in snaps:
        if t is not None:
            t.record_stream(d2h)
