"""Expert parallelism emulated on ONE GPU: the peer-transport EP layer
(``PeerEPLayer``) with W ranks that are sets of buffers on the current device,
taking turns on one stream. The on-GPU counterpart of the reference's
``simulate_ep_moe_routed`` (src/dispatch/kernels/expert_parallel.py:89-116),
which sums every rank's local contribution in one process: here every EP data
kernel runs through the C ABI exactly as on W GPUs -- ``moe_ep_dispatch``
stores each rank's rows into the owners' receive buffers (the peer table
holds the W local buffers), ``moe_ep_expert_ffn`` runs each owner's experts
and stores the rows back into the sources' return buffers, ``moe_combine``
sums each source's rows -- and stream order stands in for the flag barriers
of ``moe_ep_exchange``, so no kernel waits on another. Used by the tests (the
output must equal the 1-GPU layer byte for byte) and as a one-GPU profiling
driver for the EP kernels.
"""

from __future__ import annotations

import torch

from dispatch_b200 import _lib as L
from dispatch_b200.kernels.quantization import QuantizedStackedExpertWeights


def _ptr_table(ts: list[torch.Tensor], dev: torch.device) -> torch.Tensor:
    return torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device=dev)


def simulated_ep_forward(xs: list[torch.Tensor], router_w: torch.Tensor, weights, shared, router_cfg,
                         e_score_bias: torch.Tensor | None = None, *, check_offsets: bool = True
                         ) -> list[torch.Tensor]:
    """The expert-parallel layer with ``len(xs)`` ranks emulated on one GPU.
    ``xs[r]`` (T_r, H) 16-bit tokens of rank r (T_r may be 0); ``weights``
    all E experts (bf16 or int8, sliced per owner here), ``shared`` the
    shared expert (or None). Returns each rank's output rows."""
    from dispatch_b200.kernels.expert_parallel import _slice_experts  # noqa: PLC0415
    from dispatch_b200.kernels.grouping import _group  # noqa: PLC0415
    from dispatch_b200.kernels.layer import route  # noqa: PLC0415

    lib = L.lib()
    dev = router_w.device
    world, k = len(xs), router_cfg.top_k
    quant = isinstance(weights, QuantizedStackedExpertWeights)
    g_all = weights.gate.data if quant else weights.gate
    n_experts, inter, hidden = g_all.shape[0], g_all.shape[1], g_all.shape[2]
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not split evenly over {world} ranks")
    e_loc = n_experts // world
    act = L.dt(xs[0])
    i_sh = 0 if shared is None else shared.gate.shape[0]
    st, stream = L.status_word(dev).data_ptr(), L.stream_ptr(dev)
    t_max = max(max(x.shape[0] for x in xs), 1)
    recv_cap = world * t_max * min(k, e_loc)
    ranks = []
    for x in xs:
        idx, w = route(x, router_w, router_cfg, e_score_bias=e_score_bias)
        counts, offsets, pos, _, _, wf, _ = _group(idx, w, n_experts, want_sorted=False)
        ranks.append(dict(x=x.contiguous(), t=x.shape[0], idx=idx, counts=counts, offsets=offsets, pos=pos, wf=wf))
    counts_all = torch.stack([r["counts"] for r in ranks]).contiguous()
    dt16 = xs[0].dtype
    recv = [torch.full((recv_cap, hidden), float("nan"), dtype=dt16, device=dev) for _ in range(world)]
    ret = [torch.full((recv_cap,), -1, dtype=torch.int32, device=dev) for _ in range(world)]
    back_rows = t_max * k  # every rank's return buffer holds max_tokens * k rows, as PeerBuffers sizes them
    back = [torch.full((back_rows, hidden), float("nan"), dtype=dt16, device=dev) for _ in range(world)]
    recv_off = [torch.full((e_loc + 1,), -7, dtype=torch.int32, device=dev) for _ in range(world)]
    t_recv, t_ret, t_back = _ptr_table(recv, dev), _ptr_table(ret, dev), _ptr_table(back, dev)
    # 1. every source stores its rows into the owners' receive buffers
    for r, rk in enumerate(ranks):
        rc = lib.moe_ep_dispatch(
            L.ptr(rk["x"]) if rk["t"] else None, act, rk["t"], hidden, L.ptr(rk["idx"]) if rk["t"] else None,
            L.DT_I32, k, rk["pos"].data_ptr(), rk["offsets"].data_ptr(), counts_all.data_ptr(), r, world, n_experts,
            t_recv.data_ptr(), t_ret.data_ptr(), recv_cap, recv_off[r].data_ptr(), st, stream)
        L.check(rc, "moe_ep_dispatch")
    # 2. every owner runs its experts and stores the rows back into the sources' buffers
    ys = []
    for d, rk in enumerate(ranks):
        wl = _slice_experts(weights, d * e_loc, (d + 1) * e_loc)
        g, u, dn = (wl.gate.data, wl.up.data, wl.down.data) if quant else (wl.gate, wl.up, wl.down)
        g, u, dn = g.contiguous(), u.contiguous(), dn.contiguous()
        sc = tuple(s.contiguous() for s in (wl.gate.scale, wl.up.scale, wl.down.scale)) if quant else (None,) * 3
        t = rk["t"]
        y_sh = torch.empty(max(t, 1), hidden, dtype=dt16, device=dev)
        use_shared = shared is not None and t > 0
        nbytes = lib.moe_ffn_workspace_bytes(recv_cap, inter, t if use_shared else 0, i_sh)
        wsb = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        rc = lib.moe_ep_expert_ffn(
            recv[d].data_ptr(), act, recv_cap, hidden, recv_off[d].data_ptr(), e_loc, ret[d].data_ptr(),
            t_back.data_ptr(), world, back_rows, inter, g.data_ptr(), u.data_ptr(), dn.data_ptr(),
            L.DT_I8 if quant else act, L.ptr(sc[0]), L.ptr(sc[1]), L.ptr(sc[2]), L.dt(sc[0]) if quant else 0,
            L.ptr(rk["x"]) if use_shared else None, t if use_shared else 0, i_sh,
            L.ptr(shared.gate if use_shared else None), L.ptr(shared.up if use_shared else None),
            L.ptr(shared.down if use_shared else None), y_sh.data_ptr(), wsb.data_ptr(), nbytes, st, stream)
        L.check(rc, "moe_ep_expert_ffn")
        ys.append(y_sh if use_shared else None)
    # 3. every source combines its k returned rows per token in slot order
    outs = []
    for r, rk in enumerate(ranks):
        out = torch.empty(rk["t"], hidden, dtype=dt16, device=dev)
        if rk["t"]:
            rc = lib.moe_combine(back[r].data_ptr(), act, rk["pos"].data_ptr(), rk["wf"].data_ptr(), rk["t"], k,
                                 hidden, L.ptr(ys[r]), out.data_ptr(), L.dt(out), st, stream)
            L.check(rc, "moe_combine")
        outs.append(out)
    if check_offsets:
        # the receive offsets each owner computed from the count matrix
        torch.cuda.synchronize(dev)
        tot = counts_all.sum(0).cpu()
        for d in range(world):
            exp = torch.cat([torch.zeros(1, dtype=torch.int64), tot[d * e_loc:(d + 1) * e_loc].cumsum(0)])
            if recv_off[d].cpu().long().tolist() != exp.tolist():
                raise AssertionError(f"rank {d}: receive offsets {recv_off[d].tolist()} != {exp.tolist()}")
    return outs
