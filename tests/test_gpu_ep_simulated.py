"""Expert parallelism on ONE GPU with W simulated ranks: every EP data-movement
kernel of the peer transport (``moe_ep_dispatch``, ``moe_ep_expert_ffn`` with
its scattered return stores, ``moe_combine``) runs through the C ABI exactly as
on W GPUs, but each "rank" is a set of buffers on cuda:0 and the ranks take
turns on one stream, so stream order stands in for the barriers of
``moe_ep_exchange`` and no kernel waits on another.

Per rank r: route + group its own tokens; the (W, E) count matrix is the stack
of the ranks' counts (what the exchange all-gathers); r's dispatch stores its
rows into the owners' receive buffers (the peer table holds the W local
buffers); each owner runs the FFN over its receive buffer and stores the rows
back into the sources' return buffers; each source combines. The concatenated
outputs must equal the 1-GPU layer on the concatenated tokens byte for byte
(the reference's EP contract, src/dispatch/kernels/expert_parallel.py:119-190,
checked there only to tolerance; here exactly)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gpu_helpers import LayerWeights, randn  # noqa: E402

from dispatch_b200 import _lib as L  # noqa: E402
from dispatch_b200.kernels.expert_parallel import _slice_experts  # noqa: E402
from dispatch_b200.kernels.grouping import _group  # noqa: E402
from dispatch_b200.kernels.layer import RouterConfig, moe_layer_forward, route  # noqa: E402
from dispatch_b200.kernels.moe_forward import SharedExpertWeights, StackedExpertWeights  # noqa: E402
from dispatch_b200.kernels.quantization import QuantizedStackedExpertWeights, quantize_stacked_weights  # noqa: E402

DEV = torch.device("cuda", 0)
H, E, K, I, I_SH = 2048, 64, 6, 1408, 2816


@pytest.fixture(scope="module")
def weights() -> LayerWeights:
    return LayerWeights(h=H, i=I, e=E, i_shared=I_SH, seed=0)


@pytest.fixture(autouse=True)
def _device_status_clean():
    yield
    L.check_device_status(DEV)


def _ptr_table(ts: list[torch.Tensor]) -> torch.Tensor:
    return torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device=DEV)


def simulated_ep_forward(xs: list[torch.Tensor], router_w, ws, sh: SharedExpertWeights, cfg: RouterConfig,
                         bias) -> list[torch.Tensor]:
    """The peer-transport EP layer with len(xs) ranks emulated on one GPU."""
    lib = L.lib()
    world, k = len(xs), cfg.top_k
    e_loc = E // world
    quant = isinstance(ws, QuantizedStackedExpertWeights)
    st, stream = L.status_word(DEV).data_ptr(), L.stream_ptr(DEV)
    t_max = max(max(x.shape[0] for x in xs), 1)
    recv_cap = world * t_max * min(k, e_loc)
    ranks = []
    for x in xs:
        idx, w = route(x, router_w, cfg, e_score_bias=bias)
        counts, offsets, pos, _, _, wf, _ = _group(idx, w, E, want_sorted=False)
        ranks.append(dict(x=x, t=x.shape[0], idx=idx, counts=counts, offsets=offsets, pos=pos, wf=wf))
    counts_all = torch.stack([r["counts"] for r in ranks]).contiguous()
    recv = [torch.full((recv_cap, H), float("nan"), dtype=torch.bfloat16, device=DEV) for _ in range(world)]
    ret = [torch.full((recv_cap,), -1, dtype=torch.int32, device=DEV) for _ in range(world)]
    back_rows = t_max * k  # every rank's return buffer holds max_tokens * k rows, as PeerBuffers sizes them
    back = [torch.full((back_rows, H), float("nan"), dtype=torch.bfloat16, device=DEV) for _ in range(world)]
    recv_off = [torch.full((e_loc + 1,), -7, dtype=torch.int32, device=DEV) for _ in range(world)]
    t_recv, t_ret, t_back = _ptr_table(recv), _ptr_table(ret), _ptr_table(back)
    # 1. every source stores its rows into the owners' receive buffers
    for r, rk in enumerate(ranks):
        rc = lib.moe_ep_dispatch(
            L.ptr(rk["x"]) if rk["t"] else None, L.DT_BF16, rk["t"], H, L.ptr(rk["idx"]) if rk["t"] else None,
            L.DT_I32, k, rk["pos"].data_ptr(), rk["offsets"].data_ptr(), counts_all.data_ptr(), r, world, E,
            t_recv.data_ptr(), t_ret.data_ptr(), recv_cap, recv_off[r].data_ptr(), st, stream)
        L.check(rc, "moe_ep_dispatch")
    # 2. every owner runs its experts and stores the rows back into the sources' buffers
    ys = []
    for d, rk in enumerate(ranks):
        wl = _slice_experts(ws, d * e_loc, (d + 1) * e_loc)
        g, u, dn = (wl.gate.data, wl.up.data, wl.down.data) if quant else (wl.gate, wl.up, wl.down)
        g, u, dn = g.contiguous(), u.contiguous(), dn.contiguous()
        sc = tuple(s.contiguous() for s in (wl.gate.scale, wl.up.scale, wl.down.scale)) if quant else (None,) * 3
        t = rk["t"]
        y_sh = torch.empty(max(t, 1), H, dtype=torch.bfloat16, device=DEV)
        nbytes = lib.moe_ffn_workspace_bytes(recv_cap, I, t, I_SH)
        wsb = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
        rc = lib.moe_ep_expert_ffn(
            recv[d].data_ptr(), L.DT_BF16, recv_cap, H, recv_off[d].data_ptr(), e_loc, ret[d].data_ptr(),
            t_back.data_ptr(), world, back_rows, I, g.data_ptr(), u.data_ptr(), dn.data_ptr(),
            L.DT_I8 if quant else L.DT_BF16, L.ptr(sc[0]), L.ptr(sc[1]), L.ptr(sc[2]),
            L.dt(sc[0]) if quant else 0, L.ptr(rk["x"]) if t else None, t, I_SH, sh.gate.data_ptr(),
            sh.up.data_ptr(), sh.down.data_ptr(), y_sh.data_ptr(), wsb.data_ptr(), nbytes, st, stream)
        L.check(rc, "moe_ep_expert_ffn")
        ys.append(y_sh)
    # 3. every source combines its k returned rows per token in slot order
    outs = []
    for r, rk in enumerate(ranks):
        out = torch.empty(rk["t"], H, dtype=torch.bfloat16, device=DEV)
        if rk["t"]:
            rc = lib.moe_combine(back[r].data_ptr(), L.DT_BF16, rk["pos"].data_ptr(), rk["wf"].data_ptr(), rk["t"],
                                 k, H, ys[r].data_ptr(), out.data_ptr(), L.DT_BF16, st, stream)
            L.check(rc, "moe_combine")
        outs.append(out)
    torch.cuda.synchronize()
    # the receive offsets each owner computed from the count matrix
    tot = counts_all.sum(0).cpu()
    for d in range(world):
        exp = torch.cat([torch.zeros(1, dtype=torch.int64), tot[d * e_loc:(d + 1) * e_loc].cumsum(0)])
        assert recv_off[d].cpu().long().tolist() == exp.tolist()
    return outs


CASES = [
    # (world, tokens per rank, zipf routing, int8 experts)
    (2, [96, 96], False, False),
    (4, [128, 1, 77, 0], True, False),  # ragged ranks, one token, an empty rank
    (8, [64] * 8, False, False),
    (8, [1] * 8, True, False),  # decode: one token per rank
    (4, [200, 150, 100, 50], True, True),  # int8 experts
    (8, [33, 40, 0, 7, 128, 1, 64, 90], False, True),
]


@pytest.mark.parametrize("world,tokens,skew,quant", CASES)
@pytest.mark.parametrize("kernels", ["auto", "ep stream / 1-GPU tiled", "ep tiled / 1-GPU stream"])
def test_simulated_peer_ep_is_byte_exact_vs_one_gpu(weights: LayerWeights, world, tokens, skew, quant,
                                                    kernels) -> None:
    """``kernels`` forces the FFN kernel of the EP ranks and of the 1-GPU
    reference to differ: the rows must match byte for byte whichever kernel
    computed them, including the streaming kernel's scattered return stores."""
    lw = weights
    choice = {"auto": (L.FFN_KERNEL_AUTO, L.FFN_KERNEL_AUTO),
              "ep stream / 1-GPU tiled": (L.FFN_KERNEL_STREAM, L.FFN_KERNEL_TILED),
              "ep tiled / 1-GPU stream": (L.FFN_KERNEL_TILED, L.FFN_KERNEL_STREAM)}[kernels]
    g = torch.Generator(device="cuda").manual_seed(4000 + world * 10 + len(set(tokens)))
    xs = [randn((t, H), g, 1.0) for t in tokens]
    ws = StackedExpertWeights(lw.gate, lw.up, lw.down)
    if quant:
        ws = quantize_stacked_weights(ws, scale_dtype=torch.bfloat16)
    sh = SharedExpertWeights(*lw.shared)
    cfg = RouterConfig(top_k=K)
    bias = (-1.2 * torch.log(torch.arange(E, dtype=torch.float32, device=DEV) + 1.0)) if skew else None
    lib = L.lib()
    prev = lib.moe_set_ffn_kernel(choice[0])
    try:
        outs = simulated_ep_forward(xs, lw.router, ws, sh, cfg, bias)
        lib.moe_set_ffn_kernel(choice[1])
        ref = moe_layer_forward(torch.cat(xs), lw.router, ws, cfg, shared=sh, e_score_bias=bias).out
        torch.cuda.synchronize()
    finally:
        lib.moe_set_ffn_kernel(prev)
    got = torch.cat(outs)
    assert got.shape == ref.shape
    assert torch.equal(got, ref), f"max |diff| = {(got.float() - ref.float()).abs().max().item()}"
