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
from dispatch_b200.kernels.ep_sim import simulated_ep_forward  # noqa: E402
from dispatch_b200.kernels.layer import RouterConfig, moe_layer_forward  # noqa: E402
from dispatch_b200.kernels.moe_forward import SharedExpertWeights, StackedExpertWeights  # noqa: E402
from dispatch_b200.kernels.quantization import quantize_stacked_weights  # noqa: E402

DEV = torch.device("cuda", 0)
H, E, K, I, I_SH = 2048, 64, 6, 1408, 2816


@pytest.fixture(scope="module")
def weights() -> LayerWeights:
    return LayerWeights(h=H, i=I, e=E, i_shared=I_SH, seed=0)


@pytest.fixture(autouse=True)
def _device_status_clean():
    yield
    L.check_device_status(DEV)


CASES = [
    # (world, tokens per rank, zipf routing, int8 experts)
    (2, [96, 96], False, False),
    (4, [128, 1, 77, 0], True, False),  # ragged ranks, one token, an empty rank
    (8, [64] * 8, False, False),
    (8, [1] * 8, True, False),  # decode: one token per rank
    (4, [200, 150, 100, 50], True, True),  # int8 experts
    (8, [33, 40, 0, 7, 128, 1, 64, 90], False, True),
    (2, [2048, 2048], False, False),  # prefill: (rank, expert) groups of ~192 rows, CTA-pair tiles under AUTO
]


@pytest.mark.parametrize("world,tokens,skew,quant", CASES)
@pytest.mark.parametrize("kernels", ["auto", "ep stream / 1-GPU tiled", "ep tiled / 1-GPU stream",
                                     "ep warp / 1-GPU tiled", "ep pair / 1-GPU tiled"])
def test_simulated_peer_ep_is_byte_exact_vs_one_gpu(weights: LayerWeights, world, tokens, skew, quant,
                                                    kernels) -> None:
    """``kernels`` forces the FFN kernel of the EP ranks and of the 1-GPU
    reference to differ: the rows must match byte for byte whichever kernel
    computed them, including the streaming and CTA-pair kernels' scattered
    return stores."""
    if quant and "pair" in kernels:
        pytest.skip("the CTA-pair kernel takes 16-bit weights")
    lw = weights
    choice = {"auto": (L.FFN_KERNEL_AUTO, L.FFN_KERNEL_AUTO),
              "ep stream / 1-GPU tiled": (L.FFN_KERNEL_STREAM, L.FFN_KERNEL_TILED),
              "ep tiled / 1-GPU stream": (L.FFN_KERNEL_TILED, L.FFN_KERNEL_STREAM),
              "ep warp / 1-GPU tiled": (L.FFN_KERNEL_WARP, L.FFN_KERNEL_TILED),
              "ep pair / 1-GPU tiled": (L.FFN_KERNEL_PAIR, L.FFN_KERNEL_TILED)}[kernels]
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
