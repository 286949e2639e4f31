"""The peer-memory EP layer as a one-rank group on one GPU: every step of the
real multi-GPU path -- count exchange and barriers (exchange_kernel), the
dispatch stores into the receive buffer, the FFN whose epilogue stores rows
into the return buffer, the combine -- against the 1-GPU layer byte for
byte. With one rank every barrier waits only for its own flags, so no kernel
waits on another. The multi-rank path runs in tests/test_gpu_ep.py where
there are GPUs for it."""

from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

H, E, K, I, I_SH = 2048, 64, 6, 1408, 2816


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _make(dev, t: int, quant: bool):
    from dispatch_b200.kernels.moe_forward import SharedExpertWeights, StackedExpertWeights

    g = torch.Generator(device=dev).manual_seed(0)
    rnd = lambda *s: (torch.randn(*s, generator=g, device=dev) * 0.02).to(torch.bfloat16)  # noqa: E731
    router = rnd(E, H)
    ws = StackedExpertWeights(rnd(E, I, H), rnd(E, I, H), rnd(E, H, I))
    sh = SharedExpertWeights(rnd(I_SH, H), rnd(I_SH, H), rnd(H, I_SH))
    if quant:
        from dispatch_b200.kernels.quantization import quantize_stacked_weights

        ws = quantize_stacked_weights(ws)
    x = torch.randn(t, H, generator=torch.Generator(device=dev).manual_seed(11), device=dev).to(torch.bfloat16)
    return router, ws, sh, x


def _worker(rank: int, port: int, t: int, skew: bool, quant: bool, out_dir: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    import torch.distributed as dist

    dist.init_process_group("nccl", rank=0, world_size=1, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from dispatch_b200 import _lib as L
        from dispatch_b200.kernels.ep_peer import PeerEPLayer
        from dispatch_b200.kernels.layer import RouterConfig, moe_layer_forward

        router, ws, sh, x = _make(dev, t, quant)
        bias = (-1.2 * torch.log(torch.arange(E, dtype=torch.float32) + 1.0)).to(dev) if skew else None
        cfg = RouterConfig(top_k=K)
        layer = PeerEPLayer(router, ws, sh, cfg, rank=0, world=1, e_score_bias=bias, max_tokens=t + 3)
        outs = [layer(x), layer(x), layer(x[: (t + 1) // 2])]
        torch.cuda.synchronize()
        L.check_device_status(dev)
        ref = moe_layer_forward(x, router, ws, cfg, shared=sh, e_score_bias=bias).out
        ref_half = moe_layer_forward(x[: (t + 1) // 2].contiguous(), router, ws, cfg, shared=sh,
                                     e_score_bias=bias).out
        torch.cuda.synchronize()
        ok = [torch.equal(outs[0], ref), torch.equal(outs[1], ref), torch.equal(outs[2], ref_half)]
        diff = float((outs[0].float() - ref.float()).abs().max())
        layer.close()
        torch.save({"ok": ok, "diff": diff}, os.path.join(out_dir, "w1.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("t,skew,quant", [(256, False, False), (1, False, False), (1024, True, False),
                                          (300, True, True)])
def test_one_rank_peer_ep_is_byte_exact_vs_one_gpu(t: int, skew: bool, quant: bool, tmp_path) -> None:
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(_free_port(), t, skew, quant, str(tmp_path)), nprocs=1, join=True)
    got = torch.load(tmp_path / "w1.pt")
    assert all(got["ok"]), f"full / repeat / half equal: {got['ok']}, max |diff| {got['diff']}"
