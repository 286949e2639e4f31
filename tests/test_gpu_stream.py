"""The FFN kernels against each other, through the C ABI: the
weight-streaming kernel (one or two interleaved accumulator chains per tile)
and the tiled kernel.

Every choice must give every row the same bits: the same products summed over
the same k-blocks in the same order, whatever the tile shape or the side of
the tensor-core MMA the operands sit on. The comparison is torch.equal on the
outputs of the public calls with the kernel choice forced (moe_set_ffn_kernel),
over decode and prefill-sized batches, bf16 / f16 / int8 weights, the shared
expert, empty and ragged groups, and N or K not multiples of the tile."""

from __future__ import annotations

import contextlib

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gpu_helpers import LayerWeights, assert_parity, np32, randn  # noqa: E402

from dispatch_b200 import _lib as L  # noqa: E402
from dispatch_b200.kernels.grouped_gemm import grouped_matmul  # noqa: E402
from dispatch_b200.kernels.grouped_gemm_int8 import grouped_matmul_int8  # noqa: E402
from dispatch_b200.kernels.layer import CapturedLayer, RouterConfig, moe_layer_forward  # noqa: E402
from dispatch_b200.kernels.moe_forward import SharedExpertWeights, StackedExpertWeights  # noqa: E402
from dispatch_b200.kernels.quantization import quantize_per_channel_int8, quantize_stacked_weights  # noqa: E402
from dispatch_b200.kernels.tile_schedule import build_tile_schedule  # noqa: E402
from oracle import moe_oracle as O  # noqa: E402

DEV = torch.device("cuda", 0)


@contextlib.contextmanager
def ffn_kernel(choice: int):
    prev = L.lib().moe_set_ffn_kernel(choice)
    assert prev >= 0
    try:
        yield
    finally:
        L.lib().moe_set_ffn_kernel(prev)


@pytest.fixture(autouse=True)
def _device_status_clean():
    yield
    L.check_device_status(DEV)


def test_kernel_choice_round_trips_and_rejects_unknown() -> None:
    lib = L.lib()
    prev = lib.moe_set_ffn_kernel(L.FFN_KERNEL_STREAM)
    assert lib.moe_set_ffn_kernel(prev) == L.FFN_KERNEL_STREAM
    assert lib.moe_set_ffn_kernel(7) == -1
    assert lib.moe_set_ffn_kernel(prev) == prev


def _both(fn):
    with ffn_kernel(L.FFN_KERNEL_TILED):
        a = fn()
    with ffn_kernel(L.FFN_KERNEL_STREAM):
        b = fn()
    torch.cuda.synchronize()
    return a, b



GEMM_CASES = [
    ([5, 0, 3, 40], 24, 16),  # toy dims, an empty group, N and K below one tile
    ([1, 1, 1, 1, 1, 1], 1408, 2048),  # decode-shaped gate/up
    ([70, 0, 33, 129], 2048, 1408),  # several row tiles per group, partial tiles
    ([300, 0, 1, 257, 128], 200, 64),  # N not a multiple of 128
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize(("sizes", "n", "k"), GEMM_CASES)
def test_stream_grouped_matmul_equals_tiled(dtype, sizes, n, k) -> None:
    g = torch.Generator(device="cuda").manual_seed(31)
    sched = build_tile_schedule(torch.tensor(sizes, device=DEV), block_m=16)
    x = randn((sum(sizes), k), g, 1.0, dtype)
    w = randn((len(sizes), n, k), g, k ** -0.5, dtype)
    a, b = _both(lambda: grouped_matmul(x, w, sched))
    assert torch.equal(a, b)
    assert_parity(b, O.grouped_matmul(np32(x), np32(w), sched.group_offsets))


@pytest.mark.parametrize("scale_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize(("sizes", "n", "k"), GEMM_CASES)
def test_stream_int8_grouped_matmul_equals_tiled(scale_dtype, sizes, n, k) -> None:
    g = torch.Generator(device="cuda").manual_seed(32)
    sched = build_tile_schedule(torch.tensor(sizes, device=DEV), block_m=16)
    x = randn((sum(sizes), k), g, 1.0)
    q = quantize_per_channel_int8(randn((len(sizes), n, k), g, k ** -0.5, torch.float32), scale_dtype=scale_dtype)
    a, b = _both(lambda: grouped_matmul_int8(x, q, sched))
    assert torch.equal(a, b)


@pytest.fixture(scope="module")
def c2() -> LayerWeights:
    return LayerWeights(h=2048, i=1408, e=64, i_shared=2816, seed=3)


@pytest.mark.parametrize("t", [1, 7, 16, 128, 300, 1024, 4096])
@pytest.mark.parametrize("quant", [False, True])
def test_stream_layer_equals_tiled(c2: LayerWeights, t: int, quant: bool) -> None:
    """The whole C2 layer (routed SwiGLU + down + shared expert): the same
    bits from both kernels (the streaming one with one or two chains per
    tile, depending on the tile count), uniform and Zipf routing."""
    ws = StackedExpertWeights(c2.gate, c2.up, c2.down)
    if quant:
        ws = quantize_stacked_weights(ws, scale_dtype=torch.bfloat16)
    sh = SharedExpertWeights(*c2.shared)
    g = torch.Generator(device="cuda").manual_seed(900 + t)
    x = randn((t, 2048), g, 1.0)
    for bias in (None, -1.2 * torch.log(torch.arange(64, dtype=torch.float32, device=DEV) + 1.0)):
        a, b = _both(lambda: moe_layer_forward(x, c2.router, ws, RouterConfig(top_k=6), shared=sh,
                                               e_score_bias=bias).out)
        assert torch.equal(a, b), f"T={t}: max |diff| {(a.float() - b.float()).abs().max().item()}"


def test_automatic_choice_at_decode_gives_the_forced_kernels_bits(c2: LayerWeights) -> None:
    """AUTO (the warp-MMA kernel at this decode size) gives the same bits as
    the forced tiled and streaming kernels."""
    ws, sh = StackedExpertWeights(c2.gate, c2.up, c2.down), SharedExpertWeights(*c2.shared)
    x = randn((4, 2048), torch.Generator(device="cuda").manual_seed(5), 1.0)
    fwd = lambda: moe_layer_forward(x, c2.router, ws, RouterConfig(top_k=6), shared=sh).out  # noqa: E731
    with ffn_kernel(L.FFN_KERNEL_AUTO):
        auto = fwd()
    a, b = _both(fwd)
    assert torch.equal(auto, a) and torch.equal(auto, b)


def _pair_vs_tiled(fn):
    with ffn_kernel(L.FFN_KERNEL_TILED):
        a = fn()
    with ffn_kernel(L.FFN_KERNEL_PAIR):
        b = fn()
    torch.cuda.synchronize()
    return a, b


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize(("sizes", "n", "k"), GEMM_CASES)
def test_pair_grouped_matmul_equals_tiled(dtype, sizes, n, k) -> None:
    """The CTA-pair kernel (256 weight rows on the MMA's M side over two SMs,
    cta_group::2, and up to 256 token columns rounded to 32) gives the tiled
    kernel's bits on plain GEMMs: empty groups, groups of a few rows (token
    columns past the group holding other groups' rows or nothing), N and K
    not multiples of the tile."""
    g = torch.Generator(device="cuda").manual_seed(33)
    sched = build_tile_schedule(torch.tensor(sizes, device=DEV), block_m=16)
    x = randn((sum(sizes), k), g, 1.0, dtype)
    w = randn((len(sizes), n, k), g, k ** -0.5, dtype)
    a, b = _pair_vs_tiled(lambda: grouped_matmul(x, w, sched))
    assert torch.equal(a, b)


@pytest.mark.parametrize("t", [1, 300, 1024, 4096])
def test_pair_layer_equals_tiled(c2: LayerWeights, t: int) -> None:
    """The whole C2 layer (SwiGLU: each SM of a pair holds 64 gate rows and
    the same channels' up rows, its epilogue warps exchanging halves; down;
    shared expert): the CTA-pair kernel gives the tiled kernel's bits."""
    ws, sh = StackedExpertWeights(c2.gate, c2.up, c2.down), SharedExpertWeights(*c2.shared)
    x = randn((t, 2048), torch.Generator(device="cuda").manual_seed(950 + t), 1.0)
    for bias in (None, -1.2 * torch.log(torch.arange(64, dtype=torch.float32, device=DEV) + 1.0)):
        a, b = _pair_vs_tiled(lambda: moe_layer_forward(x, c2.router, ws, RouterConfig(top_k=6), shared=sh,
                                                        e_score_bias=bias).out)
        assert torch.equal(a, b), f"T={t}: max |diff| {(a.float() - b.float()).abs().max().item()}"


@pytest.mark.parametrize("quant", [False, True])
def test_one_token_call_forks_the_shared_expert_with_the_same_bits(c2: LayerWeights, quant: bool) -> None:
    """A one-token layer call runs the shared expert on a second stream beside
    the routed path; a larger batch runs it inside the routed launches. Each
    token's row must come out the same either way, eager and captured in a
    CUDA graph."""
    ws, sh = StackedExpertWeights(c2.gate, c2.up, c2.down), SharedExpertWeights(*c2.shared)
    if quant:
        ws = quantize_stacked_weights(ws, scale_dtype=torch.bfloat16)
    cfg = RouterConfig(top_k=6)
    x = randn((5, 2048), torch.Generator(device="cuda").manual_seed(77), 1.0)
    batch = moe_layer_forward(x, c2.router, ws, cfg, shared=sh).out
    for i in range(5):
        one = moe_layer_forward(x[i:i + 1].contiguous(), c2.router, ws, cfg, shared=sh).out
        assert torch.equal(one[0], batch[i]), f"token {i}"
    cap = CapturedLayer(x[2:3].contiguous(), c2.router, ws, cfg, shared=sh)
    for _ in range(2):
        assert torch.equal(cap.replay().out[0], batch[2])


def _warp_vs_tiled(fn):
    with ffn_kernel(L.FFN_KERNEL_TILED):
        a = fn()
    with ffn_kernel(L.FFN_KERNEL_WARP):
        b = fn()
    torch.cuda.synchronize()
    return a, b


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize(("sizes", "n", "k"), GEMM_CASES + [([40, 0, 1, 33, 7], 384, 2048)])
def test_warp_grouped_matmul_equals_tiled(dtype, sizes, n, k) -> None:
    """The warp-MMA kernel (eight warps per CTA, each a chain of mma.sync
    m16n8k16 MMAs over K in order) gives the tiled tcgen05 kernel's bits:
    groups longer than its 32-row token tile, empty groups, N and K not
    multiples of the tile."""
    g = torch.Generator(device="cuda").manual_seed(35)
    sched = build_tile_schedule(torch.tensor(sizes, device=DEV), block_m=16)
    x = randn((sum(sizes), k), g, 1.0, dtype)
    w = randn((len(sizes), n, k), g, k ** -0.5, dtype)
    a, b = _warp_vs_tiled(lambda: grouped_matmul(x, w, sched))
    assert torch.equal(a, b), f"max |diff| {(a.float() - b.float()).abs().max().item()}"


@pytest.mark.parametrize("scale_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize(("sizes", "n", "k"), GEMM_CASES)
def test_warp_int8_grouped_matmul_equals_tiled(scale_dtype, sizes, n, k) -> None:
    """int8 weights on the warp-MMA kernel (each warp converts its own rows
    into the MMA operand registers, scales applied in the epilogue): the
    tiled kernel's bits."""
    g = torch.Generator(device="cuda").manual_seed(36)
    sched = build_tile_schedule(torch.tensor(sizes, device=DEV), block_m=16)
    x = randn((sum(sizes), k), g, 1.0)
    q = quantize_per_channel_int8(randn((len(sizes), n, k), g, k ** -0.5, torch.float32), scale_dtype=scale_dtype)
    a, b = _warp_vs_tiled(lambda: grouped_matmul_int8(x, q, sched))
    assert torch.equal(a, b)


@pytest.mark.parametrize("t", [1, 7, 16, 64, 300])
@pytest.mark.parametrize("quant", [False, True])
def test_warp_layer_equals_tiled(c2: LayerWeights, t: int, quant: bool) -> None:
    """The whole C2 layer with both FFN projections on the warp-MMA kernel
    (SwiGLU pairs exchanging accumulators through shared memory, the shared
    expert as a dense segment; int8 routed experts beside the bf16 shared
    expert in one launch): the tiled kernel's bits, uniform and Zipf."""
    ws, sh = StackedExpertWeights(c2.gate, c2.up, c2.down), SharedExpertWeights(*c2.shared)
    if quant:
        ws = quantize_stacked_weights(ws, scale_dtype=torch.bfloat16)
    x = randn((t, 2048), torch.Generator(device="cuda").manual_seed(970 + t), 1.0)
    for bias in (None, -1.2 * torch.log(torch.arange(64, dtype=torch.float32, device=DEV) + 1.0)):
        a, b = _warp_vs_tiled(lambda: moe_layer_forward(x, c2.router, ws, RouterConfig(top_k=6), shared=sh,
                                                        e_score_bias=bias).out)
        assert torch.equal(a, b), f"T={t}: max |diff| {(a.float() - b.float()).abs().max().item()}"
