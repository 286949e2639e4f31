"""CPU-only checks of the C ABI and the host logic: the library loads, exports
every entry point the header declares, and the Python surface refuses
non-CUDA tensors instead of falling back to the CPU."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

from dispatch_b200 import _lib as L

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols() -> list[str]:
    text = "\n".join(h.read_text() for h in sorted((ROOT / "include").glob("*.h")))
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(moe_\w+)\s*\(", text, re.M)))


def test_header_declares_entry_points() -> None:
    syms = declared_symbols()
    for must in ("moe_route", "moe_group_tokens", "moe_grouped_gemm", "moe_expert_ffn", "moe_combine",
                 "moe_quantize_int8", "moe_layer_forward", "moe_peer_alloc", "moe_peer_import", "moe_ep_dispatch",
                 "moe_ep_expert_ffn"):
        assert must in syms


def test_library_exports_every_declared_symbol() -> None:
    lib = ctypes.CDLL(str(L.LIB_PATH))
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_python_binding_declares_every_symbol() -> None:
    assert set(declared_symbols()) <= set(L._SIGNATURES)


def test_abi_version_and_status_strings() -> None:
    lib = L.lib()
    assert lib.moe_abi_version() == 1
    assert lib.moe_status_string(L.MOE_ERR_TIMEOUT) == b"device wait timed out"
    assert lib.moe_status_string(L.MOE_ERR_BAD_EXPERT) == b"expert id out of range"


def test_entry_points_report_missing_device_without_crashing() -> None:
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = L.lib()
    rc = lib.moe_route(None, 0, None, 0, None, 1, 8, 4, 2, 0, 0, None, 1, 1, 1.0, None, None, None, None, 0, None,
                       None)
    assert rc == L.MOE_ERR_NO_DEVICE
    assert b"device" in lib.moe_last_error()


def test_workspace_helpers_are_pure_host_arithmetic() -> None:
    lib = L.lib()
    assert lib.moe_group_workspace_bytes(4096, 6, 64) >= 96 * 64 * 4
    assert lib.moe_ffn_workspace_bytes(24576, 1408, 4096, 2816) >= (24576 * 1408 + 4096 * 2816) * 2
    d = L.MoeLayerDesc()
    d.T, d.H, d.E, d.I, d.I_shared, d.k = 4096, 2048, 64, 1408, 2816, 6
    assert lib.moe_layer_workspace_bytes(ctypes.byref(d)) > 2 * 4096 * 6 * 2048 * 2


@pytest.mark.parametrize(("t", "w_dtype", "expect"), [
    (1, L.DT_BF16, L.FFN_KERNEL_WARP),     # decode: routed groups of ~0.1 rows, shared expert of 1
    (16, L.DT_BF16, L.FFN_KERNEL_WARP),    # 96 routed rows over 64 experts, shared 16
    (64, L.DT_BF16, L.FFN_KERNEL_TILED),   # routed groups of 6 rows: past the decode rule
    (1024, L.DT_BF16, L.FFN_KERNEL_TILED),  # groups of 96
    (2048, L.DT_BF16, L.FFN_KERNEL_PAIR),  # groups of 192: one well-filled pair tile
    (3072, L.DT_BF16, L.FFN_KERNEL_TILED),  # groups of 288: a last pair tile of 32 rows
    (4096, L.DT_BF16, L.FFN_KERNEL_PAIR),  # groups of 384
    (4096, L.DT_I8, L.FFN_KERNEL_TILED),   # int8 weights: the pair kernel takes 16-bit ones
    (1, L.DT_I8, L.FFN_KERNEL_WARP),
])
def test_automatic_kernel_choice_on_c2_shapes(t: int, w_dtype: int, expect: int) -> None:
    """The host-only query names the kernel AUTO launches for the C2 layer
    (H 2048, 64 experts top-6, I 1408, one shared expert over all T rows)."""
    assert L.lib().moe_ffn_kernel_auto(t * 6, 64, t, 2048, 1408, w_dtype) == expect


def test_automatic_kernel_choice_limits_wide_int8_decode() -> None:
    """int8 with K above 4096 (the C5 shapes) keeps the warp-MMA kernel only
    for about one token's routed rows; bad sizes answer -1."""
    lib = L.lib()
    assert lib.moe_ffn_kernel_auto(8, 256, 1, 7168, 2048, L.DT_I8) == L.FFN_KERNEL_WARP
    assert lib.moe_ffn_kernel_auto(16, 256, 2, 7168, 2048, L.DT_I8) == L.FFN_KERNEL_TILED
    assert lib.moe_ffn_kernel_auto(16, 256, 2, 7168, 2048, L.DT_BF16) == L.FFN_KERNEL_WARP
    assert lib.moe_ffn_kernel_auto(-1, 64, 0, 2048, 1408, L.DT_BF16) == -1
    assert lib.moe_ffn_kernel_auto(6, 0, 0, 2048, 1408, L.DT_BF16) == -1


def test_python_ops_refuse_cpu_tensors() -> None:
    from dispatch_b200.kernels.grouped_gemm import grouped_matmul
    from dispatch_b200.kernels.grouping import group_tokens_by_expert
    from dispatch_b200.kernels.tile_schedule import build_tile_schedule

    x = torch.randn(4, 16, dtype=torch.bfloat16)
    w = torch.randn(1, 16, 16, dtype=torch.bfloat16)
    sched = build_tile_schedule(torch.tensor([4]), 16)
    with pytest.raises(ValueError, match="CUDA"):
        grouped_matmul(x, w, sched)
    with pytest.raises(ValueError, match="CUDA"):
        group_tokens_by_expert(torch.zeros(3, 2, dtype=torch.long), torch.ones(3, 2), 4)


def test_grouped_matmul_validation_messages_mirror_the_reference() -> None:
    from dispatch_b200.kernels.grouped_gemm import _validated_output
    from dispatch_b200.kernels.tile_schedule import TileSchedule

    class Meta:
        is_cuda = True

    sched = TileSchedule(16, (0, 4), torch.zeros(1), torch.zeros(1), torch.zeros(1))
    x = torch.empty(4, 16, dtype=torch.float16, device="meta")
    w = torch.empty(1, 16, 16, dtype=torch.bfloat16, device="meta")
    with pytest.raises(ValueError, match="CUDA"):
        _validated_output(x, w, sched)


def test_tile_schedule_mirror_matches_reference_known_answers() -> None:
    from dispatch_b200.kernels.tile_schedule import build_tile_schedule

    s = build_tile_schedule(torch.tensor([5, 0, 3, 9]), block_m=4)
    assert s.tile_expert.tolist() == [0, 0, 2, 3, 3, 3]
    assert s.tile_valid_rows.tolist() == [4, 1, 3, 4, 4, 1]
    assert s.group_offsets == (0, 5, 5, 8, 17)
    with pytest.raises(ValueError, match="block_m"):
        build_tile_schedule(torch.tensor([4]), block_m=0)


def test_backend_registry() -> None:
    from dispatch_b200.kernels.backends import resolve_backend
    from dispatch_b200.kernels.grouped_gemm import grouped_matmul

    assert resolve_backend("b200") is grouped_matmul
    with pytest.raises(ValueError, match="unknown backend"):
        resolve_backend("naive")
