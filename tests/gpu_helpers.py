"""Shared helpers of the GPU parity tests: seeded weights generated on the
device, CPU copies for the oracle, and the two tolerances the parity bar uses."""

from __future__ import annotations

import numpy as np
import torch

# BASELINE tolerance for bf16 layer outputs vs the f32 oracle.
RTOL, ATOL = 2e-2, 1e-2
# The reference's own bar (src/dispatch/kernels/moe_forward.py:23,79-85).
REF_RTOL = 1.6e-2


def assert_parity(actual: torch.Tensor, expected: np.ndarray | torch.Tensor) -> None:
    """Both bars: rtol 2e-2 / atol 1e-2, and the reference's
    assert_matches_reference (rtol 1.6e-2, atol 1.6e-2 * max|expected|)."""
    a = actual.detach().float().cpu()
    e = torch.as_tensor(np.asarray(expected) if not isinstance(expected, torch.Tensor) else expected).float().cpu()
    torch.testing.assert_close(a, e, rtol=RTOL, atol=ATOL)
    atol = REF_RTOL * float(e.abs().max()) if e.numel() else 0.0
    torch.testing.assert_close(a, e, rtol=REF_RTOL, atol=atol)


def assert_int8_parity(actual: torch.Tensor, expected: np.ndarray | torch.Tensor) -> None:
    """The int8 bar: the reference int8 path's own check, assert_matches_reference
    (rtol 1.6e-2, atol 1.6e-2 * max|expected|) against the same int8 weights
    dequantised (tests/unit/test_grouped_gemm_int8_kernel.py:71,95 of the
    reference). Its absolute term scales with the output, as it must for
    layers whose outputs reach several units (config 5), where one bf16
    rounding of the result is already ~1e-2."""
    a = actual.detach().float().cpu()
    e = torch.as_tensor(np.asarray(expected) if not isinstance(expected, torch.Tensor) else expected).float().cpu()
    atol = REF_RTOL * float(e.abs().max()) if e.numel() else 0.0
    torch.testing.assert_close(a, e, rtol=REF_RTOL, atol=atol)


def randn(shape, gen: torch.Generator, scale: float, dtype=torch.bfloat16) -> torch.Tensor:
    return (torch.randn(*shape, generator=gen, device="cuda", dtype=torch.float32) * scale).to(dtype)


def np32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


class LayerWeights:
    """Routed experts (E, I, H)/(E, H, I), router (E, H) and an optional shared
    expert of intermediate I_s, all ~N(0, 0.02) in bf16, seeded on the device."""

    def __init__(self, h: int, i: int, e: int, i_shared: int = 0, seed: int = 0, dtype=torch.bfloat16):
        g = torch.Generator(device="cuda").manual_seed(seed)
        self.router = randn((e, h), g, 0.02, dtype)
        self.gate = randn((e, i, h), g, 0.02, dtype)
        self.up = randn((e, i, h), g, 0.02, dtype)
        self.down = randn((e, h, i), g, 0.02, dtype)
        self.shared = None
        if i_shared:
            self.shared = (randn((i_shared, h), g, 0.02, dtype), randn((i_shared, h), g, 0.02, dtype),
                           randn((h, i_shared), g, 0.02, dtype))
