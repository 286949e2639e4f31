"""Seeded input generators shared by the golden-vector script and the tests.

Inputs are drawn with numpy's PCG64 (``default_rng``), which is reproducible
across machines, so large inputs need not be stored in the fixtures.
"""

from __future__ import annotations

import numpy as np


def _bf16(x: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    return b.astype(np.uint32).view(np.float32)


def c1_inputs(num_tokens: int = 256, seed: int = 0):
    """Config 1: hidden 512, 8 experts top-2, intermediate 1024, no shared
    expert. x ~ N(0,1) fp32; router and expert weights ~ N(0, 0.02) rounded to
    bf16 (held as fp32 values, which is exact)."""
    rng = np.random.default_rng(seed)
    h, i, e = 512, 1024, 8
    x = rng.standard_normal((num_tokens, h)).astype(np.float32)
    rw = _bf16(rng.standard_normal((e, h)) * 0.02)
    gate = _bf16(rng.standard_normal((e, i, h)) * 0.02)
    up = _bf16(rng.standard_normal((e, i, h)) * 0.02)
    down = _bf16(rng.standard_normal((e, h, i)) * 0.02)
    return x, rw, gate, up, down


def toy_inputs(seed: int = 7):
    """The reference tests' toy dims: hidden 8, intermediate 16, 4 experts
    top-2, one shared expert, 7 tokens."""
    rng = np.random.default_rng(seed)
    h, i, e = 8, 16, 4
    f = lambda *s: (rng.standard_normal(s) / np.sqrt(s[-1])).astype(np.float32)  # noqa: E731
    x = rng.standard_normal((7, h)).astype(np.float32)
    return x, f(e, h), f(e, i, h), f(e, i, h), f(e, h, i), f(i, h), f(i, h), f(h, i)
