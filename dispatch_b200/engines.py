"""The kernel-race engine contract (mirror of the reference's
src/dispatch/benchmark/engines/{base,dispatch_kernels,registry}.py) with the
B200 layer as a contestant.

An engine turns stacked expert weights into a ``LayerFactory`` once
(``prepare_bf16`` / ``prepare_int8``, untimed); the factory binds a
``RaceCase`` (x, topk_idx, topk_weight f32) into a zero-argument callable whose
call is the timed routed-MoE forward. ``reference_output`` is the harness's
f32 checker, the same per-expert computation the reference uses.
"""

from __future__ import annotations

import functools
import math
from collections.abc import Callable, Sequence
from dataclasses import dataclass
from typing import Protocol

import torch

from dispatch_b200.kernels.moe_forward import StackedExpertWeights, grouped_moe_routed
from dispatch_b200.kernels.quantization import QuantizedStackedExpertWeights, grouped_moe_routed_quantized

# DeepSeek-MoE-16B / V2-Lite MoE shape (reference engines/base.py:32-35)
HIDDEN_SIZE = 2048
MOE_INTERMEDIATE_SIZE = 1408
N_ROUTED_EXPERTS = 64
NUM_EXPERTS_PER_TOK = 6
TOKEN_COUNTS = (1, 4, 16, 64, 128, 512, 2048)
DEFAULT_BLOCK_M = 16

_ROUTING_WEIGHTS: dict[str, Callable[[int], torch.Tensor]] = {
    "uniform": torch.ones,
    "zipf": lambda n: 1.0 / torch.arange(1, n + 1, dtype=torch.float32),
}
ROUTING_DISTRIBUTIONS = tuple(_ROUTING_WEIGHTS)


@dataclass(frozen=True)
class RaceCase:
    """One benchmark input; ``topk_weight`` is float32 by contract."""

    x: torch.Tensor  # (num_tokens, hidden)
    topk_idx: torch.Tensor  # (num_tokens, top_k) int64
    topk_weight: torch.Tensor  # (num_tokens, top_k) float32


BoundLayer = Callable[[], torch.Tensor]
LayerFactory = Callable[[RaceCase], BoundLayer]


class MoEEngine(Protocol):
    name: str

    def prepare_bf16(self, weights: StackedExpertWeights) -> LayerFactory: ...

    def prepare_int8(self, qweights: QuantizedStackedExpertWeights) -> LayerFactory: ...


def sample_topk_idx(num_tokens: int, n_experts: int, top_k: int, *, distribution: str,
                    generator: torch.Generator) -> torch.Tensor:
    """Synthetic routing (reference kernels/bench.py:53-68): top_k distinct
    experts per token, uniform or 1/i-skewed."""
    if distribution not in _ROUTING_WEIGHTS:
        raise ValueError(f"unknown distribution {distribution!r}; expected one of {ROUTING_DISTRIBUTIONS}")
    probs = _ROUTING_WEIGHTS[distribution](n_experts).expand(num_tokens, n_experts)
    return torch.multinomial(probs, top_k, replacement=False, generator=generator)


def make_weights(dtype: torch.dtype, *, seed: int, device: str, hidden_size: int = HIDDEN_SIZE,
                 intermediate_size: int = MOE_INTERMEDIATE_SIZE, n_experts: int = N_ROUTED_EXPERTS
                 ) -> StackedExpertWeights:
    """Seeded N(0, 1/K) expert weights (reference engines/base.py:69-88)."""
    g = torch.Generator(device=device).manual_seed(seed)

    def stack(n: int, k: int) -> torch.Tensor:
        return torch.randn(n_experts, n, k, device=device, dtype=dtype, generator=g) / math.sqrt(k)

    return StackedExpertWeights(stack(intermediate_size, hidden_size), stack(intermediate_size, hidden_size),
                                stack(hidden_size, intermediate_size))


def make_case(num_tokens: int, distribution: str, *, dtype: torch.dtype, seed: int, device: str,
              hidden_size: int = HIDDEN_SIZE, n_experts: int = N_ROUTED_EXPERTS,
              top_k: int = NUM_EXPERTS_PER_TOK) -> RaceCase:
    """Seeded case (reference engines/base.py:91-117)."""
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(num_tokens, hidden_size, device=device, dtype=dtype, generator=g)
    topk_idx = sample_topk_idx(num_tokens, n_experts, top_k, distribution=distribution,
                               generator=torch.Generator().manual_seed(seed)).to(device)
    topk_weight = torch.rand(num_tokens, top_k, device=device, dtype=torch.float32, generator=g)
    return RaceCase(x, topk_idx, topk_weight)


def reference_output(case: RaceCase, weights: StackedExpertWeights) -> torch.Tensor:
    """The harness's f32 checker (reference engines/base.py:131-139): per
    expert, rows @ W^T in float32, weighted and summed per token."""
    x = case.x.float()
    out = torch.zeros_like(x)
    for e in range(weights.num_experts):
        tok, slot = (case.topk_idx == e).nonzero(as_tuple=True)
        if tok.numel() == 0:
            continue
        xe = x[tok]
        h = torch.nn.functional.silu(xe @ weights.gate[e].float().T) * (xe @ weights.up[e].float().T)
        out.index_add_(0, tok, (h @ weights.down[e].float().T) * case.topk_weight[tok, slot].float().unsqueeze(-1))
    return out


class B200Engine:
    """dispatch's layer on the B200 kernels as a race contestant."""

    def __init__(self, *, block_m: int = DEFAULT_BLOCK_M) -> None:
        self.name = "dispatch-b200"
        self._block_m = block_m

    def prepare_bf16(self, weights: StackedExpertWeights) -> LayerFactory:
        def bind(case: RaceCase) -> BoundLayer:
            return functools.partial(grouped_moe_routed, case.x, case.topk_idx, case.topk_weight.to(case.x.dtype),
                                     weights, None, block_m=self._block_m)

        return bind

    def prepare_int8(self, qweights: QuantizedStackedExpertWeights) -> LayerFactory:
        def bind(case: RaceCase) -> BoundLayer:
            return functools.partial(grouped_moe_routed_quantized, case.x, case.topk_idx,
                                     case.topk_weight.to(case.x.dtype), qweights, None, block_m=self._block_m)

        return bind


ENGINE_NAMES = ("dispatch-b200",)


def build_engines(engine: str, block_ms: Sequence[int] = (DEFAULT_BLOCK_M,)) -> list[MoEEngine]:
    """Engine name -> contestants (reference engines/registry.py:11-32). The
    tcgen05 kernels tile rows by 128 internally, so one contestant suffices."""
    if engine not in ENGINE_NAMES:
        raise ValueError(f"unknown engine {engine!r}; expected one of {ENGINE_NAMES}")
    return [B200Engine(block_m=block_ms[0])]
