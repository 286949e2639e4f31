"""Swaps the B200 layer path into a loaded DeepSeek-style model by replacing
each MoE layer's ``moe_infer`` (mirror of the reference's
src/dispatch/kernels/integration.py:51-90, 141-195). The gate, attention and
shared experts stay the model's own code, exactly as in the reference."""

from __future__ import annotations

from collections.abc import Callable, Iterator

import torch

from dispatch_b200.kernels.moe_forward import StackedExpertWeights, grouped_moe_routed, stack_expert_weights
from dispatch_b200.kernels.quantization import (
    QuantizedStackedExpertWeights,
    grouped_moe_routed_quantized,
    quantize_stacked_weights,
)

MoEInfer = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]


def _iter_validated_moe_layers(model: torch.nn.Module) -> Iterator[tuple[torch.nn.Module, torch.nn.ModuleList]]:
    for module in model.modules():
        if not hasattr(module, "moe_infer"):
            continue
        experts = module.experts
        if not isinstance(experts, torch.nn.ModuleList):
            raise TypeError(
                f"expected {type(module).__name__}.experts to be nn.ModuleList, got {type(experts).__name__}"
            )
        yield module, experts


def patch_moe_infer(model: torch.nn.Module, matmul=None, *, block_m: int = 16) -> int:
    """Returns how many MoE layers were patched; forces eval() first (the
    model only calls moe_infer outside training)."""
    model.eval()
    patched = 0
    for module, experts in _iter_validated_moe_layers(model):
        module.moe_infer = _grouped_moe_infer(stack_expert_weights(experts), matmul, block_m)  # type: ignore[assignment]
        patched += 1
    return patched


def patch_moe_infer_quantized(model: torch.nn.Module, matmul=None, *, block_m: int = 16,
                              scale_dtype: torch.dtype = torch.float32) -> int:
    """Quantises each layer's stacked weights to int8 once, frees the
    originals, and installs the int8 path."""
    model.eval()
    patched = 0
    for module, experts in _iter_validated_moe_layers(model):
        qweights = quantize_stacked_weights(stack_expert_weights(experts), scale_dtype=scale_dtype)
        _free_expert_weights(experts)
        module.moe_infer = _grouped_moe_infer_quantized(qweights, matmul, block_m)  # type: ignore[assignment]
        patched += 1
    return patched


def _free_expert_weights(experts: torch.nn.ModuleList) -> None:
    for expert in experts:
        for name in ("gate_proj", "up_proj", "down_proj"):
            linear = getattr(expert, name)
            linear.weight = torch.nn.Parameter(linear.weight.new_empty(0), requires_grad=False)


def _grouped_moe_infer(weights: StackedExpertWeights, matmul, block_m: int) -> MoEInfer:
    @torch.no_grad()
    def moe_infer(x: torch.Tensor, flat_expert_indices: torch.Tensor, flat_expert_weights: torch.Tensor) -> torch.Tensor:
        top_k = flat_expert_indices.numel() // x.shape[0]
        return grouped_moe_routed(x, flat_expert_indices.view(-1, top_k), flat_expert_weights.view(-1, top_k),
                                  weights, matmul, block_m=block_m)

    return moe_infer


def _grouped_moe_infer_quantized(weights: QuantizedStackedExpertWeights, matmul, block_m: int) -> MoEInfer:
    @torch.no_grad()
    def moe_infer(x: torch.Tensor, flat_expert_indices: torch.Tensor, flat_expert_weights: torch.Tensor) -> torch.Tensor:
        top_k = flat_expert_indices.numel() // x.shape[0]
        return grouped_moe_routed_quantized(x, flat_expert_indices.view(-1, top_k),
                                            flat_expert_weights.view(-1, top_k), weights, matmul, block_m=block_m)

    return moe_infer
