"""The reference-facing surfaces on the GPU: the race-engine contract
(engines/base.py MoEEngine) and model patching (integration.py
patch_moe_infer*), each against an f32 computation of the same layer."""

from __future__ import annotations

import copy

import pytest
import torch
import torch.nn.functional as F  # noqa: N812

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gpu_helpers import assert_parity  # noqa: E402

from dispatch_b200.engines import B200Engine, build_engines, make_case, make_weights, reference_output  # noqa: E402
from dispatch_b200.kernels.integration import patch_moe_infer, patch_moe_infer_quantized  # noqa: E402
from dispatch_b200.kernels.moe_forward import StackedExpertWeights, assert_matches_reference  # noqa: E402
from dispatch_b200.kernels.quantization import dequantize_int8, quantize_stacked_weights  # noqa: E402

DEV = "cuda"


@pytest.mark.parametrize("num_tokens", [1, 16, 128])
@pytest.mark.parametrize("distribution", ["uniform", "zipf"])
def test_engine_bf16_matches_reference_output(num_tokens: int, distribution: str) -> None:
    weights = make_weights(torch.bfloat16, seed=0, device=DEV)
    case = make_case(num_tokens, distribution, dtype=torch.bfloat16, seed=1, device=DEV)
    (engine,) = build_engines("dispatch-b200")
    out = engine.prepare_bf16(weights)(case)()
    assert out.dtype == torch.bfloat16 and out.shape == case.x.shape
    # the race harness's own bar (run_engine_race.py refuses engines that fail it)
    assert_matches_reference(out, reference_output(case, weights))


@pytest.mark.parametrize("num_tokens", [4, 64])
def test_engine_int8_matches_dequantized_reference(num_tokens: int) -> None:
    weights = make_weights(torch.bfloat16, seed=0, device=DEV)
    q = quantize_stacked_weights(weights)
    case = make_case(num_tokens, "uniform", dtype=torch.bfloat16, seed=2, device=DEV)
    out = B200Engine().prepare_int8(q)(case)()
    deq = StackedExpertWeights(dequantize_int8(q.gate), dequantize_int8(q.up), dequantize_int8(q.down))
    assert_matches_reference(out, reference_output(case, deq))


class Expert(torch.nn.Module):
    def __init__(self, h: int, i: int):
        super().__init__()
        self.gate_proj = torch.nn.Linear(h, i, bias=False)
        self.up_proj = torch.nn.Linear(h, i, bias=False)
        self.down_proj = torch.nn.Linear(i, h, bias=False)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class DeepseekStyleMoE(torch.nn.Module):
    """A test double of a DeepSeek MoE block: softmax top-k gate, a ModuleList
    of experts, a shared expert, and a moe_infer(x, flat_ids, flat_weights)
    that loops over experts and scatter-adds, as the model's own code does."""

    def __init__(self, h: int, i: int, e: int, k: int):
        super().__init__()
        self.k = k
        self.gate = torch.nn.Linear(h, e, bias=False)
        self.experts = torch.nn.ModuleList(Expert(h, i) for _ in range(e))
        self.shared_experts = Expert(h, 2 * i)

    def forward(self, x):
        scores = F.softmax(self.gate(x), dim=-1, dtype=torch.float32)
        w, idx = torch.topk(scores, self.k, dim=-1)
        y = self.moe_infer(x, idx.view(-1), w.to(x.dtype).view(-1, 1))
        return y + self.shared_experts(x)

    @torch.no_grad()
    def moe_infer(self, x, flat_idx, flat_w):
        out = torch.zeros_like(x, dtype=torch.float32)
        tok = torch.arange(x.shape[0], device=x.device).repeat_interleave(self.k)
        for e, expert in enumerate(self.experts):
            m = flat_idx == e
            if m.any():
                out.index_add_(0, tok[m], expert(x[tok[m]]).float() * flat_w[m].float())
        return out.to(x.dtype)


def _model(n_layers: int = 2) -> torch.nn.Module:
    torch.manual_seed(0)
    layers = torch.nn.ModuleList(DeepseekStyleMoE(256, 128, 16, 4) for _ in range(n_layers))
    return torch.nn.Sequential(*layers).to(DEV, torch.bfloat16)


def test_patch_moe_infer_matches_the_models_own_moe_infer() -> None:
    model = _model()
    x = torch.randn(37, 256, device=DEV, dtype=torch.bfloat16)
    with torch.no_grad():
        expected = model(x)
    assert patch_moe_infer(model) == 2
    with torch.no_grad():
        actual = model(x)
    assert_parity(actual, expected)


def test_patch_moe_infer_quantized_matches_dequantized_model() -> None:
    model = _model(1)
    ref = copy.deepcopy(model)
    x = torch.randn(19, 256, device=DEV, dtype=torch.bfloat16)
    # the reference model with every expert weight replaced by its int8 round trip
    from dispatch_b200.kernels.quantization import quantize_per_channel_int8

    for layer in ref:
        for ex in layer.experts:
            for name in ("gate_proj", "up_proj", "down_proj"):
                lin = getattr(ex, name)
                qt = quantize_per_channel_int8(lin.weight.detach().unsqueeze(0))
                lin.weight = torch.nn.Parameter(dequantize_int8(qt).squeeze(0).to(torch.bfloat16), requires_grad=False)
    with torch.no_grad():
        expected = ref(x)
    assert patch_moe_infer_quantized(model) == 1
    with torch.no_grad():
        actual = model(x)
    assert_parity(actual, expected)
