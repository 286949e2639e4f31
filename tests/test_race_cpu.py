"""The race driver's host logic on the CPU: dispatch-b200 is registered beside
the reference's contestants (its registry keeps handing out its own), and the
summary table marks refusals and computes the reference/B200 latency ratio."""

from __future__ import annotations

import pytest

from dispatch_b200 import race


def _reference_or_skip():
    try:
        return race.import_reference()
    except ImportError as exc:  # pragma: no cover - the reference install is optional
        pytest.skip(str(exc))


def test_register_adds_dispatch_b200_beside_the_reference_engines() -> None:
    _, registry, *_ = _reference_or_skip()
    stock = tuple(registry.ENGINE_NAMES)
    race.register(registry)
    race.register(registry)  # idempotent
    assert registry.ENGINE_NAMES[: len(stock)] == stock
    assert registry.ENGINE_NAMES.count(race.B200_ENGINE) == 1
    (engine,) = registry.build_engines(race.B200_ENGINE)
    assert engine.name == race.B200_ENGINE
    naive = registry.build_engines("dispatch-naive")
    assert [e.name for e in naive] == [f"dispatch-naive-bm{b}" for b in registry.DEFAULT_BLOCK_MS]
    with pytest.raises(ValueError, match="unknown engine"):
        registry.build_engines("nope")


def test_render_marks_refusals_and_ratios() -> None:
    rows = [
        {"variant": "dispatch-naive-bm16", "precision": "bf16", "distribution": "uniform", "num_tokens": 1,
         "status": "ok", "mean_ms": 0.3},
        {"variant": "vllm", "precision": "bf16", "distribution": "uniform", "num_tokens": 1, "status": "ok",
         "mean_ms": 0.2},
        {"variant": race.B200_ENGINE, "precision": "bf16", "distribution": "uniform", "num_tokens": 1,
         "status": "ok", "mean_ms": 0.1},
        {"variant": "sglang", "precision": "bf16", "distribution": "uniform", "num_tokens": 1,
         "status": "refused", "reason": "No module named 'sglang'"},
    ]
    md = race.render(rows, [1], ["uniform"], ["bf16"])
    assert "| vllm | 0.2000 |" in md
    assert "| sglang | refused |" in md
    assert "2.00x" in md  # best reference-side 0.2 ms / B200 0.1 ms
    assert "No module named 'sglang'" in md
