"""Pins the CPU oracle to the reference: golden vectors written by the
reference itself (tests/golden/make_golden.py) and the reference tests' own
hand-computed known answers, restated here. CPU only."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
from golden_inputs import c1_inputs, toy_inputs

from oracle import moe_oracle as O

GOLD = Path(__file__).resolve().parent / "golden"


def load(name: str):
    return np.load(GOLD / f"{name}.npz")


# --- router ---------------------------------------------------------------


@pytest.mark.parametrize("case,k", [("c1", 2), ("c2u", 6), ("c2z", 6), ("e256", 8)])
def test_router_ids_bit_exact_and_weights_match_reference(case: str, k: int) -> None:
    g = load("route")
    ids, w = O.route_softmax_topk(g[f"{case}_logits"], k)
    np.testing.assert_array_equal(ids, g[f"{case}_idx"])
    np.testing.assert_allclose(w, g[f"{case}_w"], rtol=1e-6, atol=1e-7)


def test_router_logits_match_reference_gate() -> None:
    g = load("route")
    x, rw, *_ = c1_inputs(num_tokens=256)
    np.testing.assert_allclose(x @ rw.T, g["c1_logits"], rtol=1e-5, atol=1e-5)


def test_router_does_not_renormalize_by_default() -> None:
    """reference tests/unit/test_reference_moe.py:40-48."""
    g = load("route")
    _, w = O.route_softmax_topk(g["c2u_logits"], 6)
    assert not np.allclose(w.sum(-1), 1.0)
    _, wr = O.route_softmax_topk(g["c2u_logits"], 6, renormalize=True)
    np.testing.assert_allclose(wr.sum(-1), 1.0, rtol=1e-6)
    np.testing.assert_allclose(wr, w / w.sum(-1, keepdims=True), rtol=1e-6)


def test_router_selects_distinct_experts() -> None:
    g = load("route")
    ids, _ = O.route_softmax_topk(g["e256_logits"], 8)
    assert all(len(set(r.tolist())) == 8 for r in ids)


def test_router_tie_break_prefers_lower_index() -> None:
    logits = np.array([[1.0, 3.0, 3.0, 0.0, 3.0]], dtype=np.float32)
    ids, _ = O.route_softmax_topk(logits, 3)
    assert ids.tolist() == [[1, 2, 4]]


def test_sigmoid_group_router_restates_group_limited_rule() -> None:
    rng = np.random.default_rng(0)
    logits = rng.standard_normal((16, 32)).astype(np.float32)
    bias = (rng.standard_normal(32) * 0.1).astype(np.float32)
    ids, w = O.route_sigmoid_grouped(logits, bias, 4, 8, 2, routed_scaling_factor=2.5)
    s = O.sigmoid_fp32(logits)
    c = s + bias
    for t in range(16):
        gs = np.sort(c[t].reshape(8, 4), axis=-1)[:, -2:].sum(-1)
        kept = set(np.argsort(-gs, kind="stable")[:2].tolist())
        assert {int(e) // 4 for e in ids[t]} <= kept
        allowed = [e for e in range(32) if e // 4 in kept]
        best = sorted(allowed, key=lambda e: (-c[t, e], e))[:4]
        assert ids[t].tolist() == best
        np.testing.assert_allclose(w[t].sum(), 2.5, rtol=1e-5)


# --- grouping / tile schedule ---------------------------------------------


def test_group_sizes_count_every_slot_including_an_empty_expert() -> None:
    """reference tests/unit/test_grouping.py:12-17."""
    g = O.group_tokens_by_expert(np.array([[0, 2], [1, 0], [2, 2]]), np.ones((3, 2)), 4)
    assert g.group_sizes.tolist() == [2, 1, 3, 0]


def test_rows_sorted_expert_major_and_stable() -> None:
    """reference tests/unit/test_grouping.py:20-28."""
    idx = np.array([[2, 0], [0, 1], [2, 1]])
    w = np.array([[0.1, 0.2], [0.3, 0.4], [0.5, 0.6]], dtype=np.float32)
    g = O.group_tokens_by_expert(idx, w, 3)
    assert g.sorted_token_idx.tolist() == [0, 1, 1, 2, 0, 2]
    np.testing.assert_allclose(g.sorted_weight, [0.2, 0.3, 0.4, 0.6, 0.1, 0.5])


def test_ungroup_and_combine_known_answer() -> None:
    """reference tests/unit/test_grouping.py:31-42."""
    g = O.group_tokens_by_expert(np.array([[0, 1], [0, 1]]), np.array([[2.0, 3.0], [4.0, 5.0]]), 2)
    y = np.array([[1.0], [10.0], [100.0], [1000.0]], dtype=np.float32)
    assert O.ungroup_and_combine(y, g, 2).tolist() == [[2.0 + 300.0], [40.0 + 5000.0]]


def test_grouping_rejects_shape_mismatch() -> None:
    with pytest.raises(ValueError, match="shape"):
        O.group_tokens_by_expert(np.zeros((3, 2), np.int64), np.zeros((3, 3)), 4)


def test_combine_rejects_row_mismatch() -> None:
    g = O.group_tokens_by_expert(np.array([[0]]), np.ones((1, 1)), 1)
    with pytest.raises(ValueError, match="rows"):
        O.ungroup_and_combine(np.zeros((2, 4), np.float32), g, 1)


@pytest.mark.parametrize("case", ["t37_e64_k6", "t100_e256_k8", "t1_e64_k6", "t300_e8_k2"])
def test_grouping_and_schedule_match_reference(case: str) -> None:
    g = load("grouping")
    gr = O.group_tokens_by_expert(g[f"{case}_idx"], g[f"{case}_w"], g[f"{case}_group_sizes"].size)
    np.testing.assert_array_equal(gr.sorted_token_idx, g[f"{case}_sorted_token_idx"])
    np.testing.assert_array_equal(gr.sorted_weight, g[f"{case}_sorted_weight"])
    np.testing.assert_array_equal(gr.group_sizes, g[f"{case}_group_sizes"])
    s = O.build_tile_schedule(gr.group_sizes, 16)
    assert s.group_offsets == tuple(g[f"{case}_offsets"].tolist())
    np.testing.assert_array_equal(s.tile_expert, g[f"{case}_tile_expert"])
    np.testing.assert_array_equal(s.tile_row_start, g[f"{case}_tile_row_start"])
    np.testing.assert_array_equal(s.tile_valid_rows, g[f"{case}_tile_valid_rows"])
    np.testing.assert_allclose(
        O.ungroup_and_combine(g[f"{case}_y"], gr, g[f"{case}_idx"].shape[0]),
        g[f"{case}_combined"], rtol=1e-5, atol=1e-6,
    )


def test_tile_schedule_known_answers() -> None:
    """reference tests/unit/test_tile_schedule.py:12-59."""
    s = O.build_tile_schedule(np.array([5, 0, 3, 9]), 4)
    assert s.num_tiles == 6
    assert s.tile_expert.tolist() == [0, 0, 2, 3, 3, 3]
    assert s.tile_valid_rows.tolist() == [4, 1, 3, 4, 4, 1]
    assert s.group_offsets == (0, 5, 5, 8, 17)
    s = O.build_tile_schedule(np.array([6, 4]), 4)
    assert s.tile_row_start.tolist() == [0, 4, 6]
    assert s.tile_valid_rows.tolist() == [4, 2, 4]
    s = O.build_tile_schedule(np.array([0, 0, 0]), 4)
    assert s.num_tiles == 0 and s.group_offsets == (0, 0, 0, 0)
    assert s.tile_expert.dtype == np.int32
    with pytest.raises(ValueError, match="block_m"):
        O.build_tile_schedule(np.array([4]), 0)


# --- layer ------------------------------------------------------------------


def test_toy_layer_matches_reference_forward() -> None:
    g = load("moe")
    x, rw, gate, up, down, sg, su, sd = toy_inputs()
    out, ids, w = O.moe_forward(x, rw, gate, up, down, 2, shared=(sg, su, sd))
    np.testing.assert_array_equal(ids, g["toy_idx"])
    np.testing.assert_allclose(w, g["toy_w"], rtol=1e-6)
    np.testing.assert_allclose(out, g["toy_out"], rtol=1e-5, atol=1e-6)
    routed = O.grouped_moe_routed(x, ids, w, gate, up, down)
    np.testing.assert_allclose(routed, g["toy_routed"], rtol=1e-5, atol=1e-6)


def test_c1_layer_matches_reference_forward() -> None:
    g = load("moe")
    x, rw, gate, up, down = c1_inputs(num_tokens=64)
    out, ids, w = O.moe_forward(x, rw, gate, up, down, 2, logits=g["c1_logits"])
    np.testing.assert_array_equal(ids, g["c1_idx"])
    np.testing.assert_allclose(out, g["c1_out"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(out, g["c1_grouped"], rtol=1e-4, atol=1e-5)


# --- quantisation ----------------------------------------------------------


@pytest.mark.parametrize("case", ["a", "b", "c"])
def test_quantization_bit_exact_vs_reference(case: str) -> None:
    g = load("quant")
    q, s = O.quantize_per_channel_int8(g[f"{case}_w"])
    np.testing.assert_array_equal(q, g[f"{case}_q"])
    np.testing.assert_array_equal(s, g[f"{case}_s"])


def test_quantization_round_trip_within_one_step() -> None:
    """reference tests/unit/test_quantization.py:30-45."""
    g = load("quant")
    w = g["a_w"]
    q, s = O.quantize_per_channel_int8(w)
    step = np.abs(w).max(-1, keepdims=True) / 127
    assert np.all(np.abs(O.dequantize_int8(q, s) - w) <= step * 1.01)


def test_zero_channel_scale_is_one() -> None:
    w = np.zeros((1, 2, 4), np.float32)
    w[0, 1] = [1.0, -2.0, 3.0, -4.0]
    q, s = O.quantize_per_channel_int8(w)
    assert s[0, 0] == 1.0 and not q[0, 0].any()


# --- expert parallelism ------------------------------------------------------


def test_assign_experts_to_ranks() -> None:
    r = O.assign_experts_to_ranks(64, 2)
    assert (r[:32] == 0).all() and (r[32:] == 1).all()
    with pytest.raises(ValueError, match="fewer than"):
        O.assign_experts_to_ranks(1, 2)
    with pytest.raises(ValueError, match="positive"):
        O.assign_experts_to_ranks(0, 2)


@pytest.mark.parametrize("r", [1, 2, 4])
def test_ep_simulation_matches_reference(r: int) -> None:
    g = load("ep")
    np.testing.assert_array_equal(O.assign_experts_to_ranks(8, r), g[f"rank_of_{r}"])
    sim = O.simulate_ep_moe_routed(g["x"], g["idx"], g["w"], g["gate"], g["up"], g["down"], r)
    np.testing.assert_allclose(sim, g[f"sim_{r}"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(sim, g["expected"], rtol=1e-5, atol=1e-6)


def test_bf16_rounding_helper() -> None:
    import torch

    x = np.random.default_rng(0).standard_normal(1000).astype(np.float32)
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(O.round_to_bf16(x), ref)
