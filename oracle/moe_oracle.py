"""CPU oracle for the routed MoE-layer hot path -- TEST INFRASTRUCTURE ONLY.

This module is a plain numpy restatement of the reference's pure-PyTorch MoE
path (bsreecharanreddy/dispatch, ``src/dispatch/kernels``). It exists to check
the CUDA path: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it, and
only as the checker or the timed CPU baseline. The product package
(``dispatch_b200``) never imports it and has no CPU fallback.

Pinning: every function below is checked bit-exactly (integers) or at fp32
rounding level (floats) against golden vectors produced by the reference itself
(``tests/golden/make_golden.py`` imports the reference's Python modules and
writes ``tests/golden/*.npz``) plus the reference's own hand-computed known
answers (``tests/unit/test_grouping.py``, ``test_tile_schedule.py``,
``test_quantization.py``), restated in ``tests/test_oracle_golden.py``.

Two routers have no counterpart in the reference and are therefore
"parity unpinned": the renormalised softmax top-k (``norm_topk_prob=True``) is
pinned only through its un-normalised half, and the DeepSeek-V3 sigmoid
group-limited router is restated from the published routing rule.

Arithmetic conventions (shared with the CUDA kernels):
  * expert selection ranks experts by logit (softmax and sigmoid are monotone),
    ties broken towards the lower expert index, slots in descending order;
  * grouped matmuls accumulate in fp32; SwiGLU is silu(gate) * up in fp32;
  * the weighted combine sums the k slots of a token in slot order in fp32.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

# ---------------------------------------------------------------------------
# router
# ---------------------------------------------------------------------------


def softmax_fp32(logits: np.ndarray) -> np.ndarray:
    """Row softmax in fp32 with max subtraction.

    Follows ``F.softmax(self.gate(h), dim=-1, dtype=torch.float32)``
    (reference ``src/dispatch/kernels/reference_moe.py:59``).
    """
    z = logits.astype(np.float32)
    z = z - z.max(axis=-1, keepdims=True)
    e = np.exp(z, dtype=np.float32)
    return (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)


def topk_by_value(values: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest entries per row, descending, lower index first
    on ties (the observable order of ``torch.topk`` on distinct values,
    reference ``reference_moe.py:60``)."""
    n = values.shape[-1]
    # lexsort: last key is primary. Sort by (-value, index).
    idx = np.arange(n)
    out = np.empty(values.shape[:-1] + (k,), dtype=np.int64)
    flat_v = values.reshape(-1, n)
    flat_o = out.reshape(-1, k)
    for r in range(flat_v.shape[0]):
        order = np.lexsort((idx, -flat_v[r].astype(np.float64)))
        flat_o[r] = order[:k]
    return out


def route_softmax_topk(
    logits: np.ndarray, top_k: int, *, renormalize: bool = False
) -> tuple[np.ndarray, np.ndarray]:
    """Softmax top-k router: ids (T, k) int64 and fp32 weights (T, k).

    ``ReferenceMoE.route`` (reference ``reference_moe.py:56-61``) computes fp32
    softmax probabilities and keeps the top-k of them *without* renormalising.
    ``renormalize=True`` adds ``w / w.sum(-1)`` in fp32 (the DeepSeek
    ``norm_topk_prob=True`` variant; no reference test pins it).
    Selection ranks by logit, which orders experts exactly as the softmax
    probabilities do (softmax is strictly monotone).
    """
    logits = np.asarray(logits, dtype=np.float32)
    probs = softmax_fp32(logits)
    ids = topk_by_value(logits, top_k)
    w = np.take_along_axis(probs, ids, axis=-1).astype(np.float32)
    if renormalize:
        w = (w / w.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    return ids, w


def sigmoid_fp32(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.float32)
    return (np.float32(1.0) / (np.float32(1.0) + np.exp(-x, dtype=np.float32))).astype(np.float32)


def route_sigmoid_grouped(
    logits: np.ndarray,
    bias: np.ndarray,
    top_k: int,
    n_group: int,
    topk_group: int,
    *,
    routed_scaling_factor: float = 1.0,
    renormalize: bool = True,
) -> tuple[np.ndarray, np.ndarray]:
    """DeepSeek-V3 group-limited sigmoid router, restated from the published
    routing rule (no counterpart in the reference: parity unpinned).

    1. s = sigmoid(logits); c = s + bias (the load-balancing correction is
       used for selection only).
    2. group score = sum of the two largest c in each of ``n_group`` contiguous
       groups of experts.
    3. keep the ``topk_group`` best groups (descending score, lower group index
       on ties); experts outside them are excluded.
    4. pick ``top_k`` experts by c among the kept groups (descending, lower
       index on ties).
    5. weight = s of the picked expert, normalised to sum 1 when
       ``renormalize``, then multiplied by ``routed_scaling_factor``.
    """
    logits = np.asarray(logits, dtype=np.float32)
    t, e = logits.shape
    if e % n_group:
        raise ValueError(f"n_experts={e} is not divisible by n_group={n_group}")
    s = sigmoid_fp32(logits)
    c = (s + bias.astype(np.float32)[None, :]).astype(np.float32)
    per = e // n_group
    cg = c.reshape(t, n_group, per)
    # sum of top-2 per group (per >= 2 required)
    top2 = -np.sort(-cg.astype(np.float32), axis=-1)[..., :2]
    gscore = (top2[..., 0] + top2[..., 1]).astype(np.float32)
    gsel = topk_by_value(gscore, topk_group)
    mask = np.zeros((t, n_group), dtype=bool)
    np.put_along_axis(mask, gsel, True, axis=-1)
    emask = np.repeat(mask, per, axis=-1)
    masked = np.where(emask, c.astype(np.float64), -np.inf)
    ids = topk_by_value(masked, top_k)
    w = np.take_along_axis(s, ids, axis=-1).astype(np.float32)
    if renormalize:
        w = (w / w.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    w = (w * np.float32(routed_scaling_factor)).astype(np.float32)
    return ids, w


# ---------------------------------------------------------------------------
# grouping / tile schedule
# ---------------------------------------------------------------------------


@dataclass(frozen=True)
class Grouping:
    """Mirror of ``TokenGrouping`` (reference ``grouping.py:15-22``) plus the
    inverse permutation ``pos`` (flat slot t*k+s -> grouped row)."""

    sorted_token_idx: np.ndarray  # (T*k,) int64
    sorted_weight: np.ndarray  # (T*k,)
    group_sizes: np.ndarray  # (E,) int64
    pos: np.ndarray  # (T*k,) int64


def group_tokens_by_expert(
    topk_idx: np.ndarray, topk_weight: np.ndarray, n_experts: int
) -> Grouping:
    """Stable sort of the flat (token, slot) pairs by expert id.

    Follows ``group_tokens_by_expert`` (reference ``grouping.py:25-41``):
    ``argsort(flat_expert_idx, stable=True)``, token = flat // k, sizes by
    bincount. Out-of-range ids raise, as ``torch.bincount(minlength=E)`` would
    silently grow the histogram instead.
    """
    topk_idx = np.asarray(topk_idx)
    topk_weight = np.asarray(topk_weight)
    if topk_idx.shape != topk_weight.shape:
        raise ValueError(
            f"topk_idx.shape {tuple(topk_idx.shape)} != topk_weight.shape {tuple(topk_weight.shape)}"
        )
    t, k = topk_idx.shape
    flat = topk_idx.reshape(-1).astype(np.int64)
    if flat.size and (flat.min() < 0 or flat.max() >= n_experts):
        raise ValueError("expert id out of range")
    order = np.argsort(flat, kind="stable")
    pos = np.empty_like(order)
    pos[order] = np.arange(order.size)
    return Grouping(
        sorted_token_idx=(order // max(k, 1)).astype(np.int64),
        sorted_weight=topk_weight.reshape(-1)[order],
        group_sizes=np.bincount(flat, minlength=n_experts).astype(np.int64),
        pos=pos.astype(np.int64),
    )


def group_offsets(group_sizes: np.ndarray) -> np.ndarray:
    """Exclusive prefix sum, length E+1 (reference ``tile_schedule.py:32-41``)."""
    out = np.zeros(len(group_sizes) + 1, dtype=np.int64)
    np.cumsum(group_sizes, out=out[1:])
    return out


@dataclass(frozen=True)
class TileSchedule:
    block_m: int
    group_offsets: tuple[int, ...]
    tile_expert: np.ndarray
    tile_row_start: np.ndarray
    tile_valid_rows: np.ndarray

    @property
    def num_tiles(self) -> int:
        return int(self.tile_expert.shape[0])


def build_tile_schedule(group_sizes: np.ndarray, block_m: int) -> TileSchedule:
    """Per-expert block_m-row tiles (reference ``tile_schedule.py:28-50``)."""
    if block_m <= 0:
        raise ValueError(f"block_m must be positive, got {block_m}")
    offs = [0]
    te: list[int] = []
    ts: list[int] = []
    tv: list[int] = []
    for e, size in enumerate(np.asarray(group_sizes).tolist()):
        for local in range(0, size, block_m):
            te.append(e)
            ts.append(offs[-1] + local)
            tv.append(min(block_m, size - local))
        offs.append(offs[-1] + size)
    i32 = np.int32
    return TileSchedule(block_m, tuple(offs), np.array(te, i32), np.array(ts, i32), np.array(tv, i32))


# ---------------------------------------------------------------------------
# expert FFN
# ---------------------------------------------------------------------------


def grouped_matmul(x: np.ndarray, w: np.ndarray, offsets) -> np.ndarray:
    """out[rows of e] = x[rows of e] @ w[e].T in fp32 (reference
    ``moe_forward.py:39-47``, ``torch_grouped_matmul``)."""
    x = np.asarray(x, dtype=np.float32)
    w = np.asarray(w, dtype=np.float32)
    out = np.zeros((x.shape[0], w.shape[1]), dtype=np.float32)
    offsets = list(offsets)
    for e in range(len(offsets) - 1):
        s, t = int(offsets[e]), int(offsets[e + 1])
        if t > s:
            out[s:t] = x[s:t] @ w[e].T
    return out


def silu(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.float32)
    return (x / (np.float32(1.0) + np.exp(-x, dtype=np.float32))).astype(np.float32)


def swiglu_mlp(x: np.ndarray, gate: np.ndarray, up: np.ndarray, down: np.ndarray) -> np.ndarray:
    """down(silu(gate(x)) * up(x)) (reference ``reference_moe.py:25-36``)."""
    x = x.astype(np.float32)
    g = x @ gate.astype(np.float32).T
    u = x @ up.astype(np.float32).T
    return (silu(g) * u) @ down.astype(np.float32).T


def ungroup_and_combine(grouped_out: np.ndarray, grouping: Grouping, num_tokens: int) -> np.ndarray:
    """Weighted sum of each token's k rows (reference ``grouping.py:44-61``).
    Summed in slot order in fp32 (the reference's index_add_ order on CPU)."""
    if grouped_out.shape[0] != grouping.sorted_token_idx.shape[0]:
        raise ValueError(
            f"grouped_output has {grouped_out.shape[0]} rows, "
            f"grouping describes {grouping.sorted_token_idx.shape[0]}"
        )
    h = grouped_out.shape[-1]
    k = grouping.pos.size // max(num_tokens, 1) if num_tokens else 0
    out = np.zeros((num_tokens, h), dtype=np.float32)
    if num_tokens == 0:
        return out
    # weight of flat slot f lives at grouped row pos[f]
    w_flat = grouping.sorted_weight.astype(np.float32)[grouping.pos]
    for s in range(k):
        f = np.arange(num_tokens) * k + s
        out += grouped_out[grouping.pos[f]].astype(np.float32) * w_flat[f][:, None]
    return out


def grouped_moe_routed(
    x: np.ndarray,
    topk_idx: np.ndarray,
    topk_weight: np.ndarray,
    gate: np.ndarray,
    up: np.ndarray,
    down: np.ndarray,
) -> np.ndarray:
    """Routed half of the layer (reference ``moe_forward.py:61-76``):
    group -> gather -> gate/up GEMMs -> silu*up -> down GEMM -> combine."""
    e = gate.shape[0]
    g = group_tokens_by_expert(topk_idx, topk_weight, e)
    offs = group_offsets(g.group_sizes)
    xs = np.asarray(x, dtype=np.float32)[g.sorted_token_idx]
    h = silu(grouped_matmul(xs, gate, offs)) * grouped_matmul(xs, up, offs)
    y = grouped_matmul(h, down, offs)
    return ungroup_and_combine(y, g, x.shape[0])


def moe_forward(
    x: np.ndarray,
    router_w: np.ndarray,
    gate: np.ndarray,
    up: np.ndarray,
    down: np.ndarray,
    top_k: int,
    *,
    shared: tuple[np.ndarray, np.ndarray, np.ndarray] | None = None,
    renormalize: bool = False,
    logits: np.ndarray | None = None,
    topk: tuple[np.ndarray, np.ndarray] | None = None,
) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Full layer: routed + shared (reference ``reference_moe.py:74-78``).

    ``logits`` overrides ``x @ router_w.T`` (so a test can feed the exact logits
    the GPU computed); ``topk`` overrides the router entirely.
    Returns (out fp32 (T,H), topk_idx, topk_weight).
    """
    x32 = np.asarray(x, dtype=np.float32)
    if topk is None:
        if logits is None:
            logits = x32 @ np.asarray(router_w, dtype=np.float32).T
        ids, w = route_softmax_topk(logits, top_k, renormalize=renormalize)
    else:
        ids, w = topk
    out = grouped_moe_routed(x32, ids, w, gate, up, down)
    if shared is not None:
        out = out + swiglu_mlp(x32, *shared)
    return out.astype(np.float32), ids, w


# ---------------------------------------------------------------------------
# int8 weight-only quantisation
# ---------------------------------------------------------------------------

INT8_MAX = 127


def quantize_per_channel_int8(weight: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Symmetric per-(expert, out-channel) int8 (reference
    ``quantization.py:31-50``): scale = absmax/127 in fp32 (1.0 for an all-zero
    channel); q = clamp(round_half_even(w / scale), -127, 127)."""
    w = np.asarray(weight, dtype=np.float32)
    absmax = np.abs(w).max(axis=-1)
    scale = np.where(absmax == 0, np.float32(1.0), (absmax / np.float32(INT8_MAX))).astype(np.float32)
    q = np.clip(np.rint(w / scale[..., None]), -INT8_MAX, INT8_MAX).astype(np.int8)
    return q, scale


def dequantize_int8(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """q * scale in fp32 (reference ``quantization.py:53-54``)."""
    return q.astype(np.float32) * scale.astype(np.float32)[..., None]


# ---------------------------------------------------------------------------
# expert parallelism
# ---------------------------------------------------------------------------


def assign_experts_to_ranks(n_experts: int, n_ranks: int) -> np.ndarray:
    """Contiguous split (reference ``expert_parallel.py:33-41``)."""
    if n_experts <= 0 or n_ranks <= 0:
        raise ValueError(f"n_experts={n_experts} and n_ranks={n_ranks} must both be positive")
    if n_experts < n_ranks:
        raise ValueError(f"n_experts={n_experts} is fewer than n_ranks={n_ranks}")
    return (np.arange(n_experts) * n_ranks) // n_experts


def simulate_ep_moe_routed(
    x: np.ndarray,
    topk_idx: np.ndarray,
    topk_weight: np.ndarray,
    gate: np.ndarray,
    up: np.ndarray,
    down: np.ndarray,
    n_ranks: int,
) -> np.ndarray:
    """Sum over ranks of each rank's local-expert contribution (reference
    ``expert_parallel.py:44-116``): non-local slots get weight 0."""
    e = gate.shape[0]
    rank_of = assign_experts_to_ranks(e, n_ranks)
    total = np.zeros((x.shape[0], down.shape[1]), dtype=np.float32)
    for r in range(n_ranks):
        local = np.nonzero(rank_of == r)[0]
        is_local = np.isin(topk_idx, local)
        remap = np.zeros(e, dtype=np.int64)
        remap[local] = np.arange(local.size)
        lidx = remap[np.clip(topk_idx, 0, None)]
        lw = np.where(is_local, topk_weight, 0).astype(np.float32)
        total = total + grouped_moe_routed(x, lidx, lw, gate[local], up[local], down[local])
    return total


# ---------------------------------------------------------------------------
# synthetic inputs and roofline arithmetic
# ---------------------------------------------------------------------------


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 values rounded to the nearest bf16 (ties to even), returned as
    fp32. NaN/Inf are not expected in test data."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    lsb = (b >> 16) & 1
    b = (b + 0x7FFF + lsb) & 0xFFFF0000
    return b.astype(np.uint32).view(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """uint16 bit patterns of round_to_bf16(x)."""
    return (round_to_bf16(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint32) << 16).view(np.float32)


def zipf_bias(n_experts: int, s: float = 1.2) -> np.ndarray:
    """Per-expert logit bias b_e = -s * ln(e + 1): softmax weights scale by a
    Zipf(s) law over expert rank."""
    return (-s * np.log(np.arange(n_experts, dtype=np.float64) + 1.0)).astype(np.float32)


def layer_bytes(
    counts: np.ndarray, h: int, i: int, i_shared: int, n_experts: int, t: int,
    *, w_bytes: int = 2, scale_bytes: int = 0, x_bytes: int = 2,
) -> int:
    """Algorithmic bytes of one layer call: active routed experts' weights
    (+ scales), the shared expert, the router weight, x in, out."""
    active = int((np.asarray(counts) > 0).sum())
    b = active * 3 * h * i * w_bytes + active * (2 * i + h) * scale_bytes
    b += 3 * h * i_shared * 2 + n_experts * h * 2 + t * h * x_bytes + t * h * 2
    return int(b)


def layer_flops(t: int, k: int, h: int, i: int, i_shared: int, n_experts: int) -> float:
    """2*T*k*3*H*I + 2*T*3*H*I_s + 2*T*H*E."""
    return 2.0 * t * k * 3 * h * i + 2.0 * t * 3 * h * i_shared + 2.0 * t * h * n_experts
