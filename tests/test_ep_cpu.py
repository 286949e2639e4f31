"""The expert-parallel exchange on CPU: two gloo ranks run EPLayer with the
oracle standing in for the kernels (the orchestration under test is the
count exchange, split sizes, (source, expert) grouping and the two row
all-to-alls). The result must equal the single-process oracle forward over all
ranks' tokens. A second test makes one rank fail between its collectives and
checks that the other rank's next collective ends with an error instead of
waiting forever."""

from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dispatch_b200.kernels.expert_parallel import (
    EPLayer,
    Grouped,
    NcclEPBuffer,
    assign_experts_to_ranks,
    exchange_layout,
)
from oracle import moe_oracle as O

H, I, E, K, I_SH, T = 16, 24, 8, 3, 32, 13


def _weights():
    rng = np.random.default_rng(0)
    f = lambda *s: (rng.standard_normal(s) / np.sqrt(s[-1])).astype(np.float32)  # noqa: E731
    return f(E, H), f(E, I, H), f(E, I, H), f(E, H, I), (f(I_SH, H), f(I_SH, H), f(H, I_SH))


def _tokens(rank: int):
    return np.random.default_rng(100 + rank).standard_normal((T + rank, H)).astype(np.float32)


class OracleOps:
    """Compute steps of the layer restated with the CPU oracle."""

    def __init__(self, rank: int, world: int):
        self.router, gate, up, down, self.shared = _weights()
        e_loc = E // world
        sl = slice(rank * e_loc, (rank + 1) * e_loc)
        self.gate, self.up, self.down = gate[sl], up[sl], down[sl]
        self.e_loc = e_loc

    def route_and_group(self, x: torch.Tensor, n_experts: int) -> Grouped:
        xn = x.numpy()
        ids, w = O.route_softmax_topk(xn @ self.router.T, K)
        g = O.group_tokens_by_expert(ids, w, n_experts)
        offs = O.group_offsets(g.group_sizes)
        return Grouped(torch.from_numpy(g.group_sizes.astype(np.int32)), torch.from_numpy(offs.astype(np.int32)),
                       torch.from_numpy(g.pos.astype(np.int32)), torch.from_numpy(xn[g.sorted_token_idx]),
                       torch.from_numpy(w))

    def ffn(self, recv_x, recv_offsets, n_groups, x):
        xr = recv_x.numpy()
        off = recv_offsets.tolist()
        y = np.zeros((xr.shape[0], H), np.float32)
        for g in range(n_groups):
            s, t = off[g], off[g + 1]
            if t > s:
                e = g % self.e_loc
                y[s:t] = O.swiglu_mlp(xr[s:t], self.gate[e], self.up[e], self.down[e])
        ys = O.swiglu_mlp(x.numpy(), *self.shared)
        return torch.from_numpy(y), torch.from_numpy(ys)

    def combine(self, y_back, gr: Grouped, t, k, ys, out_dtype):
        y = y_back.numpy()
        pos = gr.pos.numpy()
        w = gr.topk_weight.numpy().reshape(-1)
        out = np.zeros((t, H), np.float32)
        for s in range(k):
            f = np.arange(t) * k + s
            out += y[pos[f]] * w[f][:, None]
        return torch.from_numpy(out + ys.numpy())


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int, timeout_s: float = 60.0) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


def _ep_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    _init(rank, world, port)
    try:
        from dispatch_b200.kernels.layer import RouterConfig

        layer = EPLayer(None, None, None, RouterConfig(top_k=K), rank=rank, world=world, n_experts=E,
                        ops=OracleOps(rank, world))
        out = layer(torch.from_numpy(_tokens(rank)))
        np.save(os.path.join(out_dir, f"out{rank}.npy"), out.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_ep_exchange_matches_single_process_forward(world: int, tmp_path) -> None:
    mp.spawn(_ep_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    router, gate, up, down, shared = _weights()
    xs = [_tokens(r) for r in range(world)]
    ref, _, _ = O.moe_forward(np.concatenate(xs), router, gate, up, down, K, shared=shared)
    got = np.concatenate([np.load(tmp_path / f"out{r}.npy") for r in range(world)])
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6)


def _failing_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    _init(rank, world, port, timeout_s=5.0)
    counts = torch.tensor([3, 1, 0, 2], dtype=torch.int32)
    try:
        if rank == 1:
            raise RuntimeError("rank 1 fails before its exchange")  # leaves between collectives
        try:
            exchange_layout(counts, world)
            status = "completed"
        except RuntimeError as exc:  # the peer never joins: the collective ends with an error
            status = f"error: {type(exc).__name__}"
        with open(os.path.join(out_dir, "status0.txt"), "w") as f:
            f.write(status)
    except RuntimeError:
        pass


def test_a_rank_that_leaves_makes_the_peer_collective_fail_not_hang(tmp_path) -> None:
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not finish: the failed exchange hung")
    status = (tmp_path / "status0.txt").read_text()
    assert status.startswith("error"), status


class CpuSumBuffer(NcclEPBuffer):
    """The shim with its final partial sum restated on the CPU (the product
    sums with the CUDA combine kernel)."""

    def _sum_partials(self, back, pos, t):
        out = torch.zeros(t, back.shape[1])
        for r in range(self.world):
            rows = pos[:, r]
            m = rows >= 0
            out[m] += back[rows[m].long()]
        return out


def _buffer_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    _init(rank, world, port)
    try:
        router, gate, up, down, _ = _weights()
        x = _tokens(rank)
        ids, w = O.route_softmax_topk(x @ router.T, K)
        buf = CpuSumBuffer()
        idx_t = torch.from_numpy(ids)
        per_rank, _, per_expert, in_rank, _ = buf.get_dispatch_layout(idx_t, E)
        assert per_expert.tolist() == np.bincount(ids.ravel(), minlength=E).tolist()
        recv_x, recv_idx, recv_w, per_local, handle, _ = buf.dispatch(
            torch.from_numpy(x), topk_idx=idx_t, topk_weights=torch.from_numpy(w), num_tokens_per_rank=per_rank,
            is_token_in_rank=in_rank, num_tokens_per_expert=per_expert)
        e_loc = E // world
        sl = slice(rank * e_loc, (rank + 1) * e_loc)
        # local contribution of the received tokens (slots owned elsewhere are -1)
        rx, ri, rw = recv_x.numpy(), recv_idx.numpy(), recv_w.numpy()
        local = np.zeros_like(rx)
        for j in range(rx.shape[0]):
            for s in range(K):
                if ri[j, s] >= 0:
                    e = ri[j, s]
                    local[j] += rw[j, s] * O.swiglu_mlp(rx[j:j + 1], gate[sl][e], up[sl][e], down[sl][e])[0]
        assert sum(per_local) == int((ri >= 0).sum())
        combined, _, _ = buf.combine(torch.from_numpy(local), handle)
        np.save(os.path.join(out_dir, f"buf{rank}.npy"), combined.numpy())
    finally:
        dist.destroy_process_group()


def test_deepep_compatible_buffer_round_trip_matches_routed_forward(tmp_path) -> None:
    world = 2
    mp.spawn(_buffer_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    router, gate, up, down, _ = _weights()
    for r in range(world):
        x = _tokens(r)
        ids, w = O.route_softmax_topk(x @ router.T, K)
        ref = O.grouped_moe_routed(x, ids, w, gate, up, down)
        np.testing.assert_allclose(np.load(tmp_path / f"buf{r}.npy"), ref, rtol=1e-5, atol=1e-6)


def test_exchange_layout_single_rank_is_identity() -> None:
    port = _free_port()
    _init(0, 1, port)
    try:
        counts = torch.tensor([2, 0, 5, 1], dtype=torch.int32)
        layout, recv = exchange_layout(counts, 1)
        assert layout.send_splits == [8] and layout.recv_splits == [8]
        assert layout.recv_offsets == [0, 2, 2, 7, 8]
        assert torch.equal(recv, counts)
    finally:
        dist.destroy_process_group()


def test_assign_experts_to_ranks_mirror() -> None:
    r = assign_experts_to_ranks(64, 2)
    assert r[:32].eq(0).all() and r[32:].eq(1).all()
    with pytest.raises(ValueError, match="fewer than"):
        assign_experts_to_ranks(1, 2)
    with pytest.raises(ValueError, match="positive"):
        assign_experts_to_ranks(0, 2)


def test_peer_buffers_refuse_bad_shapes_before_touching_a_device() -> None:
    from dispatch_b200.kernels.ep_peer import PeerBuffers

    common = dict(rank=0, device=torch.device("cuda", 0), max_tokens=8, top_k=2, hidden=64)
    with pytest.raises(ValueError, match="world"):
        PeerBuffers(world=17, n_experts=34, **common)
    with pytest.raises(ValueError, match="split evenly"):
        PeerBuffers(world=3, n_experts=8, **common)
    with pytest.raises(ValueError, match="16-bit"):
        PeerBuffers(world=2, n_experts=8, act_dtype=torch.float32, **common)


def test_signal_buffer_size_is_host_arithmetic() -> None:
    from dispatch_b200 import _lib as L

    lib = L.lib()
    assert lib.moe_ep_signal_bytes(8, 64) == L.EP_SIGNAL_HEADER_BYTES + 8 * 64 * 4
    assert lib.moe_ep_signal_bytes(1, 0) == L.EP_SIGNAL_HEADER_BYTES
    assert lib.moe_ep_signal_bytes(0, 64) == 0
    # 4 slots x 16 rank flags of int32 fit the header
    assert L.EP_FLAG_SLOTS * L.EP_MAX_RANKS * 4 <= L.EP_SIGNAL_HEADER_BYTES


def test_exchange_without_a_device_reports_it() -> None:
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from dispatch_b200 import _lib as L

    rc = L.lib().moe_ep_exchange(None, 0, None, None, 0, 0, 0, 1, 1, None, None)
    assert rc == L.MOE_ERR_NO_DEVICE


def test_host_batches_check_lengths_before_any_copy() -> None:
    from dispatch_b200.kernels.layer import run_host_batches

    run_host_batches(lambda x: x, [], [])  # nothing to do
    with pytest.raises(ValueError, match="outputs"):
        run_host_batches(lambda x: x, [torch.zeros(2, 8)], [])
