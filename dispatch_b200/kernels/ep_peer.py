"""Expert parallelism over NVLink peer memory: the DeepEP round trip of the
reference's make_ep_moe_infer (src/dispatch/kernels/expert_parallel.py:119-190)
with every row moved by this library's own kernels (C ABI in
include/moe_ep_b200.h).

One ``PeerEPLayer`` call on a rank's T local tokens:

1. route and group locally (stable counting sort; no row copy);
2. all-gather of the (E,) per-expert counts -> the (world, E) matrix, which
   fixes every rank's receive layout on every rank (``moe_ep_exchange``: one
   CTA stores the counts into every peer's signal buffer and exchanges flags);
3. ``moe_ep_dispatch``: each (token, slot) row is stored by this GPU straight
   into the receive buffer of the expert's owner, with its return code;
4. barrier (``moe_ep_exchange`` with no payload, stream-ordered);
5. ``moe_ep_expert_ffn``: the grouped SwiGLU FFN over the received rows (and
   the shared expert over the local tokens, in the same two launches); the
   down projection's epilogue stores each output row straight into the
   source rank's return buffer;
6. barrier;
7. the weighted combine of the k returned rows per token, in slot order.

No host synchronisation and no staging copies. Every per-row product comes
from the same kernels with the same per-row arithmetic as the 1-GPU layer and
the final sum order is the same, so the output is byte-identical to the
1-GPU result. Buffers are sized for the worst case (every slot of every
rank's ``max_tokens`` tokens landing on one rank), the way DeepEP's
low-latency buffers are sized by ``num_max_dispatch_tokens_per_rank``.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from dispatch_b200 import _lib as L


class PeerBuffers:
    """One rank's receive rows, return codes and return rows, mapped into
    every rank of the group through CUDA IPC (no multicast)."""

    def __init__(self, *, rank: int, world: int, group=None, device: torch.device, max_tokens: int, top_k: int,
                 hidden: int, n_experts: int, act_dtype: torch.dtype = torch.bfloat16):
        if not 1 <= world <= L.EP_MAX_RANKS:
            raise ValueError(f"world={world} must be in [1, {L.EP_MAX_RANKS}]")
        if n_experts % world:
            raise ValueError(f"{n_experts} experts do not split evenly over {world} ranks")
        if act_dtype not in (torch.bfloat16, torch.float16):
            raise ValueError("peer exchange moves 16-bit activation rows")
        self.rank, self.world, self.group = rank, world, group
        self.device = torch.device(device)
        self.max_tokens, self.top_k, self.hidden, self.n_experts = max_tokens, top_k, hidden, n_experts
        self.e_loc = n_experts // world
        self.act_dtype = act_dtype
        self.recv_cap = world * max_tokens * min(top_k, self.e_loc)
        self.back_rows = max_tokens * top_k
        lib = L.lib()
        self._lib = lib
        self._own: list[int] = []
        self._mapped: list[int] = []
        dev = self.device
        with torch.cuda.device(dev):
            mine = torch.tensor([dev.index], dtype=torch.int32, device=dev)
            devs = torch.empty(world, dtype=torch.int32, device=dev)
            dist.all_gather_into_tensor(devs, mine, group=group)
            bad = [int(d) for d in devs.tolist() if not lib.moe_peer_can_access(int(d))]
            if bad:
                raise RuntimeError(f"rank {rank} (cuda:{dev.index}) cannot map the memory of devices {bad}")
            sizes = (self.recv_cap * hidden * 2, self.recv_cap * 4, self.back_rows * hidden * 2,
                     lib.moe_ep_signal_bytes(world, n_experts))
            nb = len(sizes)
            self.signal_bytes = sizes[3]
            handles = (ctypes.c_uint8 * (nb * L.PEER_HANDLE_BYTES))()
            for i, n in enumerate(sizes):
                p = ctypes.c_void_p()
                L.check(lib.moe_peer_alloc(n, ctypes.byref(p)), "moe_peer_alloc")
                self._own.append(p.value)
                L.check(lib.moe_peer_export(p, ctypes.addressof(handles) + i * L.PEER_HANDLE_BYTES),
                        "moe_peer_export")
            local = torch.frombuffer(bytearray(handles), dtype=torch.uint8).to(dev)
            allh = torch.empty(world * local.numel(), dtype=torch.uint8, device=dev)
            dist.all_gather_into_tensor(allh, local, group=group)
            allh = allh.view(world, nb, L.PEER_HANDLE_BYTES).cpu()
            table = [[0] * world for _ in range(nb)]
            for s in range(world):
                for i in range(nb):
                    if s == rank:
                        table[i][s] = self._own[i]
                        continue
                    raw = bytes(allh[s, i].tolist())
                    p = ctypes.c_void_p()
                    L.check(lib.moe_peer_import(raw, ctypes.byref(p)), "moe_peer_import")
                    self._mapped.append(p.value)
                    table[i][s] = p.value
            self.recv_ptr, self.ret_ptr, self.back_ptr, self.signal_ptr = self._own
            self.t_recv = torch.tensor(table[0], dtype=torch.int64, device=dev)
            self.t_ret = torch.tensor(table[1], dtype=torch.int64, device=dev)
            self.t_back = torch.tensor(table[2], dtype=torch.int64, device=dev)
            self.t_signal = torch.tensor(table[3], dtype=torch.int64, device=dev)
            # the (world, E) count matrix lives in the signal buffer's payload area
            self.counts_all_ptr = self.signal_ptr + L.EP_SIGNAL_HEADER_BYTES
            self.epoch = 0
            self.recv_offsets = torch.zeros(self.e_loc + 1, dtype=torch.int32, device=dev)
            self._flag = torch.zeros(1, dtype=torch.int32, device=dev)
            self.barrier()
            torch.cuda.synchronize(dev)

    def barrier(self) -> None:
        """Stream-ordered barrier over the group (NCCL): kernels enqueued after
        it on any rank run after every rank's kernels enqueued before it."""
        dist.all_reduce(self._flag, group=self.group)

    def exchange(self, payload: torch.Tensor | None, slot: int, epoch: int) -> None:
        """``moe_ep_exchange``: ``payload`` (int32, or None) into row ``rank`` of
        every rank's count area, then a flag barrier on ``slot`` for ``epoch``."""
        dev = self.device
        n = 0 if payload is None else payload.numel()
        epoch = ((epoch + 2**31) % 2**32) - 2**31  # the kernel compares int32 epochs wrap-safely
        rc = self._lib.moe_ep_exchange(
            None if payload is None else payload.data_ptr(), n, self.t_signal.data_ptr(), self.signal_ptr,
            self.signal_bytes, slot, self.rank, self.world, epoch, L.status_word(dev).data_ptr(), L.stream_ptr(dev))
        L.check(rc, "moe_ep_exchange")

    def close(self) -> None:
        """Collective: unmaps the peers' buffers and frees this rank's."""
        if not self._own:
            return
        with torch.cuda.device(self.device):
            self.barrier()
            torch.cuda.synchronize(self.device)
            for p in self._mapped:
                L.check(self._lib.moe_peer_release(p), "moe_peer_release")
            self._mapped = []
            self.barrier()
            torch.cuda.synchronize(self.device)
            for p in self._own:
                L.check(self._lib.moe_peer_free(p), "moe_peer_free")
            self._own = []

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class PeerEPLayer:
    """Expert-parallel MoE layer for one rank over ``PeerBuffers`` (see the
    module docstring). Arguments as ``EPLayer``; ``max_tokens`` bounds the
    tokens per rank of any call."""

    def __init__(self, router_weight, weights, shared, router_cfg, *, rank: int, world: int, group=None,
                 e_score_bias=None, n_experts: int | None = None, weights_are_local: bool = False,
                 max_tokens: int = 4096, act_dtype: torch.dtype = torch.bfloat16,
                 buffers: PeerBuffers | None = None, overlap_shared: bool = False,
                 overlap_min_tokens: int = 1024):
        from dispatch_b200.kernels.expert_parallel import _slice_experts  # noqa: PLC0415
        from dispatch_b200.kernels.quantization import QuantizedStackedExpertWeights  # noqa: PLC0415

        self.rank, self.world, self.group = rank, world, group
        e = n_experts if n_experts is not None else weights.num_experts * (world if weights_are_local else 1)
        if e % world:
            raise ValueError(f"{e} experts do not split evenly over {world} ranks")
        self.n_experts, self.e_loc = e, e // world
        if not weights_are_local:
            weights = _slice_experts(weights, rank * self.e_loc, (rank + 1) * self.e_loc)
        self.weights, self.shared, self.cfg = weights, shared, router_cfg
        self.router_weight, self.bias = router_weight, e_score_bias
        self.top_k = router_cfg.top_k
        self.quant = isinstance(weights, QuantizedStackedExpertWeights)
        g = weights.gate.data if self.quant else weights.gate
        self.hidden, self.inter = g.shape[2], g.shape[1]
        self.act_dtype = act_dtype
        self._own_buffers = buffers is None
        self.buf = buffers or PeerBuffers(rank=rank, world=world, group=group, device=g.device,
                                          max_tokens=max_tokens, top_k=self.top_k, hidden=self.hidden,
                                          n_experts=e, act_dtype=self.act_dtype)
        # The shared expert needs only the local tokens: with overlap_shared it
        # runs on a side stream while the rows are dispatched (its GEMM CTAs
        # leave room on each SM for the small dispatch and exchange kernels).
        # Measured at 2 GPUs: 0.720 -> 0.711 ms at 4096 tokens, but 0.204 ->
        # 0.239 ms at 128 (two more launches and a stream join), so only calls
        # of at least overlap_min_tokens tokens split it off. Off by default:
        # at 8 GPUs the step was slower with it (0.92 ms), the shared GEMM's
        # persistent CTAs leaving one dispatch CTA per SM for 7x more rows.
        self.overlap_shared = overlap_shared and shared is not None
        self.overlap_min_tokens = overlap_min_tokens
        self._side: torch.cuda.Stream | None = None
        # launches of this library per call: route x2, group x2, exchange x3, dispatch, FFN x2 (+2 shared), combine
        self.launches_per_step = 13 if self.overlap_shared else 11
        # Set to a list to have each call append (phase name, CUDA event)
        # marks, recorded on the current stream after each phase.
        self.phase_events: list | None = None

    PHASES = ("route_group", "count_exchange", "dispatch", "barrier_after_dispatch", "ffn_and_return",
              "barrier_after_ffn", "combine")

    def _mark(self, name: str) -> None:
        if self.phase_events is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.phase_events.append((name, ev))

    def launches_for(self, t: int) -> int:
        """Launches of this library in one call on t tokens."""
        return 13 if (self.overlap_shared and t >= self.overlap_min_tokens) else 11

    def close(self) -> None:
        """Collective: frees the peer buffers (every rank calls it)."""
        if self._own_buffers:
            self.buf.close()

    def _shared_ffn(self, x: torch.Tensor, ys: torch.Tensor, dev: torch.device) -> None:
        """The shared expert alone (two dense GEMM launches) on the current stream."""
        lib = L.lib()
        t, h = x.shape
        sh = self.shared
        i_sh = sh.gate.shape[0]
        wq = self.weights
        g, u, d = (wq.gate.data, wq.up.data, wq.down.data) if self.quant else (wq.gate, wq.up, wq.down)
        nbytes = lib.moe_ffn_workspace_bytes(0, self.inter, t, i_sh)
        ws = L.workspace(dev, nbytes, "ep_shared_ffn")
        rc = lib.moe_expert_ffn_grouped(
            3, None, L.dt(x), 0, h, None, 1, 1, None, 0, self.inter, g.data_ptr(), u.data_ptr(), d.data_ptr(),
            L.DT_I8 if self.quant else L.dt(g), None, None, None, 0, x.data_ptr(), t, i_sh, sh.gate.data_ptr(),
            sh.up.data_ptr(), sh.down.data_ptr(), None, ys.data_ptr(), ws.data_ptr(), ws.numel(),
            L.status_word(dev).data_ptr(), L.stream_ptr(dev),
        )
        L.check(rc, "moe_expert_ffn_grouped (shared expert)")

    @torch.no_grad()
    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        dev = L.require_cuda(x, what="expert-parallel layer")
        t, h = x.shape
        if t > self.buf.max_tokens:
            raise ValueError(f"{t} tokens exceed the {self.buf.max_tokens} tokens per rank the peer buffers hold")
        if h != self.hidden or x.dtype != self.buf.act_dtype:
            raise ValueError(f"x must be ({t}, {self.hidden}) {self.buf.act_dtype}, got {tuple(x.shape)} {x.dtype}")
        x = x.contiguous()
        out = torch.empty(t, h, dtype=x.dtype, device=dev)
        self._forward(x, out, dev)
        return out

    def _route_group(self, x: torch.Tensor) -> tuple:
        """Router and grouping of this rank's rows x on the current stream:
        (ids, weights, counts, offsets, slot positions, f32 weights)."""
        from dispatch_b200.kernels.grouping import _group  # noqa: PLC0415
        from dispatch_b200.kernels.layer import route  # noqa: PLC0415

        idx, w = route(x, self.router_weight, self.cfg, e_score_bias=self.bias)
        counts, offsets, pos, _, _, wf, _ = _group(idx, w, self.n_experts, want_sorted=False)
        return idx, w, counts, offsets, pos, wf

    def _forward(self, x: torch.Tensor, out: torch.Tensor, dev: torch.device) -> None:
        """One pass of the EP round trip for x (rows of this rank) on the
        current stream; the combined rows go to `out`."""
        t, h = x.shape
        buf = self.buf
        mark_fn = self._mark
        lib = L.lib()
        st = L.status_word(dev).data_ptr()
        stream = L.stream_ptr(dev)
        k = self.top_k
        mark_fn("start")
        idx, w, counts, offsets, pos, wf = self._route_group(x)
        mark_fn("route_group")
        sh = self.shared
        i_sh = 0 if sh is None else sh.gate.shape[0]
        ys = torch.empty(t, h, dtype=x.dtype, device=dev) if sh is not None else None
        shared_done = None
        overlap = self.overlap_shared and t >= self.overlap_min_tokens
        if overlap:
            main = torch.cuda.current_stream(dev)
            if self._side is None:
                self._side = torch.cuda.Stream(dev)
            self._side.wait_stream(main)
            with torch.cuda.stream(self._side):
                self._shared_ffn(x, ys, dev)
                shared_done = torch.cuda.Event()
                shared_done.record(self._side)
            x.record_stream(self._side)
            ys.record_stream(self._side)
        buf.epoch += 1
        epoch = buf.epoch
        buf.exchange(counts, 0, epoch)
        mark_fn("count_exchange")
        rc = lib.moe_ep_dispatch(
            x.data_ptr(), L.dt(x), t, h, idx.data_ptr(), L.dt(idx), k, pos.data_ptr(), offsets.data_ptr(),
            buf.counts_all_ptr, self.rank, self.world, self.n_experts, buf.t_recv.data_ptr(),
            buf.t_ret.data_ptr(), buf.recv_cap, buf.recv_offsets.data_ptr(), st, stream,
        )
        L.check(rc, "moe_ep_dispatch")
        mark_fn("dispatch")
        buf.exchange(None, 1, epoch)
        mark_fn("barrier_after_dispatch")
        fused_shared = sh is not None and not overlap
        wq = self.weights
        g, u, d = (wq.gate.data, wq.up.data, wq.down.data) if self.quant else (wq.gate, wq.up, wq.down)
        sc = (wq.gate.scale, wq.up.scale, wq.down.scale) if self.quant else (None,) * 3
        nbytes = lib.moe_ffn_workspace_bytes(buf.recv_cap, self.inter, t if fused_shared else 0, i_sh)
        ws = L.workspace(dev, nbytes, "ep_peer_ffn")
        rc = lib.moe_ep_expert_ffn(
            buf.recv_ptr, L.dt(x), buf.recv_cap, h, buf.recv_offsets.data_ptr(), self.e_loc, buf.ret_ptr,
            buf.t_back.data_ptr(), self.world, buf.back_rows, self.inter,
            g.data_ptr(), u.data_ptr(), d.data_ptr(), L.DT_I8 if self.quant else L.dt(g),
            L.ptr(sc[0]), L.ptr(sc[1]), L.ptr(sc[2]), L.dt(sc[0]) if self.quant else 0,
            x.data_ptr() if fused_shared else None, t if fused_shared else 0, i_sh,
            L.ptr(sh.gate if fused_shared else None), L.ptr(sh.up if fused_shared else None),
            L.ptr(sh.down if fused_shared else None), L.ptr(ys if fused_shared else None), ws.data_ptr(),
            ws.numel(), st, stream,
        )
        L.check(rc, "moe_ep_expert_ffn")
        mark_fn("ffn_and_return")
        buf.exchange(None, 2, epoch)
        mark_fn("barrier_after_ffn")
        if shared_done is not None:
            torch.cuda.current_stream(dev).wait_event(shared_done)
        rc = lib.moe_combine(buf.back_ptr, L.dt(x), pos.data_ptr(), wf.data_ptr(), t, k, h, L.ptr(ys),
                             out.data_ptr(), L.dt(out), st, stream)
        L.check(rc, "moe_combine")
        mark_fn("combine")
