"""The flag exchange the expert-parallel layer uses between its kernels
(moe_ep_exchange), on one GPU: the payload lands in the count area and the
barrier completes once every flag is set; a flag that nothing sets makes the
bounded wait give up with MOE_ERR_TIMEOUT in the status word instead of
hanging, and the context stays usable."""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from dispatch_b200 import _lib as L  # noqa: E402

DEV = torch.device("cuda", 0)


class _Raw:
    """A zero-copy int32 view of raw device memory for torch.as_tensor."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<i4", "data": (ptr, False), "version": 3}


def _signal(world: int, n: int) -> int:
    p = ctypes.c_void_p()
    L.check(L.lib().moe_peer_alloc(L.lib().moe_ep_signal_bytes(world, n), ctypes.byref(p)), "moe_peer_alloc")
    return p.value


def _exchange(payload, n, table, sig, slot, rank, world, epoch, sig_bytes=None) -> None:
    sig_bytes = L.lib().moe_ep_signal_bytes(world, n) if sig_bytes is None else sig_bytes
    rc = L.lib().moe_ep_exchange(None if payload is None else payload.data_ptr(), n, table.data_ptr(), sig,
                                 sig_bytes, slot, rank, world, epoch, L.status_word(DEV).data_ptr(),
                                 L.stream_ptr(DEV))
    L.check(rc, "moe_ep_exchange")


def test_exchange_on_one_rank_copies_the_payload_and_completes() -> None:
    n = 64
    sig = _signal(1, n)
    try:
        table = torch.tensor([sig], dtype=torch.int64, device=DEV)
        area = torch.as_tensor(_Raw(sig + L.EP_SIGNAL_HEADER_BYTES, n), device=DEV)
        flags = torch.as_tensor(_Raw(sig, L.EP_FLAG_SLOTS * L.EP_MAX_RANKS), device=DEV)
        for epoch in (1, 2, 3):
            payload = torch.arange(n, dtype=torch.int32, device=DEV) * epoch
            _exchange(payload, n, table, sig, epoch % L.EP_FLAG_SLOTS, 0, 1, epoch)
            torch.cuda.synchronize()
            assert torch.equal(area, payload)
            assert int(flags[(epoch % L.EP_FLAG_SLOTS) * L.EP_MAX_RANKS]) == epoch
        L.check_device_status(DEV)
    finally:
        torch.cuda.synchronize()
        L.check(L.lib().moe_peer_free(sig), "moe_peer_free")


def test_exchange_wait_gives_up_with_timeout_status() -> None:
    """World 2 with both table entries on this rank's own buffer: flag [slot][1]
    is never stored, so the wait runs out (2 s) and reports MOE_ERR_TIMEOUT."""
    sig = _signal(2, 0)
    try:
        table = torch.tensor([sig, sig], dtype=torch.int64, device=DEV)
        _exchange(None, 0, table, sig, 1, 0, 2, 1)
        torch.cuda.synchronize()
        st = L.status_word(DEV)
        assert int(st.item()) == L.MOE_ERR_TIMEOUT
        st.zero_()
        # the context still works: a complete single-rank exchange afterwards
        one = torch.tensor([sig], dtype=torch.int64, device=DEV)
        _exchange(None, 0, one, sig, 2, 0, 1, 1)
        torch.cuda.synchronize()
        L.check_device_status(DEV)
    finally:
        torch.cuda.synchronize()
        L.check(L.lib().moe_peer_free(sig), "moe_peer_free")


def test_exchange_refuses_a_payload_larger_than_the_signal_buffers() -> None:
    """A caller that passes more payload than the signal buffers hold gets an
    argument error before anything is stored (the stores go to peer memory)."""
    sig = _signal(1, 8)
    try:
        table = torch.tensor([sig], dtype=torch.int64, device=DEV)
        payload = torch.zeros(16, dtype=torch.int32, device=DEV)
        with pytest.raises(ValueError, match="cannot hold"):
            _exchange(payload, 16, table, sig, 0, 0, 1, 1, sig_bytes=L.lib().moe_ep_signal_bytes(1, 8))
        torch.cuda.synchronize()
        L.check_device_status(DEV)
    finally:
        torch.cuda.synchronize()
        L.check(L.lib().moe_peer_free(sig), "moe_peer_free")
