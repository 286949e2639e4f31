"""The no-allocation grouping entry point, checked through the C ABI.

moe_group_tokens_noalloc serves callers that cannot allocate device memory
(for example a runtime binding the library over FFI that can only pass buffers
it already owns). It must give exactly what moe_group_tokens gives with a
caller workspace: the sort is integer work, so the comparison is bit-exact,
and it is repeated on two different calls in a row to show that what the
shared scratch array keeps from the previous call does not leak into the next.
The file name keeps pytest from collecting it before the other GPU tests.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - collected on CPU hosts too
    pytest.skip("needs a CUDA device", allow_module_level=True)

from dispatch_b200 import _lib as L  # noqa: E402

DEV = torch.device("cuda", 0)
SCRATCH_INTS = 256 * 1024  # MOE_GROUP_NOALLOC_SCRATCH_INTS


def _inputs(t: int, e: int, k: int, h: int, seed: int, idx_dtype=torch.int32, x_dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    probs = (torch.arange(1, e + 1, dtype=torch.float32) ** -1.2).expand(t, e)
    idx = torch.multinomial(probs, k, replacement=False, generator=g).to(idx_dtype).to(DEV)
    w = torch.rand(t, k, generator=g).to(DEV)
    x = torch.randn(t, h, generator=g).to(x_dtype).to(DEV)
    return idx, w, x


def _outputs(t: int, e: int, k: int, h: int, full: bool = True):
    """Output buffers pre-filled with a marker; ``full=False`` leaves out the
    optional outputs (sorted ids and weights, gathered rows)."""
    n = t * k
    out = {
        "counts": torch.full((e,), -7, dtype=torch.int32, device=DEV),
        "offsets": torch.full((e + 1,), -7, dtype=torch.int32, device=DEV),
        "pos": torch.full((n,), -7, dtype=torch.int32, device=DEV),
    }
    if full:
        out["sti"] = torch.full((n,), -7, dtype=torch.int64, device=DEV)
        out["sw"] = torch.full((n,), -7.0, dtype=torch.float32, device=DEV)
        out["xs"] = torch.zeros(n, h, dtype=torch.bfloat16, device=DEV)
    return out


def _call(noalloc: bool, idx, w, x, e: int, out) -> None:
    lib = L.lib()
    t, k = idx.shape
    h = x.shape[1]
    status = L.status_word(DEV)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    gather = "xs" in out
    common = (idx.data_ptr(), L.dt(idx), w.data_ptr(), t, k, e, out["counts"].data_ptr(), out["offsets"].data_ptr(),
              out["pos"].data_ptr(), L.ptr(out.get("sti")), L.ptr(out.get("sw")), x.data_ptr() if gather else None,
              L.dt(x) if gather else 0, h if gather else 0, L.ptr(out.get("xs")), L.DT_BF16 if gather else 0)
    if noalloc:
        rc = lib.moe_group_tokens_noalloc(*common, status.data_ptr(), stream)
    else:
        nbytes = lib.moe_group_workspace_bytes(t, k, e)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
        rc = lib.moe_group_tokens(*common, ws.data_ptr(), nbytes, status.data_ptr(), stream)
    L.check(rc, "group tokens")


@pytest.mark.parametrize("first,second", [((4096, 64, 6, 256), (300, 8, 2, 64)), ((37, 256, 8, 64), (8192, 256, 8, 64))])
def test_noalloc_grouping_matches_workspace_path_on_two_calls(first, second) -> None:
    cases = []
    for seed, (t, e, k, h) in enumerate((first, second)):
        idx, w, x = _inputs(t, e, k, h, seed)
        ref = _outputs(t, e, k, h)
        _call(False, idx, w, x, e, ref)
        cases.append((idx, w, x, e, ref, _outputs(t, e, k, h)))
    # the two no-allocation calls back to back, sharing the scratch array
    for idx, w, x, e, _, got in cases:
        _call(True, idx, w, x, e, got)
    torch.cuda.synchronize()
    L.check_device_status(DEV)
    for n_call, (idx, _, _, e, ref, got) in enumerate(cases):
        for name in ref:
            assert torch.equal(ref[name], got[name]), f"{name} differs on call {n_call} (T={idx.shape[0]}, E={e})"


@pytest.mark.parametrize("variant", ["int64 ids, f32 rows", "no optional outputs"])
def test_noalloc_grouping_variants_match_workspace_path(variant: str) -> None:
    """The other argument forms the entry point accepts: int64 expert ids with
    f32 activations converted to bf16 on the way, and the bare sort (no sorted
    ids, weights or gathered rows); again two calls in a row."""
    full = variant != "no optional outputs"
    kw = dict(idx_dtype=torch.int64, x_dtype=torch.float32) if full else {}
    shapes = ((1000, 64, 6, 128), (5, 16, 4, 64))
    cases = []
    for seed, (t, e, k, h) in enumerate(shapes):
        idx, w, x = _inputs(t, e, k, h, 10 + seed, **kw)
        ref = _outputs(t, e, k, h, full)
        _call(False, idx, w, x, e, ref)
        cases.append((idx, w, x, e, ref, _outputs(t, e, k, h, full)))
    for idx, w, x, e, _, got in cases:
        _call(True, idx, w, x, e, got)
    torch.cuda.synchronize()
    L.check_device_status(DEV)
    for n_call, (idx, _, _, e, ref, got) in enumerate(cases):
        for name in ref:
            assert torch.equal(ref[name], got[name]), f"{name} differs on call {n_call} ({variant})"


def test_noalloc_grouping_rejects_inputs_beyond_its_scratch() -> None:
    e, k = 256, 8
    t = (SCRATCH_INTS // e + 1) * 256 // k  # one 256-pair chunk more than the array holds
    lib = L.lib()
    idx = torch.zeros(t, k, dtype=torch.int32, device=DEV)
    out = {n: torch.empty(1, device=DEV) for n in ("c", "o", "p")}
    rc = lib.moe_group_tokens_noalloc(idx.data_ptr(), L.DT_I32, None, t, k, e, out["c"].data_ptr(),
                                      out["o"].data_ptr(), out["p"].data_ptr(), None, None, None, 0, 0, None, 0,
                                      None, torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == L.MOE_ERR_INVALID_ARG
    assert b"exceeds the built-in scratch" in lib.moe_last_error()
