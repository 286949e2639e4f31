"""ctypes binding of ``libmoe_b200.so`` (the C ABIs in ``include/moe_b200.h``
and ``include/moe_ep_b200.h``).

The library is built in-tree by ``dispatch_b200.build`` (nvcc, sm_100a). There
is no fallback: if the library is missing or no sm_100 device is current, every
op raises. Torch is used only for device memory, streams and dtypes; pointers
cross the ABI as plain integers.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().with_name("libmoe_b200.so")

MOE_OK = 0
MOE_ERR_INVALID_ARG = 1
MOE_ERR_UNSUPPORTED = 2
MOE_ERR_CUDA = 3
MOE_ERR_NO_DEVICE = 4
MOE_ERR_TIMEOUT = 5
MOE_ERR_BAD_EXPERT = 6
MOE_ERR_BAD_OFFSETS = 7

DT_BF16, DT_F16, DT_F32, DT_I8, DT_I32, DT_I64 = range(6)
FFN_KERNEL_AUTO, FFN_KERNEL_TILED, FFN_KERNEL_STREAM, FFN_KERNEL_PAIR, FFN_KERNEL_WARP = range(5)
ROUTER_SOFTMAX, ROUTER_SIGMOID_GROUP = 0, 1

_TORCH_DT = {
    torch.bfloat16: DT_BF16,
    torch.float16: DT_F16,
    torch.float32: DT_F32,
    torch.int8: DT_I8,
    torch.int32: DT_I32,
    torch.int64: DT_I64,
}

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_sz = ctypes.c_size_t


class MoeLayerDesc(ctypes.Structure):
    _fields_ = [
        ("T", _i64), ("H", _i64), ("E", _i64), ("I", _i64), ("I_shared", _i64),
        ("k", _i32), ("act_dtype", _i32), ("x_dtype", _i32), ("out_dtype", _i32), ("w_dtype", _i32),
        ("scale_dtype", _i32), ("router_mode", _i32), ("renorm", _i32), ("n_group", _i32),
        ("topk_group", _i32), ("routed_scaling", _f32), ("router_w_dtype", _i32),
    ]


_SIGNATURES = {
    "moe_abi_version": ([], _i32),
    "moe_set_ffn_kernel": ([_i32], _i32),
    "moe_ffn_kernel_auto": ([_i64, _i64, _i64, _i64, _i64, _i32], _i32),
    "moe_status_string": ([_i32], ctypes.c_char_p),
    "moe_last_error": ([], ctypes.c_char_p),
    "moe_device_sm_count": ([], _i32),
    "moe_route_workspace_bytes": ([_i64, _i64], _sz),
    "moe_route": (
        [_p, _i32, _p, _i32, _p, _i64, _i64, _i64, _i32, _i32, _i32, _p, _i32, _i32, _f32, _p, _p, _p, _p, _sz, _p,
         _p],
        _i32,
    ),
    "moe_group_workspace_bytes": ([_i64, _i32, _i64], _sz),
    "moe_group_tokens": (
        [_p, _i32, _p, _i64, _i32, _i64, _p, _p, _p, _p, _p, _p, _i32, _i64, _p, _i32, _p, _sz, _p, _p],
        _i32,
    ),
    "moe_group_tokens_noalloc": (
        [_p, _i32, _p, _i64, _i32, _i64, _p, _p, _p, _p, _p, _p, _i32, _i64, _p, _i32, _p, _p],
        _i32,
    ),
    "moe_grouped_gemm": ([_p, _i32, _i64, _i64, _p, _i32, _p, _i32, _i64, _i64, _p, _p, _i64, _p, _p], _i32),
    "moe_ffn_workspace_bytes": ([_i64, _i64, _i64, _i64], _sz),
    "moe_expert_ffn": (
        [_p, _i32, _i64, _i64, _p, _i64, _i64, _p, _p, _p, _i32, _p, _p, _p, _i32, _p, _i64, _i64, _p, _p, _p,
         _p, _p, _p, _sz, _p, _p],
        _i32,
    ),
    "moe_expert_ffn_part": (
        [_i32, _p, _i32, _i64, _i64, _p, _i64, _i64, _p, _p, _p, _i32, _p, _p, _p, _i32, _p, _i64, _i64, _p, _p,
         _p, _p, _p, _p, _sz, _p, _p],
        _i32,
    ),
    "moe_expert_ffn_grouped": (
        [_i32, _p, _i32, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p, _p, _p, _i32, _p, _p, _p, _i32, _p, _i64,
         _i64, _p, _p, _p, _p, _p, _p, _sz, _p, _p],
        _i32,
    ),
    "moe_combine": ([_p, _i32, _p, _p, _i64, _i32, _i64, _p, _p, _i32, _p, _p], _i32),
    "moe_quantize_int8": ([_p, _i32, _i64, _i64, _p, _p, _i32, _p], _i32),
    "moe_layer_workspace_bytes": ([ctypes.POINTER(MoeLayerDesc)], _sz),
    "moe_layer_forward": (
        [ctypes.POINTER(MoeLayerDesc), _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
         _p, _p, _sz, _p, _p],
        _i32,
    ),
    # include/moe_ep_b200.h
    "moe_peer_alloc": ([_sz, ctypes.POINTER(_p)], _i32),
    "moe_peer_free": ([_p], _i32),
    "moe_peer_export": ([_p, _p], _i32),
    "moe_peer_import": ([_p, ctypes.POINTER(_p)], _i32),
    "moe_peer_release": ([_p], _i32),
    "moe_peer_can_access": ([_i32], _i32),
    "moe_ep_dispatch": (
        [_p, _i32, _i64, _i64, _p, _i32, _i32, _p, _p, _p, _i32, _i32, _i64, _p, _p, _i64, _p, _p, _p],
        _i32,
    ),
    "moe_ep_expert_ffn": (
        [_p, _i32, _i64, _i64, _p, _i64, _p, _p, _i32, _i64, _i64, _p, _p, _p, _i32, _p, _p, _p, _i32, _p, _i64,
         _i64, _p, _p, _p, _p, _p, _sz, _p, _p],
        _i32,
    ),
    "moe_ep_signal_bytes": ([_i32, _i64], _sz),
    "moe_ep_exchange": ([_p, _i64, _p, _p, _sz, _i32, _i32, _i32, _i32, _p, _p], _i32),
}

PEER_HANDLE_BYTES = 64
EP_SIGNAL_HEADER_BYTES = 256
EP_FLAG_SLOTS = 4
EP_MAX_RANKS = 16

_lib: ctypes.CDLL | None = None
_lock = threading.Lock()


class MoeDeviceError(RuntimeError):
    """An error a kernel reported through the device status word."""


def lib() -> ctypes.CDLL:
    """The loaded library; raises ImportError if it has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise ImportError(
                        f"{LIB_PATH.name} is not built; run `python -c 'import __graft_entry__ as g; g.build()'` "
                        "(needs nvcc with sm_100a support)"
                    )
                handle = ctypes.CDLL(str(LIB_PATH))
                for name, (args, ret) in _SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.argtypes = args
                    fn.restype = ret
                _lib = handle
    return _lib


def dt(t: torch.dtype | torch.Tensor) -> int:
    d = t.dtype if isinstance(t, torch.Tensor) else t
    if d not in _TORCH_DT:
        raise ValueError(f"unsupported dtype {d}")
    return _TORCH_DT[d]


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def check(rc: int, what: str) -> None:
    """Maps an ABI status code to the exception the reference raises."""
    if rc == MOE_OK:
        return
    msg = lib().moe_last_error().decode(errors="replace")
    if rc == MOE_ERR_INVALID_ARG:
        raise ValueError(f"{what}: {msg}")
    if rc == MOE_ERR_NO_DEVICE:
        raise RuntimeError(f"{what}: needs an sm_100 CUDA device: {msg}")
    raise RuntimeError(f"{what}: {lib().moe_status_string(rc).decode()}: {msg}")


# ---------------------------------------------------------------- device state
_status: dict[int, torch.Tensor] = {}
_workspaces: dict[tuple[int, int, str], torch.Tensor] = {}


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 the kernels write errors into (0 = OK)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    s = _status.get(idx)
    if s is None:
        s = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = s
    return s


def check_device_status(device: torch.device) -> None:
    """Synchronises and raises MoeDeviceError if a kernel reported an error."""
    s = status_word(device)
    code = int(s.item())
    if code != MOE_OK:
        s.zero_()
        raise MoeDeviceError(f"device reported: {lib().moe_status_string(code).decode()} ({code})")


def workspace(device: torch.device, nbytes: int, tag: str) -> torch.Tensor:
    """A zero-initialised byte buffer cached per (device, stream, tag), at
    least ``nbytes`` long. Kernels use it as scratch within one call (the
    grouping's per-chunk histograms, the router's partial-logit slabs, the
    FFN's intermediate rows); caching per stream keeps calls on concurrent
    streams from sharing it."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, stream_ptr(device), tag)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=torch.device("cuda", idx))
        _workspaces[key] = buf
    return buf


def require_cuda(*tensors: torch.Tensor | None, what: str = "the B200 MoE kernels") -> torch.device:
    devs = {t.device for t in tensors if t is not None}
    if any(d.type != "cuda" for d in devs):
        raise ValueError(f"{what} need CUDA tensors")
    if len(devs) != 1:
        raise ValueError(f"{what} need all tensors on one CUDA device, got {sorted(map(str, devs))}")
    return next(iter(devs))
