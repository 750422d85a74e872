"""ctypes binding of libexl3_b200.so (the C ABI declared in include/exl3_b200.h).

The library is loaded from this directory (built in-tree by ``b70-inference_b200/build.py``) or from
$EXL3_B200_LIB. There is no fallback: if the library is missing, every op raises.
"""
from __future__ import annotations

import ctypes as C
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("EXL3_B200_LIB") or os.path.join(HERE, "libexl3_b200.so")

EXL3_OK, EXL3_ERR_ARG, EXL3_ERR_UNSUPPORTED, EXL3_ERR_WORKSPACE, EXL3_ERR_CUDA, EXL3_ERR_TIMEOUT = range(6)
F16, BF16, F32 = 0, 1, 2
ROUTE_SIGMOID, ROUTE_SOFTMAX, ROUTE_SQRT_SOFTPLUS = 0, 1, 2

_DTYPE = {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32}

vp, i32, i64, f32, sz = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t


class Expert(C.Structure):
    """exl3_expert: device addresses of one expert's gate/up/down trellis, suh, svh and their K."""
    _fields_ = [("trellis", vp * 3), ("suh", vp * 3), ("svh", vp * 3), ("K", C.c_int32 * 3), ("pad", C.c_int32)]


# (name, restype, argtypes)
_PROTOS = [
    ("exl3_version", i32, []),
    ("exl3_last_error", C.c_char_p, []),
    ("exl3_device_status", i32, [i32]),
    ("exl3_wait_probe", i32, [C.c_uint64, vp]),
    ("exl3_set_finisher_wait", i32, [C.c_uint64]),
    ("exl3_dequant", i32, [vp, i32, i32, i32, i32, i32, i32, vp, i32, vp]),
    ("exl3_had_r_128", i32, [vp, vp, i32, i32, i32, vp, vp, f32, vp]),
    ("exl3_pack", i32, [vp, i32, i32, i32, vp, vp]),
    ("exl3_pack_gateup", i32, [vp, vp, i32, i32, i32, i32, vp, vp]),
    ("exl3_gemv_workspace_size", sz, [i32, i32, i32]),
    ("exl3_gemv", i32, [vp, i32, i32, i32, vp, vp, vp, i32, i32, i32, i32, vp, i32, i32, vp, sz, i32, vp]),
    ("exl3_gemm_tc_workspace_size", sz, [i32, i32]),
    ("exl3_gemm_tc", i32, [vp, i32, i32, i32, vp, vp, vp, i32, i32, i32, i32, vp, i32, i32, vp, sz, vp]),
    ("exl3_gemv_noalloc", i32, [vp, i32, i32, i32, vp, vp, vp, i32, i32, i32, i32, vp, i32, i32, vp]),
    ("exl3_mgemm_workspace_size", sz, [i32, i32, i32, i32, i32]),
    ("exl3_mgemm", i32, [vp, i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, i32, vp, i32, vp, i32, i32, i32, vp, i32,
                         i32, vp, sz, vp]),
    ("exl3_silu_mul", i32, [vp, vp, vp, i64, f32, vp]),
    ("exl3_route", i32, [vp, i32, i32, i32, i32, i32, vp, vp, vp, f32, i32, vp, i32, vp, vp, vp]),
    ("exl3_route_hidden_workspace_size", sz, [i32, i32]),
    ("exl3_route_hidden", i32, [vp, i32, i32, i32, i32, vp, i32, i32, i32, vp, vp, vp, f32, i32, vp, i32, vp, vp, vp,
                                vp, sz, vp]),
    ("exl3_route_hidden_pair", i32, [vp, i32, i32, i32, i32, vp, i32, i32, i32, vp, vp, vp, f32, i32, vp, i32, vp,
                                     vp, vp, vp, i32, i32, i32, vp, vp, f32, i32, vp, i32, vp, vp, sz, vp]),
    ("exl3_router_logits", i32, [vp, i32, i32, i32, i32, vp, i32, vp, vp, vp]),
    ("exl3_moe_workspace_size", sz, [i32, i32, i32, i32, i32, i32]),
    ("exl3_moe_decode", i32, [vp, i32, i32, i32, vp, vp, i32, vp, i32, i32, i32, i32, f32, vp, i32, vp, sz, i32,
                              vp]),
    ("exl3_moe_prefill_workspace_size", sz, [i32, i32, i32, i32, i32, i32]),
    ("exl3_moe_prefill", i32, [vp, i32, i32, i32, vp, vp, i32, vp, i32, i32, i32, i32, f32, vp, i32, vp, sz, vp]),
    ("exl3_moe_align", i32, [vp, vp, i32, i32, i32, i32, i32, vp, sz, vp]),
    ("exl3_moe_prepare", i32, [vp, i32, i32, i32, vp, vp, i32, vp, i32, i32, i32, i32, vp, sz, vp]),
    ("exl3_moe_gateup", i32, [i32, i32, vp, i32, i32, i32, i32, f32, vp, sz, i32, vp]),
    ("exl3_moe_down", i32, [i32, i32, vp, i32, i32, i32, i32, vp, sz, i32, vp]),
    ("exl3_moe_combine", i32, [i32, i32, i32, i32, i32, i32, vp, i32, vp, sz, vp]),
    ("exl3_ep_buffer_bytes", sz, [i32, i32, i32, i32]),
    ("exl3_ep_recv_offsets", i32, [i32, i32, i32, i32, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t),
                                   C.POINTER(C.c_size_t)]),
    ("exl3_ep_buffer_create", i32, [sz, C.POINTER(vp), vp]),
    ("exl3_ep_buffer_open", i32, [vp, C.POINTER(vp)]),
    ("exl3_ep_buffer_close", i32, [vp]),
    ("exl3_ep_buffer_free", i32, [vp]),
    ("exl3_ep_dispatch", i32, [vp, i32, i32, i32, vp, vp, i32, i32, i32, i32, i32, i32, vp, vp, vp]),
    ("exl3_ep_combine", i32, [vp, i32, i32, i32, i32, i32, i32, vp, vp, vp]),
    ("exl3_ep_reduce", i32, [vp, i32, i32, i32, i32, i32, i32, i32, vp, vp, vp, vp]),
    ("exl3_ep_combine_reduce", i32, [vp, vp, i32, i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp]),
]

_lib = None


def lib():
    """The loaded library (raises if it is missing: there is no CPU or eager fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"exl3_b200: CUDA library not found at {LIB_PATH}; build it with "
                               f"`python b70-inference_b200/build.py`")
        L = C.CDLL(LIB_PATH)
        for name, res, args in _PROTOS:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def exported_symbols() -> list[str]:
    return [n for n, _, _ in _PROTOS]


class Exl3Error(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    if rc != EXL3_OK:
        msg = lib().exl3_last_error().decode(errors="replace")
        raise Exl3Error(f"{what}: error {rc}: {msg}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    """Raw cudaStream_t of the current stream of t's device (launches follow torch's stream semantics)."""
    return torch.cuda.current_stream(t.device).cuda_stream


def dtype_code(dt: torch.dtype) -> int:
    if dt not in _DTYPE:
        raise Exl3Error(f"unsupported dtype {dt}")
    return _DTYPE[dt]


_WS: dict = {}


def zeroed_workspace(device, nbytes: int, key: str) -> torch.Tensor:
    """A cached device buffer zeroed when (re)allocated, for entry points that need zeroed scratch on their first
    use and leave it zeroed (exl3_route_hidden's ticket)."""
    k = (str(device), "zeroed:" + key)
    buf = _WS.get(k)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(int(nbytes), 1 << 16), dtype=torch.uint8, device=device)
        _WS[k] = buf
    return buf


def workspace(device, nbytes: int, key: str = "ws") -> torch.Tensor:
    """A cached device byte buffer of at least nbytes (grown on demand, reused across calls on the same stream).
    Calls that overlap on different streams must pass their own workspace."""
    k = (str(device), key)
    buf = _WS.get(k)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(int(nbytes), 1 << 20), dtype=torch.uint8, device=device)
        _WS[k] = buf
    return buf


def require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise Exl3Error("exl3_b200 ops run on CUDA tensors only (no CPU fallback)")
