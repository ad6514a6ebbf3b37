"""ctypes binding of librespect_b200.so (the C ABI in include/respect_b200.h).

The native library is the only compute path: if it is missing or fails to
load, every operator raises. There is no CPU or library fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

# RESPECT_B200_LIB names a librespect_b200.so built elsewhere (e.g. with other compile-time options).
LIB_PATH = Path(os.environ.get("RESPECT_B200_LIB") or Path(__file__).resolve().parent / "librespect_b200.so")

RB_OK = 0
RB_ERR_INVALID_ARG, RB_ERR_UNSUPPORTED, RB_ERR_CAPACITY, RB_ERR_CUDA, RB_ERR_DEVICE_TIMEOUT, RB_ERR_WORKSPACE = 1, 2, 3, 4, 5, 6
RB_F32, RB_BF16, RB_U8, RB_I32, RB_I64 = 0, 1, 2, 3, 4
RB_MASK_BOOL, RB_MASK_ADD_BF16, RB_MASK_ADD_F32, RB_MASK_CAUSAL = 0, 1, 2, 3
COMPACT_MAX_LAYERS = 128
COMPACT_MAX_SLOTS = 1024

_DT = {torch.float32: RB_F32, torch.bfloat16: RB_BF16, torch.uint8: RB_U8, torch.bool: RB_U8,
       torch.int32: RB_I32, torch.int64: RB_I64}

c_void_p, c_int, c_int64, c_size_t, c_float = (ctypes.c_void_p, ctypes.c_int, ctypes.c_int64,
                                               ctypes.c_size_t, ctypes.c_float)


class RespectNativeError(RuntimeError):
    """A native entry point returned a non-zero rb_status."""

    def __init__(self, fn: str, status: int, message: str):
        super().__init__(f"{fn}: {message} (rb_status {status})")
        self.fn, self.status = fn, status


class AttnArgs(ctypes.Structure):
    """Mirror of rb_attn_args."""
    _fields_ = [("dtype", c_int), ("H", c_int), ("M", c_int), ("D", c_int), ("HK", c_int),
                ("NP", c_int), ("NN", c_int),
                ("q", c_void_p), ("sqh", c_int64), ("sqm", c_int64), ("sqd", c_int64),
                ("kp", c_void_p), ("skph", c_int64), ("skpn", c_int64), ("skpd", c_int64),
                ("vp", c_void_p), ("svph", c_int64), ("svpn", c_int64), ("svpd", c_int64),
                ("kn", c_void_p), ("sknh", c_int64), ("sknn", c_int64), ("sknd", c_int64),
                ("vn", c_void_p), ("svnh", c_int64), ("svnn", c_int64), ("svnd", c_int64),
                ("msk", c_void_p), ("mask_kind", c_int), ("smm", c_int64), ("smn", c_int64),
                ("causal_first", c_int),
                ("out", c_void_p), ("soh", c_int64), ("som", c_int64), ("sod", c_int64),
                ("sm_scale", c_float)]


# name -> (restype, argtypes)
SIGNATURES = {
    "rb_status_string": (ctypes.c_char_p, [c_int]),
    "rb_abi_version": (c_int, []),
    "rb_num_sms": (c_int, []),
    "rb_device_error": (c_int, [ctypes.POINTER(c_int), c_int]),
    "rb_fused_attn_hyb_workspace": (c_size_t, [c_int, c_int, c_int, c_int]),
    "rb_fused_attn_hyb": (c_int, [ctypes.POINTER(AttnArgs), c_void_p, c_size_t, c_void_p]),
    "rb_linear_workspace": (c_size_t, [c_int, c_int, c_int]),
    "rb_linear": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int, c_int, c_int,
                          c_int, c_void_p, c_size_t, c_void_p]),
    "rb_linear_bn": (c_int, [c_int, c_int]),
    "rb_linear_packed_bytes": (c_size_t, [c_int, c_int, c_int]),
    "rb_pack_linear_weight": (c_int, [c_void_p, c_int64, c_int, c_int, c_int, c_void_p, c_void_p]),
    "rb_linear_packed": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_int,
                                 c_void_p, c_size_t, c_void_p]),
    "rb_linear_swiglu_packed": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int, c_int, c_int,
                                        c_void_p]),
    "rb_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_int, c_int, c_void_p]),
    "rb_rope": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int64,
                        c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "rb_silu_mul": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p]),
    "rb_add_sq": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_void_p]),
    "rb_norm_apply": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_float, c_int, c_int, c_int,
                              c_void_p]),
    "rb_greedy_token": (c_int, [c_void_p, c_int, c_int64, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "rb_compact_kv": (c_int, [ctypes.POINTER(c_void_p), ctypes.POINTER(c_void_p), c_int, c_int, c_int,
                              c_int64, c_int64, c_int, ctypes.POINTER(ctypes.c_int32), c_int, c_int,
                              c_void_p]),
    "rb_trie_node_mask": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int64, c_void_p]),
    "rb_verify_mask": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
}

_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load librespect_b200.so once. Raises if it is missing or incomplete."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: run `python -m respect_b200.build` "
                              "(respect_b200 has no fallback path)")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)  # AttributeError if the library lacks a symbol
            fn.restype, fn.argtypes = res, args
        _lib = handle
    return _lib


def call(name: str, *args) -> None:
    """Call an entry point and raise RespectNativeError on a non-zero status."""
    st = getattr(lib(), name)(*args)
    if st != RB_OK:
        msg = lib().rb_status_string(st).decode()
        raise RespectNativeError(name, st, msg)


def dtype_code(t: torch.dtype) -> int:
    try:
        return _DT[t]
    except KeyError:
        raise TypeError(f"respect_b200: unsupported dtype {t}") from None


def stream_of(t: torch.Tensor) -> int:
    """Handle of the current CUDA stream on t's device (what torch ops use)."""
    if not t.is_cuda:
        raise ValueError("respect_b200 operators take CUDA tensors (no CPU path)")
    return torch.cuda.current_stream(t.device).cuda_stream


_ws: dict = {}


def workspace(t: torch.Tensor, nbytes: int) -> torch.Tensor | None:
    """Per-(device, stream) scratch buffer, grown on demand and kept for reuse."""
    if nbytes <= 0:
        return None
    key = (t.device, stream_of(t))
    buf = _ws.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=t.device)
        _ws[key] = buf
    return buf


def device_error(clear: bool = True) -> int:
    """Value of the device error flag set by a bounded device wait (0 = none)."""
    code = c_int(0)
    call("rb_device_error", ctypes.byref(code), int(clear))
    return code.value
