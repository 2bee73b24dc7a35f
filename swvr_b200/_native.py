"""ctypes binding of libswvr_b200.so, the C ABI declared in include/swvr_b200.h.

The library is built in-tree (``swvr_b200/_lib/libswvr_b200.so``, see ``build.py``).  There is
no fallback: if it is missing, every op raises.  Python passes device pointers, sizes, dtype
codes and the current CUDA stream; the library allocates nothing.
"""
from __future__ import annotations

import ctypes
import os
import re
from ctypes import POINTER, c_char_p, c_double, c_int, c_int32, c_int64, c_size_t, c_uint32, c_void_p

import torch

LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib")
# SWVR_LIB overrides the library file (e.g. an installed copy); default: the in-tree build.
LIB_PATH = os.environ.get("SWVR_LIB") or os.path.join(LIB_DIR, "libswvr_b200.so")
HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "swvr_b200.h")

OK, ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_CUDA, ERR_WORKSPACE = 0, -1, -2, -3, -4
F32, F64, BF16, F16 = 0, 1, 2, 3
REDUCE_NONE, REDUCE_SUM, REDUCE_MEAN = 0, 1, 2
MSE_STATS_LEN = 514  # SWVR_MSE_STATS_LEN
SELFTEST_CODE = 0x7F01  # SWVR_SELFTEST_CODE

DTYPE_CODE = {torch.float32: F32, torch.float64: F64, torch.bfloat16: BF16, torch.float16: F16}


class Problem(ctypes.Structure):
    _fields_ = [
        ("n_tokens", c_int64), ("hidden", c_int64), ("vocab", c_int64), ("embed_dim", c_int64),
        ("compute_dtype", c_int32), ("bias_dtype", c_int32),
        ("h", c_void_p), ("ldh", c_int64),
        ("W", c_void_p), ("ldw", c_int64),
        ("E", c_void_p), ("lde", c_int64),
        ("bias", c_void_p),
        ("logit_scale", c_double),
        ("chunk", c_int64),
    ]


class Grads(ctypes.Structure):
    _fields_ = [
        ("grad_O", c_void_p), ("grad_lse", c_void_p), ("O", c_void_p), ("lse", c_void_p),
        ("grad_h", c_void_p), ("grad_h_dtype", c_int32),
        ("grad_W", c_void_p), ("grad_W_dtype", c_int32), ("ld_grad_W", c_int64),
        ("grad_E", c_void_p), ("grad_E_dtype", c_int32), ("ld_grad_E", c_int64),
        ("grad_bias", c_void_p), ("grad_bias_dtype", c_int32),
        ("grad_h_acc", c_void_p), ("accumulate_grad_h", c_int32),
    ]


class ProfileRecord(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 32), ("launches", c_int64), ("total_ms", c_double)]


_SIGNATURES = {
    "swvr_abi_version": (c_int, []),
    "swvr_selftest_wait_timeout": (c_int, [c_int64, c_void_p]),
    "swvr_last_error": (c_char_p, []),
    "swvr_device_error": (c_int, [POINTER(c_uint32)]),
    "swvr_fwd_workspace_size": (c_int, [POINTER(Problem), POINTER(c_size_t)]),
    "swvr_fwd": (c_int, [POINTER(Problem), c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "swvr_fwd_partial": (c_int, [POINTER(Problem), c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "swvr_combine": (c_int, [c_int64, c_int64, c_int64, c_int32, c_void_p, c_void_p, c_void_p, c_void_p,
                             c_void_p, c_void_p]),
    "swvr_bwd_workspace_size": (c_int, [POINTER(Problem), POINTER(Grads), POINTER(c_size_t)]),
    "swvr_bwd": (c_int, [POINTER(Problem), POINTER(Grads), c_void_p, c_size_t, c_void_p]),
    "swvr_bwd_split": (c_int, [POINTER(Problem), POINTER(Grads), c_void_p, c_size_t, c_void_p]),
    "swvr_bwd_finish": (c_int, [POINTER(Problem), POINTER(Grads), c_void_p, c_size_t, c_int32, c_void_p]),
    "swvr_mse_fwd": (c_int, [c_int64, c_int64, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_double,
                             c_int32, c_void_p, c_void_p, c_void_p]),
    "swvr_mse_bwd": (c_int, [c_int64, c_int64, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_double,
                             c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "swvr_fwd_noalloc": (c_int, [POINTER(Problem), c_void_p, c_void_p, c_void_p]),
    "swvr_rmsnorm_fwd": (c_int, [c_int64, c_int64, c_void_p, c_int32, c_int64, c_void_p, c_int32, c_double, c_void_p,
                                 c_int32, c_int64, c_void_p, c_void_p]),
    "swvr_rmsnorm_bwd_workspace_size": (c_int, [c_int64, c_int64, c_int32, c_int32, POINTER(c_size_t)]),
    "swvr_rmsnorm_bwd": (c_int, [c_int64, c_int64, c_void_p, c_int32, c_void_p, c_int32, c_int64, c_void_p, c_int32,
                                 c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_void_p, c_size_t, c_void_p]),
    "swvr_profile_start": (c_int, []),
    "swvr_profile_stop": (c_int, [POINTER(ProfileRecord), c_int, POINTER(c_int)]),
}

_lib = None


def header_functions() -> list:
    """Names of the functions include/swvr_b200.h declares."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(swvr_\w+)\s*\(", text, flags=re.M)))


def lib():
    """Load (once) and return the CUDA library; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -c 'import swvr_b200.build as b; b.build()'`. "
                "swvr_b200 has no CPU or Python fallback.")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    return (lib().swvr_last_error() or b"").decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc == OK:
        return
    msg = f"{what}: {last_error()}"
    if rc == ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    raise RuntimeError(msg)


def check_device_error() -> None:
    """Raise if a bounded device-side wait expired since the last check (synchronises)."""
    code = c_uint32(0)
    check(lib().swvr_device_error(ctypes.byref(code)), "swvr_device_error")
    if code.value:
        raise RuntimeError(f"swvr_b200 kernel gave up waiting (device error site 0x{code.value:x})")


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t):
    return None if t is None else t.data_ptr()


def dtype_code(dt: torch.dtype) -> int:
    try:
        return DTYPE_CODE[dt]
    except KeyError:
        raise ValueError(f"unsupported dtype {dt}") from None


class profile:
    """Context manager counting (and event-timing) every library kernel launched inside it.

    ``result`` maps kernel name -> (launches, total milliseconds of event time)."""

    def __enter__(self):
        check(lib().swvr_profile_start(), "swvr_profile_start")
        self.result = {}
        return self

    def __exit__(self, *exc):
        recs = (ProfileRecord * 16)()
        n = c_int(0)
        check(lib().swvr_profile_stop(recs, 16, ctypes.byref(n)), "swvr_profile_stop")
        self.result = {recs[i].name.decode(): (int(recs[i].launches), float(recs[i].total_ms))
                       for i in range(min(n.value, 16))}
        return False
