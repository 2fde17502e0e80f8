"""ctypes binding of libpisa_b200.so (the C ABI declared in include/pisa_b200.h).

The CUDA library is the only compute path: importing an operator without the
built library raises ImportError, and every call on a CPU tensor raises
ValueError.  There is no CPU or Triton fallback.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().with_name("libpisa_b200.so")

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_TIMEOUT = 0, 1, 2, 3, 4
F32, BF16, F16 = 0, 1, 2
METHODS = {"pisa1": 0, "pisa2": 1, "pisa": 2}
SCHEDULES = {"grouped": 0, "fused": 1}
DTYPES = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_F = ctypes.c_float

# name -> (restype, argtypes); one entry per function of include/pisa_b200.h
SIGNATURES = {
    "pisa_version": (_I, []),
    "pisa_last_error": (ctypes.c_char_p, []),
    "pisa_mean_pool": (_I, [_P, _I, _L, _L, _L, _L, _L, _L, _L, _L, _P, _P]),
    "pisa_build_pyramid": (_I, [_P, _I, _L, _L, _L, _L, _L, _L, _L, _L, _L, _L, _P, _L, _P, _P]),
    "pisa_pyramid_update": (_I, [_P, _I, _L, _L, _L, _L, _L, _L, _L, _L, _L, _L, _P, _L, _P, _L, _P]),
    "pisa_select_blocks": (_I, [_P, _L, _L, _L, _P, _L, _L, _L, _P, _L, _P, _P, _L, _P, _L, _I,
                                _L, _L, _L, _L, _L, _L, _I, _L, _L, _L, _I, _L, _L, _L, _I, _P,
                                _P, _L, _P]),
    "pisa_select_workspace_bytes": (_L, [_L, _L, _L, _L, _L, _L, _I, _I, _L, _L, _L, _L, _L, _I, _I]),
    "pisa_select_level_plan": (_L, [_L, _L, _L, _L, _L, _L, _I, _I, _L, _L, _L, _L, _L, _I]),
    "pisa_decode_select_attend": (_I, [_P, _L, _L, _L, _P, _L, _L, _L, _P, _L, _L, _L, _P, _L, _P, _P, _L, _P, _L,
                                       _I, _L, _L, _L, _L, _L, _L, _L, _I, _L, _L, _L, _I, _L, _L, _L, _F,
                                       _P, _P, _P, _P]),
    "pisa_sparse_attn_fwd": (_I, [_P, _L, _L, _L, _P, _L, _L, _L, _P, _L, _L, _L, _P, _I, _P, _L,
                                  _I, _L, _L, _L, _L, _L, _L, _L, _L, _L, _F, _I, _P, _P, _P, _L,
                                  _P]),
    "pisa_sparse_attn_fwd_workspace_bytes": (_L, [_L, _L, _L, _L, _L, _L, _L, _L, _L, _I]),
    "pisa_sparse_attn_bwd": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _P, _L, _I, _L, _L, _L, _L, _L,
                                  _L, _L, _L, _L, _F, _I, _P, _P, _P, _P, _L, _P]),
    "pisa_sparse_attn_bwd_workspace_bytes": (_L, [_L, _L, _L, _L, _L, _L, _L]),
    "pisa_sparse_attn_bwd_tc_workspace_bytes": (_L, [_L, _L, _L, _L, _L, _L, _L, _L, _L, _I]),
    "pisa_sparse_attn_bwd_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _P, _L, _I, _L, _L, _L, _L, _L,
                                          _L, _L, _L, _L, _F, _I, _P, _P, _P, _P]),
    "pisa_sparse_attn_bwd_noalloc_max_bytes": (_L, []),
    "pisa_leaf_scores": (_I, [_P, _L, _L, _L, _P, _L, _L, _L, _P, _L, _P, _I, _P, _I, _L, _L, _L, _L,
                              _L, _L, _L, _I, _L, _L, _I, _L, _P, _P, _L, _P]),
    "pisa_leaf_scores_workspace_bytes": (_L, [_L, _L, _L, _L, _L, _L, _L, _I, _I, _L, _I]),
    "pisa_bsa_select": (_I, [_P, _L, _L, _L, _P, _L, _L, _L, _P, _L, _P, _L, _I, _L, _L, _L, _L, _L, _L, _L,
                             _L, _I, _L, _P, _P, _L, _P]),
    "pisa_bsa_workspace_bytes": (_L, [_L, _L, _L, _L, _I, _L, _I]),
    "pisa_rotary": (_I, [_P, _L, _L, _L, _P, _L, _L, _L, _P, _L, _L, _P, _I, _L, _L, _L, _L, _P]),
    "pisa_workspace_status": (_I, [_P, _P]),
    "pisa_wait_selftest": (_I, [_I, _L, _P, _L, _P]),
    "pisa_ex2_selftest": (_I, [_P, _P, _P, _L, _P]),
    "pisa_launch_count": (_L, []),
    "pisa_kernel_timing": (_I, [_I]),
    "pisa_kernel_time": (_I, [_I, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64)]),
}

_lib = None


def lib():
    """Load and type the library once (ImportError when it was never built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH.name} is not built; run `python -m nlogn_pisa_b200.build` "
                "(there is no CPU fallback)")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype, fn.argtypes = res, args
        _lib = handle
    return _lib


def check(status):
    """Map a status code to the reference's exception types."""
    if status == OK:
        return
    message = lib().pisa_last_error().decode(errors="replace")
    if status in (ERR_INVALID, ERR_UNSUPPORTED):
        raise ValueError(message)
    raise RuntimeError(f"libpisa_b200: {message}")


_checked = os.environ.get("PISA_CHECK_STATUS", "0") not in ("", "0")


def set_status_checks(enabled):
    """With checks on, every operator that ran a waiting kernel reads its
    device status word back (one 4-byte copy and a stream synchronisation)
    and raises RuntimeError when a bounded device wait expired.  Off by
    default: the common path never synchronises the host.  The environment
    variable PISA_CHECK_STATUS=1 turns checks on at import."""
    global _checked
    _checked = bool(enabled)


def status_checks():
    return _checked


def check_workspace(workspace, device):
    """Raise RuntimeError if the call that used ``workspace`` hit an expired wait."""
    if workspace is None:
        return
    with torch.cuda.device(device):
        check(lib().pisa_workspace_status(ptr(workspace), stream_of(device)))


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def int64_array(values):
    """A host int64[] for the ABI's level tables."""
    values = [int(v) for v in values]
    return (ctypes.c_int64 * max(1, len(values)))(*values)


def stream_of(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def dtype_code(t):
    try:
        return DTYPES[t.dtype]
    except KeyError:
        raise ValueError("the CUDA kernels support FP16, BF16 and FP32") from None


KERNELS = {"leaf_tiles": 0, "attn_tiles": 1, "attn_combine": 2, "pyramid": 3, "dense_level": 4, "router": 5,
           "leaf_final": 6, "bsa": 7}


def kernel_timing(enable):
    """Start (True) or stop (False) per-launch device timing of the tile kernels."""
    check(lib().pisa_kernel_timing(int(bool(enable))))


def kernel_time(name):
    """(device milliseconds, launches) of one timed kernel since its last read."""
    ms, n = ctypes.c_double(0.0), ctypes.c_int64(0)
    check(lib().pisa_kernel_time(KERNELS[name], ctypes.byref(ms), ctypes.byref(n)))
    return ms.value, n.value
