"""ctypes binding of libq2b.so (C ABI: include/q2b.h).

This is the only route from Python to the kernels.  There is no fallback:
if the library cannot be loaded, or the device is not an sm_100 GPU, every
operation raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

from . import build as _build

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_F = ctypes.c_float
_U64 = ctypes.c_uint64
_INT = ctypes.c_int

Q2B_OK = 0
Q2B_ERR_INVALID = 1
Q2B_ERR_CUDA = 2
Q2B_ERR_DEVICE = 3

MODE_RNE = 0
MODE_FOUR_SIX = 1

# name -> argtypes (all return int status, except q2b_last_error / q2b_version)
SIGNATURES = {
    "q2b_device_status": [_P],
    "q2b_abs_max": [_P, _P, _I64, _P],
    "q2b_quant_fwd": [_P, _P, _P, _P, _P, _F, _I64, _I64, _INT, _P],
    "q2b_rht_eden": [_P, _P, _P, _P, _P, _P, _INT, _P, _U64, _F, _F, _I64, _I64, _INT, _P],
    "q2b_rht_eden_noalloc": [_P, _P, _P, _P, _INT, _P, _U64, _F, _F, _I64, _I64, _INT, _P],
    "q2b_rht_eden_dual": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _INT, _P, _U64, _U64, _F, _F, _I64, _I64, _P],
    "q2b_rht_requant": [_P, _P, _P, _P, _P, _P, _INT, _P, _P, _P, _U64, _F, _F, _I64, _I64, _P],
    "q2b_gemm_nvfp4": [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P],
    "q2b_quant_fwd_ragged": [_P, _P, _P, _P, _P, _F, _I64, _I64, _INT, _P],
    "q2b_gemm_nvfp4_ex": [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P, _I64, _P],
    "q2b_quant_rows_fused": [_P, _P, _P, _P, _F, _I64, _I64, _INT, _P],
    "q2b_relu2_abs_max": [_P, _P, _P, _I64, _P],
    "q2b_adamw_step": [_P, _P, _P, _P, _INT, _I64, _F, _F, _F, _F, _F, _I64, _P, _P, _P],
    "q2b_fp4_mma_peak": [_INT, _INT, _P, _P],
}

_lib = None
_lock = threading.Lock()


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load (building first if sources are newer) the in-tree libq2b.so."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = _build.LIB_PATH
        if build_if_missing and _build.needs_build():
            _build.build()
        if not os.path.exists(path):
            raise RuntimeError(f"libq2b.so not found at {path}; run `python -m cloverlm_b200.build`")
        lib = ctypes.CDLL(path)
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = _INT
        lib.q2b_last_error.argtypes = []
        lib.q2b_last_error.restype = ctypes.c_char_p
        lib.q2b_gemm_workspace_bytes.argtypes = [_I64, _I64, _I64]
        lib.q2b_gemm_workspace_bytes.restype = _I64
        lib.q2b_version.argtypes = []
        lib.q2b_version.restype = _INT
        _lib = lib
        return lib


def lib_path() -> str:
    return _build.LIB_PATH


def check(status: int, what: str) -> None:
    if status == Q2B_OK:
        return
    msg = load().q2b_last_error().decode(errors="replace")
    if status == Q2B_ERR_INVALID:
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor):
    if not t.is_cuda:
        raise ValueError("tensor must be on a CUDA device")
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def device_status() -> int:
    """Return (and clear) the watchdog code of the current device; 0 = no timed-out wait."""
    code = ctypes.c_uint(0)
    call("q2b_device_status", ctypes.byref(code))
    return int(code.value)
