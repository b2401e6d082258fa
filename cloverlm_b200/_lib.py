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
    "q2b_watchdog_poll": [_P, _P],
    "q2b_watchdog_selftest": [_I64, _P],
    "q2b_abs_max": [_P, _P, _I64, _P],
    "q2b_quant_fwd": [_P, _P, _P, _P, _P, _F, _I64, _I64, _INT, _P],
    "q2b_rht_eden": [_P, _P, _P, _P, _P, _P, _INT, _P, _U64, _F, _F, _I64, _I64, _INT, _P],
    "q2b_rht_eden_noalloc": [_P, _P, _P, _P, _INT, _P, _U64, _F, _F, _I64, _I64, _INT, _P],
    "q2b_rht_eden_dual": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _INT, _P, _U64, _U64, _F, _F, _I64, _I64, _P],
    "q2b_rht_requant": [_P, _P, _P, _P, _P, _P, _INT, _P, _P, _P, _U64, _F, _F, _I64, _I64, _P],
    "q2b_gemm_nvfp4": [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P],
    "q2b_gemm_nvfp4_f32": [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P],
    "q2b_gemm_nvfp4_add": [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P],
    "q2b_gemm_nvfp4_relu2": [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P],
    "q2b_gemm_nvfp4_relu2_bwd": [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P],
    "q2b_quant_fwd_ragged": [_P, _P, _P, _P, _P, _F, _I64, _I64, _INT, _P],
    "q2b_gemm_nvfp4_ex": [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P, _I64, _P],
    "q2b_quant_rows_fused": [_P, _P, _P, _P, _F, _I64, _I64, _INT, _P],
    "q2b_relu2_abs_max": [_P, _P, _P, _I64, _P],
    "q2b_relu2_bwd": [_P, _P, _P, _I64, _P],
    "q2b_softmax_xent_bf16": [_P, _P, _P, _F, _I64, _I64, _P],
    "q2b_rope_norm_fwd": [_P, _P, _P, _P, _P, _I64, _INT, _INT, _P],
    "q2b_rope_norm_bwd": [_P, _P, _P, _P, _P, _P, _P, _I64, _INT, _INT, _P],
    "q2b_add_rmsnorm_amax": [_P, _P, _P, _P, _P, _P, _P, _I64, _INT, _F, _P],
    "q2b_rmsnorm_bwd": [_P, _P, _P, _I64, _P, _P, _P, _P, _P, _I64, _INT, _P],
    "q2b_adamw_step": [_P, _P, _P, _P, _INT, _I64, _F, _F, _F, _F, _F, _I64, _P, _P, _P],
    "q2b_fp4_mma_peak": [_INT, _P, _P],
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


class WatchdogTimeout(RuntimeError):
    """A bounded wait inside a libq2b kernel gave up; outputs since then are invalid."""


class WatchdogMonitor:
    """Makes a watchdog trip visible on the normal training path without a sync.

    ``poll()`` is called once per step (the optimizer and the data-parallel
    exchange call it): it checks the word copied by the previous poll, if the
    stream has passed that copy, and raises WatchdogTimeout when it is set;
    then it queues the next asynchronous copy (q2b_watchdog_poll) into pinned
    host memory.  A trip is therefore reported at most one step late."""

    def __init__(self, device: torch.device):
        self.device = device
        self.words = torch.zeros(2, dtype=torch.int32).pin_memory()
        self.events = [None, None]
        self.slot = 0

    def _check(self, slot: int, block: bool) -> None:
        ev = self.events[slot]
        if ev is None:
            return
        if block:
            ev.synchronize()
        elif not ev.query():
            return
        code = int(self.words[slot].item()) & 0xFFFFFFFF
        self.events[slot] = None
        if code:
            raise WatchdogTimeout(f"a libq2b kernel wait timed out (watchdog code {code}); results computed since "
                                  f"then are invalid -- clear with q2b_device_status after handling")

    def poll(self) -> None:
        other = self.slot ^ 1
        self._check(other, block=False)
        self._check(self.slot, block=False)
        stream = torch.cuda.current_stream(self.device)
        ptr_ = ctypes.c_void_p(self.words.data_ptr() + 4 * self.slot)
        with torch.cuda.device(self.device):
            call("q2b_watchdog_poll", ptr_, ctypes.c_void_p(stream.cuda_stream))
            ev = torch.cuda.Event()
            ev.record(stream)
        self.events[self.slot] = ev
        self.slot = other

    def check_now(self) -> None:
        """Block until every queued poll has landed and raise if any saw a trip."""
        self._check(0, block=True)
        self._check(1, block=True)


_monitors: dict = {}


def watchdog(device: torch.device) -> WatchdogMonitor:
    """The process-wide WatchdogMonitor of `device`."""
    key = torch.device(device).index if torch.device(device).index is not None else torch.cuda.current_device()
    mon = _monitors.get(key)
    if mon is None:
        mon = _monitors[key] = WatchdogMonitor(torch.device("cuda", key))
    return mon
