"""CPU oracle for the Quartet-II NVFP4 hot path -- TEST INFRASTRUCTURE ONLY.

This package is the checker the CUDA path of ``cloverlm_b200`` is compared
against.  Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline``
leg of ``bench.py`` (plus its ``--impl reference`` arm) may import it; the
product library never does, and has no CPU fallback.

It wraps ``liboracle.so`` (``q2b_oracle.c``, a plain-C restatement of the
reference kernels; see that file's header for the file:line of every routine
it follows) with numpy arrays, and composes the reference's Python-level
operations from it:

  quant_fp4            quartet2/python/quartet2/quant.py:114-138
  rht128_quant_eden    quartet2/python/quartet2/quant.py:320-397
  quant_had_eden       quartet2/python/quartet2/quant.py:141-213
  rht128_requant       quartet2/python/quartet2/quant.py:402-491
  swizzle_hadamard     quartet2/python/quartet2/rht.py:65-82
  dequant              quartet2/python/quartet2/linear.py:106-144 (_dq_fp4)

Arrays: bf16 tensors are passed as numpy ``uint16`` bit patterns; E2M1 codes
as ``uint8`` [rows, cols/2] (low nibble = even element); E4M3 scales as
``uint8`` in the blocked 128x4 layout, flat; tensor scales as Python floats.

Parity status: pinned.  The restatement is checked against (a) the reference's
own semantics tests restated here (bit-exact equality of the 16x128-slice and
full-matrix rotations, quartet2/test/test_rht.py:49-59; the effective-bitwidth
floors of quartet2/test/test_rounding.py:95-133), (b) golden vectors produced
by the reference's Python emulation ``src/fake_quartet.py`` (tests/golden/),
and (c) on a GPU box, the reference's own CUDA kernels built from source into
``oracle/_ref`` (tests/test_gpu_ref_pin.py).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None


def build(force: bool = False) -> str:
    """Compile liboracle.so with the committed Makefile (gcc only)."""
    src = os.path.join(_HERE, "q2b_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE, "liboracle.so"])
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        F = ctypes.c_float
        L.oq_bf16_to_f32.argtypes = [ctypes.c_uint16]; L.oq_bf16_to_f32.restype = F
        L.oq_f32_to_bf16.argtypes = [F]; L.oq_f32_to_bf16.restype = ctypes.c_uint16
        L.oq_f32_to_e2m1.argtypes = [F]; L.oq_f32_to_e2m1.restype = ctypes.c_uint8
        L.oq_e2m1_to_f32.argtypes = [ctypes.c_uint8]; L.oq_e2m1_to_f32.restype = F
        L.oq_f32_to_e4m3.argtypes = [F]; L.oq_f32_to_e4m3.restype = ctypes.c_uint8
        L.oq_e4m3_to_f32.argtypes = [ctypes.c_uint8]; L.oq_e4m3_to_f32.restype = F
        L.oq_sr_e4m3.argtypes = [F, ctypes.c_uint16]; L.oq_sr_e4m3.restype = ctypes.c_uint8
        L.oq_sf_offset.argtypes = [I64, I64, I64]; L.oq_sf_offset.restype = I64
        L.oq_amax_bf16.argtypes = [P, I64, P]; L.oq_amax_bf16.restype = None
        L.oq_quant_fwd.argtypes = [P, I64, I64, F, F, ctypes.c_int, P, P, P]; L.oq_quant_fwd.restype = None
        L.oq_build_rht_matrix.argtypes = [P, P]; L.oq_build_rht_matrix.restype = None
        L.oq_rotate.argtypes = [P, I64, I64, P, ctypes.c_int, P]; L.oq_rotate.restype = None
        L.oq_eden_pass1.argtypes = [P, I64, I64, F, P, P, P, P]; L.oq_eden_pass1.restype = None
        L.oq_philox.argtypes = [ctypes.c_uint64, ctypes.c_uint32, P]; L.oq_philox.restype = None
        L.oq_sr_scales.argtypes = [P, I64, I64, ctypes.c_uint32, F, ctypes.c_uint64, P, P]; L.oq_sr_scales.restype = None
        L.oq_dequant_bf16.argtypes = [P, P, F, I64, I64, P]; L.oq_dequant_bf16.restype = None
        L.oq_dequant_f32.argtypes = [P, P, F, I64, I64, P]; L.oq_dequant_f32.restype = None
        L.oq_num_threads.argtypes = []; L.oq_num_threads.restype = ctypes.c_int
        L.oq_set_num_threads.argtypes = [ctypes.c_int]; L.oq_set_num_threads.restype = None
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def set_num_threads(n: int) -> None:
    lib().oq_set_num_threads(int(n))


def num_threads() -> int:
    return int(lib().oq_num_threads())


# ---------------------------------------------------------------- formats

def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


E2M1_GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                      -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)


def e4m3_table() -> np.ndarray:
    L = lib()
    return np.array([L.oq_e4m3_to_f32(i) for i in range(256)], dtype=np.float32)


def sf_offsets(rows: int, cols16: int) -> np.ndarray:
    """offsets[r, k] = position of scale (r, k) in the blocked 128x4 layout."""
    r = np.arange(rows, dtype=np.int64)[:, None]
    k = np.arange(cols16, dtype=np.int64)[None, :]
    nkt = cols16 // 4
    return (((r >> 7) * nkt + (k >> 2)) << 9) | ((r & 31) << 4) | (((r >> 5) & 3) << 2) | (k & 3)


def unblock(sf_flat: np.ndarray, rows: int, cols16: int) -> np.ndarray:
    return np.asarray(sf_flat).reshape(-1)[sf_offsets(rows, cols16)]


def to_blocked(sf: np.ndarray) -> np.ndarray:
    rows, cols16 = sf.shape
    out = np.empty(rows * cols16, dtype=sf.dtype)
    out[sf_offsets(rows, cols16)] = sf
    return out


def unpack_codes(codes: np.ndarray) -> np.ndarray:
    c = np.asarray(codes, dtype=np.uint8)
    return np.stack([c & 15, c >> 4], axis=-1).reshape(c.shape[0], -1)


def dequant(codes: np.ndarray, sf_flat: np.ndarray, ts: float) -> np.ndarray:
    """fp32 code * scale * tensor_scale (the value the GEMM consumes)."""
    rows, half = codes.shape
    out = np.empty((rows, half * 2), dtype=np.float32)
    lib().oq_dequant_f32(_p(np.ascontiguousarray(codes)), _p(np.ascontiguousarray(sf_flat)), float(ts),
                         rows, half * 2, _p(out))
    return out


def dequant_bf16(codes: np.ndarray, sf_flat: np.ndarray, ts: float) -> np.ndarray:
    rows, half = codes.shape
    out = np.empty((rows, half * 2), dtype=np.uint16)
    lib().oq_dequant_bf16(_p(np.ascontiguousarray(codes)), _p(np.ascontiguousarray(sf_flat)), float(ts),
                          rows, half * 2, _p(out))
    return out


# ------------------------------------------------------------- operations

def amax(x_bf16: np.ndarray) -> float:
    out = np.zeros(1, dtype=np.float32)
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    lib().oq_amax_bf16(_p(x), x.size, _p(out))
    return float(out[0])


def quant_fp4(x_bf16: np.ndarray, amax_value: float | None = None, scale_override: float = 1.0,
              four_six: bool = True):
    """RNE (four_six=False) or four-over-six RTN NVFP4 quantization.

    Returns (codes [rows, cols/2] uint8, sf blocked uint8 [rows*cols/16], ts float).
    """
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    rows, cols = x.shape
    if rows % 128 or cols % 128:
        raise ValueError("rows and cols must be multiples of 128")
    a = amax(x) if amax_value is None else float(np.float32(amax_value))
    codes = np.empty((rows, cols // 2), dtype=np.uint8)
    sf = np.empty(rows * cols // 16, dtype=np.uint8)
    ts = np.zeros(1, dtype=np.float32)
    lib().oq_quant_fwd(_p(x), rows, cols, a, float(np.float32(scale_override)), int(bool(four_six)),
                       _p(codes), _p(sf), _p(ts))
    return codes, sf, float(ts[0])


def swizzle_hadamard(h: np.ndarray) -> np.ndarray:
    """Row reorder of rht.py:65-82, on any [128, k] array."""
    r = np.empty_like(h)
    reorder = [0, 1, 2, 3, 16, 17, 18, 19, 32, 33, 34, 35, 48, 49, 50, 51]
    for k in range(0, 128, 64):
        for l in range(4):
            for j in range(16):
                r[k + 16 * l + j] = h[k + 4 * l + reorder[j]]
    return r


def rht_matrix_from_slice(h16_bf16: np.ndarray) -> np.ndarray:
    """Effective 128x128 (bf16 bits) matrix the rht128_* kernels apply, given their 16x128 input."""
    h16 = np.ascontiguousarray(h16_bf16, dtype=np.uint16)
    assert h16.shape == (16, 128)
    out = np.empty((128, 128), dtype=np.uint16)
    lib().oq_build_rht_matrix(_p(h16), _p(out))
    return out


def rotate(x_bf16: np.ndarray, H_bf16: np.ndarray, transpose: bool = False) -> np.ndarray:
    """fp32 (x or x^T) rotated in 128-groups along the last dim: y_g = x_g @ H^T."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    H = np.ascontiguousarray(H_bf16, dtype=np.uint16)
    rows, cols = x.shape
    R, C = (cols, rows) if transpose else (rows, cols)
    out = np.empty((R, C), dtype=np.float32)
    lib().oq_rotate(_p(x), rows, cols, _p(H), int(bool(transpose)), _p(out))
    return out


def eden_pass1(v: np.ndarray, scale_override: float):
    """EDEN pass 1 on rotated values. Returns (codes, scratch bf16 [rows, cols/16], max_bits)."""
    v = np.ascontiguousarray(v, dtype=np.float32)
    rows, cols = v.shape
    fp4_max = np.float32(6.0 / scale_override)
    inv = np.float32(1.0) / fp4_max
    codes = np.empty((rows, cols // 2), dtype=np.uint8)
    scratch = np.empty((rows, cols // 16), dtype=np.uint16)
    rowmax = np.empty(rows, dtype=np.float32)
    mb = np.zeros(1, dtype=np.uint32)
    lib().oq_eden_pass1(_p(v), rows, cols, float(inv), _p(codes), _p(scratch), _p(rowmax), _p(mb))
    return codes, scratch, int(mb[0])


def sr_scales(scratch: np.ndarray, max_bits: int, seed: int, fp8_max: float = 256.0):
    scratch = np.ascontiguousarray(scratch, dtype=np.uint16)
    rows, cols16 = scratch.shape
    sf = np.empty(rows * cols16, dtype=np.uint8)
    ts = np.zeros(1, dtype=np.float32)
    inv = np.float32(1.0) / np.float32(fp8_max)
    lib().oq_sr_scales(_p(scratch), rows, cols16, int(max_bits), float(inv), int(seed) & (2**64 - 1), _p(sf), _p(ts))
    return sf, float(ts[0])


def quant_had_eden(x_bf16: np.ndarray, H_bf16: np.ndarray, seed: int, scale_override: float = 1.0,
                   transpose: bool = False, fp8_max: float = 256.0):
    """Rotate by a full 128x128 H (y = x H^T per group) then EDEN-quantize (quant.py:141-213)."""
    v = rotate(x_bf16, H_bf16, transpose)
    codes, scratch, mb = eden_pass1(v, scale_override)
    sf, ts = sr_scales(scratch, mb, seed, fp8_max)
    return codes, sf, ts


def rht128_quant_eden(x_bf16: np.ndarray, h16_bf16: np.ndarray, seed: int, scale_override: float = 1.0,
                      transpose: bool = False, fp8_max: float = 256.0):
    """Randomized-Hadamard rotation from the 16x128 slice, then EDEN (quant.py:320-397)."""
    return quant_had_eden(x_bf16, rht_matrix_from_slice(h16_bf16), seed, scale_override, transpose, fp8_max)


def rht128_requant(codes: np.ndarray, sf_flat: np.ndarray, ts: float, h16_bf16: np.ndarray, seed: int,
                   scale_override: float = 1.0, fp8_max: float = 256.0):
    """Dequantize to bf16, transpose, rotate, EDEN (quant.py:402-491, rht128_requant.cu)."""
    xb = dequant_bf16(codes, sf_flat, ts)
    return quant_had_eden(xb, rht_matrix_from_slice(h16_bf16), seed, scale_override, True, fp8_max)


def hadamard128_bf16() -> np.ndarray:
    """bf16(scipy.linalg.hadamard(128) / sqrt(128)) (linear.py:9-15), Sylvester construction."""
    n = 128
    H = np.ones((1, 1))
    while H.shape[0] < n:
        H = np.block([[H, H], [H, -H]])
    return f32_to_bf16((H * n ** -0.5).astype(np.float32))


def philox(seed: int, ctr: int) -> np.ndarray:
    out = np.zeros(4, dtype=np.uint32)
    lib().oq_philox(int(seed) & (2**64 - 1), int(ctr) & 0xFFFFFFFF, _p(out))
    return out


# ------------------------------------------------- whole linear, fwd + bwd

BWD_SCALE_OVERRIDE = (17 / 16) * 0.93


def linear_fwd_bwd(x_bf16: np.ndarray, w_bf16: np.ndarray, dy_bf16: np.ndarray, h16_bf16: np.ndarray,
                   seeds=(1, 2, 3, 4), four_six: bool = True):
    """CPU restatement of Quartet_II_fn forward + backward (reference
    quartet2/python/quartet2/linear.py:155-233) for x [M, K], w [N, K],
    dy [M, N], a given (already sign-randomized) 16x128 Hadamard slice and
    the four stochastic-rounding seeds (E, E^T, W^T, X^T).

    Returns (y, dx, dw) as fp32 arrays; the GEMMs are fp32 products of the
    dequantized NVFP4 operands, rounded to bf16 like the GPU epilogue."""
    so = BWD_SCALE_OVERRIDE
    xq = quant_fp4(x_bf16, four_six=four_six)
    wq = quant_fp4(w_bf16, four_six=four_six)
    y = dequant(*xq) @ dequant(*wq).T
    H = rht_matrix_from_slice(h16_bf16)
    e = quant_had_eden(dy_bf16, H, seeds[0], so, transpose=False)
    et = quant_had_eden(dy_bf16, H, seeds[1], so, transpose=True)
    wt = rht128_requant(wq[0], wq[1], wq[2], h16_bf16, seeds[2], so)
    xt = rht128_requant(xq[0], xq[1], xq[2], h16_bf16, seeds[3], so)
    dx = dequant(*e) @ dequant(*wt).T
    dw = dequant(*et) @ dequant(*xt).T
    rb = lambda a: bf16_to_f32(f32_to_bf16(a.astype(np.float32)))
    return rb(y), rb(dx), rb(dw)
