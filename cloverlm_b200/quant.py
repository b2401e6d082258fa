"""NVFP4 quantizers -- drop-in for ``quartet2.quant`` (reference file
quartet2/python/quartet2/quant.py; paths are relative to the reference
project root).

Same names, keyword arguments, output shapes, dtypes, layouts and assertion
behaviour as the reference, backed by libq2b (sm_100a CUDA through the C ABI
of include/q2b.h).  The torch custom ops keep the reference's op names
(``quartet2::four_six``, ``quartet2::rtn``, ``quartet2::eden``,
``quartet2::rht128_eden``, ``quartet2::group_transform_eden``,
``quartet2::had128_requant``, ``quartet2::dequant_tp_had_quant``) so
``torch.compile(fullgraph=True)`` traces them the same way.

Differences from the reference, all deliberate:
  * kernels run on the current torch stream (the reference uses the legacy
    default stream);
  * stochastic-rounding noise is keyed by the index of the scale (the
    reference reuses noise across rows that share a thread/block index);
  * ``NVFP4QuantMode.EDEN`` in ``quant_fp4`` runs the EDEN estimator per
    16-element group with an identity rotation (``quant_had_eden`` with
    H = I) -- the reference's test-only ``eden_fp4`` kernel
    (quartet2/csrc/round_eden_fp4.cu) is not reproduced bit for bit.
"""
from __future__ import annotations

from collections import namedtuple
from enum import Enum

import torch

from . import _lib

_FP8_MAX = 256.0


def _seed_value(seed) -> int:
    if isinstance(seed, torch.Tensor):
        return int(seed.item()) & (2**64 - 1)
    return int(seed) & (2**64 - 1)


# --------------------------------------------------------------- custom ops

@torch.library.custom_op("quartet2::four_six", mutates_args=("o", "s", "t"))
def _four_six_fp4_op(o: torch.Tensor, s: torch.Tensor, t: torch.Tensor, x: torch.Tensor, amax: torch.Tensor,
                     scale_override: float) -> None:
    with torch.cuda.device(x.device):
        _lib.call("q2b_quant_fwd", _lib.ptr(o), _lib.ptr(s), _lib.ptr(t), _lib.ptr(x), _lib.ptr(amax),
                  float(scale_override), x.shape[0], x.shape[1], _lib.MODE_FOUR_SIX, _lib.stream_of(x))


@torch.library.custom_op("quartet2::rtn", mutates_args=("o", "s", "t"))
def _rtn_fp4_op(o: torch.Tensor, s: torch.Tensor, t: torch.Tensor, x: torch.Tensor, amax: torch.Tensor,
                scale_override: float) -> None:
    with torch.cuda.device(x.device):
        _lib.call("q2b_quant_fwd", _lib.ptr(o), _lib.ptr(s), _lib.ptr(t), _lib.ptr(x), _lib.ptr(amax),
                  float(scale_override), x.shape[0], x.shape[1], _lib.MODE_RNE, _lib.stream_of(x))


def _rht_eden_call(o, s, t, scratch_scales, scratch_max, h, x, seed, fp4_max, fp8_max, transpose):
    rows, cols = x.shape
    with torch.cuda.device(x.device):
        _lib.call("q2b_rht_eden", _lib.ptr(o), _lib.ptr(s), _lib.ptr(t), _lib.ptr(scratch_scales),
                  _lib.ptr(scratch_max), _lib.ptr(h), h.shape[0], _lib.ptr(x), _seed_value(seed),
                  float(fp4_max), float(fp8_max), rows, cols, int(bool(transpose)), _lib.stream_of(x))


@torch.library.custom_op("quartet2::eden", mutates_args=("o", "s", "t"))
def _eden_fp4_op(o: torch.Tensor, s: torch.Tensor, t: torch.Tensor, x: torch.Tensor, amax: torch.Tensor,
                 scale_override: float, seed: torch.Tensor) -> None:
    eye = torch.eye(128, dtype=torch.bfloat16, device=x.device)
    scratch = torch.empty(x.numel() // 16, dtype=torch.bfloat16, device=x.device)
    smax = torch.empty((), dtype=torch.uint32, device=x.device)
    _rht_eden_call(o, s, t, scratch, smax, eye, x, seed, 6.0 / scale_override, _FP8_MAX, False)


@torch.library.custom_op("quartet2::group_transform_eden",
                         mutates_args=("o", "s", "t", "scratch_scales", "scratch_max"))
def _group_transform_128_eden(o: torch.Tensor, s: torch.Tensor, t: torch.Tensor, scratch_scales: torch.Tensor,
                              scratch_max: torch.Tensor, h: torch.Tensor, x: torch.Tensor, seed: torch.Tensor,
                              fp4_max: float, fp8_max: float, transpose: bool) -> None:
    _rht_eden_call(o, s, t, scratch_scales, scratch_max, h, x, seed, fp4_max, fp8_max, transpose)


@torch.library.custom_op("quartet2::rht128_eden", mutates_args=("o", "s", "t", "scratch_scales", "scratch_max"))
def _transform_rht128_eden(o: torch.Tensor, s: torch.Tensor, t: torch.Tensor, scratch_scales: torch.Tensor,
                           scratch_max: torch.Tensor, h: torch.Tensor, x: torch.Tensor, seed: torch.Tensor,
                           fp4_max: float, fp8_max: float, transpose: bool) -> None:
    _rht_eden_call(o, s, t, scratch_scales, scratch_max, h, x, seed, fp4_max, fp8_max, transpose)


@torch.library.custom_op("quartet2::rht128_eden_dual",
                         mutates_args=("o", "s", "t", "scratch_scales", "scratch_max",
                                       "ot", "st", "tt", "scratch_scales_t", "scratch_max_t"))
def _transform_rht128_eden_dual(o: torch.Tensor, s: torch.Tensor, t: torch.Tensor, scratch_scales: torch.Tensor,
                                scratch_max: torch.Tensor, ot: torch.Tensor, st: torch.Tensor, tt: torch.Tensor,
                                scratch_scales_t: torch.Tensor, scratch_max_t: torch.Tensor, h: torch.Tensor,
                                x: torch.Tensor, seed: torch.Tensor, seed_t: torch.Tensor, fp4_max: float,
                                fp8_max: float) -> None:
    rows, cols = x.shape
    with torch.cuda.device(x.device):
        _lib.call("q2b_rht_eden_dual", _lib.ptr(o), _lib.ptr(s), _lib.ptr(t), _lib.ptr(scratch_scales),
                  _lib.ptr(scratch_max), _lib.ptr(ot), _lib.ptr(st), _lib.ptr(tt), _lib.ptr(scratch_scales_t),
                  _lib.ptr(scratch_max_t), _lib.ptr(h), h.shape[0], _lib.ptr(x), _seed_value(seed),
                  _seed_value(seed_t), float(fp4_max), float(fp8_max), rows, cols, _lib.stream_of(x))


def _requant_call(o, s, t, scratch_scales, scratch_max, h, x, x_group_scales, x_tensor_scale, seed, fp4_max,
                  fp8_max):
    rows, half = x.shape
    with torch.cuda.device(x.device):
        _lib.call("q2b_rht_requant", _lib.ptr(o), _lib.ptr(s), _lib.ptr(t), _lib.ptr(scratch_scales),
                  _lib.ptr(scratch_max), _lib.ptr(h), h.shape[0], _lib.ptr(x), _lib.ptr(x_group_scales),
                  _lib.ptr(x_tensor_scale), _seed_value(seed), float(fp4_max), float(fp8_max), rows, half * 2,
                  _lib.stream_of(x))


@torch.library.custom_op("quartet2::had128_requant", mutates_args=("o", "s", "t", "scratch_scales", "scratch_max"))
def _rht128_requant(o: torch.Tensor, s: torch.Tensor, t: torch.Tensor, scratch_scales: torch.Tensor,
                    scratch_max: torch.Tensor, h: torch.Tensor, x: torch.Tensor, x_group_scales: torch.Tensor,
                    x_tensor_scale: torch.Tensor, seed: torch.Tensor, fp4_max: float, fp8_max: float) -> None:
    _requant_call(o, s, t, scratch_scales, scratch_max, h, x, x_group_scales, x_tensor_scale, seed, fp4_max, fp8_max)


@torch.library.custom_op("quartet2::dequant_tp_had_quant",
                         mutates_args=("o", "s", "t", "scratch_scales", "scratch_max"))
def _dequant_tp_had_quant(o: torch.Tensor, s: torch.Tensor, t: torch.Tensor, scratch_scales: torch.Tensor,
                          scratch_max: torch.Tensor, h: torch.Tensor, x: torch.Tensor, x_group_scales: torch.Tensor,
                          x_tensor_scale: torch.Tensor, seed: torch.Tensor, fp4_max: float, fp8_max: float) -> None:
    _requant_call(o, s, t, scratch_scales, scratch_max, h, x, x_group_scales, x_tensor_scale, seed, fp4_max, fp8_max)


NVFP4Quant = namedtuple("NVFP4Quant", ["fp4", "micro_scales", "tensor_scale"])


class NVFP4QuantMode(Enum):
    RNE = 0
    FOUR_SIX = 1
    EDEN = 2


def quant_fp4(x, *, scale_override: float, amax: torch.Tensor = None, mode=NVFP4QuantMode.RNE,
              seed: torch.Tensor = None) -> NVFP4Quant:
    """Forward NVFP4 quantization (reference quant.py:114-138)."""
    q = torch.empty((x.shape[0], x.shape[1] // 2), device=x.device, dtype=torch.uint8)
    s = torch.empty((x.shape[0], x.shape[1] // 16), device=x.device, dtype=torch.float8_e4m3fn)
    assert x.dtype == torch.bfloat16
    assert x.is_cuda
    assert x.is_contiguous()
    assert x.shape[0] % 128 == 0
    assert x.shape[1] % 128 == 0

    if amax is None:
        amax = abs_max(x)
    else:
        assert amax.dtype == torch.float32
    global_scale = torch.empty((), device=x.device, dtype=torch.float32)
    if mode == NVFP4QuantMode.FOUR_SIX:
        _four_six_fp4_op(q, s.view(torch.uint8), global_scale, x.detach(), amax, scale_override)
    elif mode == NVFP4QuantMode.RNE:
        _rtn_fp4_op(q, s.view(torch.uint8), global_scale, x.detach(), amax, scale_override)
    elif mode == NVFP4QuantMode.EDEN:
        assert seed is not None
        _eden_fp4_op(q, s.view(torch.uint8), global_scale, x.detach(), amax, scale_override, seed)
    else:
        raise ValueError(f"Unknown NVFP4QuantMode: {mode}")
    return NVFP4Quant(q, s, global_scale)


@torch.library.custom_op("quartet2::abs_max", mutates_args=())
def abs_max(x: torch.Tensor) -> torch.Tensor:
    """max |x| as an fp32 0-d tensor (replaces the reference's torch.compile reduction, linear.py:146-148)."""
    assert x.dtype == torch.bfloat16 and x.is_cuda
    x = x.contiguous()
    out = torch.empty((), device=x.device, dtype=torch.float32)
    with torch.cuda.device(x.device):
        _lib.call("q2b_abs_max", _lib.ptr(out), _lib.ptr(x), x.numel(), _lib.stream_of(x))
    return out


@abs_max.register_fake
def _abs_max_fake(x: torch.Tensor) -> torch.Tensor:
    return torch.empty((), device=x.device, dtype=torch.float32)


def _alloc_outputs(x, rows, cols, out, group_scales, tensor_scale, scratch_scales, scratch_amax):
    if out is None:
        out = torch.empty((rows, cols // 2), dtype=torch.uint8, device=x.device)
    else:
        out = out.reshape(-1, out.shape[-1])
    if group_scales is None:
        group_scales = torch.empty((rows, cols // 16), device=x.device, dtype=torch.float8_e4m3fn)
    else:
        group_scales = group_scales.reshape(-1, group_scales.shape[-1])
    if tensor_scale is None:
        tensor_scale = torch.empty((), device=x.device, dtype=torch.float32)
    if scratch_scales is None:
        scratch_scales = torch.empty((rows * cols // 16), device=x.device, dtype=torch.bfloat16)
    if scratch_amax is None:
        scratch_amax = torch.empty((), device=x.device, dtype=torch.uint32)
    return out, group_scales, tensor_scale, scratch_scales, scratch_amax


def _default_seed(seed):
    if seed is None:
        seed = torch.randint(0, 2**32, (), dtype=torch.int64)
    return seed


def quant_had_eden(*, out: torch.Tensor = None, group_scales: torch.Tensor = None, tensor_scale: torch.Tensor = None,
                   scratch_scales: torch.Tensor = None, scratch_amax: torch.Tensor = None, h: torch.Tensor,
                   x: torch.Tensor, seed: torch.Tensor = None, scale_override: float = 1.0, transpose: bool = False):
    """Rotate x (or x^T) by an explicit 128x128 `h` as x h^T per 128-group, then EDEN (reference quant.py:141-213)."""
    seed = _default_seed(seed)
    assert x.dim() == 2
    rows, cols = x.shape
    if transpose:
        rows, cols = cols, rows
    assert x.dtype == torch.bfloat16
    assert x.is_cuda
    assert x.is_contiguous()
    assert h.dtype == torch.bfloat16
    assert h.is_cuda
    assert h.is_contiguous()
    assert h.shape == (128, 128)
    out, group_scales, tensor_scale, scratch_scales, scratch_amax = _alloc_outputs(
        x, rows, cols, out, group_scales, tensor_scale, scratch_scales, scratch_amax)
    _group_transform_128_eden(out, group_scales.view(torch.uint8), tensor_scale, scratch_scales, scratch_amax, h, x,
                              seed, fp4_max=6.0 / scale_override, fp8_max=_FP8_MAX, transpose=transpose)
    group_scales = group_scales.reshape(rows, cols // 16)
    return NVFP4Quant(out, group_scales, tensor_scale)


def rht128_quant_eden(*, out: torch.Tensor = None, group_scales: torch.Tensor = None,
                      tensor_scale: torch.Tensor = None, scratch_scales: torch.Tensor = None,
                      scratch_amax: torch.Tensor = None, h: torch.Tensor, x: torch.Tensor, seed: torch.Tensor = None,
                      scale_override: float = 1.0, transpose: bool = False):
    """Randomized-Hadamard rotation from the top 16x128 slice `h`, then EDEN (reference quant.py:320-397)."""
    seed = _default_seed(seed)
    assert x.dim() == 2
    rows, cols = x.shape
    if transpose:
        rows, cols = cols, rows
    assert x.dtype == torch.bfloat16
    assert x.is_cuda
    assert x.is_contiguous()
    assert h.dtype == torch.bfloat16
    assert h.is_cuda
    assert h.is_contiguous()
    out, group_scales, tensor_scale, scratch_scales, scratch_amax = _alloc_outputs(
        x, rows, cols, out, group_scales, tensor_scale, scratch_scales, scratch_amax)
    _transform_rht128_eden(out, group_scales.view(torch.uint8), tensor_scale, scratch_scales, scratch_amax, h, x,
                           seed, fp4_max=6.0 / scale_override, fp8_max=_FP8_MAX, transpose=transpose)
    group_scales = group_scales.reshape(rows, cols // 16)
    return NVFP4Quant(out, group_scales, tensor_scale)


def rht128_quant_eden_dual(*, h: torch.Tensor, x: torch.Tensor, seed: torch.Tensor = None,
                           seed_t: torch.Tensor = None, scale_override: float = 1.0,
                           scratch_amax: torch.Tensor = None, scratch_amax_t: torch.Tensor = None,
                           scratch_scales: torch.Tensor = None, scratch_scales_t: torch.Tensor = None):
    """Both ``rht128_quant_eden(transpose=False)`` and ``(transpose=True)`` from ONE read of x.

    Returns (NVFP4Quant of x, NVFP4Quant of x^T).  No reference counterpart: it
    fuses the two calls Quartet_II_fn.backward makes on the output gradient
    (reference linear.py:222,229)."""
    seed = _default_seed(seed)
    seed_t = _default_seed(seed_t)
    assert x.dim() == 2 and x.dtype == torch.bfloat16 and x.is_cuda and x.is_contiguous()
    assert h.dtype == torch.bfloat16 and h.is_cuda and h.is_contiguous()
    M, N = x.shape
    dev = x.device
    o = torch.empty((M, N // 2), dtype=torch.uint8, device=dev)
    s = torch.empty((M, N // 16), dtype=torch.float8_e4m3fn, device=dev)
    t = torch.empty((), dtype=torch.float32, device=dev)
    ot = torch.empty((N, M // 2), dtype=torch.uint8, device=dev)
    st = torch.empty((N, M // 16), dtype=torch.float8_e4m3fn, device=dev)
    tt = torch.empty((), dtype=torch.float32, device=dev)
    sc = torch.empty((M * N // 16,), dtype=torch.bfloat16, device=dev) if scratch_scales is None else scratch_scales
    sct = torch.empty((M * N // 16,), dtype=torch.bfloat16, device=dev) if scratch_scales_t is None \
        else scratch_scales_t
    if scratch_amax is None:
        scratch_amax = torch.empty((), dtype=torch.uint32, device=dev)
    if scratch_amax_t is None:
        scratch_amax_t = torch.empty((), dtype=torch.uint32, device=dev)
    _transform_rht128_eden_dual(o, s.view(torch.uint8), t, sc, scratch_amax, ot, st.view(torch.uint8), tt, sct,
                                scratch_amax_t, h, x, seed, seed_t, fp4_max=6.0 / scale_override, fp8_max=_FP8_MAX)
    return NVFP4Quant(o, s, t), NVFP4Quant(ot, st, tt)


def _requant(fn, *, out, group_scales, tensor_scale, scratch_scales, scratch_amax, h, x, x_group_scales,
             x_tensor_scale, seed, scale_override):
    seed = _default_seed(seed)
    assert x.dim() == 2
    rows, cols = x.shape
    rows, cols = 2 * cols, rows  # transpose and take into account 2 vals per element
    assert x.dtype == torch.uint8
    assert x.is_cuda
    assert x.is_contiguous()
    assert x_group_scales.dtype == torch.float8_e4m3fn
    assert x_group_scales.shape[0] == x.shape[0]
    assert x_group_scales.shape[1] == x.shape[1] // 8
    assert x_group_scales.is_cuda
    assert x_group_scales.is_contiguous()
    assert x_tensor_scale.dim() == 0
    assert x_tensor_scale.dtype == torch.float32
    assert h.dtype == torch.bfloat16
    assert h.is_cuda
    assert h.is_contiguous()
    out, group_scales, tensor_scale, scratch_scales, scratch_amax = _alloc_outputs(
        x, rows, cols, out, group_scales, tensor_scale, scratch_scales, scratch_amax)
    fn(out, group_scales.view(torch.uint8), tensor_scale, scratch_scales, scratch_amax, h, x,
       x_group_scales.view(torch.uint8), x_tensor_scale, seed, fp4_max=6.0 / scale_override, fp8_max=_FP8_MAX)
    group_scales = group_scales.reshape(rows, cols // 16)
    return NVFP4Quant(out, group_scales, tensor_scale)


def rht128_requant(*, out: torch.Tensor = None, group_scales: torch.Tensor = None, tensor_scale: torch.Tensor = None,
                   scratch_scales: torch.Tensor = None, scratch_amax: torch.Tensor = None, h: torch.Tensor,
                   x: torch.Tensor, x_group_scales: torch.Tensor, x_tensor_scale: torch.Tensor,
                   seed: torch.Tensor = None, scale_override: float = 1.0):
    """Requantize an NVFP4 tensor as x^T h^T with EDEN (reference quant.py:402-491)."""
    return _requant(_rht128_requant, out=out, group_scales=group_scales, tensor_scale=tensor_scale,
                    scratch_scales=scratch_scales, scratch_amax=scratch_amax, h=h, x=x,
                    x_group_scales=x_group_scales, x_tensor_scale=x_tensor_scale, seed=seed,
                    scale_override=scale_override)


# Output position p of each 16-group holds element _DQ_TP_ORDER[p] (reference quant.py:240-243).
_DQ_TP_ORDER = [0, 1, 8, 9, 2, 3, 10, 11, 4, 5, 12, 13, 6, 7, 14, 15]


def dequant_tp_had_eden(*, out: torch.Tensor = None, group_scales: torch.Tensor = None,
                        tensor_scale: torch.Tensor = None, scratch_scales: torch.Tensor = None,
                        scratch_amax: torch.Tensor = None, h: torch.Tensor, x: torch.Tensor,
                        x_group_scales: torch.Tensor, x_tensor_scale: torch.Tensor, seed: int = None,
                        scale_override: float = 1.0):
    """Requantize with an explicit 128x128 `h`; within each group of 16 the output
    elements come in the order [0, 1, 8, 9, 2, 3, 10, 11, ...] (reference quant.py:216-317)."""
    assert h.shape == (128, 128)
    perm = torch.tensor([16 * (p // 16) + _DQ_TP_ORDER[p % 16] for p in range(128)], device=h.device)
    hp = h[perm].contiguous()
    return _requant(_dequant_tp_had_quant, out=out, group_scales=group_scales, tensor_scale=tensor_scale,
                    scratch_scales=scratch_scales, scratch_amax=scratch_amax, h=hp, x=x,
                    x_group_scales=x_group_scales, x_tensor_scale=x_tensor_scale, seed=seed,
                    scale_override=scale_override)
