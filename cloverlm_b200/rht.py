"""Rotation helpers -- drop-in for ``quartet2.rht`` (reference file
quartet2/python/quartet2/rht.py).

``transform_128`` / ``transform_rht128`` return the rotated bf16 tensor
without quantizing it.  In the reference they are test-support kernels; here
they are plain GEMMs of each 128-group with the (effective) rotation matrix,
run by torch on the GPU, because nothing on the training path needs them.
The quantizing rotations (``quant.rht128_quant_eden`` and friends) run in
libq2b's tcgen05 kernel.
"""
from __future__ import annotations

import torch

_REORDER = [0, 1, 2, 3, 16, 17, 18, 19, 32, 33, 34, 35, 48, 49, 50, 51]


def swizzle_hadamard(hadamard_matrix):
    """Row reorder under which transform_128(x, swizzle_hadamard(h)) == transform_rht128(x, h[:16]) (rht.py:65-82)."""
    r = torch.empty_like(hadamard_matrix)
    for k in range(0, 128, 64):
        for l in range(4):
            for j in range(16):
                r[k + 16 * l + j, :] = hadamard_matrix[k + 4 * l + _REORDER[j], :]
    return r


def rht_matrix_from_slice(h16: torch.Tensor) -> torch.Tensor:
    """The 128x128 matrix the rht128 kernels apply, given its top 16x128 slice:
    F[R, c] = h16[R % 16, c] * H8[R // 16, c // 16] (Sylvester), rows swizzled."""
    assert h16.shape == (16, 128)
    R = torch.arange(128, device=h16.device)
    c = torch.arange(128, device=h16.device)
    par = torch.zeros(128, 128, dtype=torch.int64, device=h16.device)
    v = (R[:, None] // 16) & (c[None, :] // 16)
    while bool(v.any()):
        par ^= v & 1
        v = v >> 1
    sign = (1 - 2 * par).to(h16.dtype)
    F = h16[R % 16] * sign
    return swizzle_hadamard(F)


def _rotate(x, h, transpose):
    if transpose:
        x = x.T
    r = x.reshape(-1, 128) @ h.T
    return r.reshape(x.shape).contiguous()


def transform_128(*, out: torch.Tensor = None, h: torch.Tensor, x: torch.Tensor, transpose: bool = False):
    assert h.dim() == 2 and h.shape == (128, 128)
    assert x.dtype == torch.bfloat16
    assert x.is_cuda and x.is_contiguous() and h.is_cuda and h.is_contiguous()
    original_shape = x.shape
    if transpose:
        assert len(original_shape) == 2
    r = _rotate(x.reshape(-1, x.shape[-1]), h, transpose)
    if out is not None:
        out.copy_(r.reshape(out.shape))
        return out
    return r if transpose else r.reshape(original_shape)


def transform_rht128(*, out: torch.Tensor = None, h: torch.Tensor, x: torch.Tensor, transpose: bool = False):
    assert h.dim() == 2 and h.shape == (16, 128)
    return transform_128(out=out, h=rht_matrix_from_slice(h), x=x, transpose=transpose)
