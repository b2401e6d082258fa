"""Quartet-II NVFP4 linear layer -- drop-in for ``quartet2.linear`` (reference
file quartet2/python/quartet2/linear.py; paths are relative to the reference
project root).

Forward (reference linear.py:155-196): abs-max of input and weight, four-over-
six (or RNE) NVFP4 quantization of both, NVFP4 GEMM; the NVFP4 operands are
saved for backward.  Backward (linear.py:200-233): a freshly sign-randomized
128-point Hadamard rotation, EDEN quantization of the output gradient E and
of E^T (here from ONE read of E by the dual-orientation kernel), EDEN
requantization of the saved W^T and X^T, and two NVFP4 GEMMs for dX and dW.

Every kernel is libq2b's (sm_100a CUDA through the C ABI of include/q2b.h);
the GEMM replaces the reference's flashinfer.mm_fp4(backend="cudnn").
"""
from __future__ import annotations

import torch

from . import _lib
from .quant import (NVFP4QuantMode, abs_max, quant_fp4, rht128_quant_eden, rht128_quant_eden_dual,
                    rht128_requant)

__all__ = [
    "Quartet_II_linear", "Quartet_II_fn", "_fp4_mm", "_dq_fp4", "abs_max", "to_blocked", "unblock",
    "get_hadamard_matrix", "rerotate_hadamard", "register_optimizer_hook",
]


def get_hadamard_matrix(group_size: int, dtype: torch.dtype, device: torch.device):
    """Sylvester Hadamard matrix scaled by 1/sqrt(n), as the reference builds it
    from scipy.linalg.hadamard (linear.py:9-15); entries are then rounded to `dtype`."""
    H = torch.ones(1, 1, dtype=torch.float64)
    while H.shape[0] < group_size:
        H = torch.cat([torch.cat([H, H], 1), torch.cat([H, -H], 1)], 0)
    if H.shape[0] != group_size:
        raise ValueError("group_size must be a power of two")
    return (H * group_size ** -0.5).to(dtype=dtype, device=device).requires_grad_(False)


def rerotate_hadamard(hadamard_matrix):
    """Random +-1 sign per column (the inner dimension of the TN GEMMs), linear.py:25-31."""
    signs = torch.randint(0, 2, (hadamard_matrix.size(0),), device=hadamard_matrix.device,
                          dtype=hadamard_matrix.dtype) * 2 - 1
    return hadamard_matrix * signs[None, :]


@torch.library.custom_op("quartet2::fp4_mm", mutates_args=())
def _fp4_mm(x_fp4: torch.Tensor, w_fp4: torch.Tensor, x_mx: torch.Tensor, w_mx: torch.Tensor,
            alpha: torch.Tensor) -> torch.Tensor:
    """out[m, n] = alpha * dq(x)[m, :] . dq(w)[n, :] in bf16 (reference linear.py:34-56)."""
    m, packed_k = x_fp4.shape
    k = packed_k * 2
    n = w_fp4.shape[0]
    out = torch.empty([m, n], device=x_fp4.device, dtype=torch.bfloat16)
    if alpha.dtype != torch.float32:
        alpha = alpha.float()
    with torch.cuda.device(x_fp4.device):
        _lib.call("q2b_gemm_nvfp4", _lib.ptr(out), _lib.ptr(x_fp4), _lib.ptr(w_fp4), _lib.ptr(x_mx),
                  _lib.ptr(w_mx), _lib.ptr(alpha), m, n, k, _lib.stream_of(x_fp4))
    return out


@_fp4_mm.register_fake
def _fp4_mm_fake(x_fp4, w_fp4, x_mx, w_mx, alpha):
    return torch.empty((x_fp4.shape[0], w_fp4.shape[0]), device=x_fp4.device, dtype=torch.bfloat16)


@torch.library.custom_op("quartet2::fp4_mm_f32", mutates_args=())
def _fp4_mm_f32(x_fp4: torch.Tensor, w_fp4: torch.Tensor, x_mx: torch.Tensor, w_mx: torch.Tensor,
                alpha: torch.Tensor) -> torch.Tensor:
    """_fp4_mm with an fp32 output (the accumulator times alpha, unrounded): the weight
    gradient of an fp32 master weight, produced in the parameter's dtype (q2b_gemm_nvfp4_f32)."""
    m, packed_k = x_fp4.shape
    n = w_fp4.shape[0]
    out = torch.empty([m, n], device=x_fp4.device, dtype=torch.float32)
    if alpha.dtype != torch.float32:
        alpha = alpha.float()
    with torch.cuda.device(x_fp4.device):
        _lib.call("q2b_gemm_nvfp4_f32", _lib.ptr(out), _lib.ptr(x_fp4), _lib.ptr(w_fp4), _lib.ptr(x_mx),
                  _lib.ptr(w_mx), _lib.ptr(alpha), m, n, packed_k * 2, _lib.stream_of(x_fp4))
    return out


@_fp4_mm_f32.register_fake
def _fp4_mm_f32_fake(x_fp4, w_fp4, x_mx, w_mx, alpha):
    return torch.empty((x_fp4.shape[0], w_fp4.shape[0]), device=x_fp4.device, dtype=torch.float32)


def _fp4_mm_add(out, x_fp4, w_fp4, x_mx, w_mx, alpha):
    """out += _fp4_mm(...) in place (bf16 adds; q2b_gemm_nvfp4_add); returns out."""
    m, packed_k = x_fp4.shape
    n = w_fp4.shape[0]
    assert out.dtype == torch.bfloat16 and out.is_contiguous() and out.shape == (m, n)
    alpha = alpha.float()
    with torch.cuda.device(x_fp4.device):
        _lib.call("q2b_gemm_nvfp4_add", _lib.ptr(out), _lib.ptr(x_fp4), _lib.ptr(w_fp4), _lib.ptr(x_mx),
                  _lib.ptr(w_mx), _lib.ptr(alpha), m, n, packed_k * 2, _lib.stream_of(x_fp4))
    return out


def _fp4_mm_relu2(x_fp4, w_fp4, x_mx, w_mx, alpha):
    """(a, relu(a)^2, max relu(a)^2) for a = _fp4_mm(...) in one GEMM (q2b_gemm_nvfp4_relu2)."""
    m, packed_k = x_fp4.shape
    n = w_fp4.shape[0]
    a = torch.empty([m, n], device=x_fp4.device, dtype=torch.bfloat16)
    h = torch.empty_like(a)
    amax = torch.empty((), device=x_fp4.device, dtype=torch.float32)
    alpha = alpha.float()
    with torch.cuda.device(x_fp4.device):
        _lib.call("q2b_gemm_nvfp4_relu2", _lib.ptr(a), _lib.ptr(h), _lib.ptr(amax), _lib.ptr(x_fp4), _lib.ptr(w_fp4),
                  _lib.ptr(x_mx), _lib.ptr(w_mx), _lib.ptr(alpha), m, n, packed_k * 2, _lib.stream_of(x_fp4))
    return a, h, amax


def _fp4_mm_relu2_bwd(x_fp4, w_fp4, x_mx, w_mx, alpha, a):
    """2 * relu(a) * _fp4_mm(...) in one GEMM (q2b_gemm_nvfp4_relu2_bwd); a bf16 [m, n]."""
    m, packed_k = x_fp4.shape
    n = w_fp4.shape[0]
    a = a.reshape(m, n).contiguous()
    out = torch.empty([m, n], device=x_fp4.device, dtype=torch.bfloat16)
    alpha = alpha.float()
    with torch.cuda.device(x_fp4.device):
        _lib.call("q2b_gemm_nvfp4_relu2_bwd", _lib.ptr(out), _lib.ptr(a), _lib.ptr(x_fp4), _lib.ptr(w_fp4),
                  _lib.ptr(x_mx), _lib.ptr(w_mx), _lib.ptr(alpha), m, n, packed_k * 2, _lib.stream_of(x_fp4))
    return out


def to_blocked(input_matrix) -> torch.Tensor:
    """[H, W] scale matrix -> flat blocked 128x4 layout (linear.py:64-94)."""
    rows, cols = input_matrix.shape
    n_row_blocks = (rows + 127) // 128
    n_col_blocks = (cols + 3) // 4
    assert (rows, cols) == (n_row_blocks * 128, n_col_blocks * 4)
    blocks = input_matrix.view(n_row_blocks, 128, n_col_blocks, 4).permute(0, 2, 1, 3)
    rearranged = blocks.reshape(-1, 4, 32, 4).transpose(1, 2).reshape(-1, 32, 16)
    return rearranged.flatten()


def unblock(blocked_scales, rows, cols):
    """Inverse of to_blocked for a [rows, cols/16] scale matrix (linear.py:97-103)."""
    n_row_blocks, n_col_blocks = rows // 128, (cols // 16) // 4
    rearranged = blocked_scales.reshape(-1, 32, 4, 4)
    rearranged = rearranged.permute(0, 2, 1, 3).reshape(-1, n_col_blocks, 128, 4)
    rearranged = rearranged.permute(0, 2, 1, 3)
    return rearranged.reshape(n_row_blocks * 128, n_col_blocks * 4)


_E2M1 = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]


def _dq_fp4(x_e2m1: torch.Tensor, x_e4m3: torch.Tensor, alpha):
    """Dequantize NVFP4 codes + blocked scales * alpha to bf16 (linear.py:106-144)."""
    codes = x_e2m1.view(torch.uint8).to(torch.int32)
    unpacked = torch.stack([codes & 0xF, (codes >> 4) & 0xF], dim=-1).flatten(start_dim=-2)
    grid = torch.tensor(_E2M1, dtype=torch.float32, device=x_e2m1.device)
    vals = grid[unpacked]
    scales = unblock(x_e4m3.to(torch.float32), x_e2m1.shape[0], x_e2m1.shape[1] * 2)
    out = (vals.unflatten(dim=-1, sizes=(-1, 16)) * scales[..., None]).flatten(start_dim=-2) * alpha
    return out.to(torch.bfloat16)


def _quantize_weight(weight, weight_amax, mode, cache):
    """bf16 (under autocast), abs-max and NVFP4 quantization of a layer weight.

    `cache` (a dict owned by the layer, or None) keeps the result while the weight is
    unchanged: it is keyed by the weight's storage pointer, its autograd version counter
    (bumped by every in-place update, including QuartetAdamW's) and the identity of the
    abs-max tensor the optimizer hands over each step.  The reference quantizes the weight
    in every forward; the result is identical, so a step with several micro-batches
    quantizes each weight once."""
    key = None
    if cache is not None and not torch.compiler.is_compiling():
        key = (weight.data_ptr(), weight._version, id(weight_amax) if weight_amax is not None else None)
        hit = cache.get("q")
        if hit is not None and cache.get("key") == key:
            return hit
    w = weight
    if torch.is_autocast_enabled("cuda"):
        w = w.to(torch.bfloat16)
    w = w.contiguous()
    if weight_amax is None:
        weight_amax = abs_max(w)
    q = quant_fp4(w, amax=weight_amax, scale_override=1.0, mode=mode)
    if key is not None:
        cache["q"], cache["key"] = q, key
    return q


class Quartet_II_fn(torch.autograd.Function):
    group_size = 16

    @staticmethod
    def forward(ctx, input, weight, had, mode: NVFP4QuantMode, disable_backward_quant: bool = False,
                weight_amax: torch.Tensor = None, input_amax: torch.Tensor = None,
                scratch_amax: torch.Tensor = None, weight_cache: dict = None):
        ctx.batch = input.shape[0]
        ctx.seq = input.shape[1]
        ctx.in_dim = weight.shape[1]
        ctx.out_dim = weight.shape[0]
        ctx.disable_backward_quant = disable_backward_quant
        ctx.scratch_amax = scratch_amax
        ctx.had = had
        ctx.w_dtype = weight.dtype

        weight_in = weight
        if torch.is_autocast_enabled("cuda"):
            input = input.to(torch.bfloat16)
        elif weight.dtype != torch.bfloat16:
            raise TypeError("Weight must be bfloat16. Either set `dtype=torch.bfloat16` or enable autocast`")
        elif input.dtype != torch.bfloat16:
            raise TypeError("Input must be bfloat16. Either cast input to bfloat16 or enable autocast`")

        forward_scale_override = 1.0
        flat_input = input.reshape(-1, input.shape[-1]).contiguous()
        if input_amax is None:
            input_amax = abs_max(flat_input)
        input_fp4 = quant_fp4(flat_input, amax=input_amax, scale_override=forward_scale_override, mode=mode)
        weight_fp4 = _quantize_weight(weight_in, weight_amax, mode, weight_cache)
        ctx.save_for_backward(input_fp4.fp4, input_fp4.micro_scales, input_fp4.tensor_scale,
                              weight_fp4.fp4, weight_fp4.micro_scales, weight_fp4.tensor_scale)
        res = _fp4_mm(input_fp4.fp4, weight_fp4.fp4, input_fp4.micro_scales, weight_fp4.micro_scales,
                      alpha=input_fp4.tensor_scale * weight_fp4.tensor_scale)
        return res.reshape(ctx.batch, ctx.seq, ctx.out_dim)

    @staticmethod
    def backward(ctx, grad_output):
        xfp4, xs, xm, wfp4, ws, wm = ctx.saved_tensors
        if torch.is_autocast_enabled("cuda"):
            grad_output = grad_output.to(torch.bfloat16)
        flat_grad_output = grad_output.reshape(-1, grad_output.shape[-1]).contiguous()
        grad_input, grad_weight = quartet_backward(flat_grad_output, xfp4, xs, xm, wfp4, ws, wm, ctx.had,
                                                   ctx.scratch_amax, ctx.disable_backward_quant,
                                                   wgrad_f32=ctx.w_dtype == torch.float32)
        return grad_input.reshape(ctx.batch, ctx.seq, ctx.in_dim), grad_weight, None, None, None, None, None, None, None


def quartet_backward(flat_grad_output, xfp4, xs, xm, wfp4, ws, wm, had, scratch_amax, disable_backward_quant=False,
                     wgrad_f32=False, relu2_input=None, grad_input_acc=None):
    """dX and dW of one Quartet-II linear from the saved NVFP4 operands (linear.py:200-233):
    rerotate H, EDEN of E and E^T (one pass), requantize W^T and X^T, two NVFP4 GEMMs.
    With wgrad_f32 (an fp32 master weight under autocast) dW is written in fp32 by the
    GEMM, where the reference's bf16 dW is cast to the parameter's dtype afterwards.
    With relu2_input (the pre-activation a of an input x = relu(a)^2) the dgrad GEMM's
    epilogue applies the ReLU^2 backward and the result is dL/da instead of dL/dx.  With
    grad_input_acc (a bf16 [M, K] tensor) dX is added into it by the dgrad GEMM, which
    returns it."""
    backward_scale_override = (17 / 16) * 0.93
    had = rerotate_hadamard(had)
    if disable_backward_quant:
        xr = _dq_fp4(xfp4, xs, xm)
        wr = _dq_fp4(wfp4, ws, wm)
        return flat_grad_output @ wr, flat_grad_output.T @ xr
    h16 = had[:16, :].contiguous()
    # E and E^T from one pass over the output gradient
    e_q, et_q = rht128_quant_eden_dual(h=h16, x=flat_grad_output, scale_override=backward_scale_override,
                                       scratch_amax=scratch_amax)
    wt_q = rht128_requant(x=wfp4, x_group_scales=ws, x_tensor_scale=wm, h=h16,
                          scale_override=backward_scale_override, scratch_amax=scratch_amax)
    if grad_input_acc is not None:
        grad_input = _fp4_mm_add(grad_input_acc, e_q.fp4, wt_q.fp4, e_q.micro_scales, wt_q.micro_scales,
                                 e_q.tensor_scale * wt_q.tensor_scale)
    elif relu2_input is None:
        grad_input = _fp4_mm(e_q.fp4, wt_q.fp4, e_q.micro_scales, wt_q.micro_scales,
                             alpha=e_q.tensor_scale * wt_q.tensor_scale)
    else:
        grad_input = _fp4_mm_relu2_bwd(e_q.fp4, wt_q.fp4, e_q.micro_scales, wt_q.micro_scales,
                                       e_q.tensor_scale * wt_q.tensor_scale, relu2_input)
    xt_q = rht128_requant(x=xfp4, x_group_scales=xs, x_tensor_scale=xm, h=h16,
                          scale_override=backward_scale_override, scratch_amax=scratch_amax)
    mm = _fp4_mm_f32 if wgrad_f32 else _fp4_mm
    grad_weight = mm(et_q.fp4, xt_q.fp4, et_q.micro_scales, xt_q.micro_scales,
                     alpha=et_q.tensor_scale * xt_q.tensor_scale)
    return grad_input, grad_weight


class Quartet_II_linear(torch.nn.Linear):
    """nn.Linear whose forward/backward run the Quartet-II NVFP4 recipe.

    As in the reference (linear.py:236-256) the bias parameter exists but is
    not added by forward."""

    def __init__(self, *args, four_over_six=True, **kwargs):
        super().__init__(*args, **kwargs)
        self.mode = NVFP4QuantMode.FOUR_SIX if four_over_six else NVFP4QuantMode.RNE
        self.weight_abs_max = None
        had = get_hadamard_matrix(128, torch.bfloat16, self.weight.device) if self.weight.device.type != "meta" else None
        self.register_buffer("had", had, persistent=False)
        self.register_buffer("scratch_amax", torch.empty((), dtype=torch.uint32, device=self.weight.device),
                             persistent=False)
        self._weight_cache = {}  # the weight's NVFP4 quantization while it is unchanged (_quantize_weight)

    def _apply(self, fn):
        old_device = self.weight.device
        super()._apply(fn)
        if old_device.type == "meta" and self.weight.device.type != "meta":
            self.had = get_hadamard_matrix(128, torch.bfloat16, self.weight.device)
        return self

    def forward(self, x, disable_backward_quant=False, input_abs_max=None):
        return Quartet_II_fn.apply(x, self.weight[...], self.had, self.mode, disable_backward_quant,
                                   self.weight_abs_max, input_abs_max, self.scratch_amax, self._weight_cache)


def register_optimizer_hook(model: torch.nn.Module, optimizer: torch.optim.Optimizer):
    """After every optimizer step cache each Quartet layer's weight abs-max (linear.py:259-270)."""
    opt_params = {id(p) for group in optimizer.param_groups for p in group["params"]}
    quartet_modules = [m for m in model.modules() if isinstance(m, Quartet_II_linear) and id(m.weight) in opt_params]

    def hook(opt, args, kwargs):
        for m in quartet_modules:
            w = m.weight.detach()
            if w.dtype != torch.bfloat16:
                w = w.to(torch.bfloat16)
            m.weight_abs_max = abs_max(w)

    return optimizer.register_step_post_hook(hook)
