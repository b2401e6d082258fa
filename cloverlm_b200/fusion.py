"""Fusions across the ops around the Quartet-II linear.

``shared_input_forward(x, layers)`` -- several Quartet_II_linear layers that
read the same activation (the attention projections lq, lk, lv of
src/models/transformer.py:316-322,341-344 all take X).  The reference runs
three independent Quartet_II_fn calls, each computing abs-max(X) and
quantizing X; here X is quantized once and the three forward GEMMs share its
NVFP4 copy.  Forward outputs are bit-identical to separate calls.  Backward
runs each layer's own backward (quartet_backward, with its own randomized
Hadamard draw) and sums the input gradients in the dgrad GEMMs themselves
(the second and third add into the first's output); only the order of the
random draws differs from separate calls.

``relu2_abs_max(a)`` -- the MLP's ReLU² activation (src/models/mlp.py:34-38,
the `act` of MLP2L.l1, mlp.py:96-99,113-118) computed together with the
abs-max of its bf16 output, so the next Quartet layer gets ``input_abs_max``
and skips its own pass over the activation.

``mlp_relu2(x, l1, l2)`` -- the whole MLP2L with ReLU² (mlp.py:113-118): the
first linear's GEMM writes the pre-activation, its ReLU² and the ReLU²'s
abs-max from its epilogue, and in backward the second linear's dgrad GEMM
applies the ReLU² gradient in its epilogue, so neither the activation nor its
gradient makes an extra round trip through HBM.  Outputs and gradients are
bit-identical to l2(relu2_abs_max(l1(x))) with the same random draws.
"""
from __future__ import annotations

import torch

from . import _lib
from .linear import Quartet_II_linear, _fp4_mm, _fp4_mm_relu2, _quantize_weight, quartet_backward
from .quant import NVFP4QuantMode, abs_max, quant_fp4


class _SharedInputQuartet(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, mode, input_amax, n, *args):
        weights, weight_amaxes, hads, scratches = args[:n], args[n:2 * n], args[2 * n:3 * n], args[3 * n:4 * n]
        caches = args[4 * n:5 * n]
        if torch.is_autocast_enabled("cuda"):
            x = x.to(torch.bfloat16)
        elif x.dtype != torch.bfloat16:
            raise TypeError("Input must be bfloat16. Either cast input to bfloat16 or enable autocast`")
        flat = x.reshape(-1, x.shape[-1]).contiguous()
        if input_amax is None:
            input_amax = abs_max(flat)
        xq = quant_fp4(flat, amax=input_amax, scale_override=1.0, mode=mode)
        outs, saved = [], [xq.fp4, xq.micro_scales, xq.tensor_scale]
        for w, wa, cache in zip(weights, weight_amaxes, caches):
            if not torch.is_autocast_enabled("cuda") and w.dtype != torch.bfloat16:
                raise TypeError("Weight must be bfloat16. Either set `dtype=torch.bfloat16` or enable autocast`")
            wq = _quantize_weight(w, wa, mode, cache)
            y = _fp4_mm(xq.fp4, wq.fp4, xq.micro_scales, wq.micro_scales, alpha=xq.tensor_scale * wq.tensor_scale)
            outs.append(y.reshape(*x.shape[:-1], w.shape[0]))
            saved += [wq.fp4, wq.micro_scales, wq.tensor_scale]
        ctx.save_for_backward(*saved)
        ctx.hads, ctx.scratches, ctx.n, ctx.x_shape = hads, scratches, n, x.shape
        ctx.w_f32 = [w.dtype == torch.float32 for w in weights]
        return tuple(outs)

    @staticmethod
    def backward(ctx, *grads):
        saved = ctx.saved_tensors
        xfp4, xs, xm = saved[:3]
        dx, dws = None, []
        for i, g in enumerate(grads):
            if g is None:
                dws.append(None)
                continue
            wfp4, ws, wm = saved[3 + 3 * i:6 + 3 * i]
            if torch.is_autocast_enabled("cuda"):
                g = g.to(torch.bfloat16)
            # the first input gradient is written, the others are added into it by their dgrad GEMMs
            gi, gw = quartet_backward(g.reshape(-1, g.shape[-1]).contiguous(), xfp4, xs, xm, wfp4, ws, wm,
                                      ctx.hads[i], ctx.scratches[i], wgrad_f32=ctx.w_f32[i], grad_input_acc=dx)
            dx = gi
            dws.append(gw)
        dx = None if dx is None else dx.reshape(ctx.x_shape)
        return (dx, None, None, None, *dws, *([None] * (4 * ctx.n)))


def shared_input_forward(x: torch.Tensor, layers, input_abs_max: torch.Tensor | None = None):
    """Outputs of ``layers`` (Quartet_II_linear, same in_features and mode) on one input x,
    quantizing x once."""
    layers = list(layers)
    if not layers or not all(isinstance(m, Quartet_II_linear) for m in layers):
        raise TypeError("shared_input_forward takes Quartet_II_linear layers")
    if len({m.in_features for m in layers}) != 1 or len({m.mode for m in layers}) != 1:
        raise ValueError("layers must share in_features and mode")
    n = len(layers)
    args = ([m.weight[...] for m in layers] + [m.weight_abs_max for m in layers] + [m.had for m in layers]
            + [m.scratch_amax for m in layers] + [m._weight_cache for m in layers])
    return _SharedInputQuartet.apply(x, layers[0].mode, input_abs_max, n, *args)


# ----------------------------------------------------------------- ReLU^2 + abs-max

class _Relu2AbsMax(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a):
        a = a.contiguous()
        y = torch.empty_like(a, dtype=torch.bfloat16)
        amax = torch.empty((), dtype=torch.float32, device=a.device)
        with torch.cuda.device(a.device):
            _lib.call("q2b_relu2_abs_max", _lib.ptr(y), _lib.ptr(amax), _lib.ptr(a), a.numel(), _lib.stream_of(a))
        ctx.save_for_backward(a)
        ctx.mark_non_differentiable(amax)
        return y, amax

    @staticmethod
    def backward(ctx, gy, gamax):
        (a,) = ctx.saved_tensors
        # d relu(a)^2 / da = 2 relu(a), one pass (q2b_relu2_bwd)
        gy = gy.to(torch.bfloat16).contiguous()
        da = torch.empty_like(a)
        if a.numel() % 8 == 0:
            with torch.cuda.device(a.device):
                _lib.call("q2b_relu2_bwd", _lib.ptr(da), _lib.ptr(a), _lib.ptr(gy), a.numel(), _lib.stream_of(a))
            return da
        return (gy.float() * (2.0 * torch.relu(a.float()))).to(a.dtype)


def relu2_abs_max(a: torch.Tensor):
    """(relu(a)^2 in bf16, max |relu(a)^2| as an fp32 0-d tensor) for bf16 a, one pass."""
    if a.dtype != torch.bfloat16 or not a.is_cuda:
        raise TypeError("relu2_abs_max takes a bf16 CUDA tensor")
    return _Relu2AbsMax.apply(a)


# ------------------------------------------------------------------ fused MLP

class _QuartetMLPRelu2(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, input_amax, mode, w1, w1_amax, had1, scratch1, cache1, w2, w2_amax, had2, scratch2, cache2):
        if torch.is_autocast_enabled("cuda"):
            x = x.to(torch.bfloat16)
        elif x.dtype != torch.bfloat16 or w1.dtype != torch.bfloat16 or w2.dtype != torch.bfloat16:
            raise TypeError("Input and weights must be bfloat16. Either cast them to bfloat16 or enable autocast`")
        flat = x.reshape(-1, x.shape[-1]).contiguous()
        if input_amax is None:
            input_amax = abs_max(flat)
        xq = quant_fp4(flat, amax=input_amax, scale_override=1.0, mode=mode)
        w1q = _quantize_weight(w1, w1_amax, mode, cache1)
        a, h, hamax = _fp4_mm_relu2(xq.fp4, w1q.fp4, xq.micro_scales, w1q.micro_scales,
                                    xq.tensor_scale * w1q.tensor_scale)
        hq = quant_fp4(h, amax=hamax, scale_override=1.0, mode=mode)
        del h
        w2q = _quantize_weight(w2, w2_amax, mode, cache2)
        z = _fp4_mm(hq.fp4, w2q.fp4, hq.micro_scales, w2q.micro_scales, alpha=hq.tensor_scale * w2q.tensor_scale)
        ctx.save_for_backward(xq.fp4, xq.micro_scales, xq.tensor_scale, w1q.fp4, w1q.micro_scales, w1q.tensor_scale,
                              a, hq.fp4, hq.micro_scales, hq.tensor_scale, w2q.fp4, w2q.micro_scales,
                              w2q.tensor_scale)
        ctx.hads, ctx.scratches = (had1, had2), (scratch1, scratch2)
        ctx.w_f32 = (w1.dtype == torch.float32, w2.dtype == torch.float32)
        ctx.x_shape = x.shape
        return z.reshape(*x.shape[:-1], w2.shape[0])

    @staticmethod
    def backward(ctx, gz):
        (xf, xs, xm, w1f, w1s, w1m, a, hf, hs, hm, w2f, w2s, w2m) = ctx.saved_tensors
        gz = gz.to(torch.bfloat16)
        flat = gz.reshape(-1, gz.shape[-1]).contiguous()
        # the second linear's backward; its dgrad GEMM applies the ReLU^2 gradient: dL/da
        da, dw2 = quartet_backward(flat, hf, hs, hm, w2f, w2s, w2m, ctx.hads[1], ctx.scratches[1],
                                   wgrad_f32=ctx.w_f32[1], relu2_input=a)
        dx, dw1 = quartet_backward(da, xf, xs, xm, w1f, w1s, w1m, ctx.hads[0], ctx.scratches[0],
                                   wgrad_f32=ctx.w_f32[0])
        return (dx.reshape(ctx.x_shape), None, None, dw1, None, None, None, None, dw2, None, None, None, None)


def mlp_relu2(x: torch.Tensor, l1: Quartet_II_linear, l2: Quartet_II_linear, input_abs_max: torch.Tensor = None):
    """l2(relu(l1(x))^2) with the activation and its gradient in the two GEMMs' epilogues."""
    if not (isinstance(l1, Quartet_II_linear) and isinstance(l2, Quartet_II_linear)):
        raise TypeError("mlp_relu2 takes two Quartet_II_linear layers")
    if l1.mode != l2.mode or l1.out_features != l2.in_features:
        raise ValueError("l1 and l2 must chain (l1.out_features == l2.in_features) and share the mode")
    return _QuartetMLPRelu2.apply(x, input_abs_max, l1.mode, l1.weight[...], l1.weight_abs_max, l1.had,
                                  l1.scratch_amax, l1._weight_cache, l2.weight[...], l2.weight_abs_max, l2.had,
                                  l2.scratch_amax, l2._weight_cache)
