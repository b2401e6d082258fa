"""Forward-only NVFP4 linear for inference -- the vLLM plugin path of the
reference (src/evals/vllm_plugin/quartet2_quant.py:45-140,
``QuartetIILinearMethod``) on libq2b.

The weight is quantized once (four-over-six, tensor scale from its abs-max),
exactly as ``process_weights_after_loading`` does, including the zero rows
that pad ``out_features`` to a multiple of 128 (quartet2_quant.py:80-99).

``apply`` differs from the reference in how it treats the activation rows:
the reference pads them to a multiple of 128 with ``F.pad``, quantizes and
multiplies the padded matrix and slices the output (quartet2_quant.py:110-137).
Here the activations are quantized and multiplied as they are
(``q2b_quant_rows_fused`` -- abs-max, scale and codes in one launch -- for
decode-sized inputs, ``q2b_abs_max`` + ``q2b_quant_fwd_ragged`` for larger
ones, then ``q2b_gemm_nvfp4_ex`` with both tensor scales passed as pointers,
so no product kernel runs): the GEMM reads rows past M
as zeros through its TMA descriptor and stores only rows < M, and at
decode-sized M it splits K across the SMs and sums the partial tiles in fp32.
The codes and scales of the real rows are the ones the padded path produces
(zero padding rows change neither the abs-max nor any group); the output
equals the padded path's up to fp32 summation order when K is split.
As in the reference, the bias is added to the bf16 output.  The quantizer
and the GEMM are torch custom ops (``quartet2::quant_rows``,
``quartet2::quant_rows_amax``, ``quartet2::fp4_mm_rows``) with fake
implementations, like the reference's ``quartet2::four_six`` and
``quartet2::fp4_mm``, so ``torch.compile(fullgraph=True)`` traces ``apply``.
"""
from __future__ import annotations

import threading
from typing import NamedTuple

import torch
import torch.nn.functional as F

from . import _lib
from .quant import NVFP4QuantMode, abs_max, quant_fp4


class PreparedWeight(NamedTuple):
    """Quantized weight as ``process_weights_after_loading`` stores it on the layer
    (``weight_fp4``, ``weight_micro_scales``, ``weight_tensor_scale``, ``w_pad``)."""
    fp4: torch.Tensor            # uint8 [N_pad, K/2]
    micro_scales: torch.Tensor   # float8_e4m3fn [N_pad, K/16], blocked layout
    tensor_scale: torch.Tensor   # fp32 []
    out_features: int
    w_pad: int


def prepare_weight(weight: torch.Tensor) -> PreparedWeight:
    """quartet2_quant.py:74-99: pad out_features to 128, abs-max, four-over-six quantization."""
    out_features = weight.shape[0]
    rem = out_features % 128
    w_pad = 128 - rem if rem else 0
    if w_pad:
        weight = F.pad(weight, (0, 0, 0, w_pad))
    weight = weight.to(torch.bfloat16).contiguous()
    wq = quant_fp4(weight, amax=abs_max(weight), scale_override=1.0, mode=NVFP4QuantMode.FOUR_SIX)
    return PreparedWeight(wq.fp4, wq.micro_scales, wq.tensor_scale, out_features, w_pad)


_ws_lock = threading.Lock()
_workspaces: dict = {}


def _workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor | None:
    """Zero-filled split-K workspace, one per (device, stream); the GEMM leaves it zero after every call."""
    if nbytes <= 0:
        return None
    key = (device.index, stream)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(nbytes, dtype=torch.uint8, device=device)
            _workspaces[key] = ws
        return ws


# Inputs up to this many 16-element groups are quantized by the one-launch
# cluster kernel (abs-max, scale and codes together); larger ones by the
# grid-wide abs-max and quantizer kernels.
FUSED_MAX_GROUPS = 1 << 12  # measured: faster up to ~2k groups, slower than the grid kernels at 14k


def quant_rows(x: torch.Tensor, amax: torch.Tensor | None = None):
    """Four-over-six quantization of bf16 x [M, K] for any M >= 1.

    Returns (codes uint8 [M, K/2], scales float8_e4m3fn [ceil(M/128)*128, K/16]
    in the blocked layout with zero rows past M, tensor scale fp32 [])."""
    assert x.dtype == torch.bfloat16 and x.is_cuda and x.dim() == 2
    x = x.contiguous()
    if amax is None:
        return _quant_rows_op(x)
    return _quant_rows_amax_op(x, amax)


def _quant_rows_out(x):
    m, k = x.shape
    m_pad = (m + 127) // 128 * 128
    codes = torch.empty((m, k // 2), dtype=torch.uint8, device=x.device)
    ts = torch.empty((), dtype=torch.float32, device=x.device)
    return m, k, m_pad, codes, ts


@torch.library.custom_op("quartet2::quant_rows", mutates_args=())
def _quant_rows_op(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Abs-max + four-over-six quantization of x [M, K], any M (torch op so torch.compile traces it)."""
    m, k, m_pad, codes, ts = _quant_rows_out(x)
    with torch.cuda.device(x.device):
        if m * k // 16 <= FUSED_MAX_GROUPS:
            scales = torch.empty((m_pad, k // 16), dtype=torch.float8_e4m3fn, device=x.device)
            _lib.call("q2b_quant_rows_fused", _lib.ptr(codes), _lib.ptr(scales), _lib.ptr(ts), _lib.ptr(x), 1.0,
                      m, k, _lib.MODE_FOUR_SIX, _lib.stream_of(x))
            return codes, scales, ts
        amax = abs_max(x)
        scales = torch.zeros((m_pad, k // 16), dtype=torch.float8_e4m3fn, device=x.device)
        _lib.call("q2b_quant_fwd_ragged", _lib.ptr(codes), _lib.ptr(scales), _lib.ptr(ts), _lib.ptr(x),
                  _lib.ptr(amax), 1.0, m, k, _lib.MODE_FOUR_SIX, _lib.stream_of(x))
    return codes, scales, ts


@torch.library.custom_op("quartet2::quant_rows_amax", mutates_args=())
def _quant_rows_amax_op(x: torch.Tensor, amax: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Four-over-six quantization of x [M, K], any M, with the tensor abs-max given."""
    m, k, m_pad, codes, ts = _quant_rows_out(x)
    scales = torch.zeros((m_pad, k // 16), dtype=torch.float8_e4m3fn, device=x.device)
    with torch.cuda.device(x.device):
        _lib.call("q2b_quant_fwd_ragged", _lib.ptr(codes), _lib.ptr(scales), _lib.ptr(ts), _lib.ptr(x),
                  _lib.ptr(amax), 1.0, m, k, _lib.MODE_FOUR_SIX, _lib.stream_of(x))
    return codes, scales, ts


def _quant_rows_fake_impl(x):
    m, k = x.shape
    m_pad = (m + 127) // 128 * 128
    return (torch.empty((m, k // 2), dtype=torch.uint8, device=x.device),
            torch.empty((m_pad, k // 16), dtype=torch.float8_e4m3fn, device=x.device),
            torch.empty((), dtype=torch.float32, device=x.device))


@_quant_rows_op.register_fake
def _quant_rows_fake(x):
    return _quant_rows_fake_impl(x)


@_quant_rows_amax_op.register_fake
def _quant_rows_amax_fake(x, amax):
    return _quant_rows_fake_impl(x)


def fp4_mm_rows(x_fp4: torch.Tensor, w_fp4: torch.Tensor, x_mx: torch.Tensor, w_mx: torch.Tensor,
                alpha: torch.Tensor, alpha_b: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 [M, N] = alpha (* alpha_b) * dq(x) @ dq(w)^T for any M >= 1 (x_mx padded to whole 128-row blocks)."""
    if alpha.dtype != torch.float32:
        alpha = alpha.float()
    if alpha_b is not None and alpha_b.dtype != torch.float32:
        alpha_b = alpha_b.float()
    return _fp4_mm_rows_op(x_fp4, w_fp4, x_mx, w_mx, alpha, alpha_b)


@torch.library.custom_op("quartet2::fp4_mm_rows", mutates_args=())
def _fp4_mm_rows_op(x_fp4: torch.Tensor, w_fp4: torch.Tensor, x_mx: torch.Tensor, w_mx: torch.Tensor,
                    alpha: torch.Tensor, alpha_b: torch.Tensor | None) -> torch.Tensor:
    m, packed_k = x_fp4.shape
    k = packed_k * 2
    n = w_fp4.shape[0]
    out = torch.empty((m, n), dtype=torch.bfloat16, device=x_fp4.device)
    with torch.cuda.device(x_fp4.device):
        lib = _lib.load()
        nbytes = int(lib.q2b_gemm_workspace_bytes(m, n, k))
        stream = _lib.stream_of(x_fp4)
        ws = _workspace(x_fp4.device, stream.value, nbytes)
        _lib.call("q2b_gemm_nvfp4_ex", _lib.ptr(out), _lib.ptr(x_fp4), _lib.ptr(w_fp4), _lib.ptr(x_mx),
                  _lib.ptr(w_mx), _lib.ptr(alpha), _lib.ptr(alpha_b), m, n, k, _lib.ptr(ws),
                  nbytes if ws is not None else 0, stream)
    return out


@_fp4_mm_rows_op.register_fake
def _fp4_mm_rows_fake(x_fp4, w_fp4, x_mx, w_mx, alpha, alpha_b):
    return torch.empty((x_fp4.shape[0], w_fp4.shape[0]), dtype=torch.bfloat16, device=x_fp4.device)


def apply(prepared: PreparedWeight, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """QuartetIILinearMethod.apply (quartet2_quant.py:101-140) without row padding."""
    orig_shape = x.shape
    flat = x.reshape(-1, x.shape[-1])
    if flat.dtype != torch.bfloat16:
        flat = flat.to(torch.bfloat16)
    codes, scales, ts = quant_rows(flat)
    out = fp4_mm_rows(codes, prepared.fp4, scales, prepared.micro_scales, ts, prepared.tensor_scale)
    if prepared.w_pad:
        out = out[:, :prepared.out_features]
    out = out.reshape(*orig_shape[:-1], out.shape[-1])
    if bias is not None:
        out = out + bias
    return out


class QuartetIIInferenceLinear(torch.nn.Module):
    """A forward-only layer holding a prepared weight; ``forward`` = ``apply``."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None = None):
        super().__init__()
        p = prepare_weight(weight)
        self.register_buffer("weight_fp4", p.fp4)
        self.register_buffer("weight_micro_scales", p.micro_scales)
        self.register_buffer("weight_tensor_scale", p.tensor_scale)
        self.out_features = p.out_features
        self.w_pad = p.w_pad
        self.bias = None if bias is None else torch.nn.Parameter(bias.detach().clone(), requires_grad=False)

    def prepared(self) -> PreparedWeight:
        return PreparedWeight(self.weight_fp4, self.weight_micro_scales, self.weight_tensor_scale,
                              self.out_features, self.w_pad)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return apply(self.prepared(), x, self.bias)
