"""GPU parity of the inference linear (reference QuartetIILinearMethod,
src/evals/vllm_plugin/quartet2_quant.py:45-140) at decode and prefill M.

The reference pads the activation rows to a multiple of 128; ours does not.
Checks: the quantized rows are bit-identical to quantizing the zero-padded
matrix; the output is within the GEMM bar (1e-2 relative Frobenius) of an
fp32 matmul of the dequantized operands and matches the padded path to bf16
rounding; the split-K workspace is left zero; bias and leading dims behave as
in the reference."""
import pytest
import torch
import torch.nn.functional as F

import oracle
from cloverlm_b200 import _lib
from cloverlm_b200.inference import (QuartetIIInferenceLinear, _workspaces, apply, fp4_mm_rows, prepare_weight,
                                     quant_rows)
from cloverlm_b200.linear import _fp4_mm
from cloverlm_b200.quant import NVFP4QuantMode, abs_max, quant_fp4
from helpers import u8

pytestmark = pytest.mark.gpu

REL_FRO_TOL = 1e-2


@pytest.fixture(autouse=True)
def _no_watchdog():
    yield
    assert _lib.device_status() == 0, "a kernel wait timed out"


def _inputs(m, k, n, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16).cuda()
    return x, w


def _padded_reference(x, p):
    """The reference's apply: pad rows to 128, quantize, GEMM, slice."""
    m = x.shape[0]
    pad = (-m) % 128
    xp = F.pad(x, (0, 0, 0, pad))
    q = quant_fp4(xp, amax=abs_max(xp), scale_override=1.0, mode=NVFP4QuantMode.FOUR_SIX)
    out = _fp4_mm(q.fp4, p.fp4, q.micro_scales, p.micro_scales, q.tensor_scale * p.tensor_scale)
    return out[:m, :p.out_features], q


@pytest.mark.parametrize("m", [1, 5, 64, 128, 200, 256])
def test_ragged_quant_matches_padded_rows(m):
    x, _ = _inputs(m, 512, 128, seed=m)
    codes, scales, ts = quant_rows(x)
    xp = F.pad(x, (0, 0, 0, (-m) % 128))
    q = quant_fp4(xp, amax=abs_max(xp), scale_override=1.0, mode=NVFP4QuantMode.FOUR_SIX)
    assert torch.equal(codes, q.fp4[:m])
    assert torch.equal(scales.view(torch.uint8), q.micro_scales.view(torch.uint8))
    assert ts.item() == q.tensor_scale.item()


@pytest.mark.parametrize("m,k", [(1, 128), (3, 256), (2, 384), (130, 128), (64, 14336), (700, 3584)])
@pytest.mark.parametrize("path", ["fused", "two_kernel"])
def test_ragged_quant_both_paths_match_padded_rows(m, k, path):
    """The one-launch cluster path (abs-max + codes) and the abs-max + ragged-quantizer path, on
    row counts and widths whose group counts are not multiples of a warp."""
    x, _ = _inputs(m, k, 128, seed=m * 7 + k)
    codes, scales, ts = quant_rows(x) if path == "fused" else quant_rows(x, amax=abs_max(x))
    xp = F.pad(x, (0, 0, 0, (-m) % 128))
    q = quant_fp4(xp, amax=abs_max(xp), scale_override=1.0, mode=NVFP4QuantMode.FOUR_SIX)
    assert torch.equal(codes, q.fp4[:m])
    assert torch.equal(scales.view(torch.uint8), q.micro_scales.view(torch.uint8))
    assert ts.item() == q.tensor_scale.item()


def test_fused_rows_rne_mode_matches_quant_fp4():
    m, k = 9, 640
    x, _ = _inputs(m, k, 128, seed=3)
    codes = torch.empty((m, k // 2), dtype=torch.uint8, device="cuda")
    scales = torch.full((128 * k // 16,), 0xFF, dtype=torch.uint8, device="cuda")  # pad rows must come back 0
    ts = torch.empty((), device="cuda")
    _lib.call("q2b_quant_rows_fused", _lib.ptr(codes), _lib.ptr(scales), _lib.ptr(ts), _lib.ptr(x), 1.0, m, k,
              _lib.MODE_RNE, _lib.stream_of(x))
    xp = F.pad(x, (0, 0, 0, 128 - m))
    q = quant_fp4(xp, amax=abs_max(xp), scale_override=1.0, mode=NVFP4QuantMode.RNE)
    assert torch.equal(codes, q.fp4[:m])
    assert torch.equal(scales, q.micro_scales.view(torch.uint8).reshape(-1))
    assert ts.item() == q.tensor_scale.item()


@pytest.mark.parametrize("m,k,n", [(1, 3584, 3584), (8, 3584, 10752), (64, 14336, 3584), (1, 512, 384),
                                   (37, 1024, 640), (256, 3584, 3584), (300, 512, 256), (4096, 3584, 3584)])
def test_apply_matches_padded_path_and_fp32(m, k, n):
    x, w = _inputs(m, k, n, seed=m + n)
    p = prepare_weight(w)
    out = apply(p, x)
    assert out.shape == (m, n) and out.dtype == torch.bfloat16
    ref, q = _padded_reference(x, p)
    # same quantized operands, so the padded path is the exact oracle up to fp32 summation order
    rel_pad = ((out.float() - ref.float()).norm() / ref.float().norm()).item()
    assert rel_pad < 4e-3, rel_pad
    A = torch.from_numpy(oracle.dequant(u8(q.fp4), u8(q.micro_scales).reshape(-1), q.tensor_scale.item())).cuda()[:m]
    B = torch.from_numpy(oracle.dequant(u8(p.fp4), u8(p.micro_scales).reshape(-1), p.tensor_scale.item())).cuda()
    exact = (A @ B.T)[:, :n]
    rel = ((out.float() - exact).norm() / exact.norm()).item()
    assert rel <= REL_FRO_TOL, rel


def test_split_k_workspace_is_left_zero_and_reused():
    x, w = _inputs(3, 3584, 3584, seed=11)
    p = prepare_weight(w)
    assert _lib.load().q2b_gemm_workspace_bytes(3, 3584, 3584) > 0  # this shape splits K
    a = apply(p, x)
    b = apply(p, x)
    # fp32 partial sums arrive in any order; both calls agree to bf16 rounding
    assert ((a.float() - b.float()).norm() / a.float().norm()).item() < 4e-3
    assert len(_workspaces) > 0
    for ws in _workspaces.values():
        assert int(ws.count_nonzero().item()) == 0


def test_weight_padding_bias_and_leading_dims():
    g = torch.Generator().manual_seed(5)
    w = (torch.randn(200, 256, generator=g) * 0.02).to(torch.bfloat16).cuda()  # 200 -> padded to 256 rows
    bias = torch.randn(200, generator=g).to(torch.bfloat16).cuda()
    layer = QuartetIIInferenceLinear(w, bias)
    assert layer.w_pad == 56
    x = torch.randn(2, 3, 256, generator=g).to(torch.bfloat16).cuda()
    y = layer(x)
    assert y.shape == (2, 3, 200)
    y0 = apply(layer.prepared(), x.reshape(6, 256)).reshape(2, 3, 200)
    assert torch.equal(y, y0 + bias)


def test_gemm_rows_exact_small_integers():
    """Unit scales and integer-valued products are exact in fp32, split or not."""
    for m in (1, 7, 130):
        g = torch.Generator().manual_seed(m)
        k, n = 2048, 256
        ca = torch.randint(0, 256, (m, k // 2), generator=g, dtype=torch.uint8)
        cb = torch.randint(0, 256, (n, k // 2), generator=g, dtype=torch.uint8)
        m_pad = (m + 127) // 128 * 128
        sa = torch.full((m_pad * k // 16,), 0x38, dtype=torch.uint8)
        sb = torch.full((n * k // 16,), 0x38, dtype=torch.uint8)
        one = torch.ones((), device="cuda")
        out = fp4_mm_rows(ca.cuda(), cb.cuda(), sa.view(torch.float8_e4m3fn).cuda(), sb.view(torch.float8_e4m3fn).cuda(),
                          one)
        ca_pad = torch.zeros((m_pad, k // 2), dtype=torch.uint8)
        ca_pad[:m] = ca
        A = torch.from_numpy(oracle.dequant(ca_pad.numpy(), sa.numpy(), 1.0)).double()[:m]
        B = torch.from_numpy(oracle.dequant(cb.numpy(), sb.numpy(), 1.0)).double()
        ref = (A @ B.T).to(torch.bfloat16)
        assert torch.equal(out.cpu(), ref), m


def test_apply_compiles_fullgraph():
    """The ops of apply are torch custom ops (as the reference's quantizers and _fp4_mm are), so
    torch.compile traces the inference linear without graph breaks (vLLM compiles its models)."""
    x, w = _inputs(5, 512, 384, seed=21)
    p = prepare_weight(w)
    compiled = torch.compile(lambda t: apply(p, t), fullgraph=True)
    a, b = compiled(x), apply(p, x)
    assert a.shape == b.shape
    assert ((a.float() - b.float()).norm() / b.float().norm()).item() < 4e-3
