"""Pins the CPU oracle against the reference's OWN CUDA kernels.

oracle/_ref/libq2ref.so is built from the reference sources (oracle/Makefile,
target `ref`, run by __graft_entry__.build() where the reference tree is
present) and travels to the GPU box; these tests run the reference kernels
there and compare them with the oracle on the same inputs.  Differences come
only from the reference's approximate reciprocal (rcp.approx) and its
tensor-core summation order; the measured fractions are asserted small.
The stochastic rounding of the scales is keyed differently by design, so the
EDEN comparison is on the codes, the pre-rounding bf16 scales (scratch) and
the global max, which fix the result up to that noise.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

import oracle
from helpers import bf16_bits, randn_bf16, student_t_bf16, u8

pytestmark = pytest.mark.gpu

REF_SO = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "libq2ref.so")
BWD_SO = (17 / 16) * 0.93
APPROX_RCP_FRACTION = 2e-3   # codes/scales flipped by rcp.approx vs IEEE reciprocal


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(REF_SO):
        pytest.skip("reference kernels not built (oracle/_ref/libq2ref.so)")
    L = ctypes.CDLL(REF_SO)
    P, F, L64, I = ctypes.c_void_p, ctypes.c_float, ctypes.c_long, ctypes.c_int
    L.qref_quant_fwd.argtypes = [P, P, P, P, P, F, L64, L64, I]
    L.qref_rht128_eden.argtypes = [P, P, P, P, P, P, P, L64, F, F, I, I, I, I]
    L.qref_rht128_requant.argtypes = [P, P, P, P, P, P, P, P, P, L64, F, F, I, I]
    L.qref_last_error.restype = ctypes.c_char_p
    return L


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _ok(L, rc):
    assert rc == 0, L.qref_last_error().decode()
    torch.cuda.synchronize()


@pytest.mark.parametrize("four_six", [False, True])
@pytest.mark.parametrize("shape", [(1024, 3584), (2048, 3584)])
def test_oracle_matches_reference_quant_fwd(ref, four_six, shape):
    x = randn_bf16(*shape, seed=17, outliers=1e-3, device="cuda")
    amax = x.float().abs().max().reshape(())
    y = torch.empty(shape[0], shape[1] // 2, dtype=torch.uint8, device="cuda")
    s = torch.empty(shape[0] * shape[1] // 16, dtype=torch.uint8, device="cuda")
    t = torch.empty((), device="cuda")
    _ok(ref, ref.qref_quant_fwd(_p(y), _p(s), _p(t), _p(x), _p(amax), 1.0, shape[0], shape[1], int(four_six)))
    codes, sf, ts = oracle.quant_fp4(bf16_bits(x), four_six=four_six)
    assert t.item() == np.float32(ts)
    assert (u8(y) != codes).mean() <= APPROX_RCP_FRACTION
    assert (u8(s) != sf).mean() <= APPROX_RCP_FRACTION


def _ref_rht(ref, x, h, seed, transpose, full_h, so=BWD_SO):
    M, N = x.shape
    rows, cols = (N, M) if transpose else (M, N)
    y = torch.empty(rows, cols // 2, dtype=torch.uint8, device="cuda")
    s = torch.empty(rows * cols // 16, dtype=torch.uint8, device="cuda")
    t = torch.empty((), device="cuda")
    scratch = torch.empty(rows * cols // 16, dtype=torch.bfloat16, device="cuda")
    mx = torch.zeros((), dtype=torch.int32, device="cuda")
    fp4_max = 6.0 / so
    _ok(ref, ref.qref_rht128_eden(_p(y), _p(s), _p(t), _p(scratch), _p(mx), _p(h), _p(x), seed, fp4_max, 256.0,
                                  M, N, int(transpose), int(full_h)))
    return y, s, t, scratch, mx


def _h(seed):
    from cloverlm_b200.linear import get_hadamard_matrix
    g = torch.Generator().manual_seed(seed)
    H = get_hadamard_matrix(128, torch.bfloat16, "cpu")
    signs = (torch.randint(0, 2, (128,), generator=g) * 2 - 1).to(torch.bfloat16)
    return (H * signs[None, :]).contiguous()


@pytest.mark.parametrize("transpose", [False, True])
@pytest.mark.parametrize("shape", [(1024, 640), (2048, 3584)])
def test_oracle_matches_reference_rht128_eden(ref, shape, transpose):
    x = student_t_bf16(*shape, seed=1, device="cuda")
    H = _h(2)
    h16 = H[:16].contiguous()
    y, s, t, scratch, mx = _ref_rht(ref, x, h16.cuda(), 42, transpose, False)
    v = oracle.rotate(bf16_bits(x), oracle.rht_matrix_from_slice(bf16_bits(h16)), transpose)
    codes, osc, mb = oracle.eden_pass1(v, BWD_SO)
    assert (u8(y) != codes).mean() <= APPROX_RCP_FRACTION
    assert (bf16_bits(scratch).reshape(osc.shape) != osc).mean() <= APPROX_RCP_FRACTION
    assert int(mx.item()) & 0xFFFFFFFF == mb
    _, ts = oracle.sr_scales(osc, mb, seed=0)
    assert t.item() == np.float32(ts)


def test_reference_slice_identity(ref):
    """The reference's own rht128 (16-row slice) and group-transform (full
    swizzled matrix) kernels agree bit for bit (its test_rht.py:49-59), and
    our oracle reproduces that identity."""
    x = randn_bf16(1024, 640, seed=4, device="cuda")
    H = (_h(3).float() * 128 ** 0.5).to(torch.bfloat16)
    from cloverlm_b200.rht import swizzle_hadamard
    a = _ref_rht(ref, x, H[:16].contiguous().cuda(), 42, False, False, so=1.0)
    b = _ref_rht(ref, x, swizzle_hadamard(H).contiguous().cuda(), 42, False, True, so=1.0)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1]) and a[2].item() == b[2].item()


@pytest.mark.parametrize("shape", [(1024, 640), (2048, 3584)])
def test_oracle_matches_reference_requant(ref, shape):
    from cloverlm_b200.quant import NVFP4QuantMode, quant_fp4
    x = randn_bf16(*shape, seed=9, outliers=1e-3, device="cuda")
    q, s, t = quant_fp4(x, scale_override=1.0, mode=NVFP4QuantMode.FOUR_SIX)
    M, N = shape
    h16 = _h(5)[:16].contiguous()
    y = torch.empty(N, M // 2, dtype=torch.uint8, device="cuda")
    so_ = torch.empty(N * M // 16, dtype=torch.uint8, device="cuda")
    ts_ = torch.empty((), device="cuda")
    scratch = torch.empty(N * M // 16, dtype=torch.bfloat16, device="cuda")
    mx = torch.zeros((), dtype=torch.int32, device="cuda")
    _ok(ref, ref.qref_rht128_requant(_p(y), _p(so_), _p(ts_), _p(scratch), _p(mx), _p(h16.cuda()), _p(q),
                                     _p(s), _p(t), 7, 6.0 / BWD_SO, 256.0, M, N))
    xb = oracle.dequant_bf16(u8(q), u8(s).reshape(-1), t.item())
    v = oracle.rotate(xb, oracle.rht_matrix_from_slice(bf16_bits(h16)), True)
    codes, osc, mb = oracle.eden_pass1(v, BWD_SO)
    assert (u8(y) != codes).mean() <= APPROX_RCP_FRACTION
    assert (bf16_bits(scratch).reshape(osc.shape) != osc).mean() <= APPROX_RCP_FRACTION
    assert int(mx.item()) & 0xFFFFFFFF == mb
