"""CPU tests of the oracle (the C restatement in oracle/): number formats
against torch's own conversions, the reference's semantic identities and
effective-bitwidth floors (quartet2/test/test_rht.py, test_rounding.py), and
golden vectors from the reference's Python emulation (tests/golden/)."""
import os

import numpy as np
import pytest
import torch

import oracle
from helpers import bf16_bits, eff_bits, randn_bf16

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "fake_quartet_golden.npz")
BWD_SO = (17 / 16) * 0.93


def test_bf16_conversion_matches_torch():
    x = torch.randn(100000) * torch.exp(torch.randn(100000) * 10)
    ours = oracle.f32_to_bf16(x.numpy())
    np.testing.assert_array_equal(ours, bf16_bits(x.to(torch.bfloat16)))


def test_e4m3_conversion_matches_torch():
    L = oracle.lib()
    vals = np.concatenate([np.random.default_rng(0).uniform(-460, 460, 20000),
                           np.random.default_rng(1).uniform(-0.02, 0.02, 20000),
                           np.array([0.0, -0.0, 2 ** -9, 2 ** -10, 448.0, -448.0, 0.015625, 240.0, 232.0])])
    vals = vals.astype(np.float32)
    ref = torch.from_numpy(vals).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    ours = np.array([L.oq_f32_to_e4m3(float(v)) for v in vals], dtype=np.uint8)
    # torch does not saturate (|v| > 448 rounds to NaN); compare in range only
    ok = np.abs(vals) <= 448
    np.testing.assert_array_equal(ours[ok], ref[ok])
    table = oracle.e4m3_table()
    tref = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    fin = ~np.isnan(tref)
    np.testing.assert_array_equal(table[fin], tref[fin])


def test_e2m1_round_to_nearest_even_and_saturation():
    L = oracle.lib()
    cases = {0.0: 0, 0.25: 0, 0.26: 1, 0.75: 2, 1.25: 2, 1.75: 4, 2.5: 4, 3.5: 6, 5.0: 6, 5.01: 7, 6.0: 7, 100.0: 7,
             -0.1: 8, -0.75: 10, -7.0: 15}
    for v, code in cases.items():
        assert L.oq_f32_to_e2m1(v) == code, v
    for c in range(16):
        assert L.oq_f32_to_e2m1(L.oq_e2m1_to_f32(c)) == c


def test_sf_layout_roundtrip():
    sf = np.arange(256 * 32, dtype=np.int32).reshape(256, 32)
    np.testing.assert_array_equal(oracle.unblock(oracle.to_blocked(sf), 256, 32), sf)
    assert oracle.lib().oq_sf_offset(1, 0, 32) == 16 and oracle.lib().oq_sf_offset(32, 0, 32) == 4


def test_philox_known_answers():
    # Philox-4x32-10 known-answer vectors of the Random123 distribution (Salmon et al.)
    L = oracle.lib()
    import ctypes
    out = np.zeros(4, dtype=np.uint32)
    L.oq_philox(0, 0, out.ctypes.data_as(ctypes.c_void_p))
    np.testing.assert_array_equal(out, [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8])


@pytest.mark.parametrize("mode,floor", [(False, 3.38), (True, 3.52)])
def test_rtn_effective_bitwidth_floor(mode, floor):
    x = randn_bf16(1024, 2048, seed=42)
    c, s, ts = oracle.quant_fp4(bf16_bits(x), four_six=mode)
    assert eff_bits(x.float().numpy(), oracle.dequant(c, s, ts)) > floor


@pytest.mark.parametrize("transpose", [False, True])
def test_rht_slice_equals_swizzled_full_matrix(transpose):
    """quartet2/test/test_rht.py:49-59 restated: bit-exact agreement of the
    16-row-slice path and the explicit swizzle_hadamard(H) path."""
    x = bf16_bits(randn_bf16(256, 640, seed=3))
    H = oracle.hadamard128_bf16()
    signs = np.random.default_rng(0).integers(0, 2, 128)
    Hs = H ^ (signs.astype(np.uint16) << 15)[None, :]  # column sign flips
    a = oracle.rht128_quant_eden(x, Hs[:16].copy(), seed=42, transpose=transpose)
    b = oracle.quant_had_eden(x, oracle.swizzle_hadamard(Hs), seed=42, transpose=transpose)
    for u, v in zip(a, b):
        np.testing.assert_array_equal(u, v)


@pytest.mark.parametrize("transpose", [False, True])
def test_eden_bitwidth_floors(transpose):
    x = randn_bf16(1024, 1024, seed=9)
    H = oracle.hadamard128_bf16()
    ref = oracle.rotate(bf16_bits(x), oracle.swizzle_hadamard(H), transpose)
    c, s, ts = oracle.rht128_quant_eden(bf16_bits(x), H[:16].copy(), seed=1, transpose=transpose)
    assert eff_bits(ref, oracle.dequant(c, s, ts)) > 3.2
    eye = oracle.f32_to_bf16(np.eye(128, dtype=np.float32))
    c, s, ts = oracle.quant_had_eden(bf16_bits(x), eye, seed=1, transpose=transpose)
    xt = x.float().numpy().T if transpose else x.float().numpy()
    assert eff_bits(xt, oracle.dequant(c, s, ts)) > 3.37


def test_requant_close_to_quantizing_the_dequantized_tensor():
    """quartet2/test/test_rounding.py:117-123: requantizing an NVFP4 tensor
    (dequantize to bf16, transpose, EDEN) is within > 4.2 bits of an
    independent EDEN quantization of the same dequantized transpose."""
    x = randn_bf16(1024, 512, seed=5)
    eye = oracle.f32_to_bf16(np.eye(128, dtype=np.float32))
    c, s, ts = oracle.quant_had_eden(bf16_bits(x), eye, seed=1)
    ref = oracle.quant_had_eden(oracle.dequant_bf16(c, s, ts), eye, seed=2, transpose=True)
    H = oracle.hadamard128_bf16()
    rq = oracle.rht128_requant(c, s, ts, H[:16].copy(), seed=3)
    rot = oracle.rotate(oracle.dequant_bf16(c, s, ts), oracle.swizzle_hadamard(H), True)
    assert eff_bits(oracle.dequant(*ref), oracle.dequant(*oracle.quant_had_eden(
        oracle.dequant_bf16(c, s, ts), eye, seed=4, transpose=True))) > 4.2
    assert eff_bits(rot, oracle.dequant(*rq)) > 3.2


def test_sr_is_unbiased_on_the_grid():
    L = oracle.lib()
    rng = np.random.default_rng(0)
    for v in [1.03, 17.3, 200.1, 0.02]:
        lo_b = L.oq_f32_to_e4m3(v)
        draws = np.array([L.oq_e4m3_to_f32(L.oq_sr_e4m3(v, int(n))) for n in rng.integers(0, 65536, 4000)])
        assert abs(draws.mean() - v) / v < 0.01, (v, draws.mean())
        assert len(np.unique(draws)) <= 2


def _golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("name", ["normal_outliers", "student_t"])
@pytest.mark.parametrize("four_six", [True, False])
def test_rtn_against_reference_emulation(name, four_six):
    """The reference's emulation (src/fake_quartet.py) computes with bf16
    intermediates and ties away from zero, so it pins semantics
    statistically: our restatement of the CUDA kernel is never worse and
    quantizes to the same grid up to those rounding differences."""
    d = _golden()
    x = d[f"rtn_{name}_x"]
    y = oracle.bf16_to_f32(d[f"rtn_{name}_{'46' if four_six else 'rne'}_y"])
    c, s, ts = oracle.quant_fp4(x, four_six=four_six)
    dq = oracle.dequant(c, s, ts)
    xf = oracle.bf16_to_f32(x)
    sse_ours, sse_ref = ((xf - dq) ** 2).sum(), ((xf - y) ** 2).sum()
    assert sse_ours <= 1.01 * sse_ref
    assert abs(eff_bits(xf, dq) - eff_bits(xf, y)) < 0.35
    # group scales agree to within one bf16-rounding step of the emulation's scale arithmetic
    g = lambda a: np.abs(a.reshape(-1, 16)).max(1)
    ratio = g(y)[g(dq) > 0] / g(dq)[g(dq) > 0]
    assert np.median(ratio) > 0.99 and np.median(ratio) < 1.01


def test_eden_rotation_against_reference_emulation():
    """The emulation's rotated abs-max pins the rotation (x @ H^T per 128-group,
    not x @ H) to within fp32 summation order; EDEN accuracy is at least the
    emulation's."""
    d = _golden()
    x, H, y = d["eden_x"], d["eden_h"], d["eden_y"]
    v = oracle.rotate(x, H, False)
    amax = float(d["eden_next_amax"][0])
    assert abs(float(np.abs(v).max()) - amax) <= 1e-6 * amax
    assert abs(float(np.abs(oracle.rotate(x, H.T.copy(), False)).max()) - amax) > 1e-3 * amax
    c, s, ts = oracle.quant_had_eden(x, H, seed=1, scale_override=BWD_SO)
    assert eff_bits(v, oracle.dequant(c, s, ts)) >= eff_bits(v, y) - 0.02


def test_linear_fwd_bwd_shapes_and_accuracy():
    rng = np.random.default_rng(0)
    M, K, N = 256, 256, 384
    x = oracle.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    w = oracle.f32_to_bf16((0.05 * rng.standard_normal((N, K))).astype(np.float32))
    dy = oracle.f32_to_bf16(rng.standard_normal((M, N)).astype(np.float32))
    h16 = oracle.hadamard128_bf16()[:16].copy()
    y, dx, dw = oracle.linear_fwd_bwd(x, w, dy, h16)
    X, W, DY = (oracle.bf16_to_f32(a) for a in (x, w, dy))
    assert y.shape == (M, N) and dx.shape == (M, K) and dw.shape == (N, K)
    assert eff_bits(X @ W.T, y) > 2.8
    cos = lambda a, b: float((a * b).sum() / np.sqrt((a * a).sum() * (b * b).sum()))
    assert cos(dx, DY @ W) > 0.97 and cos(dw, DY.T @ X) > 0.97
