"""CPU tests of the host layer's pure-torch pieces: the blocked 128x4 scale
layout (linear.to_blocked / unblock) and _dq_fp4 against the oracle, and the
fake (meta) implementations that torch.compile uses to trace the ops that
return new tensors (quartet2::fp4_mm, quant_rows, quant_rows_amax,
fp4_mm_rows, abs_max)."""
import numpy as np
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import oracle
from cloverlm_b200 import inference as I
from cloverlm_b200 import linear as L
from cloverlm_b200 import quant as Q


@pytest.mark.parametrize("rows,cols16", [(128, 4), (256, 64), (384, 224)])
def test_to_blocked_and_unblock_follow_the_oracle_layout(rows, cols16):
    rng = np.random.default_rng(rows * 1000 + cols16)
    sf = rng.integers(0, 256, size=(rows, cols16), dtype=np.uint8)
    blocked = L.to_blocked(torch.from_numpy(sf)).numpy()
    np.testing.assert_array_equal(blocked, oracle.to_blocked(sf))
    back = L.unblock(torch.from_numpy(blocked), rows, cols16 * 16).numpy()
    np.testing.assert_array_equal(back, sf)


def test_dq_fp4_matches_the_oracle_bit_for_bit():
    rng = np.random.default_rng(7)
    rows, cols = 256, 512
    codes = rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
    sf = rng.integers(0x08, 0x7F, size=(rows, cols // 16), dtype=np.uint8)  # finite, non-negative E4M3
    sf_flat = oracle.to_blocked(sf)
    ts = np.float32(0.3716)
    ours = L._dq_fp4(torch.from_numpy(codes), torch.from_numpy(sf_flat).view(torch.float8_e4m3fn), float(ts))
    ref = oracle.f32_to_bf16(oracle.dequant(codes, sf_flat, float(ts)))
    np.testing.assert_array_equal(ours.view(torch.int16).numpy().view(np.uint16), ref)


def test_fake_implementations_give_the_shapes_torch_compile_traces():
    with FakeTensorMode():
        m, k, n = 7, 256, 384
        x = torch.empty((m, k), dtype=torch.bfloat16)
        codes, scales, ts = torch.ops.quartet2.quant_rows(x)
        assert codes.shape == (m, k // 2) and codes.dtype == torch.uint8
        assert scales.shape == (128, k // 16) and scales.dtype == torch.float8_e4m3fn
        assert ts.shape == () and ts.dtype == torch.float32
        amax = torch.empty((), dtype=torch.float32)
        codes2, scales2, _ = torch.ops.quartet2.quant_rows_amax(x, amax)
        assert codes2.shape == codes.shape and scales2.shape == scales.shape
        w = torch.empty((n, k // 2), dtype=torch.uint8)
        w_sf = torch.empty((n, k // 16), dtype=torch.float8_e4m3fn)
        y = torch.ops.quartet2.fp4_mm_rows(codes, w, scales, w_sf, ts, None)
        assert y.shape == (m, n) and y.dtype == torch.bfloat16
        xp = torch.empty((128, k // 2), dtype=torch.uint8)
        xs = torch.empty((128, k // 16), dtype=torch.float8_e4m3fn)
        y2 = torch.ops.quartet2.fp4_mm(xp, w, xs, w_sf, ts)
        assert y2.shape == (128, n) and y2.dtype == torch.bfloat16
        a = torch.ops.quartet2.abs_max(x)
        assert a.shape == () and a.dtype == torch.float32
    assert I is not None and Q is not None  # importing them registers the ops
