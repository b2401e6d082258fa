"""The allocation-free EDEN entry point, q2b_rht_eden_noalloc.

Some callers cannot allocate device memory: an operator running inside a host
framework that owns all device memory through its own pool and passes the
operator nothing but its inputs and outputs, or a latency-critical path that
cannot afford cudaMalloc's implicit synchronization.  For them libq2b keeps
the EDEN scratch (bf16 pre-rounding scales and the max word) in a static
device buffer of fixed size.  These tests call that entry point through the C
ABI and check it against q2b_rht_eden with caller-provided scratch, on two
calls in a row (the second call must not see the first call's leftovers).
The file is named to be collected last.
"""
import ctypes

import pytest
import torch

from cloverlm_b200 import _lib
from cloverlm_b200.linear import get_hadamard_matrix

pytestmark = pytest.mark.gpu

BWD_SO = (17 / 16) * 0.93
MAX_ELEMS = 16 * 2**20 * 8  # Q2B_NOALLOC_MAX_ELEMS in include/q2b.h


def _outputs(rows, cols, dev):
    return (torch.empty(rows, cols // 2, dtype=torch.uint8, device=dev),
            torch.empty(rows * cols // 16, dtype=torch.uint8, device=dev),
            torch.empty((), dtype=torch.float32, device=dev))


def _h16(seed, dev):
    g = torch.Generator().manual_seed(seed)
    H = get_hadamard_matrix(128, torch.bfloat16, "cpu")
    signs = (torch.randint(0, 2, (128,), generator=g) * 2 - 1).to(torch.bfloat16)
    return (H * signs[None, :])[:16].contiguous().to(dev)


def _run(x, h, seed, transpose, noalloc):
    M, N = x.shape
    rows, cols = (N, M) if transpose else (M, N)
    codes, sf, ts = _outputs(rows, cols, x.device)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    fp4_max = 6.0 / BWD_SO
    if noalloc:
        _lib.call("q2b_rht_eden_noalloc", _lib.ptr(codes), _lib.ptr(sf), _lib.ptr(ts), _lib.ptr(h), 16,
                  _lib.ptr(x), seed, fp4_max, 256.0, M, N, int(transpose), st)
    else:
        scratch = torch.empty(M * N // 16, dtype=torch.bfloat16, device=x.device)
        smax = torch.empty((), dtype=torch.int32, device=x.device)
        _lib.call("q2b_rht_eden", _lib.ptr(codes), _lib.ptr(sf), _lib.ptr(ts), _lib.ptr(scratch), _lib.ptr(smax),
                  _lib.ptr(h), 16, _lib.ptr(x), seed, fp4_max, 256.0, M, N, int(transpose), st)
    torch.cuda.synchronize()
    return codes, sf, ts


def test_noalloc_matches_allocating_entry_point_twice():
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(2024)
    # first call: a large-magnitude input in row orientation; second call: a
    # smaller, differently shaped input, transposed -- its max must not be
    # polluted by the first call's scales left in the shared buffer.
    cases = [
        (torch.randn(2048, 3584, device=dev, generator=g).mul_(50.0).to(torch.bfloat16), 11, False),
        (torch.randn(1024, 640, device=dev, generator=g).to(torch.bfloat16), 12, True),
    ]
    h = _h16(3, dev)
    for x, seed, transpose in cases:
        got = _run(x, h, seed, transpose, noalloc=True)
        ref = _run(x, h, seed, transpose, noalloc=False)
        # same kernels on the same inputs: equal bit for bit (tighter than the
        # 1e-4 byte-mismatch tolerance the oracle comparisons use)
        assert torch.equal(got[0], ref[0])
        assert torch.equal(got[1], ref[1])
        assert got[2].item() == ref[2].item()
    assert _lib.device_status() == 0


def test_noalloc_accepts_exactly_the_limit():
    """M*N == Q2B_NOALLOC_MAX_ELEMS fills the whole scale area; the max word just past it
    must stay separate (bit-identical to the allocating entry point)."""
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(16384, 8192, device=dev, generator=g).to(torch.bfloat16)
    assert x.numel() == MAX_ELEMS
    h = _h16(5, dev)
    for transpose in (False, True):
        got = _run(x, h, 21, transpose, noalloc=True)
        ref = _run(x, h, 21, transpose, noalloc=False)
        assert torch.equal(got[0], ref[0])
        assert torch.equal(got[1], ref[1])
        assert got[2].item() == ref[2].item()
    assert _lib.device_status() == 0


def test_noalloc_rejects_inputs_beyond_the_static_limit():
    dev = torch.device("cuda:0")
    x = torch.empty(128, 128, dtype=torch.bfloat16, device=dev)  # pointer only; never read
    h = _h16(0, dev)
    codes, sf, ts = _outputs(128, 128, dev)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # one 128x128 tile past the limit, and far past it
    for rows, cols in ((MAX_ELEMS // 128 + 128, 128), (MAX_ELEMS // 8192 + 2, 8192)):
        if rows % 128:
            rows += 128 - rows % 128
        with pytest.raises(ValueError, match="exceeds the static scratch limit"):
            _lib.call("q2b_rht_eden_noalloc", _lib.ptr(codes), _lib.ptr(sf), _lib.ptr(ts), _lib.ptr(h), 16,
                      _lib.ptr(x), 1, 6.0, 256.0, rows, cols, 0, st)
