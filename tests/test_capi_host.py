"""CPU tests of the boundary: libq2b.so loads without a GPU, exports every
entry point include/q2b.h declares, and rejects bad arguments with the
reference's messages before touching the device."""
import ctypes
import os
import re

import pytest
import torch

from cloverlm_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "q2b.h")).read()
    return sorted(set(re.findall(r"^(?:int|int64_t|const char\*)\s+(q2b_\w+)\(", text, re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 9
    for n in names:
        assert hasattr(lib, n), n
    assert set(_lib.SIGNATURES) <= set(names)
    # every int-returning entry point has its argument types declared for ctypes
    # (an undeclared one would pass 64-bit sizes and floats wrongly)
    assert set(names) - {"q2b_last_error", "q2b_version", "q2b_gemm_workspace_bytes"} <= set(_lib.SIGNATURES)
    assert lib.q2b_version() >= 100


FAKE = ctypes.c_void_p(0x10000)  # aligned, never dereferenced: validation fails first


@pytest.mark.parametrize("cols,msg", [(64, "cols must be divisible by 128"), (100, "cols must be divisible by 128")])
def test_quant_fwd_rejects_bad_cols(cols, msg):
    with pytest.raises(ValueError, match=msg):
        _lib.call("q2b_quant_fwd", FAKE, FAKE, FAKE, FAKE, FAKE, 1.0, 128, cols, 1, None)


def test_quant_fwd_rejects_bad_rows_mode_and_pointers():
    with pytest.raises(ValueError, match="rows must be divisible by 128"):
        _lib.call("q2b_quant_fwd", FAKE, FAKE, FAKE, FAKE, FAKE, 1.0, 100, 128, 1, None)
    with pytest.raises(ValueError, match="unknown mode"):
        _lib.call("q2b_quant_fwd", FAKE, FAKE, FAKE, FAKE, FAKE, 1.0, 128, 128, 7, None)
    with pytest.raises(ValueError, match="not aligned to 16 bytes"):
        _lib.call("q2b_quant_fwd", ctypes.c_void_p(0x10004), FAKE, FAKE, FAKE, FAKE, 1.0, 128, 128, 1, None)
    with pytest.raises(ValueError, match="is null"):
        _lib.call("q2b_quant_fwd", FAKE, FAKE, None, FAKE, FAKE, 1.0, 128, 128, 1, None)


def test_eden_and_requant_reject_bad_arguments():
    with pytest.raises(ValueError, match="rows must be divisible by 128"):
        _lib.call("q2b_rht_eden", FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 16, FAKE, 1, 6.0, 256.0, 96, 128, 0, None)
    with pytest.raises(ValueError, match="16 \\(Hadamard slice\\) or 128 rows"):
        _lib.call("q2b_rht_eden", FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 32, FAKE, 1, 6.0, 256.0, 128, 128, 0, None)
    with pytest.raises(ValueError, match="cols must be divisible by 128"):
        _lib.call("q2b_rht_requant", FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 16, FAKE, FAKE, FAKE, 1, 6.0, 256.0,
                  128, 200, None)
    with pytest.raises(ValueError, match="distinct max words"):
        _lib.call("q2b_rht_eden_dual", FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 16, FAKE,
                  1, 2, 6.0, 256.0, 128, 128, None)


def test_gemm_rejects_bad_shapes():
    with pytest.raises(ValueError, match="M must be divisible by 128"):
        _lib.call("q2b_gemm_nvfp4", FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 100, 128, 128, None)
    with pytest.raises(ValueError, match="K must be divisible by 64"):
        _lib.call("q2b_gemm_nvfp4", FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 128, 128, 80, None)


def test_ragged_entry_points_reject_bad_arguments():
    with pytest.raises(ValueError, match="rows must be positive"):
        _lib.call("q2b_quant_fwd_ragged", FAKE, FAKE, FAKE, FAKE, FAKE, 1.0, 0, 128, 1, None)
    with pytest.raises(ValueError, match="cols must be divisible by 128"):
        _lib.call("q2b_quant_fwd_ragged", FAKE, FAKE, FAKE, FAKE, FAKE, 1.0, 3, 200, 1, None)
    with pytest.raises(ValueError, match="N must be divisible by 128"):
        _lib.call("q2b_gemm_nvfp4_ex", FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, None, 1, 100, 128, None, 0, None)
    with pytest.raises(ValueError, match="workspace must be 16-byte aligned"):
        _lib.call("q2b_gemm_nvfp4_ex", FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, None, 1, 128, 128, ctypes.c_void_p(0x10004),
                  64, None)
    with pytest.raises(ValueError, match="rows must be positive"):
        _lib.call("q2b_quant_rows_fused", FAKE, FAKE, FAKE, FAKE, 1.0, 0, 128, 1, None)
    with pytest.raises(ValueError, match="unknown mode"):
        _lib.call("q2b_quant_rows_fused", FAKE, FAKE, FAKE, FAKE, 1.0, 1, 128, 5, None)
    # no split plan for a shape the GEMM rejects
    assert _lib.load().q2b_gemm_workspace_bytes(1, 100, 128) == 0


def test_adamw_rejects_bad_arguments():
    with pytest.raises(ValueError, match="n must be positive"):
        _lib.call("q2b_adamw_step", FAKE, FAKE, FAKE, FAKE, 0, 0, 1e-3, 0.9, 0.99, 1e-8, 0.0, 1, None, None, None)
    with pytest.raises(ValueError, match="step must be >= 1"):
        _lib.call("q2b_adamw_step", FAKE, FAKE, FAKE, FAKE, 0, 8, 1e-3, 0.9, 0.99, 1e-8, 0.0, 0, None, None, None)
    with pytest.raises(ValueError, match="betas"):
        _lib.call("q2b_adamw_step", FAKE, FAKE, FAKE, FAKE, 0, 8, 1e-3, 1.0, 0.99, 1e-8, 0.0, 1, None, None, None)
    with pytest.raises(ValueError, match="is null"):
        _lib.call("q2b_adamw_step", None, FAKE, FAKE, FAKE, 0, 8, 1e-3, 0.9, 0.99, 1e-8, 0.0, 1, None, None, None)


def test_fp4_mma_peak_rejects_bad_arguments():
    with pytest.raises(ValueError, match="multiple of 4"):
        _lib.call("q2b_fp4_mma_peak", 6, None, None)
    with pytest.raises(ValueError, match="multiple of 4"):
        _lib.call("q2b_fp4_mma_peak", 0, None, None)


def test_last_error_is_thread_local_text():
    with pytest.raises(ValueError):
        _lib.call("q2b_gemm_nvfp4", FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 100, 128, 128, None)
    assert b"divisible" in _lib.load().q2b_last_error()


def test_python_layer_asserts_like_the_reference():
    from cloverlm_b200.quant import quant_fp4
    with pytest.raises(AssertionError):
        quant_fp4(torch.zeros(128, 128, dtype=torch.float32), scale_override=1.0)  # dtype
    with pytest.raises(AssertionError):
        quant_fp4(torch.zeros(128, 128, dtype=torch.bfloat16), scale_override=1.0)  # not CUDA


def test_no_cuda_means_loud_failure():
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    from cloverlm_b200.linear import _fp4_mm
    with pytest.raises((ValueError, RuntimeError)):
        _fp4_mm(torch.zeros(128, 64, dtype=torch.uint8), torch.zeros(128, 64, dtype=torch.uint8),
                torch.zeros(1024, dtype=torch.uint8), torch.zeros(1024, dtype=torch.uint8), torch.ones(()))
