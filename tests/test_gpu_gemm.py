"""GPU parity of the tcgen05 NVFP4 GEMM: within 1e-2 relative Frobenius error
of an fp32 matmul of the dequantized operands (the bar BASELINE.json sets)."""
import numpy as np
import pytest
import torch

import oracle
from cloverlm_b200 import _lib
from cloverlm_b200.linear import _dq_fp4, _fp4_mm
from cloverlm_b200.quant import NVFP4QuantMode, quant_fp4
from helpers import u8

pytestmark = pytest.mark.gpu

REL_FRO_TOL = 1e-2


@pytest.fixture(autouse=True)
def _no_watchdog():
    yield
    assert _lib.device_status() == 0, "a kernel wait timed out"


def _blocky(rows, cols, seed):
    """Values whose magnitude varies by 2^[-6, 6] per (row, 16-block): a scale
    factor applied to the wrong row or block shows up as a large error."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g)
    e = torch.randint(-6, 7, (rows, cols // 16), generator=g).float()
    x = x * torch.exp2(e).repeat_interleave(16, dim=1)
    return x.to(torch.bfloat16).cuda()


def _dq(q):
    return _dq_fp4(q.fp4, q.micro_scales, 1.0).float() * q.tensor_scale.float()


def _dq_exact(q):
    """fp32 dequantization without bf16 rounding (oracle)."""
    return torch.from_numpy(oracle.dequant(u8(q.fp4), u8(q.micro_scales).reshape(-1), q.tensor_scale.item())).cuda()


def _check(M, N, K, seed, blocky=False):
    mk = _blocky if blocky else (lambda r, c, s: torch.randn(r, c, generator=torch.Generator().manual_seed(s))
                                 .to(torch.bfloat16).cuda())
    a = mk(M, K, seed)
    b = mk(N, K, seed + 1)
    qa = quant_fp4(a, scale_override=1.0, mode=NVFP4QuantMode.FOUR_SIX)
    qb = quant_fp4(b, scale_override=1.0, mode=NVFP4QuantMode.FOUR_SIX)
    out = _fp4_mm(qa.fp4, qb.fp4, qa.micro_scales, qb.micro_scales, qa.tensor_scale * qb.tensor_scale)
    assert out.dtype == torch.bfloat16 and out.shape == (M, N)
    ref = _dq_exact(qa) @ _dq_exact(qb).T
    rel = ((out.float() - ref).norm() / ref.norm()).item()
    assert rel <= REL_FRO_TOL, rel
    return rel


@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (128, 256, 256), (256, 384, 384), (128, 128, 640),
                                   (384, 512, 1024), (1024, 3584, 3584), (256, 896, 3584),
                                   # 256x256-divisible shapes take the 2-SM (cta_group::2) kernel
                                   (256, 256, 128), (512, 768, 384), (768, 512, 640), (2048, 2048, 2048)])
def test_gemm_random(M, N, K):
    rel = _check(M, N, K, seed=M + N + K)
    assert rel < 5e-3  # bf16 output rounding dominates


@pytest.mark.parametrize("M,N,K", [(128, 256, 512), (512, 256, 768), (256, 128, 1152)])
def test_gemm_blocky_scales(M, N, K):
    _check(M, N, K, seed=7, blocky=True)


@pytest.mark.parametrize("M,N,K", [(4096, 3584, 3584), (2048, 2560, 1408), (2048, 2560, 8192), (2560, 2048, 640),
                                   (4096, 896, 3584), (896, 3584, 8192), (2176, 2688, 1408)])
def test_gemm_pair_kernel_shapes(M, N, K):
    """Shapes whose 256x256 tiles fill the SM pairs take the cta_group::2 kernel (ragged K tails included;
    M or N = 128 mod 256 leave a half tile read as zeros and clipped on store)."""
    rel = _check(M, N, K, seed=M + K)
    assert rel < 5e-3


def test_gemm_large_k_wgrad_shape():
    # wgrad-like: long contraction (tokens), small output
    _check(512, 512, 16384, seed=3)


def test_gemm_exact_small_integers():
    """Codes with unit scales and ts=1 make the product exact in fp32."""
    M, N, K = 256, 256, 512
    g = torch.Generator().manual_seed(0)
    ca = torch.randint(0, 256, (M, K // 2), generator=g, dtype=torch.uint8)
    cb = torch.randint(0, 256, (N, K // 2), generator=g, dtype=torch.uint8)
    # scale byte 0x38 = 1.0 in E4M3
    sa = torch.full((M * K // 16,), 0x38, dtype=torch.uint8)
    sb = torch.full((N * K // 16,), 0x38, dtype=torch.uint8)
    one = torch.ones((), device="cuda")
    out = _fp4_mm(ca.cuda(), cb.cuda(), sa.view(torch.float8_e4m3fn).cuda(), sb.view(torch.float8_e4m3fn).cuda(), one)
    A = torch.from_numpy(oracle.dequant(ca.numpy(), sa.numpy(), 1.0)).double()
    B = torch.from_numpy(oracle.dequant(cb.numpy(), sb.numpy(), 1.0)).double()
    ref = (A @ B.T).to(torch.bfloat16)
    assert torch.equal(out.cpu(), ref)


def test_gemm_rejects_bad_shapes():
    a = torch.zeros(128, 40, dtype=torch.uint8, device="cuda")
    s = torch.zeros(128 * 5, dtype=torch.uint8, device="cuda").view(torch.float8_e4m3fn)
    with pytest.raises(ValueError, match="K must be divisible by 64"):
        _fp4_mm(a, a, s, s, torch.ones((), device="cuda"))


@pytest.mark.gpu
def test_fp4_mma_peak_probe_runs_in_range():
    """The FP4 tensor-pipe probe completes with no watchdog trip, at a rate
    between a plausible floor and twice the nominal dense FP4 figure."""
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream(dev)
    _lib.call("q2b_fp4_mma_peak", 64, None, stream.cuda_stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    _lib.call("q2b_fp4_mma_peak", 1024, None, stream.cuda_stream)
    e1.record(stream)
    e1.synchronize()
    assert _lib.device_status() == 0
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    tflops = (sms // 2) * 1024 * 2.0 * 256 * 256 * 64 / (e0.elapsed_time(e1) / 1e3) / 1e12
    assert 2000 < tflops < 18000, tflops


@pytest.mark.parametrize("M,N,K", [(2048, 2560, 1408), (4096, 3584, 2048), (896, 3584, 4096), (384, 256, 640),
                                   (128, 896, 512), (896, 14336, 4096), (16384, 896, 1024)])
def test_gemm_fp32_output_is_the_unrounded_bf16_result(M, N, K):
    """q2b_gemm_nvfp4_f32 (fp32 D, for fp32 weight gradients) holds alpha * the fp32
    accumulator: rounded to bf16 it equals the bf16 GEMM bit for bit, and it is within
    the GEMM tolerance of the fp32 product of the dequantized operands."""
    from cloverlm_b200.linear import _fp4_mm_f32
    g = torch.Generator().manual_seed(M + N)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    b = torch.randn(N, K, generator=g).to(torch.bfloat16).cuda()
    qa = quant_fp4(a, scale_override=1.0, mode=NVFP4QuantMode.FOUR_SIX)
    qb = quant_fp4(b, scale_override=1.0, mode=NVFP4QuantMode.FOUR_SIX)
    alpha = qa.tensor_scale * qb.tensor_scale
    f32 = _fp4_mm_f32(qa.fp4, qb.fp4, qa.micro_scales, qb.micro_scales, alpha)
    bf = _fp4_mm(qa.fp4, qb.fp4, qa.micro_scales, qb.micro_scales, alpha)
    assert f32.dtype == torch.float32 and f32.shape == (M, N)
    assert torch.equal(f32.to(torch.bfloat16), bf)
    ref = _dq_exact(qa) @ _dq_exact(qb).T
    assert ((f32 - ref).norm() / ref.norm()).item() < 1e-4  # fp32 accumulation only


@pytest.mark.parametrize("M,N,K", [(2048, 2560, 1408), (4096, 3584, 896), (384, 256, 640), (2176, 2688, 1408)])
def test_gemm_add_accumulates_into_the_output(M, N, K):
    """q2b_gemm_nvfp4_add: D += bf16(alpha * A B^T), each element the bf16 sum of the old value and
    the bf16 GEMM result (TMA reductions on the 2-SM path, bf16 adds on the 1-SM path): equal to
    (D + _fp4_mm(...)) in bf16 up to one rounding step in at most 1e-3 of the elements."""
    from cloverlm_b200.linear import _fp4_mm_add
    g = torch.Generator().manual_seed(M + K)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    b = torch.randn(N, K, generator=g).to(torch.bfloat16).cuda()
    d0 = torch.randn(M, N, generator=g).to(torch.bfloat16).cuda()
    qa = quant_fp4(a, scale_override=1.0, mode=NVFP4QuantMode.FOUR_SIX)
    qb = quant_fp4(b, scale_override=1.0, mode=NVFP4QuantMode.FOUR_SIX)
    alpha = qa.tensor_scale * qb.tensor_scale
    got = _fp4_mm_add(d0.clone(), qa.fp4, qb.fp4, qa.micro_scales, qb.micro_scales, alpha)
    want = (d0.float() + _fp4_mm(qa.fp4, qb.fp4, qa.micro_scales, qb.micro_scales, alpha).float()).to(torch.bfloat16)
    diff = (got.view(torch.int16).int() - want.view(torch.int16).int()).abs()
    assert int(diff.max()) <= 1 and (diff != 0).float().mean().item() <= 1e-3
    assert _lib.device_status() == 0


@pytest.mark.parametrize("M,N,K", [(32768, 896, 3584), (896, 3584, 32768), (2176, 2688, 1408)])
def test_gemm_half_tiles_bit_identical_to_cudnn(M, N, K):
    """The pair kernel with a half last tile (the GQA K/V projections' 896 columns or rows) gives the
    same bits as the reference's GEMM (FlashInfer's cuDNN NVFP4 path)."""
    mm_fp4 = pytest.importorskip("flashinfer").mm_fp4
    from cloverlm_b200.quant import NVFP4QuantMode, quant_fp4
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = quant_fp4(torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16), scale_override=1.0,
                  mode=NVFP4QuantMode.FOUR_SIX)
    B = quant_fp4(torch.randn(N, K, device="cuda", generator=g).to(torch.bfloat16), scale_override=1.0,
                  mode=NVFP4QuantMode.FOUR_SIX)
    alpha = A.tensor_scale * B.tensor_scale
    ours = _fp4_mm(A.fp4, B.fp4, A.micro_scales, B.micro_scales, alpha)
    ref = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    mm_fp4(A.fp4, B.fp4.T, A.micro_scales.view(torch.float8_e4m3fn).view(-1, K // 16),
           B.micro_scales.view(torch.float8_e4m3fn).view(-1, K // 16).T, alpha, torch.bfloat16, ref, block_size=16,
           use_8x4_sf_layout=False, backend="cudnn", use_nvfp4=True)
    assert torch.equal(ours, ref)
