"""The vLLM plugin mirror (cloverlm_b200/vllm_plugin.py) of the reference's
src/evals/vllm_plugin/quartet2_quant.py: registration and weight creation on
the CPU, load-time quantization and apply against cloverlm_b200.inference on
the GPU.  Skipped where vLLM cannot be imported."""
import pytest
import torch

vllm_plugin = pytest.importorskip("cloverlm_b200.vllm_plugin", reason="vLLM not importable")


@pytest.fixture(autouse=True)
def _single_rank(monkeypatch):
    """vLLM parameters ask for their tensor-parallel rank; these tests run outside a vLLM engine."""
    import vllm.model_executor.parameter as vp
    monkeypatch.setattr(vp, "get_tensor_model_parallel_rank", lambda: 0)
    monkeypatch.setattr(vp, "get_tensor_model_parallel_world_size", lambda: 1)


def test_config_and_weight_creation():
    cfg = vllm_plugin.QuartetIIConfig.from_config({})
    assert cfg.get_name() == "quartet2"
    assert vllm_plugin.QuartetIIConfig.get_min_capability() == 100
    assert cfg.get_supported_act_dtypes() == [torch.bfloat16]
    assert cfg.get_quant_method(torch.nn.Linear(4, 4), "x") is None  # only vLLM LinearBase layers
    layer = torch.nn.Module()
    method = vllm_plugin.QuartetIILinearMethod(cfg)
    method.create_weights(layer, 256, [128, 200], 256, 328, torch.bfloat16, weight_loader=lambda *a: None)
    assert layer.weight.shape == (328, 256) and layer.weight.dtype == torch.bfloat16


@pytest.mark.gpu
def test_apply_matches_inference_module():
    from cloverlm_b200 import inference
    cfg = vllm_plugin.QuartetIIConfig()
    method = vllm_plugin.QuartetIILinearMethod(cfg)
    layer = torch.nn.Module()
    method.create_weights(layer, 512, [200], 512, 200, torch.bfloat16, weight_loader=lambda *a: None)
    g = torch.Generator().manual_seed(0)
    with torch.no_grad():
        layer.weight.data = (torch.randn(200, 512, generator=g) * 0.02).to(torch.bfloat16).cuda()
    method.process_weights_after_loading(layer)
    assert layer.w_pad == 56 and layer.weight_fp4.shape == (256, 256)
    x = torch.randn(3, 7, 512, generator=g).to(torch.bfloat16).cuda()
    bias = torch.randn(200, generator=g).to(torch.bfloat16).cuda()
    y = method.apply(layer, x, bias)
    ref = inference.apply(inference.prepare_weight(layer.weight.data), x, bias)
    assert y.shape == (3, 7, 200)
    assert ((y.float() - ref.float()).norm() / ref.float().norm()).item() < 4e-3
