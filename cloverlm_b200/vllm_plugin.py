"""vLLM quantization plugin "quartet2" on libq2b -- the drop-in for the
reference's src/evals/vllm_plugin/quartet2_quant.py (QuartetIIConfig,
QuartetIILinearMethod).  Importing this module registers the config under
the same name, so a model configured with ``quantization="quartet2"`` runs
its linears through ``cloverlm_b200.inference``: weights quantized once after
loading (four-over-six, rows padded to 128 as the reference does), activations
quantized without row padding, GEMM through the tcgen05 kernels.  Import this
module instead of the reference's plugin module (both register "quartet2").
"""
from __future__ import annotations

import torch
from vllm.model_executor.layers.linear import LinearBase, LinearMethodBase
from vllm.model_executor.layers.quantization import register_quantization_config
from vllm.model_executor.layers.quantization.base_config import QuantizationConfig, QuantizeMethodBase
from vllm.model_executor.parameter import ModelWeightParameter

from .inference import PreparedWeight, apply, prepare_weight


@register_quantization_config("quartet2")
class QuartetIIConfig(QuantizationConfig):
    """quartet2_quant.py:17-43: bf16 activations, Blackwell (SM 10.0) and up, no config files."""

    def get_name(self) -> str:
        return "quartet2"

    def get_supported_act_dtypes(self) -> list:
        return [torch.bfloat16]

    @classmethod
    def get_min_capability(cls) -> int:
        return 100

    @staticmethod
    def get_config_filenames() -> list[str]:
        return []

    @classmethod
    def from_config(cls, config: dict) -> "QuartetIIConfig":
        return cls()

    def get_quant_method(self, layer: torch.nn.Module, prefix: str) -> QuantizeMethodBase | None:
        if isinstance(layer, LinearBase):
            return QuartetIILinearMethod(self)
        return None


class QuartetIILinearMethod(LinearMethodBase):
    """quartet2_quant.py:45-140 with cloverlm_b200.inference behind it."""

    def __init__(self, config: QuartetIIConfig):
        self.config = config

    def create_weights(self, layer: torch.nn.Module, input_size_per_partition: int,
                       output_partition_sizes: list[int], input_size: int, output_size: int,
                       params_dtype: torch.dtype, **extra_weight_attrs):
        weight = ModelWeightParameter(
            data=torch.empty(sum(output_partition_sizes), input_size_per_partition, dtype=params_dtype),
            input_dim=1, output_dim=0, weight_loader=extra_weight_attrs.get("weight_loader"))
        layer.register_parameter("weight", weight)

    def process_weights_after_loading(self, layer: torch.nn.Module) -> None:
        p = prepare_weight(layer.weight.data)
        layer.weight_fp4 = p.fp4
        layer.weight_micro_scales = p.micro_scales
        layer.weight_tensor_scale = p.tensor_scale
        layer.w_pad = p.w_pad

    def apply(self, layer: torch.nn.Module, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        p = PreparedWeight(layer.weight_fp4, layer.weight_micro_scales, layer.weight_tensor_scale,
                           layer.weight.shape[0], layer.w_pad)
        return apply(p, x, bias)
