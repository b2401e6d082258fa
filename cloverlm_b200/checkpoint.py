"""NVFP4 on-disk checkpoint format of the reference and its loaders.

Format (src/evals/hf_model/convert_checkpoint.py:35-56,194-207): every
quantizable 2-D block weight ``transformer.<key>`` (not the embedding, not
the output head, not norms; ``_is_quantizable``, :59-65) is stored as three
tensors

  ``<key>``          float4_e2m1fn_x2 [rows, cols/2]   E2M1 codes, low nibble = even column
  ``<key>_scale``    float8_e4m3fn    [rows, cols/16]  block scales in the blocked 128x4
                                                        layout the GEMM consumes, viewed 2-D
  ``<key>_scale_2``  float32          []               tensor scale

quantized four-over-six with the tensor scale from the weight's abs-max; all
other tensors are stored in the target dtype.  Rows and columns are padded to
multiples of 128 for quantization and the codes and scale matrix are then
sliced back to [rows, ...] exactly as the reference slices them (for the 4B
model every quantized weight is already a multiple of 128, so nothing is cut).

Loaders:
  * ``dequant_nvfp4_state_dict`` -- the reference's loader
    (src/evals/hf_model/modeling_cloverlm.py:16-37): codes * scales * ts -> bf16.
  * ``prepared_weights`` -- B200 addition: hands the stored codes and blocked
    scales straight to the inference GEMM (``cloverlm_b200.inference``) with no
    dequantize/requantize round trip; the result equals
    ``inference.prepare_weight`` of the original bf16 weight.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .inference import PreparedWeight
from .linear import _dq_fp4
from .quant import NVFP4QuantMode, quant_fp4

NVFP4_GROUP_SIZE = 16


def is_quantizable(key: str) -> bool:
    """convert_checkpoint.py:59-65: 2-D block weights, not the embedding or the output head."""
    if "emb.weight" in key or key.endswith("linear.weight"):
        return False
    return ".weight" in key


def quantize_weight_nvfp4(w: torch.Tensor, device: str | torch.device = "cuda"):
    """convert_checkpoint.py:35-56: (codes float4_e2m1fn_x2, scales float8_e4m3fn, tensor scale), on CPU."""
    assert w.ndim == 2
    rows, cols = w.shape
    pad_r, pad_c = (-rows) % 128, (-cols) % 128
    if pad_r or pad_c:
        w = F.pad(w, (0, pad_c, 0, pad_r))
    wd = w.to(device=device, dtype=torch.bfloat16).contiguous()
    q = quant_fp4(wd, scale_override=1.0, mode=NVFP4QuantMode.FOUR_SIX)
    fp4 = q.fp4[:rows, :cols // 2].view(torch.float4_e2m1fn_x2)
    scales = q.micro_scales[:rows, :cols // NVFP4_GROUP_SIZE]
    return fp4.cpu(), scales.cpu(), q.tensor_scale.cpu()


def convert_state_dict(state_dict: dict, dtype: torch.dtype = torch.bfloat16, nvfp4: bool = True,
                       device: str | torch.device = "cuda") -> dict:
    """convert_checkpoint.py:182-207: prefix keys with ``transformer.`` and quantize block weights."""
    out = {}
    for k, v in state_dict.items():
        hf_key = f"transformer.{k}"
        if nvfp4 and v.ndim == 2 and is_quantizable(hf_key):
            packed, scale, scale2 = quantize_weight_nvfp4(v, device)
            out[hf_key] = packed
            out[f"{hf_key}_scale"] = scale
            out[f"{hf_key}_scale_2"] = scale2
        else:
            out[hf_key] = v.clone().to(dtype)
    return out


def save(state_dict: dict, path: str) -> None:
    """Write a converted state dict as safetensors (convert_checkpoint.py:213-217)."""
    from safetensors.torch import save_file
    save_file(state_dict, path)


def load(path: str) -> dict:
    from safetensors.torch import load_file
    return load_file(path)


def nvfp4_keys(raw_sd: dict) -> list[str]:
    return sorted(k.removesuffix("_scale_2") for k in raw_sd if k.endswith("_scale_2"))


def dequant_nvfp4_state_dict(raw_sd: dict, dtype: torch.dtype = torch.bfloat16,
                             device: str | torch.device = "cuda") -> dict:
    """modeling_cloverlm.py:16-37: NVFP4 triples -> dense ``dtype`` tensors (on CPU)."""
    bases = set(nvfp4_keys(raw_sd))
    result = {}
    for key, tensor in raw_sd.items():
        if key.endswith(("_scale", "_scale_2")):
            continue
        if key in bases:
            fp4 = tensor.to(device)
            scales = raw_sd[f"{key}_scale"].to(device)
            ts = raw_sd[f"{key}_scale_2"].float().item()
            result[key] = _dq_fp4(fp4, scales, ts).to(dtype).cpu()
        else:
            result[key] = tensor.to(dtype) if tensor.is_floating_point() else tensor
    return result


def prepared_weights(raw_sd: dict, device: str | torch.device = "cuda") -> dict:
    """NVFP4 triples -> ``inference.PreparedWeight`` on ``device`` without dequantization.

    Needs rows and columns that are multiples of 128 (the stored scale matrix
    is then the whole blocked buffer); other shapes were cut by the converter
    and are rejected."""
    out = {}
    for key in nvfp4_keys(raw_sd):
        fp4 = raw_sd[key]
        rows, half = fp4.shape
        if rows % 128 or (half * 2) % 128:
            raise ValueError(f"{key}: [{rows}, {half * 2}] is not a multiple of 128; use dequant_nvfp4_state_dict")
        codes = fp4.view(torch.uint8).to(device).contiguous()
        scales = raw_sd[f"{key}_scale"].to(device).contiguous()
        ts = raw_sd[f"{key}_scale_2"].to(device=device, dtype=torch.float32).reshape(())
        out[key] = PreparedWeight(codes, scales, ts, rows, 0)
    return out
