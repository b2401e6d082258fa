"""NVFP4 checkpoint format (reference src/evals/hf_model/convert_checkpoint.py
and modeling_cloverlm.py:16-37): key rules, safetensors round trip, the
dequantizing loader against the oracle (CPU), and on the GPU the converter
against quant_fp4 and the direct loader against inference.prepare_weight."""
import os

import numpy as np
import pytest
import torch

import oracle
from cloverlm_b200 import checkpoint as ck
from helpers import u8


def test_quantizable_keys_follow_the_reference_rule():
    assert ck.is_quantizable("transformer.blocks.0.mhsa.lq.weight")
    assert ck.is_quantizable("transformer.blocks.3.mlp.l1.weight")
    assert not ck.is_quantizable("transformer.emb.weight")
    assert not ck.is_quantizable("transformer.linear.weight")
    assert not ck.is_quantizable("transformer.blocks.0.mhsa.scale")


def _synthetic_triple(rows, cols, seed):
    g = torch.Generator().manual_seed(seed)
    codes = torch.randint(0, 256, (rows, cols // 2), generator=g, dtype=torch.uint8)
    scales = torch.randint(0x20, 0x50, (rows * cols // 16,), generator=g, dtype=torch.uint8)
    return (codes.view(torch.float4_e2m1fn_x2), scales.view(torch.float8_e4m3fn).reshape(rows, cols // 16),
            torch.tensor(0.37, dtype=torch.float32))


def test_safetensors_round_trip_and_cpu_dequant_matches_oracle(tmp_path):
    fp4, sc, ts = _synthetic_triple(256, 384, seed=1)
    sd = {"transformer.blocks.0.mlp.l1.weight": fp4, "transformer.blocks.0.mlp.l1.weight_scale": sc,
          "transformer.blocks.0.mlp.l1.weight_scale_2": ts, "transformer.emb.weight": torch.randn(8, 4)}
    path = os.path.join(tmp_path, "model.safetensors")
    ck.save(sd, path)
    raw = ck.load(path)
    assert ck.nvfp4_keys(raw) == ["transformer.blocks.0.mlp.l1.weight"]
    dense = ck.dequant_nvfp4_state_dict(raw, device="cpu")
    assert set(dense) == {"transformer.blocks.0.mlp.l1.weight", "transformer.emb.weight"}
    ref = oracle.dequant(u8(fp4.view(torch.uint8)), u8(sc.view(torch.uint8)).reshape(-1), float(ts))
    want = torch.from_numpy(ref).to(torch.bfloat16)
    assert torch.equal(dense["transformer.blocks.0.mlp.l1.weight"], want)
    assert dense["transformer.emb.weight"].dtype == torch.bfloat16


@pytest.mark.gpu
def test_converter_matches_quant_fp4_and_direct_loader_matches_prepare_weight():
    from cloverlm_b200 import inference
    from cloverlm_b200.quant import NVFP4QuantMode, quant_fp4
    g = torch.Generator().manual_seed(3)
    w = (torch.randn(384, 512, generator=g) * 0.02).to(torch.bfloat16)
    conv = ck.convert_state_dict({"blocks.0.mlp.l1.weight": w, "emb.weight": torch.randn(16, 8)})
    key = "transformer.blocks.0.mlp.l1.weight"
    q = quant_fp4(w.cuda(), scale_override=1.0, mode=NVFP4QuantMode.FOUR_SIX)
    assert torch.equal(conv[key].view(torch.uint8), q.fp4.cpu())
    assert torch.equal(conv[key + "_scale"].view(torch.uint8), q.micro_scales.view(torch.uint8).cpu())
    assert conv[key + "_scale_2"].item() == q.tensor_scale.item()
    direct = ck.prepared_weights(conv)[key]
    ref = inference.prepare_weight(w.cuda())
    x = torch.randn(5, 512, generator=g).to(torch.bfloat16).cuda()
    assert torch.equal(direct.fp4, ref.fp4) and torch.equal(direct.micro_scales.view(torch.uint8),
                                                            ref.micro_scales.view(torch.uint8))
    a, b = inference.apply(direct, x).float(), inference.apply(ref, x).float()
    assert ((a - b).norm() / b.norm()).item() < 4e-3  # same operands; split-K sums in any order
    # the dequantizing loader on the GPU equals the oracle's dequantization
    dense = ck.dequant_nvfp4_state_dict(conv)
    want = oracle.dequant(u8(q.fp4), u8(q.micro_scales).reshape(-1), q.tensor_scale.item())
    assert torch.equal(dense[key], torch.from_numpy(want).to(torch.bfloat16))
