"""Fused AdamW + post-step abs-max (q2b_adamw_step, cloverlm_b200.optim.QuartetAdamW)
against torch.optim.AdamW(fused=True), the reference's optimizer
(src/models/parametrizations.py:311), and the abs-max its hook computes
(quartet2/python/quartet2/linear.py:259-270)."""
import ctypes

import pytest
import torch

from cloverlm_b200 import _lib
from cloverlm_b200.linear import Quartet_II_linear
from cloverlm_b200.optim import QuartetAdamW

pytestmark = pytest.mark.gpu

HP = dict(lr=3e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)


def _pair(shape, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randn(shape, device="cuda", generator=g) * 0.02
    a = torch.nn.Parameter(w.clone())
    b = torch.nn.Parameter(w.clone())
    return a, b, g


@pytest.mark.parametrize("grad_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(384, 512), (1001,), (3, 7)])
def test_matches_torch_fused_adamw(shape, grad_dtype):
    a, b, g = _pair(shape, seed=sum(shape))
    ours = QuartetAdamW([a], **HP)
    ref = torch.optim.AdamW([b], fused=True, **HP)
    if grad_dtype != torch.float32:
        a.grad_dtype = None  # bf16 gradients of fp32 weights, as the NVFP4 wgrad GEMM produces them
    for _ in range(4):
        grad = (torch.randn(shape, device="cuda", generator=g) * 0.1).to(grad_dtype)
        a.grad = grad.clone()
        b.grad = grad.float().clone()
        ours.step()
        ref.step()
    torch.testing.assert_close(a.detach(), b.detach(), rtol=2e-6, atol=1e-8)
    torch.testing.assert_close(ours.state[a]["exp_avg"], ref.state[b]["exp_avg"], rtol=2e-6, atol=1e-9)
    torch.testing.assert_close(ours.state[a]["exp_avg_sq"], ref.state[b]["exp_avg_sq"], rtol=2e-6, atol=1e-12)


def test_abs_max_and_bf16_copy_in_the_same_pass_any_alignment():
    n = 4099
    base = torch.randn(n + 3, device="cuda") * 0.05
    for off in (0, 1, 3):  # offsets 1 and 3 take the scalar path
        w = base[off:off + n].clone() if off == 0 else base.clone()[off:off + n]
        m = torch.zeros_like(base)[off:off + n]
        v = torch.zeros_like(base)[off:off + n]
        grad = torch.randn(n, device="cuda")
        wb = torch.empty(n + 3, dtype=torch.bfloat16, device="cuda")[off:off + n]
        amax = torch.full((), 123.0, device="cuda")
        w_ref = w.clone()
        _lib.call("q2b_adamw_step", _lib.ptr(w), _lib.ptr(m), _lib.ptr(v), _lib.ptr(grad), 0, n, 1e-2, 0.9, 0.99,
                  1e-8, 0.0, 1, _lib.ptr(wb), _lib.ptr(amax), _lib.stream_of(w))
        torch.cuda.synchronize()
        assert amax.item() == w.to(torch.bfloat16).abs().max().item()
        assert torch.equal(wb, w.to(torch.bfloat16))
        # step 1 with zero weight decay: w - lr * g / (|g| + eps) (bias corrections cancel)
        torch.testing.assert_close(w, w_ref - 1e-2 * grad / (grad.abs() + 1e-8), rtol=1e-6, atol=1e-7)


def test_attach_replaces_the_optimizer_hook():
    torch.manual_seed(0)
    model = torch.nn.Sequential(Quartet_II_linear(256, 384, bias=False, device="cuda"),
                                Quartet_II_linear(384, 256, bias=False, device="cuda"))
    opt = QuartetAdamW(model.parameters(), **HP)
    assert opt.attach(model) == 2
    x = torch.randn(1, 256, 256, device="cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = model(x)
    y.float().pow(2).mean().backward()
    opt.step()
    for layer in model:
        assert layer.weight_abs_max is not None
        # the reference hook's value: abs-max of the bf16 weight (linear.py:259-270)
        assert layer.weight_abs_max.item() == layer.weight.detach().to(torch.bfloat16).abs().max().item()
    # the next forward uses the cached value
    with torch.autocast("cuda", dtype=torch.bfloat16):
        model(x).float().sum().backward()
    assert _lib.device_status() == 0


def test_register_optimizer_hook_caches_the_bf16_weight_abs_max():
    """register_optimizer_hook (reference linear.py:259-270): after every optimizer step each
    Quartet layer the optimizer updates holds abs_max of its bf16 weight, and the next forward
    uses it (its output equals a forward that computes the abs-max itself)."""
    from cloverlm_b200.linear import register_optimizer_hook
    torch.manual_seed(1)
    model = torch.nn.Sequential(Quartet_II_linear(256, 384, bias=False, device="cuda"),
                                Quartet_II_linear(384, 256, bias=False, device="cuda"))
    other = Quartet_II_linear(256, 128, bias=False, device="cuda")  # not in the optimizer: untouched
    opt = torch.optim.AdamW(model.parameters(), lr=1e-2)
    handle = register_optimizer_hook(torch.nn.ModuleList([model, other]), opt)
    x = torch.randn(1, 128, 256, device="cuda")
    for _ in range(2):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            model(x).float().pow(2).mean().backward()
        opt.step()
        opt.zero_grad()
        for layer in model:
            want = layer.weight.detach().to(torch.bfloat16).float().abs().max()
            assert layer.weight_abs_max.item() == want.item()
        assert other.weight_abs_max is None
    with torch.autocast("cuda", dtype=torch.bfloat16):
        cached = model[0](x)
        model[0].weight_abs_max = None
        fresh = model[0](x)
    assert torch.equal(cached, fresh)
    handle.remove()
    opt.step()
    assert _lib.device_status() == 0
