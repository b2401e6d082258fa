"""The CloverLM block glue kernels and the model / training step built on them.

Each libq2b glue kernel is checked against a plain PyTorch fp32 restatement of the
reference's operations (src/models/transformer.py:39-74 RoPE, mlp.py:5-6 sphere norm,
transformer.py:380-395 residual RMSNorm, mlp.py:34-38 ReLU^2), forward and backward.
A two-block model is then checked against the same model with those operations done
by PyTorch, and a few optimizer steps must lower the loss."""
import math

import pytest
import torch
import torch.nn.functional as F

from cloverlm_b200 import _lib
from cloverlm_b200.model import (CloverLM, CloverLMConfig, _TiedHeadCrossEntropy, add_rmsnorm_amax, rope_sphere_norm,
                                 rope_table)

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_watchdog():
    yield
    assert _lib.device_status() == 0, "a kernel wait timed out"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def torch_rope_norm(x, table, scale, heads):
    """The reference's apply_rope (bf16 result) then sphere_norm, then * scale, in fp32."""
    x = x.float().unflatten(-1, (heads, 128))
    T = x.shape[-3]
    cos = table[:T, :, 0].repeat_interleave(2, dim=-1)[:, None, :]
    sin = table[:T, :, 1].repeat_interleave(2, dim=-1)[:, None, :]
    xr = torch.empty_like(x)
    xr[..., 0::2] = -x[..., 1::2]
    xr[..., 1::2] = x[..., 0::2]
    y = (x * cos + xr * sin).to(torch.bfloat16).float()
    n = F.normalize(y, dim=-1)
    return n if scale is None else n * scale.reshape(1, 1, heads, 1)


@pytest.mark.parametrize("heads,use_scale", [(28, True), (7, False), (2, True)])
def test_rope_norm_forward_and_backward_match_torch(heads, use_scale):
    torch.manual_seed(0)
    B, T = 2, 256
    table = rope_table(T, 128, 1024.0, "cuda")
    x = torch.randn(B, T, heads * 128, device="cuda").to(torch.bfloat16)
    scale = (torch.rand(1, heads, 1, 1, device="cuda") * 4 + 9) if use_scale else None
    out = rope_sphere_norm(x.requires_grad_(), table, scale.requires_grad_() if use_scale else None, heads, T)
    xr = x.detach().float().requires_grad_()
    sr = scale.detach().clone().requires_grad_() if use_scale else None
    ref = torch_rope_norm(xr, table, sr, heads)
    assert out.shape == (B, T, heads, 128) and out.dtype == torch.bfloat16
    assert _rel(out, ref) < 4e-3
    g = torch.randn_like(ref)
    out.backward(g.to(torch.bfloat16))
    ref.backward(g.to(torch.bfloat16).float())
    assert _rel(x.grad, xr.grad) < 1e-2
    if use_scale:
        # both sum dout * n over bf16-rounded normalized values (the reference's autograd
        # saves the bf16 normalized Q for the scale's gradient too)
        assert _rel(scale.grad, sr.grad) < 5e-3


def test_add_rmsnorm_amax_forward_and_backward_match_torch():
    torch.manual_seed(1)
    rows, d, eps = 300, 3584, float(torch.finfo(torch.float32).eps)
    x = torch.randn(rows, d, device="cuda", requires_grad=True)
    y = (torch.randn(rows, d, device="cuda") * 0.3).to(torch.bfloat16).requires_grad_()
    w = (1 + 0.1 * torch.randn(d, device="cuda")).requires_grad_()
    xo, xb, amax = add_rmsnorm_amax(x, y, w, eps)
    xr, yr, wr = x.detach().clone().requires_grad_(), y.detach().float().requires_grad_(), w.detach().clone().requires_grad_()
    ref = xr + F.rms_norm(yr, (d,), wr, eps)
    torch.testing.assert_close(xo, ref, rtol=1e-5, atol=1e-5)
    assert torch.equal(xb, xo.to(torch.bfloat16))
    assert amax.item() == xb.float().abs().max().item()
    g32 = torch.randn(rows, d, device="cuda")
    gb = torch.randn(rows, d, device="cuda").to(torch.bfloat16)
    torch.autograd.backward([xo, xb], [g32, gb])
    (ref * (g32 + gb.float())).sum().backward()
    assert _rel(x.grad, xr.grad) < 1e-6
    assert _rel(y.grad, yr.grad) < 1e-2
    assert _rel(w.grad, wr.grad) < 1e-4


def test_relu2_backward_kernel():
    from cloverlm_b200.fusion import relu2_abs_max
    a = torch.randn(64, 1024, device="cuda").to(torch.bfloat16).requires_grad_()
    h, amax = relu2_abs_max(a)
    g = torch.randn_like(h)
    h.backward(g)
    want = (2.0 * torch.relu(a.detach().float()) * g.float()).to(torch.bfloat16)
    assert torch.equal(a.grad, want)


def test_chunked_tied_head_cross_entropy_matches_torch():
    torch.manual_seed(2)
    n, d, V = 5000, 256, 1000
    h = torch.randn(n, d, device="cuda", requires_grad=True)
    w = (torch.randn(V, d, device="cuda") * 0.05).requires_grad_()
    t = torch.randint(0, V, (n,), device="cuda")
    loss = _TiedHeadCrossEntropy.apply(h, w, t)
    hr, wr = h.detach().clone().requires_grad_(), w.detach().clone().requires_grad_()
    ref = F.cross_entropy((hr.to(torch.bfloat16) @ wr.to(torch.bfloat16).T).float(), t)
    assert abs(loss.item() - ref.item()) < 1e-4 * ref.item()
    (2.0 * loss).backward()
    (2.0 * ref).backward()
    assert _rel(h.grad, hr.grad) < 1e-2 and _rel(w.grad, wr.grad) < 1e-2


TINY = CloverLMConfig(vocab_size=512, num_blocks=2, heads=2, d_head=128, ratio=2, exp_factor=4, context=256)


def _batch(cfg, B, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    ids = torch.randint(0, cfg.vocab_size, (B, cfg.context + 1), device="cuda", generator=g)
    return ids[:, :-1].contiguous(), ids[:, 1:].contiguous()


def _torch_glue_loss(model, ids, targets):
    """The same model with RoPE/norm, residual RMSNorms and the head in plain PyTorch."""
    from cloverlm_b200.fusion import relu2_abs_max, shared_input_forward
    cfg = model.cfg
    B, T = ids.shape
    table = model.rope(T, ids.device)
    x = F.embedding(ids, model.emb.weight)
    for blk in model.blocks:
        xb = x.to(torch.bfloat16)
        q, k, v = shared_input_forward(xb, [blk.lq, blk.lk, blk.lv])
        q = torch_rope_norm(q, table, blk.scale, cfg.heads).to(torch.bfloat16)
        k = torch_rope_norm(k, table, None, cfg.groups).to(torch.bfloat16)
        v = v.view(B, T, cfg.groups, cfg.d_head)
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                           is_causal=True, scale=1.0, enable_gqa=True)
        y = blk.lo(o.transpose(1, 2).reshape(B, T, cfg.d))
        x = x + F.rms_norm(y.float(), (cfg.d,), blk.att_norm, cfg.norm_eps)
        h, _ = relu2_abs_max(blk.l1(x.to(torch.bfloat16)))
        x = x + F.rms_norm(blk.l2(h).float(), (cfg.d,), blk.mlp_norm, cfg.norm_eps)
    with torch.autocast("cuda", enabled=False):
        hN = F.rms_norm(x, (cfg.d,), model.out_norm, cfg.norm_eps)
        logits = (hN.to(torch.bfloat16) @ model.emb.weight.to(torch.bfloat16).T).float()
        return F.cross_entropy(logits.reshape(-1, cfg.vocab_size), targets.reshape(-1))


def test_tiny_model_matches_torch_glue_and_backward_is_sound():
    torch.manual_seed(3)
    model = CloverLM(TINY, device="cuda")
    ids, targets = _batch(TINY, 2, seed=5)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        loss = model(ids, targets)
        ref = _torch_glue_loss(model, ids, targets)
    assert abs(loss.item() - math.log(TINY.vocab_size)) < 0.5
    assert abs(loss.item() - ref.item()) < 2e-3 * ref.item()
    torch.manual_seed(11)
    loss.backward()
    ours = {n: p.grad.clone() for n, p in model.named_parameters()}
    model.zero_grad(set_to_none=True)
    torch.manual_seed(11)
    ref.backward()
    for n, p in model.named_parameters():
        assert torch.isfinite(ours[n]).all(), n
        cos = F.cosine_similarity(ours[n].flatten().double(), p.grad.flatten().double(), dim=0).item()
        # same Hadamard and SR draws; the glue's rounding differences still move a few EDEN
        # decisions, and the embedding gradient collects them from every block
        assert cos > 0.95, (n, cos)


def test_training_steps_lower_the_loss():
    from cloverlm_b200.optim import QuartetAdamW
    from cloverlm_b200.train import TrainStep
    torch.manual_seed(4)
    model = CloverLM(TINY, device="cuda")
    opt = QuartetAdamW(model.parameters(), lr=3e-3, betas=(0.9, 0.95), eps=1e-6, weight_decay=0.0)
    step = TrainStep(model, opt)
    batches = [_batch(TINY, 2, seed=s) for s in (1, 2)]
    first = step(batches).item()
    for _ in range(25):
        last = step(batches).item()
    assert math.isfinite(last) and last < first - 1.0, (first, last)
    for blk in model.blocks:  # the optimizer keeps the Quartet layers' weight abs-max current
        for lin in (blk.lq, blk.lk, blk.lv, blk.lo, blk.l1, blk.l2):
            assert lin.weight_abs_max.item() == lin.weight.detach().to(torch.bfloat16).float().abs().max().item()


@pytest.mark.parametrize("rows,V", [(300, 1000), (64, 32768), (3, 8)])
def test_softmax_xent_kernel_matches_torch(rows, V):
    torch.manual_seed(5)
    x = (torch.randn(rows, V, device="cuda") * 4).to(torch.bfloat16)
    t = torch.randint(0, V, (rows,), device="cuda")
    inv_n = 1.0 / 777
    g = x.clone()
    row_loss = torch.empty(rows, dtype=torch.float32, device="cuda")
    _lib.call("q2b_softmax_xent_bf16", _lib.ptr(g), _lib.ptr(row_loss), _lib.ptr(t), inv_n, rows, V, _lib.stream_of(g))
    xf = x.float().requires_grad_()
    ref = F.cross_entropy(xf, t, reduction="none")
    torch.testing.assert_close(row_loss, ref.detach(), rtol=1e-5, atol=1e-5)
    (ref.sum() * inv_n).backward()
    want = xf.grad.to(torch.bfloat16)
    # the same fp32 formula up to the reduction order of the log-sum-exp: equal or one bf16 step apart
    diff = (g.float() - want.float()).abs()
    assert (diff <= want.float().abs() * 2 ** -7 + 1e-12).all()
