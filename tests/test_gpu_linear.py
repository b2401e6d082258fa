"""Quartet_II_linear end to end on the GPU, restating the checks of the
reference's quartet2/test/test_linear.py: backward accuracy of a three-layer
ReLU network against fp32 gradients as the number of averaged backward passes
grows (effective bits and cosine floors of test_linear.py:95-129), forward
accuracy, autocast with fp32 weights, torch.compile of the forward; plus the
fusions of cloverlm_b200.fusion (shared-input Q/K/V forward, ReLU^2 with the
abs-max of its output)."""
import pytest
import torch

from cloverlm_b200 import _lib
from cloverlm_b200.fusion import relu2_abs_max, shared_input_forward
from cloverlm_b200.linear import Quartet_II_linear

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_watchdog():
    yield
    assert _lib.device_status() == 0, "a kernel wait timed out"


def _quality(res, ref):
    """(relative mean squared error, effective bits, cosine-like ratio) as the reference reports them."""
    res, ref = res.float(), ref.float()
    qe = (res - ref).pow(2).mean() / ref.pow(2).mean()
    return qe.item(), (-torch.log2(qe) / 2).item(), ((res.flatten() @ ref.flatten()) / (ref.flatten() @ ref.flatten())).item()


def _three_layers(H, seed):
    torch.manual_seed(seed)
    layers = [Quartet_II_linear(H, H, bias=False, device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    with torch.no_grad():
        for m in layers:
            m.weight /= H ** 0.5 * m.weight.std()
    return layers


def _run(layers, x, head, y, exact):
    h = x
    for i, m in enumerate(layers):
        h = m(h, disable_backward_quant=exact)
        if i < 2:
            h = torch.relu(h)
    return (h @ head - y).pow(2).mean()


@pytest.mark.parametrize("steps,floors", [(1, (1.9, 2.5, 3.8, 0.06)), (4, (2.9, 3.4, 4.0, 0.02)),
                                          (16, (3.9, 4.5, 6.4, 0.01)), (64, (4.9, 5.5, 7.5, 0.01)),
                                          (256, (5.9, 6.5, 8.1, 0.005))])
def test_backward_accuracy(steps, floors):
    B, T, H = 8, 16, 256
    layers = _three_layers(H, seed=42)
    torch.manual_seed(43)
    x = torch.randn(B, T, H, device="cuda", dtype=torch.bfloat16)
    y = torch.randn(B, T, 1, device="cuda", dtype=torch.bfloat16)
    head = torch.randn(H, 1, device="cuda", dtype=torch.bfloat16)
    _run(layers, x, head, y, exact=True).backward()
    ref = [m.weight.grad.float().clone() for m in layers]
    for m in layers:
        m.weight.grad = None
    loss = _run(layers, x, head, y, exact=False)
    acc = [torch.zeros_like(r) for r in ref]
    for _ in range(steps):
        loss.backward(retain_graph=True)
        for a, m in zip(acc, layers):
            a += m.weight.grad.float()
            m.weight.grad = None
    for i, (a, r) in enumerate(zip(acc, ref)):
        _, bits, cos = _quality(a / steps, r)
        assert bits >= floors[i], (i, bits)
        assert abs(cos - 1.0) < floors[3], (i, cos)


def test_forward_accuracy_and_autocast():
    """test_linear.py:136-153 (cos > 0.999, bits > 2.8), averaged over five seeds: one sample of the
    projection ratio moves by ~1e-3 from seed to seed."""
    q16, q32 = [], []
    for seed in range(5):
        torch.manual_seed(seed)
        w = Quartet_II_linear(128, 256, device="cuda", dtype=torch.bfloat16)
        x = torch.randn(1, 512, 128, device="cuda", dtype=torch.bfloat16)
        q16.append(_quality(w(x), x @ w.weight.T))
        w32 = Quartet_II_linear(128, 256, device="cuda")  # fp32 weights, bf16 compute under autocast
        x32 = torch.randn(1, 512, 128, device="cuda")
        with torch.autocast("cuda"):
            q32.append(_quality(w32(x32), x32 @ w32.weight.T))
    for q in (q16, q32):
        assert sum(c for _, _, c in q) / len(q) > 0.999, q
        assert min(b for _, b, _ in q) > 2.8, q


def test_compile_forward_fullgraph():
    w = Quartet_II_linear(128, 256, device="cuda", dtype=torch.bfloat16)
    x = torch.randn(1, 128, 128, device="cuda", dtype=torch.bfloat16)
    y = torch.compile(lambda t: w(t), fullgraph=True)(x)
    assert torch.equal(y, w(x))


def test_shared_input_qkv_forward_identical_backward_sound():
    torch.manual_seed(1)
    d, dkv = 512, 256
    lq = Quartet_II_linear(d, d, bias=False, device="cuda", dtype=torch.bfloat16)
    lk = Quartet_II_linear(d, dkv, bias=False, device="cuda", dtype=torch.bfloat16)
    lv = Quartet_II_linear(d, dkv, bias=False, device="cuda", dtype=torch.bfloat16)
    x = torch.randn(2, 128, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    q, k, v = shared_input_forward(x, [lq, lk, lv])
    assert torch.equal(q, lq(x)) and torch.equal(k, lk(x)) and torch.equal(v, lv(x))
    gq, gk, gv = (torch.randn_like(t) for t in (q, k, v))
    torch.autograd.backward([q, k, v], [gq, gk, gv])
    fused = [x.grad.clone()] + [m.weight.grad.clone() for m in (lq, lk, lv)]
    # exact (unquantized-backward) gradients of the same forward
    x.grad = None
    for m in (lq, lk, lv):
        m.weight.grad = None
    outs = [m(x, disable_backward_quant=True) for m in (lq, lk, lv)]
    torch.autograd.backward(outs, [gq, gk, gv])
    exact = [x.grad.clone()] + [m.weight.grad.clone() for m in (lq, lk, lv)]
    for f, e in zip(fused, exact):
        _, bits, cos = _quality(f, e)
        assert bits > 1.7 and abs(cos - 1.0) < 0.1, (bits, cos)


def test_relu2_abs_max_matches_torch():
    torch.manual_seed(2)
    a = torch.randn(3, 1000, 7, device="cuda", dtype=torch.bfloat16, requires_grad=True)  # 21000: a tail of 0
    a2 = torch.randn(4097, device="cuda", dtype=torch.bfloat16, requires_grad=True)       # tail of 1
    for t in (a, a2):
        y, amax = relu2_abs_max(t)
        ref = torch.relu(t.detach()) ** 2
        assert torch.equal(y, ref)
        assert amax.item() == ref.float().abs().max().item()
        g = torch.randn_like(y)
        (gy,) = torch.autograd.grad(y, t, g)
        torch.testing.assert_close(gy.float(), (g.float() * 2 * torch.relu(t.detach().float())), rtol=1e-2, atol=1e-2)


def test_mlp_relu2_fusion_feeds_the_next_layer_its_abs_max():
    torch.manual_seed(3)
    l1 = Quartet_II_linear(256, 512, bias=False, device="cuda", dtype=torch.bfloat16)
    l2 = Quartet_II_linear(512, 256, bias=False, device="cuda", dtype=torch.bfloat16)
    x = torch.randn(1, 256, 256, device="cuda", dtype=torch.bfloat16)
    a = l1(x)
    h, amax = relu2_abs_max(a)
    assert torch.equal(l2(h, input_abs_max=amax), l2(torch.relu(a) ** 2))


def test_training_step_captures_in_a_cuda_graph():
    """Forward + backward of a Quartet layer (quantizers, EDEN, requant, three NVFP4 GEMMs, the
    randomized Hadamard draw) records into one CUDA graph: no host synchronisation on the path.
    Replays give the eager forward bit for bit; each replay draws fresh Hadamard signs from torch's
    graph-safe generator (as eager steps do), so its gradients differ from the last replay's but
    stay as close to the exact gradients as eager ones."""
    torch.manual_seed(4)
    layer = Quartet_II_linear(256, 384, bias=False, device="cuda", dtype=torch.bfloat16)
    x = torch.randn(1, 256, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    dy = torch.randn(1, 256, 384, device="cuda", dtype=torch.bfloat16)
    layer(x, disable_backward_quant=True).backward(dy)
    exact = (x.grad.clone(), layer.weight.grad.clone())
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):  # warm-up on the capture stream
            layer.weight.grad = None
            x.grad = None
            layer(x).backward(dy)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    layer.weight.grad = None
    x.grad = None
    with torch.cuda.graph(g):
        y = layer(x)
        y.backward(dy)
    outs = []
    for _ in range(2):
        g.replay()
        torch.cuda.synchronize()
        outs.append((y.clone(), x.grad.clone(), layer.weight.grad.clone()))
    with torch.no_grad():
        eager = layer(x)
    assert torch.equal(outs[0][0], eager) and torch.equal(outs[1][0], eager)
    assert not torch.equal(outs[0][1], outs[1][1])  # a new random rotation per replay
    for _, gx, gw in outs:
        for got, ref in ((gx, exact[0]), (gw, exact[1])):
            _, bits, cos = _quality(got, ref)
            assert bits > 1.7 and abs(cos - 1.0) < 0.1, (bits, cos)


def test_weight_quantization_is_reused_only_while_the_weight_is_unchanged():
    """Quartet_II_linear keeps its weight's NVFP4 quantization between forwards (a step's
    micro-batches quantize each weight once); any update -- an in-place torch op, a
    QuartetAdamW step, a new abs-max from the optimizer -- makes the next forward
    quantize again, so outputs always equal a fresh quantization."""
    from cloverlm_b200.optim import QuartetAdamW
    torch.manual_seed(5)
    lin = Quartet_II_linear(256, 384, bias=False, device="cuda")
    x = torch.randn(1, 128, 256, device="cuda")

    def fresh():
        lin._weight_cache.clear()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            return lin(x)

    with torch.autocast("cuda", dtype=torch.bfloat16):
        y0 = lin(x)
        q0 = lin._weight_cache["q"]
        y1 = lin(x)
    assert lin._weight_cache["q"] is q0 and torch.equal(y0, y1)
    with torch.no_grad():
        lin.weight.mul_(1.5)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y2 = lin(x)
    assert lin._weight_cache["q"] is not q0 and torch.equal(y2, fresh())
    opt = QuartetAdamW(lin.parameters(), lr=1e-2)
    opt.attach(lin)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        lin(x).float().pow(2).mean().backward()
    q1 = lin._weight_cache["q"]
    opt.step()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y3 = lin(x)
    assert lin._weight_cache["q"] is not q1 and torch.equal(y3, fresh())


@pytest.mark.parametrize("M,K,H", [(2048, 512, 2560), (256, 256, 384)])
def test_fused_mlp_relu2_equals_the_unfused_chain(M, K, H):
    """fusion.mlp_relu2 (ReLU^2 + abs-max in the first GEMM's epilogue, the ReLU^2 gradient in
    the second linear's dgrad epilogue) is bit-identical to l2(relu2_abs_max(l1(x))), forward
    and backward, with the same random draws -- on shapes the 2-SM kernel takes (first case)
    and on shapes that use the GEMM + separate-kernel path (second)."""
    from cloverlm_b200.fusion import mlp_relu2, relu2_abs_max
    torch.manual_seed(9)
    l1 = Quartet_II_linear(K, H, bias=False, device="cuda")
    l2 = Quartet_II_linear(H, K, bias=False, device="cuda")
    x = torch.randn(1, M, K, device="cuda")
    grads = []
    for fused in (True, False):
        xi = x.clone().requires_grad_()
        for m in (l1, l2):
            m.weight.grad = None
        with torch.autocast("cuda", dtype=torch.bfloat16):
            if fused:
                z = mlp_relu2(xi, l1, l2)
            else:
                h, amax = relu2_abs_max(l1(xi))
                z = l2(h, input_abs_max=amax)
        torch.manual_seed(21)
        z.float().pow(2).mean().backward()
        grads.append((z.detach(), xi.grad, l1.weight.grad.clone(), l2.weight.grad.clone()))
    for a, b in zip(*grads):
        assert torch.equal(a, b)
