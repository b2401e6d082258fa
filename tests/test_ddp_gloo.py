"""Multi-process tests of the data-parallel gradient exchange
(cloverlm_b200/ddp.py) on CPU with the gloo backend, world size 2."""
import contextlib
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _worker_average(rank, world, port, q, mode):
    from cloverlm_b200.ddp import GradAllReduce
    _init(rank, world, port)
    torch.manual_seed(0)
    layers = [torch.nn.Linear(8, 4, bias=False).to(torch.bfloat16) for _ in range(3)]
    comm = GradAllReduce([l.weight for l in layers], mode=mode)
    for step in range(2):
        for l in layers:
            l.weight.grad = None
        # each rank its own tokens (data parallel), layers used one after another
        g = torch.Generator().manual_seed(100 * rank + step)
        x = torch.randn(16, 8, generator=g).to(torch.bfloat16)
        for l in layers:
            l(x).float().pow(2).sum().backward()
        comm.wait()
        q.put((rank, step, [l.weight.grad.float().clone() for l in layers]))
    comm.close()
    dist.destroy_process_group()


def _local_grads(rank, step):
    torch.manual_seed(0)
    layers = [torch.nn.Linear(8, 4, bias=False).to(torch.bfloat16) for _ in range(3)]
    g = torch.Generator().manual_seed(100 * rank + step)
    x = torch.randn(16, 8, generator=g).to(torch.bfloat16)
    out = []
    for l in layers:
        l(x).float().pow(2).sum().backward()
        out.append(l.weight.grad.float())
    return out


@pytest.mark.parametrize("mode", ["overlap", "flat"])
def test_grad_allreduce_averages_across_ranks(mode):
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_average, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world * 2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, step, grads in results:
        expect = [(a + b) / 2 for a, b in zip(_local_grads(0, step), _local_grads(1, step))]
        for g, e in zip(grads, expect):
            # bf16 gradients, bf16 reduction: compare at bf16 resolution
            torch.testing.assert_close(g, e.to(torch.bfloat16).float(), rtol=2e-2, atol=2e-2)


def _worker_failing(rank, world, port, q):
    from cloverlm_b200.ddp import GradAllReduce
    _init(rank, world, port, timeout_s=5)
    w = torch.nn.Parameter(torch.ones(4, dtype=torch.bfloat16))
    comm = GradAllReduce([w])
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()  # flush before the abrupt exit
        os._exit(3)  # a rank that dies between steps
    try:
        (w.float() * 2).sum().backward()
        comm.wait()
        q.put((rank, "no error"))
    except Exception as e:  # the surviving rank sees the failure on the host
        q.put((rank, type(e).__name__))


def test_rank_failure_surfaces_as_host_error_not_hang():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_failing, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    msgs = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert msgs[1] == "left"
    assert msgs[0] != "no error"


def _worker_accumulate(rank, world, port, q, bucket_mb, mode):
    from cloverlm_b200.ddp import GradAllReduce
    _init(rank, world, port)
    torch.manual_seed(0)
    layers = [torch.nn.Linear(8, 4, bias=False) for _ in range(3)]
    unused = torch.nn.Parameter(torch.ones(5))  # never receives a gradient
    comm = GradAllReduce([l.weight for l in layers] + [unused], mode=mode, bucket_mb=bucket_mb)
    for step in range(2):
        for l in layers:
            l.weight.grad = None
        for micro in range(2):  # the reference's accumulation loop (src/train.py:314-330)
            g = torch.Generator().manual_seed(1000 * rank + 10 * step + micro)
            x = torch.randn(16, 8, generator=g)
            ctx = comm.no_sync() if micro == 0 else contextlib.nullcontext()
            with ctx:
                for l in layers:
                    l(x).float().pow(2).sum().backward()
        comm.wait()
        q.put((rank, step, [l.weight.grad.clone() for l in layers],
               [comm.reduced_grad(l.weight).float().clone() for l in layers], comm.reduced_grad(unused).float()))
    comm.close()
    dist.destroy_process_group()


def _local_accumulated(rank, step):
    torch.manual_seed(0)
    layers = [torch.nn.Linear(8, 4, bias=False) for _ in range(3)]
    for micro in range(2):
        g = torch.Generator().manual_seed(1000 * rank + 10 * step + micro)
        x = torch.randn(16, 8, generator=g)
        for l in layers:
            l(x).float().pow(2).sum().backward()
    return [l.weight.grad for l in layers]


@pytest.mark.parametrize("bucket_mb,mode", [(256.0, "overlap"), (1e-4, "overlap"), (1e-4, "flat")])
def test_accumulation_under_no_sync_averages_the_summed_gradients(bucket_mb, mode):
    """Two micro-batches per step, the first under no_sync(): every rank ends with the
    average over ranks of its summed micro-batch gradients (bf16 exchange), whether all
    parameters share one bucket or each has its own; an unused parameter contributes zeros."""
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_accumulate, args=(r, world, port, q, bucket_mb, mode))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world * 2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, step, grads, reduced, unused in results:
        expect = [(a + b) / 2 for a, b in zip(_local_accumulated(0, step), _local_accumulated(1, step))]
        for g, r, e in zip(grads, reduced, expect):
            torch.testing.assert_close(r, e.to(torch.bfloat16).float(), rtol=2e-2, atol=2e-2)
            torch.testing.assert_close(g, r)  # copied back into .grad (fp32)
        assert torch.equal(unused, torch.zeros(5))


def _worker_double_backward(rank, world, port, q):
    from cloverlm_b200.ddp import GradAllReduce
    _init(rank, world, port)
    w = torch.nn.Parameter(torch.ones(4))
    comm = GradAllReduce([w])
    try:
        (w * 2).sum().backward()
        (w * 3).sum().backward()  # a second synchronizing backward without no_sync()
        q.put((rank, "no error"))
    except RuntimeError as e:
        q.put((rank, "no_sync" in str(e)))
    dist.destroy_process_group()


def test_second_sync_backward_without_no_sync_is_an_error():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_double_backward, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    msgs = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert msgs[0] is True and msgs[1] is True
