"""One data-parallel training step of a Quartet-II model, as the reference runs it.

The reference's loop (src/train.py:314-345): the step's batch is split into
micro-batches; all but the last run their backward under DDP's ``no_sync()``
(gradients accumulate locally), each loss is scaled by 1/accumulation, the
last backward exchanges the gradients (DDP buckets,
src/models/utils_models.py:37), the step loss is all-reduced with AVG, and the
optimizer steps.  Here the exchange is ``ddp.GradAllReduce`` (bf16 buckets
all-reduced by NCCL as they fill during the last backward) and the optimizer is
``optim.QuartetAdamW``, which reads the averaged bf16 gradients straight from
the buckets and hands every Quartet layer its post-step weight abs-max.
Autocast is bf16 as in the reference (its GradScaler is disabled for bf16).
"""
from __future__ import annotations

import contextlib

import torch
import torch.distributed as dist

from .ddp import GradAllReduce
from .optim import QuartetAdamW


class TrainStep:
    def __init__(self, model: torch.nn.Module, optimizer: QuartetAdamW, comm: GradAllReduce | None = None):
        self.model = model
        self.opt = optimizer
        self.comm = comm
        optimizer.attach(model)

    def __call__(self, micro_batches) -> torch.Tensor:
        """micro_batches: [(ids, targets), ...] on the device.  Returns the step's mean loss
        (0-d fp32 device tensor, averaged over micro-batches and ranks)."""
        n = len(micro_batches)
        total = torch.zeros((), dtype=torch.float32, device=micro_batches[0][0].device)
        for i, (ids, targets) in enumerate(micro_batches):
            sync = self.comm is None or i == n - 1
            ctx = contextlib.nullcontext() if sync else self.comm.no_sync()
            with ctx:
                with torch.autocast("cuda", dtype=torch.bfloat16):
                    loss = self.model(ids, targets) / n
                total += loss.detach()
                loss.backward()
        grad_of = None
        if self.comm is not None:
            self.comm.wait()
            if dist.get_backend(self.comm.group) == "nccl":
                dist.all_reduce(total, op=dist.ReduceOp.AVG, group=self.comm.group)
            else:
                dist.all_reduce(total, group=self.comm.group)
                total /= self.comm.world
            if not self.comm.copy_back:
                grad_of = self.comm.reduced_grad
        self.opt.step(grad_of=grad_of)
        self.opt.zero_grad(set_to_none=True)
        return total
