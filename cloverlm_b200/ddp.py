"""Data-parallel gradient exchange for Quartet-II layers.

The reference trains with torch DDP (fp32 gradient buckets, src/train.py:121,
src/models/utils_models.py:37).  Here the weight gradients of the NVFP4 GEMM
(bf16, straight from the wgrad epilogue) are all-reduced in bf16 as soon as
each one is ready -- from a post-accumulate-grad hook, asynchronously, on the
process group's own stream -- so the exchange of layer i overlaps the
backward of the layers after it.  With NCCL the reduction is AVG over NVLink;
with gloo (CPU tests) it is SUM followed by a division at wait().
"""
from __future__ import annotations

from typing import Iterable

import torch
import torch.distributed as dist


class GradAllReduce:
    def __init__(self, params: Iterable[torch.nn.Parameter], group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.native_avg = dist.get_backend(group) == "nccl"
        self._works: list[tuple[object, torch.Tensor]] = []
        self._hooks = [p.register_post_accumulate_grad_hook(self._on_grad) for p in params]

    def _on_grad(self, p: torch.nn.Parameter) -> None:
        g = p.grad
        if g is None:
            return
        op = dist.ReduceOp.AVG if self.native_avg else dist.ReduceOp.SUM
        work = dist.all_reduce(g, op=op, group=self.group, async_op=True)
        self._works.append((work, g))

    def wait(self) -> None:
        """Block the current stream until every launched all-reduce has finished."""
        for work, g in self._works:
            work.wait()
            if not self.native_avg:
                g.div_(self.world)
        self._works.clear()

    def close(self) -> None:
        self.wait()
        for h in self._hooks:
            h.remove()
        self._hooks.clear()
