"""Data-parallel gradient exchange for Quartet-II training.

The reference trains with torch DDP (fp32 gradient buckets, src/train.py:121,
src/models/utils_models.py:37) and accumulates micro-batches under
``no_sync()`` (src/train.py:314-330).  Here the gradients are exchanged in
bf16 (NCCL AVG over NVLink) through flat buckets:

* parameters are assigned to buckets of about ``bucket_mb`` MB in the reverse
  of the order given (the order their gradients become ready in backward);
* on a synchronizing backward, a post-accumulate-grad hook packs each
  finished gradient into its bucket slot (bf16) and, once every slot of a
  bucket is filled, launches that bucket's all-reduce asynchronously, so the
  exchange overlaps the rest of the backward (``mode="overlap"``);
  ``mode="flat"`` packs the same way but reduces everything in one call from
  ``wait()`` (no NCCL kernel beside the backward's kernels);
* inside ``no_sync()`` the hooks do nothing: gradients accumulate locally in
  ``.grad`` and only the last micro-batch's backward exchanges them;
* ``wait()`` makes the current stream wait for every bucket, then (with
  ``copy_back=True``, the default) writes the averaged gradient back into
  each ``.grad``; an optimizer that reads bf16 gradients can instead take
  ``reduced_grad(p)`` and skip that pass.

With NCCL the reduction is AVG; with gloo (CPU tests) it is SUM followed by a
division.  Parameters whose gradient never arrives in a step contribute
zeros.
"""
from __future__ import annotations

import contextlib
from typing import Iterable

import torch
import torch.distributed as dist


class GradAllReduce:
    def __init__(self, params: Iterable[torch.nn.Parameter], group=None, mode: str = "overlap",
                 bucket_mb: float = 256.0, copy_back: bool = True):
        if mode not in ("overlap", "flat"):
            raise ValueError(f"unknown mode {mode!r}")
        self.group = group
        self.mode = mode
        self.copy_back = copy_back
        self.world = dist.get_world_size(group)
        self.native_avg = dist.get_backend(group) == "nccl"
        self.params = [p for p in params if p.requires_grad]
        # buckets in gradient-ready order (reverse of the order given)
        limit = float("inf") if mode == "flat" else bucket_mb * (1 << 20) / 2  # elements of bf16
        self.buckets: list[list[torch.nn.Parameter]] = []
        cur, size = [], 0
        for p in reversed(self.params):
            if cur and size + p.numel() > limit:
                self.buckets.append(cur)
                cur, size = [], 0
            cur.append(p)
            size += p.numel()
        if cur:
            self.buckets.append(cur)
        self._where: dict[int, tuple[int, int]] = {}
        for b, ps in enumerate(self.buckets):
            off = 0
            for p in ps:
                self._where[id(p)] = (b, off)
                off += p.numel()
        self._flat: list[torch.Tensor | None] = [None] * len(self.buckets)
        self._pending = [0] * len(self.buckets)
        self._filled: list[set] = [set() for _ in self.buckets]
        self._launched = [False] * len(self.buckets)
        self._works: list[tuple[object, int]] = []
        self._active = False
        self._sync_enabled = True
        self._hooks = [p.register_post_accumulate_grad_hook(self._on_grad) for p in self.params]

    # ------------------------------------------------------------ buckets
    def _bucket(self, b: int, device) -> torch.Tensor:
        if self._flat[b] is None:
            n = sum(p.numel() for p in self.buckets[b])
            self._flat[b] = torch.empty(n, dtype=torch.bfloat16, device=device)
        return self._flat[b]

    def _slot(self, p: torch.nn.Parameter) -> torch.Tensor:
        b, off = self._where[id(p)]
        return self._bucket(b, p.device)[off:off + p.numel()].view_as(p)

    def reduced_grad(self, p: torch.nn.Parameter) -> torch.Tensor:
        """The averaged bf16 gradient of `p` (valid after wait())."""
        return self._slot(p)

    def _launch(self, b: int) -> None:
        op = dist.ReduceOp.AVG if self.native_avg else dist.ReduceOp.SUM
        work = dist.all_reduce(self._flat[b], op=op, group=self.group, async_op=True)
        self._works.append((work, b))
        self._launched[b] = True

    def _on_grad(self, p: torch.nn.Parameter) -> None:
        if not self._sync_enabled or p.grad is None:
            return
        b, _ = self._where[id(p)]
        if id(p) in self._filled[b]:
            raise RuntimeError("a parameter's gradient was produced twice in one synchronizing backward; "
                               "run earlier micro-batches under no_sync()")
        self._slot(p).copy_(p.grad)
        self._filled[b].add(id(p))
        self._active = True
        if self.mode == "overlap" and len(self._filled[b]) == len(self.buckets[b]):
            self._launch(b)

    @contextlib.contextmanager
    def no_sync(self):
        """Backward passes inside accumulate into .grad without any exchange."""
        prev = self._sync_enabled
        self._sync_enabled = False
        try:
            yield
        finally:
            self._sync_enabled = prev

    def wait(self) -> None:
        """Make the current stream wait until every gradient of this step is averaged."""
        if not self._active:
            return
        for b, ps in enumerate(self.buckets):
            if self._launched[b]:
                continue
            for p in ps:  # parameters without a gradient this step contribute zeros
                if id(p) not in self._filled[b]:
                    self._slot(p).zero_()
            self._launch(b)
        for work, b in self._works:
            work.wait()
            if not self.native_avg:
                self._flat[b].div_(self.world)
        if self.copy_back:
            for p in self.params:
                if p.grad is not None:
                    p.grad.copy_(self._slot(p))
        self._works.clear()
        self._filled = [set() for _ in self.buckets]
        self._launched = [False] * len(self.buckets)
        self._active = False

    def close(self) -> None:
        self.wait()
        for h in self._hooks:
            h.remove()
        self._hooks.clear()
