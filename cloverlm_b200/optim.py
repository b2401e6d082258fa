"""AdamW whose step also yields each Quartet weight's post-step abs-max.

The reference trains hidden weights with ``torch.optim.AdamW(fused=True)``
(src/models/parametrizations.py:311) and registers ``register_optimizer_hook``
(quartet2/python/quartet2/linear.py:259-270), which after every step re-reads
each Quartet weight to cache ``weight_abs_max`` for the next forward.
``QuartetAdamW`` runs one libq2b kernel per parameter (``q2b_adamw_step``)
that updates the fp32 weight and both moments and reduces max|bf16(w_new)| in the
same pass; ``attach(model)`` routes that value into the Quartet layers, so the
hook's extra read of every weight disappears.  Each step also polls the
library's device watchdog (asynchronously, see ``_lib.WatchdogMonitor``), so a
kernel wait that timed out raises on the training path within a step.  The update is torch's AdamW
(decoupled weight decay) in the operation order of its fused CUDA kernel.
"""
from __future__ import annotations

import torch

from . import _lib
from .linear import Quartet_II_linear


class QuartetAdamW(torch.optim.Optimizer):
    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 1e-2, check_watchdog: bool = True):
        if lr < 0.0 or eps < 0.0 or weight_decay < 0.0:
            raise ValueError("lr, eps and weight_decay must be non-negative")
        if not (0.0 <= betas[0] < 1.0 and 0.0 <= betas[1] < 1.0):
            raise ValueError(f"invalid betas {betas}")
        super().__init__(params, dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay))
        self._amax_modules: dict[int, torch.nn.Module] = {}
        self.check_watchdog = check_watchdog

    def attach(self, model: torch.nn.Module) -> int:
        """Give every Quartet_II_linear whose weight this optimizer updates its weight_abs_max
        from the fused step (replaces register_optimizer_hook); returns the number of layers."""
        mine = {id(p) for g in self.param_groups for p in g["params"]}
        for m in model.modules():
            if isinstance(m, Quartet_II_linear) and id(m.weight) in mine:
                self._amax_modules[id(m.weight)] = m
        return len(self._amax_modules)

    @torch.no_grad()
    def step(self, closure=None, grad_of=None):
        """One AdamW step.  grad_of(p), when given, supplies each parameter's gradient in
        place of p.grad (for example the averaged bf16 gradient of a data-parallel
        exchange, GradAllReduce.reduced_grad), so no copy back into .grad is needed."""
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        device = None
        for group in self.param_groups:
            beta1, beta2 = group["betas"]
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.dtype != torch.float32 or not p.is_cuda or not p.is_contiguous():
                    raise TypeError("QuartetAdamW updates contiguous fp32 CUDA parameters")
                g = p.grad if grad_of is None else grad_of(p)
                if g.dtype not in (torch.float32, torch.bfloat16) or g.shape != p.shape:
                    raise TypeError("gradient must be fp32 or bf16 with the parameter's shape")
                g = g.contiguous()
                state = self.state[p]
                if not state:
                    state["step"] = 0
                    state["exp_avg"] = torch.zeros_like(p, memory_format=torch.contiguous_format)
                    state["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.contiguous_format)
                state["step"] += 1
                mod = self._amax_modules.get(id(p))
                amax = torch.empty((), dtype=torch.float32, device=p.device) if mod is not None else None
                with torch.cuda.device(p.device):
                    _lib.call("q2b_adamw_step", _lib.ptr(p), _lib.ptr(state["exp_avg"]), _lib.ptr(state["exp_avg_sq"]),
                              _lib.ptr(g), int(g.dtype == torch.bfloat16), p.numel(), float(group["lr"]),
                              float(beta1), float(beta2), float(group["eps"]), float(group["weight_decay"]),
                              int(state["step"]), None, _lib.ptr(amax), _lib.stream_of(p))
                # the update is not a torch op: record it, so caches keyed by the version see it
                torch.autograd.graph.increment_version(p)
                if mod is not None:
                    mod.weight_abs_max = amax
                device = p.device
        if device is not None and self.check_watchdog:
            # once per step, without a sync: raises if a kernel wait timed out in an earlier step
            _lib.watchdog(device).poll()
        return loss
