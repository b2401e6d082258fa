"""TEST / BASELINE INFRASTRUCTURE -- the reference's own CPU path, timed.

The reference's CPU implementation of the Quartet-II linear is its fake-quant
emulation, src/fake_quartet.py (FakeQuartetFn: Triton RTN / four-over-six and
EDEN kernels, F.linear GEMMs), which runs on host cores under the Triton
interpreter (TRITON_INTERPRET=1).  This module imports that file unmodified --
from the installed reference (baseline/_ref/fake_quartet.py, made by
`pip install --target baseline/_ref <reference>`) or from $CLOVERLM_REF/src --
and times FakeQuartetFn forward + backward on a bounded sample.

Three adjustments make it run on a CPU, none of which changes its arithmetic
(tests/golden/make_golden.py uses the same two launch adjustments):
  * the @triton.autotune launchers need a GPU to benchmark configs, so each
    kernel is launched through its underlying JIT function with BLOCK_SIZE=2048
    (64*32, the first of its autotuned configs);
  * FakeQuartetFn.forward is wrapped in torch.compile, which is disabled here
    (TORCHDYNAMO_DISABLE=1): the same Python runs eagerly;
  * the interpreter's bf16 tl.dot is wrong, so the sample runs in fp32 (inputs
    holding bf16 values), which is also what the GPU path computes in.
The CPU number is a reported baseline, not a target.

Run as a script it prints one JSON object (used by bench.py in a subprocess,
so the interpreter setting never reaches the GPU process).
"""
from __future__ import annotations

import importlib.util
import json
import os
import platform
import sys
import time

os.environ.setdefault("TRITON_INTERPRET", "1")
os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def find_fake_quartet() -> str | None:
    cands = [os.path.join(ROOT, "baseline", "_ref", "fake_quartet.py")]
    ref = os.environ.get("CLOVERLM_REF", os.path.join(os.path.dirname(ROOT), "reference"))
    cands.append(os.path.join(ref, "src", "fake_quartet.py"))
    for c in cands:
        if os.path.exists(c):
            return c
    return None


class _DirectLaunch:
    """Stands in for an @triton.autotune kernel: kernel[grid](**kw) launches kernel.fn with BLOCK_SIZE=2048."""

    def __init__(self, autotuned, block=2048):
        self.fn = autotuned.fn
        self.block = block

    def __getitem__(self, grid):
        g = grid({"BLOCK_SIZE": self.block}) if callable(grid) else grid

        def launch(**kw):
            return self.fn[g](**kw, BLOCK_SIZE=self.block)
        return launch


def load_fake_quartet():
    path = find_fake_quartet()
    if path is None:
        raise FileNotFoundError("the reference's src/fake_quartet.py was not found (baseline/_ref or $CLOVERLM_REF)")
    spec = importlib.util.spec_from_file_location("fake_quartet", path)
    fq = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(fq)
    fq._rtn_1x16s_fp4_kernel = _DirectLaunch(fq._rtn_1x16s_fp4_kernel)
    fq._eden_1x16s_fp4_kernel = _DirectLaunch(fq._eden_1x16s_fp4_kernel)
    import torch
    fq.FakeQuartetFn.hadamard_matrix = fq.get_hadamard_matrix(128, dtype=torch.float32, device="cpu")
    return fq, path


def time_linear(fq, tokens: int, k: int, n: int, reps: int = 1, seed: int = 0):
    """FakeQuartetFn forward + backward of one linear: X [tokens, k], W [n, k] (bf16 values
    held in fp32).  Returns (seconds, flops) summed over reps."""
    import torch
    g = torch.Generator().manual_seed(seed)
    secs = 0.0
    for _ in range(reps):
        x = torch.randn(1, tokens, k, generator=g).to(torch.bfloat16).float().requires_grad_()
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16).float().requires_grad_()
        dy = torch.randn(1, tokens, n, generator=g).to(torch.bfloat16).float()
        t0 = time.perf_counter()
        y = fq.FakeQuartetFn.apply(x, w, fq.AmaxStorage(), False, False, False, True)
        y.backward(dy)
        secs += time.perf_counter() - t0
    return secs, 6.0 * tokens * k * n * reps


def main(argv=None) -> int:
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=128)
    ap.add_argument("--k", type=int, default=1024)
    ap.add_argument("--n", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1)
    a = ap.parse_args(argv)
    import torch
    fq, path = load_fake_quartet()
    for i in range(a.warmup):
        time_linear(fq, a.tokens, a.k, a.n, seed=100 + i)
    per_step = []
    flops = 0.0
    for i in range(a.steps):
        s, f = time_linear(fq, a.tokens, a.k, a.n, seed=i)
        per_step.append(s)
        flops += f
    cpu = platform.processor() or platform.machine()
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    cpu = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    print(json.dumps({"seconds": sum(per_step), "seconds_per_step": per_step, "flops": flops,
                      "flops_per_s": flops / sum(per_step), "tokens": a.tokens, "k": a.k, "n": a.n,
                      "steps": a.steps, "warmup": a.warmup, "torch_threads": torch.get_num_threads(),
                      "os_cpu_count": os.cpu_count(), "cpu_model": cpu,
                      "source": os.path.relpath(path, ROOT) if path.startswith(ROOT) else "reference src/fake_quartet.py"}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
