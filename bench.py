#!/usr/bin/env python
"""Benchmark of the Quartet-II NVFP4 training path on B200.

Headline workload (the "train tokens/s at 1/2/4/8"
half of its metric): one data-parallel training step of CloverLM-4B with every
block linear a Quartet-II NVFP4 layer (cloverlm_b200.model / .train): 29
blocks, d 3584, 28 heads x 128 with 7 KV heads, MLP 14336 (ReLU^2), vocab
32768 tied, seq 2048, 32 sequences per GPU per step (2 micro-batches of 16,
the first under no_sync), bf16 autocast, fused AdamW, and on N > 1 GPUs the
bf16 gradient all-reduce (NCCL) overlapped with the last backward.  Weak
scaling: every rank trains on its own 65536 tokens per step.  `value` is the
whole job's tokens/s from CUDA events, max over ranks.

At N = 1 the line also carries BASELINE config 3 (`linear_set`: fwd+bwd of the
four 4B linear shapes at 65536 tokens, TFLOP/s -- the other half of the
metric), config 2 (`quantizer_sweep`, GB/s), config 5 (`small_m`), the FP4
tensor-pipe ceiling the GEMM's roofline is quoted against, and `cpu_baseline`:
the reference's own fake-quant CPU path (src/fake_quartet.py under the Triton
interpreter) timed on this box's host cores.

`--impl reference` runs only that reference CPU path, one bounded sample per
step, and reports it in the same unit.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

SHAPES = [("qkv", 3584, 10752), ("attn_out", 3584, 3584), ("mlp_up", 3584, 14336), ("mlp_down", 14336, 3584)]
METRIC = "Quartet-II linear fwd+bwd TFLOP/s at 4B shapes; train tokens/s at 1/2/4/8"
UNIT = "tokens/s"
# libq2b kernels each C-ABI call launches (memsets not counted)
KERNELS_PER_CALL = {"q2b_abs_max": 1, "q2b_quant_fwd": 1, "q2b_rht_eden": 2, "q2b_rht_eden_dual": 3,
                    "q2b_rht_requant": 2, "q2b_gemm_nvfp4": 1, "q2b_gemm_nvfp4_f32": 1, "q2b_gemm_nvfp4_ex": 1, "q2b_relu2_abs_max": 1,
                    "q2b_relu2_bwd": 1, "q2b_rope_norm_fwd": 1, "q2b_rope_norm_bwd": 1,
                    "q2b_add_rmsnorm_amax": 1, "q2b_rmsnorm_bwd": 1, "q2b_adamw_step": 1,
                    "q2b_watchdog_poll": 0}


# DRAM bytes (read + write) of one pair-GEMM launch of the training step's shapes, from the ncu
# capture summarised in profiles/gemm_nvfp4_2sm_fwd_mlp_down_32k.txt (MLP-down forward, M=32768
# N=3584 K=14336): 551.5 MB against 528.1 MB algorithmic (1.04x).
GEMM_TRAFFIC_PER_LAUNCH = 551.5e6
GEMM_TRAFFIC_NOTE = ("dram read+write of one MLP-down forward launch (M=32768, N=3584, K=14336) under ncu; "
                     "algorithmic 528.1 MB, ratio 1.04")


def load_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p.get("hbm_gbs", 6650.0), "bf16_tflops": p.get("bf16_tflops", 1590.0),
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", 1400.0), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi sampler running during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        loaded = [s for s in sm if s > 500] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------ instrumentation

class Instrument:
    """Bench-only accounting while `active`: libq2b kernel launches per C-ABI call, and
    CUDA-event durations of every NVFP4 GEMM launch (the dominant kernel) on the
    launching stream."""

    def __init__(self):
        import torch
        from cloverlm_b200 import _lib, fusion
        from cloverlm_b200 import linear as L
        self.torch = torch
        self.active = False
        self.launches = 0
        self.gemm = []  # (start event, end event, flop, pair kernel?)
        self._lib, self._L, self._fusion = _lib, L, fusion
        self._orig_call = _lib.call
        _lib.call = self._call
        # every NVFP4 GEMM wrapper of the training step, wherever it is referenced
        for mod, name in ((L, "_fp4_mm"), (L, "_fp4_mm_f32"), (L, "_fp4_mm_relu2_bwd"), (L, "_fp4_mm_add"),
                          (L, "_fp4_mm_relu2"), (fusion, "_fp4_mm"), (fusion, "_fp4_mm_relu2")):
            setattr(mod, name, self._wrap(getattr(mod, name), name))

    def _call(self, name, *a):
        if self.active:
            self.launches += KERNELS_PER_CALL.get(name, 0)
        return self._orig_call(name, *a)

    def _wrap(self, fn, name):
        if getattr(fn, "_bench_wrapped", False):
            return fn
        codes = 1 if name == "_fp4_mm_add" else 0  # position of A's codes (the add form takes out first)

        def timed(*args, **kw):
            if not self.active:
                return fn(*args, **kw)
            torch = self.torch
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            out = fn(*args, **kw)
            e.record()
            a_fp4, b_fp4 = args[codes], args[codes + 1]
            m, n, k = a_fp4.shape[0], b_fp4.shape[0], a_fp4.shape[1] * 2
            self.gemm.append((s, e, 2.0 * m * n * k, m % 128 == 0 and n % 128 == 0))  # the pair kernel's rule
            return out
        timed._bench_wrapped = True
        return timed

    def reset(self):
        self.launches = 0
        self.gemm = []

    def gemm_summary(self, steps: int) -> dict:
        ms = [s.elapsed_time(e) for s, e, _, _ in self.gemm]
        flop = [f for _, _, f, _ in self.gemm]
        pair = [p for _, _, _, p in self.gemm]
        tot_ms, tot_f = sum(ms), sum(flop)
        pms = sum(m for m, p in zip(ms, pair) if p)
        pf = sum(f for f, p in zip(flop, pair) if p)
        return {"launches_per_step": len(ms) // max(steps, 1), "ms_per_step": tot_ms / max(steps, 1),
                "tflops": tot_f / (tot_ms / 1e3) / 1e12 if tot_ms else None,
                "pair_kernel_share_of_flop": pf / tot_f if tot_f else None,
                "pair_kernel_tflops": pf / (pms / 1e3) / 1e12 if pms else None}


# ----------------------------------------------------- the reference's CPU path

def reference_cpu(tokens: int, k: int, n: int, warmup: int, steps: int, timeout: int = 900) -> dict:
    """The reference's fake-quant Quartet-II linear (src/fake_quartet.py, Triton interpreter
    on host cores) timed by oracle/ref_cpu.py in a subprocess."""
    cmd = [sys.executable, os.path.join(ROOT, "oracle", "ref_cpu.py"), "--tokens", str(tokens), "--k", str(k),
           "--n", str(n), "--warmup", str(warmup), "--steps", str(steps)]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout)
    if res.returncode != 0:
        raise RuntimeError("reference CPU path failed: " + res.stderr[-2000:])
    return json.loads(res.stdout.strip().splitlines()[-1])


def cpu_entry(r: dict, flops_per_token: float) -> dict:
    """A timed reference CPU sample as a model-equivalent tokens/s figure."""
    return {"value": r["flops_per_s"] / flops_per_token, "unit": UNIT, "cores": r["torch_threads"],
            "kind": "reference",
            "sample": (f"the reference's fake-quant Quartet-II linear (src/fake_quartet.py FakeQuartetFn, Triton "
                       f"interpreter, fp32) fwd+bwd on X [{r['tokens']}, {r['k']}], W [{r['n']}, {r['k']}] x "
                       f"{r['steps']}: {r['flops_per_s'] / 1e9:.3f} GFLOP/s, divided by the 4B model's "
                       f"{flops_per_token / 1e9:.1f} GFLOP of Quartet-linear work per token (the rest of the "
                       f"model is not counted, which favours the CPU)"),
            "linear_gflops": r["flops_per_s"] / 1e9, "seconds": r["seconds"],
            "cpu_model": r["cpu_model"], "os_cpu_count": r["os_cpu_count"], "torch_threads": r["torch_threads"],
            "source": r["source"]}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from cloverlm_b200.model import CloverLMConfig
    cfg = CloverLMConfig()
    fpt = cfg.linear_flops_per_token()
    r = reference_cpu(args.ref_tokens, args.ref_k, args.ref_n, args.warmup, args.steps)
    cb = cpu_entry(r, fpt)
    line = {
        "impl": "reference", "metric": METRIC, "value": cb["value"], "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * r["seconds"] / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (bf16 values)",
        "data": "synthetic", "config": train_config(args, 1) | {"note": "bounded sample on host cores; each step "
                                                                        "one fake-quant linear fwd+bwd"},
        "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ config 4: training

def train_config(args, world: int) -> dict:
    return {"workload": "CloverLM-4B training step (BASELINE config 4): 29 blocks, d 3584, 28 heads x 128 "
                        "(7 KV heads), MLP 14336 ReLU^2, vocab 32768 tied, every block linear Quartet-II NVFP4",
            "model": "CloverLM-4B", "seq_len": 2048, "micro_batch": args.micro_batch,
            "accumulation": args.accum, "sequences_per_gpu": args.micro_batch * args.accum,
            "global_batch": world * args.micro_batch * args.accum, "parallelism": f"dp{world}",
            "note": "32 sequences per GPU per step reached with 2 micro-batches of 16 under no_sync "
                    "(32 x 2048 tokens of activations do not fit beside the optimizer state in 180 GB)",
            "l2": "inputs larger than L2 (every activation >= 235 MB)"}


def train_measure(args, world: int, rank: int, local: int, dev, inst: Instrument) -> dict:
    import torch
    import torch.distributed as dist

    from cloverlm_b200.ddp import GradAllReduce
    from cloverlm_b200.model import CloverLM, CloverLMConfig
    from cloverlm_b200.optim import QuartetAdamW
    from cloverlm_b200.train import TrainStep

    cfg = CloverLMConfig()
    torch.manual_seed(0)  # the same initial weights on every rank (what DDP's broadcast establishes)
    model = CloverLM(cfg, device=dev)
    opt = QuartetAdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), eps=1e-6, weight_decay=0.0)
    comm = None
    if world > 1:
        comm = GradAllReduce(list(model.parameters()), mode="overlap", bucket_mb=args.bucket_mb, copy_back=False)
    step = TrainStep(model, opt, comm)
    # exposed exchange: device time the compute stream stalls in comm.wait() (the last buckets'
    # all-reduces that the backward did not hide), CUDA events around the wait on that stream
    waits = []
    if comm is not None:
        inner_wait = comm.wait

        def timed_wait():
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            inner_wait()
            b.record()
            waits.append((a, b))
        comm.wait = timed_wait
    gen = torch.Generator(device=dev).manual_seed(654356 + rank * 2097593)  # per-rank data (utils_data.py:266-269)
    shape = (args.accum, args.micro_batch, cfg.context + 1)
    pool = [torch.randint(0, cfg.vocab_size, shape, device=dev, generator=gen) for _ in range(4)]

    def split(ids):
        return [(ids[i, :, :-1], ids[i, :, 1:]) for i in range(args.accum)]

    losses = []
    for i in range(args.warmup):
        losses.append(step(split(pool[i % 4])).item())
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    inst.reset()
    inst.active = True
    waits.clear()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(args.steps):
        loss = step(split(pool[i % 4]))
    ev1.record()
    torch.cuda.synchronize()
    inst.active = False
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    losses.append(loss.item())
    ms = ev0.elapsed_time(ev1) / args.steps
    exposed_ms = sum(a.elapsed_time(b) for a, b in waits) / args.steps if waits else 0.0
    gemm = inst.gemm_summary(args.steps)
    launches = inst.launches // args.steps
    mem = torch.cuda.max_memory_allocated(dev)

    # end to end: every step's token ids copied from pinned host memory, its loss read back
    host_ids = pool[0].cpu().pin_memory()
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()
    h2d = host_ids.numel() * host_ids.element_size()

    def e2e_step():
        ids = host_ids.to(dev, non_blocking=True)
        out = step(split(ids))
        loss_host.copy_(out, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.e2e_steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.e2e_steps
    if world > 1:
        t = torch.tensor([ms, e2e_ms, exposed_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms, exposed_ms = t.tolist()
    tokens = args.accum * args.micro_batch * cfg.context
    out = {
        "ms_per_step": ms, "tokens_per_gpu": tokens, "value": world * tokens / (ms / 1e3),
        "e2e": {"value": world * tokens / (e2e_ms / 1e3), "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                "note": "TrainStep on token ids copied from pinned host memory every step, loss read back"},
        "model_tflops": world * tokens * cfg.train_flops_per_token() / (ms / 1e3) / 1e12,
        "linear_tflops": world * tokens * cfg.linear_flops_per_token() / (ms / 1e3) / 1e12,
        "gemm": gemm, "gpu_launches": launches, "clocks": clocks,
        "loss_first_last": [losses[0], losses[-1]], "max_memory_gb": mem / 1e9,
        "params": sum(p.numel() for p in model.parameters()),
    }
    if comm is not None:
        nbytes = sum(f.numel() * f.element_size() for f in comm._flat if f is not None)
        out["exchange"] = {"bytes_per_gpu": nbytes, "buckets": len(comm.buckets),
                           "exposed_ms_per_step": exposed_ms, "exposed_share_of_step": exposed_ms / ms,
                           "note": "device time the compute stream waits in GradAllReduce.wait() per step "
                                   "(CUDA events on that stream, max over ranks); the rest of the all-reduce "
                                   "time overlaps the last backward"}
    if comm is not None:
        comm.close()
    del model, opt, comm, step, pool
    import gc
    gc.collect()
    torch.cuda.empty_cache()
    return out


# --------------------------------------------------------- config 3: linear set

def linear_set_measure(dev, tokens: int, steps: int, warmup: int, inst: Instrument) -> dict:
    """fwd+bwd of the four 4B linear shapes at `tokens` tokens through
    Quartet_II_linear; TFLOP/s = 6 * M * sum(K*N) per step."""
    import torch
    from cloverlm_b200 import linear as L
    M = tokens
    g = torch.Generator(device=dev).manual_seed(1234)
    layers, xs, dys = [], [], []
    for name, K, N in SHAPES:
        lay = L.Quartet_II_linear(K, N, bias=False, device=dev, dtype=torch.bfloat16)
        with torch.no_grad():
            lay.weight.normal_(0.0, 0.02, generator=torch.Generator(device=dev).manual_seed(99 + K + N))
        layers.append(lay)
        xs.append(torch.randn(M, K, device=dev, dtype=torch.bfloat16, generator=g).requires_grad_(True))
        dys.append(torch.randn(M, N, device=dev, dtype=torch.bfloat16, generator=g))

    def step():
        for lay, x, dy in zip(layers, xs, dys):
            lay.weight.grad = None
            x.grad = None
            lay(x.view(1, M, -1)).backward(dy.view(1, M, -1))

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    inst.reset()
    inst.active = True
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(steps):
        step()
    ev1.record()
    torch.cuda.synchronize()
    inst.active = False
    ms = ev0.elapsed_time(ev1) / steps
    flop = 6.0 * M * sum(k * n for _, k, n in SHAPES)
    out = {"workload": "BASELINE config 3: QKV 3584->10752, O 3584->3584, up 3584->14336, down 14336->3584 "
                       "(fused-QKV shapes) fwd+bwd through Quartet_II_linear",
           "tokens": M, "ms_per_step": ms, "tflops": flop / (ms / 1e3) / 1e12, "gemm": inst.gemm_summary(steps),
           "gpu_launches": inst.launches // steps}
    del layers, xs, dys
    torch.cuda.empty_cache()
    return out


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from cloverlm_b200 import _lib
    from cloverlm_b200.model import CloverLMConfig

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    _lib.load(build_if_missing=False)
    inst = Instrument()
    tr = train_measure(args, world, rank, local, dev, inst)
    peaks = load_peaks()
    cfg = CloverLMConfig()
    fp4_peak = fp4_mma_peak_report(dev)
    if world > 1:  # the slowest rank's ceiling
        t = torch.tensor([fp4_peak["tflops"]], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        fp4_peak["tflops"] = t.item()
    peak = fp4_peak["tflops"] if fp4_peak else 4.0 * peaks["bf16_tflops_sustained"]
    achieved = tr["gemm"]["tflops"]
    line = {
        "metric": METRIC, "value": tr["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": tr["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "nvfp4 linears (e2m1 x e4m3 block-16, fp32 accumulate), bf16 autocast "
                                      "elsewhere, fp32 master weights",
        "data": "synthetic (uniform token ids, per-rank seeds; random-init weights)",
        "config": train_config(args, world) | {"tokens_per_gpu": tr["tokens_per_gpu"],
                                               "allreduce": "bf16 NCCL AVG, 256 MB buckets launched during the "
                                                            "last backward" if world > 1 else None},
        "e2e": tr["e2e"],
        "roofline": {"bound": "tensor", "kernel": "q2b_gemm_nvfp4 (gemm_nvfp4_2sm_kernel for the 256-aligned "
                                                  "shapes, gemm_nvfp4_kernel otherwise) inside the training step",
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak if achieved else None, "traffic": GEMM_TRAFFIC_PER_LAUNCH,
                     "traffic_note": GEMM_TRAFFIC_NOTE,
                     "peak_note": ("FP4 tensor-pipe ceiling measured in this run by q2b_fp4_mma_peak"
                                   if fp4_peak else "4 x measured sustained bf16 (MEASURED_PEAKS.json)"),
                     "frac_of_4x_bf16_sustained": achieved / (4.0 * peaks["bf16_tflops_sustained"]) if achieved
                     else None,
                     "gemm_share_of_step": tr["gemm"]["ms_per_step"] / tr["ms_per_step"]},
        "gpu_launches": tr["gpu_launches"],
        "clocks": tr["clocks"],
        "train": {k: tr[k] for k in ("model_tflops", "linear_tflops", "gemm", "loss_first_last", "max_memory_gb",
                                     "params", "exchange") if k in tr},
        "lib": _lib.lib_path(),
    }
    if fp4_peak:
        line["roofline"]["fp4_mma_peak_measured"] = fp4_peak
    if world == 1 and not args.no_linear_set:
        ls = linear_set_measure(dev, args.tokens, args.linear_steps, args.warmup, inst)
        ls["frac_of_fp4_peak"] = ls["tflops"] / peak
        line["linear_set"] = ls
    if world == 1 and not args.no_small_m:
        line["small_m"] = small_m_report(dev)
    if world == 1 and not args.no_quant_sweep:
        line["quantizer_sweep"] = quant_sweep_report(dev)
    if world == 1 and not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = cpu_entry(reference_cpu(128, 1024, 1024, 0, 1), cfg.linear_flops_per_token())
        except Exception as e:  # reported, not fatal: the GPU numbers stand on their own
            line["cpu_baseline"] = {"value": None, "unit": UNIT, "error": str(e)[-300:]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def fp4_mma_peak_report(dev, iters: int = 4096, reps: int = 3) -> dict:
    """The tensor pipe's FP4 ceiling on this GPU: q2b_fp4_mma_peak (back-to-back
    cta_group::2 M256 N256 K64 NVFP4 MMAs on resident shared-memory operands,
    one SM pair per two SMs), timed with CUDA events; median of `reps`."""
    import torch
    from cloverlm_b200 import _lib
    stream = torch.cuda.current_stream(dev)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    _lib.call("q2b_fp4_mma_peak", 256, None, stream.cuda_stream)
    times = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        _lib.call("q2b_fp4_mma_peak", iters, None, stream.cuda_stream)
        e1.record(stream)
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    ms = sorted(times)[len(times) // 2]
    flop = (sms // 2) * iters * 2.0 * 256 * 256 * 64
    return {"tflops": flop / (ms / 1e3) / 1e12, "ms": ms, "iters": iters, "sm_pairs": sms // 2,
            "note": "q2b_fp4_mma_peak: back-to-back cta_group::2 M256 N256 K64 block-scaled MMAs, "
                    "operands resident in shared memory"}


SWEEP_M = [1024, 16384, 65536]
SWEEP_K = [3584, 14336]


def quant_sweep_report(dev, reps: int = 5) -> dict:
    """quantizers on bf16 [M, K] ~ Student-t(df=3)/sqrt(3), seed 1, through the public
    API.  Each call is timed alone with CUDA events after a 256 MB write that evicts L2, so no input
    is served from L2.  Algorithmic bytes per element: abs-max 2; RTN (RNE, four-over-six) 2 + 0.5625;
    EDEN with the randomized Hadamard rotation 2 + 0.5625 per orientation, the dual-orientation call
    reading x once (2 + 2 * 0.5625).  The bf16 scale scratch the two-pass scheme writes and re-reads
    (0.25 B/elem per orientation) is not counted as algorithmic."""
    import torch

    from cloverlm_b200.linear import get_hadamard_matrix
    from cloverlm_b200.quant import NVFP4QuantMode, abs_max, quant_fp4, rht128_quant_eden, rht128_quant_eden_dual

    peaks = load_peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    h = get_hadamard_matrix(128, torch.bfloat16, dev)[:16].contiguous()
    seed = torch.tensor(1)

    def timed(fn):
        ts = []
        for _ in range(reps + 1):
            flush.zero_()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize(dev)
            ts.append(a.elapsed_time(b))
        return statistics.median(ts[1:])

    out = {"unit": "GB/s", "hbm_peak_gbs": peaks["hbm_gbs"], "peak_source": peaks["source"],
           "config": "BASELINE config 2: Student-t(3)/sqrt(3) bf16, seed 1; L2 evicted before every call",
           "shapes": {}}
    g = torch.Generator(device=dev).manual_seed(1)
    for M in SWEEP_M:
        for K in SWEEP_K:
            z = torch.randn(M, K, device=dev, generator=g)
            chi = torch.randn(3, M, K, device=dev, generator=g).pow_(2).sum(0)
            x = (z / torch.sqrt(chi / 3.0) / 3.0 ** 0.5).to(torch.bfloat16)
            del z, chi
            am = abs_max(x)
            n = M * K
            rows = {
                "abs_max": (2.0, lambda: abs_max(x)),
                "rtn_rne": (2.5625, lambda: quant_fp4(x, scale_override=1.0, amax=am, mode=NVFP4QuantMode.RNE)),
                "rtn_four_six": (2.5625, lambda: quant_fp4(x, scale_override=1.0, amax=am,
                                                          mode=NVFP4QuantMode.FOUR_SIX)),
                "eden_rht_rows": (2.5625, lambda: rht128_quant_eden(h=h, x=x, seed=seed, transpose=False)),
                "eden_rht_cols": (2.5625, lambda: rht128_quant_eden(h=h, x=x, seed=seed, transpose=True)),
                "eden_rht_dual": (3.125, lambda: rht128_quant_eden_dual(h=h, x=x, seed=seed, seed_t=seed)),
            }
            res = {}
            for name, (bpe, fn) in rows.items():
                ms = timed(fn)
                gbs = n * bpe / (ms * 1e-3) / 1e9
                res[name] = {"gbs": round(gbs, 1), "frac_hbm": round(gbs / peaks["hbm_gbs"], 3), "us": round(ms * 1e3, 1)}
            out["shapes"][f"{M}x{K}"] = res
            del x
    del flush
    torch.cuda.empty_cache()
    return out


SMALL_M = [1, 8, 64, 256, 4096]


def small_m_report(dev, reps: int = 200) -> dict:
    """forward-only inference linears with pre-quantized weights at decode and
    prefill M, through cloverlm_b200.inference.apply (no row padding, split-K at small M).  Each call
    is captured in a CUDA graph (as vLLM runs decode) and replayed `reps` times; the time per call is
    device time from CUDA events.  `padded_us` is the reference's algorithm (rows padded to 128,
    quantized, multiplied and sliced) on the same kernels, captured the same way."""
    import torch
    import torch.nn.functional as F

    from cloverlm_b200 import inference
    from cloverlm_b200.linear import _fp4_mm
    from cloverlm_b200.quant import NVFP4QuantMode, abs_max, quant_fp4

    def graph_time(fn):
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(3):
                fn()
        torch.cuda.current_stream(dev).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):  # same stream as the warm-up: reuses its split-K workspace
            fn()
        g.replay()
        torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) * 1e3 / reps

    out = {"unit": "us per call (CUDA graph replay, device time)", "reps": reps,
           "config": "BASELINE config 5: W pre-quantized four-over-six from N(0,0.02), X ~ N(0,1) bf16",
           "shapes": {}}
    gen = torch.Generator(device=dev).manual_seed(7)
    for name, K, N in SHAPES:
        w = (torch.randn(N, K, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
        prep = inference.prepare_weight(w)
        rows = {}
        for m in SMALL_M:
            x = torch.randn(m, K, device=dev, generator=gen).to(torch.bfloat16)

            def ours():
                return inference.apply(prep, x)

            def padded():
                xp = F.pad(x, (0, 0, 0, (-m) % 128))
                q = quant_fp4(xp, amax=abs_max(xp), scale_override=1.0, mode=NVFP4QuantMode.FOUR_SIX)
                return _fp4_mm(q.fp4, prep.fp4, q.micro_scales, prep.micro_scales,
                               q.tensor_scale * prep.tensor_scale)[:m]

            t_ours = graph_time(ours)
            t_pad = graph_time(padded)
            rows[str(m)] = {"ours_us": round(t_ours, 2), "padded_us": round(t_pad, 2),
                            "tflops": round(2.0 * m * N * K / (t_ours * 1e-6) / 1e12, 2)}
        out["shapes"][f"{name} {K}->{N}"] = rows
    return out


KERNEL_CASES = {
    # name: (what, shape) -- single-kernel workloads of the training step's shapes, for ncu captures
    "gemm_fwd": "q2b_gemm_nvfp4 (pair kernel, bf16 out): MLP-down forward, M=32768 N=3584 K=14336",
    "gemm_wgrad": "q2b_gemm_nvfp4_f32 (pair kernel, fp32 out): MLP-up wgrad, M=14336 N=3584 K=32768",
    "gemm_qkv_65k": "q2b_gemm_nvfp4 (pair kernel, bf16 out): config-3 fused-QKV forward, M=65536 N=10752 K=3584",
    "gemm_up_wgrad_65k": "q2b_gemm_nvfp4 (pair kernel, bf16 out): config-3 MLP-up wgrad, M=14336 N=3584 K=65536",
    "eden_dual": "q2b_rht_eden_dual: E [32768, 14336] -> E and E^T",
    "requant": "q2b_rht_requant: NVFP4 X [32768, 14336] -> X^T",
    "quant_fwd": "q2b_quant_fwd four-over-six: [32768, 14336]",
}


def kernel_case(name: str, reps: int = 3) -> None:
    """Run one kernel of the training step `reps` times on its own (inputs > L2, a few GB on the
    device): the workload an ncu capture of that kernel uses.  Prints the mean CUDA-event time."""
    import torch

    from cloverlm_b200 import _lib
    from cloverlm_b200.linear import _fp4_mm, _fp4_mm_f32, get_hadamard_matrix
    from cloverlm_b200.quant import NVFP4QuantMode, quant_fp4, rht128_quant_eden_dual, rht128_requant
    torch.cuda.set_device(0)
    _lib.load(build_if_missing=False)
    g = torch.Generator(device="cuda").manual_seed(11)

    def rnd(r, c):
        return torch.randn(r, c, device="cuda", generator=g).to(torch.bfloat16)

    def q(r, c):
        return quant_fp4(rnd(r, c), scale_override=1.0, mode=NVFP4QuantMode.FOUR_SIX)

    h = get_hadamard_matrix(128, torch.bfloat16, "cuda")[:16].contiguous()
    if name == "gemm_fwd":
        a, b = q(32768, 14336), q(3584, 14336)
        fn = lambda: _fp4_mm(a.fp4, b.fp4, a.micro_scales, b.micro_scales, a.tensor_scale * b.tensor_scale)
    elif name == "gemm_wgrad":
        a, b = q(14336, 32768), q(3584, 32768)
        fn = lambda: _fp4_mm_f32(a.fp4, b.fp4, a.micro_scales, b.micro_scales, a.tensor_scale * b.tensor_scale)
    elif name == "gemm_qkv_65k":
        a, b = q(65536, 3584), q(10752, 3584)
        fn = lambda: _fp4_mm(a.fp4, b.fp4, a.micro_scales, b.micro_scales, a.tensor_scale * b.tensor_scale)
    elif name == "gemm_up_wgrad_65k":
        a, b = q(14336, 65536), q(3584, 65536)
        fn = lambda: _fp4_mm(a.fp4, b.fp4, a.micro_scales, b.micro_scales, a.tensor_scale * b.tensor_scale)
    elif name == "eden_dual":
        x = rnd(32768, 14336)
        fn = lambda: rht128_quant_eden_dual(h=h, x=x, seed=torch.tensor(1), seed_t=torch.tensor(2))
    elif name == "requant":
        xq = q(32768, 14336)
        fn = lambda: rht128_requant(x=xq.fp4, x_group_scales=xq.micro_scales, x_tensor_scale=xq.tensor_scale, h=h,
                                    seed=torch.tensor(3))
    elif name == "quant_fwd":
        x = rnd(32768, 14336)
        fn = lambda: quant_fp4(x, scale_override=1.0, mode=NVFP4QuantMode.FOUR_SIX)
    else:
        raise SystemExit(f"unknown kernel case {name!r}; choose from {sorted(KERNEL_CASES)}")
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    print(json.dumps({"kernel_case": name, "what": KERNEL_CASES[name], "ms": e0.elapsed_time(e1) / reps}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--micro-batch", dest="micro_batch", type=int, default=16)
    ap.add_argument("--accum", type=int, default=2, help="micro-batches per step (the first ones under no_sync)")
    ap.add_argument("--bucket-mb", dest="bucket_mb", type=float, default=256.0)
    ap.add_argument("--e2e-steps", dest="e2e_steps", type=int, default=4)
    ap.add_argument("--tokens", type=int, default=65536, help="tokens of the config-3 linear-set section")
    ap.add_argument("--linear-steps", dest="linear_steps", type=int, default=10)
    ap.add_argument("--ref-tokens", dest="ref_tokens", type=int, default=128)
    ap.add_argument("--ref-k", dest="ref_k", type=int, default=512)
    ap.add_argument("--ref-n", dest="ref_n", type=int, default=512)
    ap.add_argument("--no-linear-set", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-small-m", action="store_true", help="skip the inference-linear latency section")
    ap.add_argument("--no-quant-sweep", action="store_true", help="skip the quantizer sweep section")
    ap.add_argument("--kernel-case", dest="kernel_case", choices=sorted(KERNEL_CASES),
                    help="run one kernel of the training step on its own (for ncu captures) and exit")
    args = ap.parse_args()
    if args.kernel_case:
        kernel_case(args.kernel_case)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
