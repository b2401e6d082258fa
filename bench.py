#!/usr/bin/env python
"""Benchmark of the Quartet-II NVFP4 linear hot path on B200.

Workload (the one its headline metric is quoted on):
the CloverLM-4B linear set -- QKV 3584->10752, attention output 3584->3584,
MLP up 3584->14336, MLP down 14336->3584 -- at M = 65536 tokens per GPU.
One step = forward + backward of all four Quartet-II linears through the
public API (Quartet_II_linear), i.e. abs-max, four-over-six quantization,
NVFP4 GEMM, randomized-Hadamard EDEN quantization of E and E^T,
requantization of W^T and X^T, dgrad and wgrad NVFP4 GEMMs.  On N > 1 GPUs
each rank runs its own 65536 tokens (weak scaling) and the bf16 weight
gradients are all-reduced (NCCL, AVG) as the data-parallel exchange step.

FLOP per step per GPU = 6 * M * sum(K*N) = 60.6 TFLOP.  Inputs are synthetic
(seeded N(0,1) activations/gradients, N(0, 0.02) weights) and larger than L2.

`--impl reference` times the reference algorithm on the host cores instead:
the CPU restatement in oracle/ (the reference's own implementation is CUDA
plus a Triton emulation, neither of which runs on host cores), on a bounded
token sample of the same four linears.
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
UNIT = "TFLOP/s"
KERNELS_PER_CALL = {"q2b_abs_max": 1, "q2b_quant_fwd": 1, "q2b_rht_eden": 2, "q2b_rht_eden_dual": 3,
                    "q2b_rht_requant": 2, "q2b_gemm_nvfp4": 1}


# Average DRAM bytes (read + write) per gemm_nvfp4_2sm_kernel launch over one step of this workload,
# from the ncu launch list summarised in profiles/step_launches_4b_linear_set.txt.
GEMM_DRAM_BYTES_PER_LAUNCH = 1671.3e6


def flops_per_token() -> float:
    return 6.0 * sum(k * n for _, k, n in SHAPES)


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


# ------------------------------------------------------------ CPU (oracle)

def cpu_step_tokens() -> int:
    return int(os.environ.get("Q2B_CPU_SAMPLE_TOKENS", "128"))


def run_cpu_sample(tokens: int, seed: int = 0):
    """One fwd+bwd of the four linears on `tokens` tokens with the CPU oracle.
    Returns (seconds, flops)."""
    import numpy as np

    import oracle
    rng = np.random.default_rng(seed)
    h16 = oracle.hadamard128_bf16()[:16].copy()
    t_total = 0.0
    for i, (_, K, N) in enumerate(SHAPES):
        x = oracle.f32_to_bf16(rng.standard_normal((tokens, K), dtype=np.float32))
        w = oracle.f32_to_bf16((0.02 * rng.standard_normal((N, K))).astype(np.float32))
        dy = oracle.f32_to_bf16(rng.standard_normal((tokens, N), dtype=np.float32))
        t0 = time.perf_counter()
        oracle.linear_fwd_bwd(x, w, dy, h16, seeds=(4 * i + 1, 4 * i + 2, 4 * i + 3, 4 * i + 4))
        t_total += time.perf_counter() - t0
    return t_total, flops_per_token() * tokens


def cpu_baseline_entry(tokens: int, reps: int = 1) -> dict:
    import oracle
    secs, flops = 0.0, 0.0
    for r in range(reps):
        s, f = run_cpu_sample(tokens, seed=r)
        secs += s
        flops += f
    return {"value": flops / secs / 1e12, "unit": UNIT, "cores": oracle.num_threads(), "kind": "port",
            "sample": f"fwd+bwd of the four 4B linears on {tokens} tokens x {reps} (oracle/ C restatement, "
                      f"{oracle.num_threads()} threads; GEMMs as fp32 numpy matmuls)"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle
    tokens = cpu_step_tokens()
    for _ in range(args.warmup):
        run_cpu_sample(tokens)
    secs, flops = 0.0, 0.0
    for k in range(args.steps):
        s, f = run_cpu_sample(tokens, seed=k + 1)
        secs += s
        flops += f
    value = flops / secs / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * secs / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "4B Quartet-II linear set fwd+bwd (QKV 3584->10752, O 3584->3584, "
                               "up 3584->14336, down 14336->3584)", "tokens_per_step": tokens,
                   "note": "bounded token sample on host cores"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": oracle.num_threads(), "kind": "port",
                         "sample": f"{tokens} tokens per step, oracle/ C restatement on {oracle.num_threads()} "
                                   f"host threads"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------- GPU

def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    import cloverlm_b200
    from cloverlm_b200 import _lib
    from cloverlm_b200 import linear as L

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    _lib.load(build_if_missing=False)

    M = args.tokens
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    layers, xs, dys = [], [], []
    for name, K, N in SHAPES:
        lay = L.Quartet_II_linear(K, N, bias=False, device=dev, dtype=torch.bfloat16)
        with torch.no_grad():
            lay.weight.normal_(0.0, 0.02, generator=torch.Generator(device=dev).manual_seed(99 + K + N))
        layers.append(lay)
        xs.append(torch.randn(M, K, device=dev, dtype=torch.bfloat16, generator=g).requires_grad_(True))
        dys.append(torch.randn(M, N, device=dev, dtype=torch.bfloat16, generator=g))

    comm = None
    if world > 1:
        from cloverlm_b200.ddp import GradAllReduce
        comm = GradAllReduce([lay.weight for lay in layers], mode=os.environ.get("Q2B_DDP_MODE", "overlap"))

    # bench-only instrumentation: kernel launches and GEMM launch durations
    counters = {"launches": 0, "gemm_events": [], "gemm_bytes": 0.0}
    orig_call = _lib.call
    state = {"timing": False}

    def counting_call(name, *a):
        if state["timing"]:
            counters["launches"] += KERNELS_PER_CALL.get(name, 0)
        return orig_call(name, *a)

    _lib.call = counting_call
    orig_mm = L._fp4_mm

    def timed_mm(x_fp4, w_fp4, x_mx, w_mx, alpha):
        if not state["timing"]:
            return orig_mm(x_fp4, w_fp4, x_mx, w_mx, alpha)
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        out = orig_mm(x_fp4, w_fp4, x_mx, w_mx, alpha)
        e.record()
        m, n, k = x_fp4.shape[0], w_fp4.shape[0], x_fp4.shape[1] * 2
        counters["gemm_events"].append((s, e, 2.0 * m * n * k))
        counters["gemm_bytes"] += m * k / 2 + n * k / 2 + (m + n) * k / 16 + 2 * m * n
        return out

    L._fp4_mm = timed_mm

    def step():
        for lay, x, dy in zip(layers, xs, dys):
            lay.weight.grad = None
            x.grad = None
            y = lay(x.view(1, M, -1))
            y.backward(dy.view(1, M, -1))
        if comm is not None:
            comm.wait()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    state["timing"] = True
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        step()
    ev1.record()
    torch.cuda.synchronize()
    state["timing"] = False
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    gemm_ms = sum(s.elapsed_time(e) for s, e, _ in counters["gemm_events"])
    gemm_flops = sum(f for _, _, f in counters["gemm_events"])
    n_gemm = len(counters["gemm_events"])
    gemm_alg_bytes = counters["gemm_bytes"]
    launches = counters["launches"] // args.steps

    # ---- end to end: inputs from pinned host memory, result read back, every step
    host_x = [x.detach().cpu().pin_memory() for x in xs]
    host_dy = [dy.cpu().pin_memory() for dy in dys]
    h2d = sum(t.numel() * t.element_size() for t in host_x + host_dy)
    res_host = torch.empty(len(layers), dtype=torch.float32).pin_memory()
    d2h = res_host.numel() * res_host.element_size()

    copy_stream = torch.cuda.Stream(dev)

    def e2e_step():
        # every layer's inputs go host -> device on a copy stream, issued up front, so the
        # PCIe transfers of later layers overlap the compute of earlier ones
        cur = torch.cuda.current_stream(dev)
        copy_stream.wait_stream(cur)
        staged = []
        with torch.cuda.stream(copy_stream):
            for hx, hdy in zip(host_x, host_dy):
                x = hx.to(dev, non_blocking=True)
                dy = hdy.to(dev, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy_stream)
                staged.append((x, dy, ev))
        norms = []
        for lay, (x, dy, ev) in zip(layers, staged):
            cur.wait_event(ev)
            x.record_stream(cur)
            dy.record_stream(cur)
            x.requires_grad_(True)
            lay.weight.grad = None
            y = lay(x.view(1, M, -1))
            y.backward(dy.view(1, M, -1))
            norms.append(lay.weight.grad.float().norm())
        if comm is not None:
            comm.wait()
        res_host.copy_(torch.stack(norms), non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps

    if world > 1:
        t = torch.tensor([ms, e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = t.tolist()
    if comm is not None:
        comm.close()

    flops_step = flops_per_token() * M
    value = world * flops_step / (ms / 1e3) / 1e12
    peaks = load_peaks()
    fp4_peak = 4.0 * peaks["bf16_tflops_sustained"]
    achieved = gemm_flops / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else None
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "nvfp4 (e2m1 x e4m3 block-16, fp32 accumulate, bf16 io)",
        "data": "synthetic (seeded N(0,1) activations and gradients, N(0,0.02) weights)",
        "config": {"workload": "4B Quartet-II linear set fwd+bwd: QKV 3584->10752, O 3584->3584, "
                               "up 3584->14336, down 14336->3584 (BASELINE config 3)",
                   "tokens_per_gpu": M, "tokens_per_s": world * M / (ms / 1e3),
                   "parallelism": f"dp{world}",
                   "allreduce": (f"bf16 NCCL AVG ({comm.mode})" if comm is not None else None),
                   "l2": "inputs larger than L2 (>= 470 MB per operand)"},
        "e2e": {"value": world * flops_step / (e2e_ms / 1e3) / 1e12, "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "note": "Quartet_II_linear API; activations and output gradients copied from pinned host "
                        "memory each step (on a copy stream, overlapping earlier layers' compute), "
                        "weight-gradient norms read back"},
        "roofline": {"bound": "tensor", "kernel": "gemm_nvfp4_2sm_kernel", "achieved": achieved,
                     "peak": fp4_peak, "unit": "TFLOP/s",
                     "frac": (achieved / fp4_peak) if achieved else None,
                     "traffic": GEMM_DRAM_BYTES_PER_LAUNCH,
                     "algorithmic_bytes_per_launch": gemm_alg_bytes / max(n_gemm, 1),
                     "peak_note": "dense NVFP4 = 4 x measured sustained bf16 (MEASURED_PEAKS.json "
                                  f"{peaks['source']}); nominal dense fp4 9000 TFLOP/s",
                     "gemm_launches_per_step": n_gemm // max(args.steps, 1),
                     "gemm_share_of_step": (gemm_ms / args.steps) / ms},
        "gpu_launches": launches,
        "clocks": clocks,
        "lib": _lib.lib_path(),
    }
    if world == 1:
        pk = fp4_mma_peak_report(dev)
        line["roofline"]["fp4_mma_peak_measured"] = pk
        if achieved:
            line["roofline"]["frac_of_fp4_mma_peak"] = achieved / pk["tflops"]
    if world == 1 and not args.no_small_m:
        line["small_m"] = small_m_report(dev)
    if world == 1 and not args.no_quant_sweep:
        line["quantizer_sweep"] = quant_sweep_report(dev)
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_entry(cpu_step_tokens())
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
    EDEN with the randomized Hadamard rotation 2 + 0.5625 + 0.25 (bf16 scale scratch written and read
    by the stochastic-rounding pass) per orientation, the dual-orientation call reading x once."""
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
                "eden_rht_rows": (2.8125, lambda: rht128_quant_eden(h=h, x=x, seed=seed, transpose=False)),
                "eden_rht_cols": (2.8125, lambda: rht128_quant_eden(h=h, x=x, seed=seed, transpose=True)),
                "eden_rht_dual": (3.625, lambda: rht128_quant_eden_dual(h=h, x=x, seed=seed, seed_t=seed)),
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=65536)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-small-m", action="store_true", help="skip the inference-linear latency section")
    ap.add_argument("--no-quant-sweep", action="store_true", help="skip the quantizer sweep section")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
