#!/usr/bin/env python
"""Benchmark of the DoRA hot path on B200: one adapted linear layer, forward + backward.

Workload (the high-rank single-layer configuration): W0 [28672 x 8192] bf16
~N(0, 0.02), rank 384, A kaiming-uniform, B ~N(0, 0.01), scale 1.0, X
[16384 x 8192] bf16 ~N(0, 1), seeded synthetic data.  One step is
    y = base(x) + DoRA delta   (factored norm + fused compose)
    y.backward(dy)             (fused compose backward, LoRA and base GEMMs)
through ``dorafactors_b200.layer.DoraLinear``, i.e. the PEFT wiring of
``DoraLinearLayer``.  The metric is whole-job tokens/s; the line also carries
the factored norm's tensor TFLOP/s and the compose kernels' HBM GB/s against
the measured peaks, each timed with CUDA events around every native call of
the timed steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]

N > 1 (launched by torchrun, one process per GPU): token data parallelism.
Every rank runs the full layer on its own 16384 tokens (weak scaling) and the
LoRA / magnitude gradients are all-reduced over NCCL each step, each one as
soon as autograd has accumulated it, the exchange data-parallel training
performs.

Extra keys of the same line (not the headline value): ``dropin_unfused`` (the
same layer wired as PEFT's unchanged DoraLinearVariant, delta then a separate
``result + delta``), ``rowshard`` (the 70B-class layer, W0 28672 x 8192 and
8192 x 28672, r=256, 32768 tokens, out-features sharded over the N ranks with
the output all-gather fused into the compose, strong scaling), at 1 GPU
``rank_sweep`` (the factored norm on W0 8192 x 8192 for r = 16 .. 1024 and the
compose kernels at 8192 x 8192, each call timed alone) and, at 8 GPUs,
``model`` (the Llama-style decoder with DoRA on all seven projections, one
4096-token sequence per GPU, data parallel).

``--impl reference`` times the reference's own eager CPU implementation (its
``DoraLinearLayer`` from dora.py / dora_fused.py, byte-compiled into
oracle/_ref by oracle/build_ref.py) on the host cores with every thread the
process may use, each step a forward + backward on a 4096-token sample of the
same workload over the full weight, on rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

OUT_F, IN_F, RANK, TOKENS, SCALE = 28672, 8192, 384, 16384, 1.0
METRIC = "DoRA layer fwd+bwd tokens/s, norm TFLOP/s & compose HBM GB/s vs peak"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
CPU_SAMPLE_TOKENS = 4096  # tokens per host-core step: a quarter of the workload's 16384
CPU_PORT_TOKENS = 512  # the same with the numpy port (no reference build present)


def workload_config(parallelism: str) -> dict:
    return {
        "workload": f"dora_linear_fwd_bwd out={OUT_F} in={IN_F} r={RANK} tokens={TOKENS}/rank bf16",
        "out_features": OUT_F,
        "in_features": IN_F,
        "rank": RANK,
        "tokens_per_rank": TOKENS,
        "scale": SCALE,
        "l2": "inputs larger than L2 (x 268 MB, each activation 940 MB), no flush needed",
        "parallelism": parallelism,
    }


def load_peaks() -> tuple[dict, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


# Algorithmic work per native call (bf16, e = 2 bytes).
def compose_fwd_bytes(T, out, e=2):
    return e * 4 * T * out + e * out  # read lora, base, g; write out, inner


def compose_bwd_bytes(T, out, e=2):
    return e * 4 * T * out + 2 * e * out  # read d_out, inner, g; write d_lora, d_base, d_g


def norm_flops(out, inp, r):
    return 2 * out * inp * r + 2 * r * r * inp + 2 * out * r * r  # W0 A^T, A A^T, B G


def norm_bytes(out, inp, r, e=2):
    return e * (out * inp + r * inp + out * r) + e * out  # read W0, A, B; write the norm


# ---------------------------------------------------------------------------
# Clock sampling during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.gpu_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first(self, timeout_s: float = 3.0) -> None:
        """Block until nvidia-smi has printed its first sample (it takes a moment to
        start), so that a short measured region still gets sampled."""
        t0 = time.time()
        while self.proc is not None and not self.lines and time.time() - t0 < timeout_s:
            time.sleep(0.02)

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self._t is not None:
            self._t.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


def physical_gpu_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        parts = [p.strip() for p in vis.split(",") if p.strip()]
        if local_rank < len(parts) and parts[local_rank].isdigit():
            return int(parts[local_rank])
    return local_rank


# ---------------------------------------------------------------------------
# Per-call CUDA-event timing of the native entry points
# ---------------------------------------------------------------------------
class NativeTimer:
    """Wraps the native calls with CUDA events on the current stream while enabled."""

    NAMES = ("weight_norm", "compose_fwd", "compose_bwd", "linear_output_fwd", "linear_output_bwd",
             "linear_output_fwd_allgather", "linear_output_bwd_strided")

    def __init__(self):
        import torch

        from dorafactors_b200 import _native

        self.torch = torch
        self.native = _native
        self.enabled = False
        self.events: dict = {n: [] for n in self.NAMES}
        self.orig = {n: getattr(_native, n) for n in self.NAMES}
        for n in self.NAMES:
            setattr(_native, n, self._wrap(n, self.orig[n]))

    def _wrap(self, name, fn):
        def wrapped(*a, **k):
            if not self.enabled:
                return fn(*a, **k)
            s = self.torch.cuda.Event(enable_timing=True)
            e = self.torch.cuda.Event(enable_timing=True)
            s.record()
            r = fn(*a, **k)
            e.record()
            self.events[name].append((s, e))
            return r

        return wrapped

    def summary(self) -> dict:
        out = {}
        for n, evs in self.events.items():
            if evs:
                ms = [s.elapsed_time(e) for s, e in evs]
                out[n] = {"calls": len(ms), "avg_ms": sum(ms) / len(ms), "total_ms": sum(ms)}
        return out

    def reset(self):
        self.events = {n: [] for n in self.NAMES}

    def restore(self):
        for n in self.NAMES:
            setattr(self.native, n, self.orig[n])


# ---------------------------------------------------------------------------
# Native arm
# ---------------------------------------------------------------------------
def build_layer(device, seed):
    import math

    import torch
    from torch import nn

    from dorafactors_b200.layer import DoraLinear

    g = torch.Generator(device=device).manual_seed(seed)
    base = nn.Linear(IN_F, OUT_F, bias=False, device=device, dtype=torch.bfloat16)
    with torch.no_grad():
        base.weight.copy_((torch.randn(OUT_F, IN_F, device=device, generator=g) * 0.02).bfloat16())
    mod = DoraLinear(base, r=RANK, scaling=SCALE, init_lora_B_zero=False)
    with torch.no_grad():
        bound = 1.0 / math.sqrt(IN_F)  # kaiming_uniform(a=sqrt(5)) bound for fan_in = IN_F
        mod.lora_A.weight.copy_(((torch.rand(RANK, IN_F, device=device, generator=g) * 2 - 1) * bound).bfloat16())
        mod.lora_B.weight.copy_((torch.randn(OUT_F, RANK, device=device, generator=g) * 0.01).bfloat16())
        mod.reset_magnitude()
    x = torch.randn(TOKENS, IN_F, device=device, generator=g).bfloat16()
    dy = torch.randn(TOKENS, OUT_F, device=device, generator=g).bfloat16()
    return mod, x, dy


def run_native(args) -> None:
    import torch
    import torch.distributed as dist

    from dorafactors_b200 import _native

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    torch.backends.cuda.matmul.allow_tf32 = False

    mod, x_dev, dy = build_layer(device, 1234 + rank)
    x = x_dev.clone().requires_grad_(True)
    params = [mod.lora_A.weight, mod.lora_B.weight, mod.lora_magnitude_vector.weight]

    reducer = None
    if world > 1:
        from dorafactors_b200.parallel import GradAllReducer

        # Each gradient's all-reduce starts as soon as it is accumulated and runs
        # under the rest of the backward (the base layer's dX GEMM).
        reducer = GradAllReducer(params)

    def step(xin):
        for p in params:
            p.grad = None
        xin.grad = None
        y = mod(xin)
        y.backward(dy)
        if reducer is not None:
            reducer.wait()

    def barrier():
        if world > 1:
            dist.barrier()

    timer = NativeTimer()
    for _ in range(args.warmup):
        step(x)
    torch.cuda.synchronize()
    barrier()
    clocks = ClockSampler(physical_gpu_index(local_rank))
    clocks.start()
    launches0 = _native.launch_count()
    timer.enabled = True
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier()
    t0.record()
    for _ in range(args.steps):
        step(x)
    t1.record()
    torch.cuda.synchronize()
    barrier()
    timer.enabled = False
    launches = _native.launch_count() - launches0
    ms = t0.elapsed_time(t1) / args.steps
    kern = timer.summary()
    peak_mem = torch.cuda.max_memory_allocated(device)

    # End to end through the public API: every step copies its 268 MB input from
    # pinned host memory and reads the magnitude gradient back, inside the timed
    # region.  The copy for step i+1 runs on a second stream while step i
    # computes (double-buffered input, as a data loader would feed it).
    x_host = x_dev.detach().cpu().pin_memory()
    dm_host = torch.empty(OUT_F, dtype=torch.bfloat16).pin_memory()
    copy_stream = torch.cuda.Stream(device)
    bufs = [torch.empty_like(x_dev).requires_grad_(True) for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]

    def issue_copy(i):
        b = i % 2
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(free[b])
            with torch.no_grad():
                bufs[b].copy_(x_host, non_blocking=True)
            ready[b].record(copy_stream)

    def e2e_steps(n):
        issue_copy(0)
        for i in range(n):
            b = i % 2
            torch.cuda.current_stream().wait_event(ready[b])
            if i + 1 < n:
                issue_copy(i + 1)
            step(bufs[b])
            free[b].record()
            dm_host.copy_(mod.lora_magnitude_vector.weight.grad, non_blocking=True)

    e2e_steps(max(1, args.warmup))
    torch.cuda.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    e2e_steps(args.steps)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    clk = clocks.stop()

    if world > 1:
        t = torch.tensor([ms, e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = float(t[0]), float(t[1])

    # Extra measurements (not the headline value): the unfused drop-in wiring of
    # the same layer, then the row-sharded 70B-class layer on both of its shapes.
    dropin = None if args.no_extras else measure_dropin(mod, x, dy, params, reducer, timer, args, world, device)
    del bufs, x_host
    rowshard = None
    if not args.no_extras:
        rowshard = {f"{o}x{i}": measure_rowshard(o, i, args, world, rank, device, timer) for o, i in ROWSHARD_SHAPES}
    sweep = None
    if not args.no_extras and world == 1:
        timer.enabled = False
        # The sweep times single calls of a few tens of microseconds: after the
        # power-capped GEMM-heavy steps above, one idle second lets the SM clock
        # return from its capped state, and the clocks seen during the sweep are
        # reported with it.
        time.sleep(1.0)
        sweep_clocks = ClockSampler(physical_gpu_index(local_rank))
        sweep_clocks.start()
        sweep_clocks.wait_first()
        sweep = measure_rank_sweep(device)
        sweep["clocks"] = sweep_clocks.stop()
    model = None
    if not args.no_extras and world == MODEL_EXTRA_WORLD:
        timer.enabled = False
        model = measure_model(args.layers, args.seq, MODEL_EXTRA_STEPS, args.warmup, world, rank, local_rank, device)

    if rank == 0:
        peaks, peak_src = load_peaks()
        kernels = {}
        hbm_bytes = {
            "compose_fwd": compose_fwd_bytes(TOKENS, OUT_F),
            "linear_output_fwd": compose_fwd_bytes(TOKENS, OUT_F),
            "compose_bwd": compose_bwd_bytes(TOKENS, OUT_F),
            "linear_output_bwd": compose_bwd_bytes(TOKENS, OUT_F),
        }
        for name, st in kern.items():
            if name in hbm_bytes:
                a = hbm_bytes[name] / (st["avg_ms"] * 1e-3) / 1e9
                kernels[name] = {**st, "algorithmic_bytes": hbm_bytes[name], "achieved_gbs": a,
                                 "frac": a / peaks["hbm_gbs"]}
            elif name == "weight_norm":
                # Timed inside a long step: against the sustained (power-capped) GEMM peak.
                a = norm_flops(OUT_F, IN_F, RANK) / (st["avg_ms"] * 1e-3) / 1e12
                kernels[name] = {**st, "algorithmic_flops": norm_flops(OUT_F, IN_F, RANK), "achieved_tflops": a,
                                 "peak_tflops": peaks["bf16_tflops_sustained"], "peak_kind": "sustained",
                                 "frac": a / peaks["bf16_tflops_sustained"]}
        dom = max(kern, key=lambda n: kern[n]["total_ms"]) if kern else None
        roof = None
        if dom in hbm_bytes:
            roof = {"kernel": dom, "bound": "hbm", "achieved": kernels[dom]["achieved_gbs"],
                    "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": kernels[dom]["frac"],
                    "traffic": read_traffic(dom), "algorithmic_bytes": hbm_bytes[dom], "peak_source": peak_src}
        elif dom == "weight_norm":
            roof = {"kernel": dom, "bound": "tensor", "achieved": kernels[dom]["achieved_tflops"],
                    "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s", "frac": kernels[dom]["frac"],
                    "traffic": read_traffic(dom), "algorithmic_flops": norm_flops(OUT_F, IN_F, RANK),
                    "peak_source": peak_src}
        value = TOKENS * world / (ms * 1e-3)
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded normal / kaiming-uniform weights, normal tokens)",
            "config": workload_config("single" if world == 1 else f"dp{world}"),
            "roofline": roof,
            "kernels": kernels,
            "e2e": {"value": TOKENS * world / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": TOKENS * IN_F * 2, "d2h_bytes_per_step": OUT_F * 2},
            "gpu_launches": launches,
            "clocks": clk,
            "peak_mem_gb": peak_mem / 1e9,
        }
        if dropin is not None:
            line["dropin_unfused"] = dropin
        if rowshard is not None:
            line["rowshard"] = rowshard
        if model is not None:
            line["model"] = model
        if sweep is not None:
            line["rank_sweep"] = sweep
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_sample()
        print(json.dumps(line), flush=True)
    timer.restore()
    if reducer is not None:
        reducer.remove()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _max_over_ranks(values: list[float], world: int, device) -> list[float]:
    import torch
    import torch.distributed as dist

    if world == 1:
        return values
    t = torch.tensor(values, device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t]


def measure_dropin(mod, x, dy, params, reducer, timer, args, world, device) -> dict:
    """The same layer wired as PEFT's unchanged DoraLinearVariant.forward wires it
    (variants.py:214-284): delta = DoraLinearLayer.forward(x, ..., base_result=result),
    then a separate y = result + delta, and autograd adds d_y and d_base for the base
    branch.  Timed like the headline step, for comparison with the fused layer output."""
    import torch

    layer = mod.lora_magnitude_vector

    def step():
        for p in params:
            p.grad = None
        x.grad = None
        result = mod.base_layer(x)
        delta = layer(x, lora_A=mod.lora_A, lora_B=mod.lora_B, scaling=SCALE, base_layer=mod.base_layer,
                      base_result=result)
        y = result + delta
        y.backward(dy)
        if reducer is not None:
            reducer.wait()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    timer.reset()
    timer.enabled = True
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    timer.enabled = False
    (ms,) = _max_over_ranks([e0.elapsed_time(e1) / args.steps], world, device)
    kern = {k: {"calls": v["calls"], "avg_ms": v["avg_ms"]} for k, v in timer.summary().items()}
    return {"what": "DoraLinearLayer.forward (delta) + separate result + delta, unchanged PEFT variant wiring",
            "ms_per_step": ms, "tokens_per_s": TOKENS * world / (ms * 1e-3), "kernels": kern}


SWEEP_RANKS = (16, 64, 128, 256, 512, 1024)
SWEEP_DIM = 8192


def measure_rank_sweep(device, iters: int = 10, warmup: int = 3) -> dict:
    """Rank sweep on a fixed layer (W0 8192 x 8192 bf16 ~N(0, 0.02), r in 16..1024,
    8192 tokens): the factored norm per rank, rated against HBM and the tensor pipe
    (it crosses from HBM-bound to tensor-bound near r = 281), and the compose forward
    and backward at 8192 x 8192.  Calls are timed back to back with CUDA events after
    a 256 MB write that evicts L2; W0 (134 MB) is larger than L2 (126 MB)."""
    import math

    import torch

    from dorafactors_b200 import _native

    peaks, _ = load_peaks()
    n = SWEEP_DIM
    g = torch.Generator(device=device).manual_seed(8192)
    W = (torch.randn(n, n, device=device, generator=g) * 0.02).bfloat16()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)

    def timed(fn) -> float:
        for _ in range(warmup):
            fn()
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            fn()
        e.record()
        e.synchronize()
        return s.elapsed_time(e) / iters

    out = {"workload": f"W0 {n}x{n} bf16, r in {list(SWEEP_RANKS)}, {n} tokens; {iters} calls back to back "
                       f"after an L2-evicting write",
           "norm": {}}
    for r in SWEEP_RANKS:
        A = ((torch.rand(r, n, device=device, generator=g) * 2 - 1) / math.sqrt(n)).bfloat16()
        B = (torch.randn(n, r, device=device, generator=g) * 0.01).bfloat16()
        norm = torch.empty(n, dtype=torch.bfloat16, device=device)
        ms = timed(lambda: _native.weight_norm(W, A, B, 1.0, norm))
        f, b = norm_flops(n, n, r), norm_bytes(n, n, r)
        tf, gbs = f / (ms * 1e-3) / 1e12, b / (ms * 1e-3) / 1e9
        bound = "hbm" if f / b < peaks["bf16_tflops"] * 1e12 / (peaks["hbm_gbs"] * 1e9) else "tensor"
        out["norm"][str(r)] = {"ms": ms, "gflop": f / 1e9, "tflops": tf, "tensor_frac": tf / peaks["bf16_tflops"],
                               "bytes": b, "gbs": gbs, "hbm_frac": gbs / peaks["hbm_gbs"], "bound": bound,
                               "frac": gbs / peaks["hbm_gbs"] if bound == "hbm" else tf / peaks["bf16_tflops"]}
    a = torch.randn(n, n, device=device, generator=g).bfloat16()
    c = torch.randn(n, n, device=device, generator=g).bfloat16()
    mag = (torch.rand(n, device=device, generator=g) + 0.5).bfloat16()
    o1, o2, dg = torch.empty_like(a), torch.empty_like(a), torch.empty(n, dtype=torch.bfloat16, device=device)
    for name, fn, nbytes in (
        ("linear_output_fwd", lambda: _native.linear_output_fwd(a, c, None, mag, 1.0, o1, o2), compose_fwd_bytes(n, n)),
        ("linear_output_bwd", lambda: _native.linear_output_bwd(a, c, mag, 1.0, o1, o2, dg), compose_bwd_bytes(n, n)),
    ):
        ms = timed(fn)
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"ms": ms, "bytes": nbytes, "gbs": gbs, "hbm_frac": gbs / peaks["hbm_gbs"]}
    del W, flush, a, c, o1, o2
    torch.cuda.empty_cache()
    return out


ROWSHARD_SHAPES = ((28672, 8192), (8192, 28672))
ROWSHARD_RANK, ROWSHARD_TOKENS = 256, 32768
NVLINK_GBS = 770.0  # measured peer copy per direction per GPU on this platform


def measure_rowshard(out_f, in_f, args, world, rank, device, timer) -> dict:
    """Out-feature row sharding of one 70B-class layer (strong scaling): W0 [out x in]
    bf16 ~N(0, 0.02), r = 256, 32768 tokens ~N(0, 1), s = 1.0.  Every rank holds out/P
    rows, runs the native norm and the fused compose + all-gather (its output columns
    stored into every rank's buffer over NVLink), and in backward the strided fused
    backward with the dX all-reduce overlapped.  Returns step time (max over ranks),
    tokens/s and per-kernel rooflines."""
    import math

    import torch
    import torch.distributed as dist

    from dorafactors_b200 import _native
    from dorafactors_b200.parallel import RowShardedDoraLinear

    r, T, scale = ROWSHARD_RANK, ROWSHARD_TOKENS, 1.0
    g = torch.Generator(device=device).manual_seed(4321)  # identical full tensors on every rank
    W = (torch.randn(out_f, in_f, device=device, generator=g) * 0.02).bfloat16()
    A = ((torch.rand(r, in_f, device=device, generator=g) * 2 - 1) / math.sqrt(in_f)).bfloat16()
    B = (torch.randn(out_f, r, device=device, generator=g) * 0.01).bfloat16()
    norm = torch.empty(out_f, dtype=torch.bfloat16, device=device)
    _native.weight_norm(W, A, B, scale, norm)
    layer = RowShardedDoraLinear.from_full(W, None, A, B, norm.clone(), scale)
    del W, B
    x = torch.randn(T, in_f, device=device, generator=g).bfloat16().requires_grad_(True)
    dy = torch.randn(T, out_f, device=device, generator=g).bfloat16()
    params = [layer.lora_A, layer.lora_B, layer.magnitude]

    def step():
        for p_ in params:
            p_.grad = None
        x.grad = None
        y = layer(x)
        y.backward(dy)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    timer.reset()
    timer.enabled = True
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    timer.enabled = False
    kern = timer.summary()
    if world == 1 and "linear_output_fwd" in kern:  # one shard: the plain layer-output kernel runs
        kern["linear_output_fwd_allgather"] = kern.pop("linear_output_fwd")
    names = ("weight_norm", "linear_output_fwd_allgather", "linear_output_bwd_strided")
    vals = _max_over_ranks([t0.elapsed_time(t1) / args.steps] + [kern.get(n, {}).get("avg_ms", 0.0) for n in names],
                           world, device)
    ms, k_ms = vals[0], dict(zip(names, vals[1:]))
    peaks, _ = load_peaks()
    w = layer.weight.shape[0]
    e = 2
    out = {"workload": f"row-sharded dora_linear_fwd_bwd out={out_f} in={in_f} r={r} tokens={T} bf16",
           "ranks": world, "rows_per_rank": w, "scaling": "strong", "ms_per_step": ms,
           "tokens_per_s": T / (ms * 1e-3), "kernels": {}}
    if k_ms["weight_norm"] > 0:
        f = norm_flops(w, in_f, r)
        a = f / (k_ms["weight_norm"] * 1e-3) / 1e12
        out["kernels"]["weight_norm"] = {"avg_ms": k_ms["weight_norm"], "algorithmic_flops": f, "achieved_tflops": a,
                                         "frac": a / peaks["bf16_tflops_sustained"], "peak": "bf16 sustained"}
    if k_ms["linear_output_fwd_allgather"] > 0:
        t = k_ms["linear_output_fwd_allgather"] * 1e-3
        # Local HBM: read lora + result, write inner + own y, plus the peers' columns
        # landing in this rank's y; NVLink: this rank's columns to every peer.
        hbm = e * T * w * 4 + e * T * w * (world - 1) + e * w
        link = e * T * w * (world - 1)
        bound = max(hbm / (peaks["hbm_gbs"] * 1e9), link / (NVLINK_GBS * 1e9))
        out["kernels"]["compose_allgather"] = {
            "avg_ms": k_ms["linear_output_fwd_allgather"], "hbm_bytes": hbm, "nvlink_bytes_out": link,
            "hbm_gbs": hbm / t / 1e9, "allgather_gbs": link / t / 1e9, "bound": "nvlink" if link / NVLINK_GBS >
            hbm / peaks["hbm_gbs"] else "hbm", "frac": bound / t,
            "peaks": {"hbm_gbs": peaks["hbm_gbs"], "nvlink_gbs": NVLINK_GBS}}
    if k_ms["linear_output_bwd_strided"] > 0:
        b = compose_bwd_bytes(T, w)
        a = b / (k_ms["linear_output_bwd_strided"] * 1e-3) / 1e9
        out["kernels"]["linear_output_bwd"] = {"avg_ms": k_ms["linear_output_bwd_strided"], "algorithmic_bytes": b,
                                               "achieved_gbs": a, "frac": a / peaks["hbm_gbs"]}
    layer.pool.close()
    del layer, x, dy
    torch.cuda.empty_cache()
    return out


def read_traffic(kernel: str):
    """DRAM bytes per launch from the committed ncu summary, if one exists for this kernel."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    try:
        with open(p) as f:
            for line in f:
                parts = line.split()
                if len(parts) >= 2 and parts[0] == kernel:
                    return float(parts[1])
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------
# CPU baseline / reference arm: the reference's own eager DoRA layer on the
# host cores (its dora.py / dora_fused.py, byte-compiled into oracle/_ref by
# oracle/build_ref.py), or the numpy oracle when that build is absent.
# ---------------------------------------------------------------------------
def cpu_threads() -> int:
    """Host threads this process may use (its CPU affinity, not OMP_NUM_THREADS)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover - non-Linux
        return os.cpu_count() or 1


def extrapolate_full_step(t_norm: float, t_step: float, tokens: int, full_tokens: int = TOKENS) -> float:
    """Seconds of one full-workload step estimated from a step on ``tokens`` tokens
    (``t_step``, which includes one factored norm) and the norm alone (``t_norm``):
    the token-proportional part scales, the norm does not."""
    return t_norm + max(t_step - t_norm, 0.0) * (full_tokens / tokens)


class CpuLayerStep:
    """One forward + backward of the adapted linear on the host cores, on ``tokens``
    tokens of the benchmark workload (full 28672 x 8192 r=384 bf16 weight, s=1.0).

    kind "reference": the reference's ``DoraLinearLayer`` (dora.py:1380-1484) on its
    eager CPU path, wired as ``DoraLinearVariant.forward`` wires it with no bias and
    no dropout (``y = result + delta``, variants.py:214-284), loss gradient ``dy``;
    the norm alone is ``_get_weight_norm_linear`` (dora.py:1024-1153).
    kind "port": the numpy oracle's restatement of the same step.
    """

    def __init__(self, tokens: int, seed: int = 0):
        import math

        import torch

        self.tokens = tokens
        self.threads = cpu_threads()
        torch.set_num_threads(self.threads)  # torchrun exports OMP_NUM_THREADS=1
        g = torch.Generator().manual_seed(seed)
        W = (torch.randn(OUT_F, IN_F, generator=g) * 0.02).bfloat16()
        A = ((torch.rand(RANK, IN_F, generator=g) * 2 - 1) / math.sqrt(IN_F)).bfloat16()
        B = (torch.randn(OUT_F, RANK, generator=g) * 0.01).bfloat16()
        try:
            from oracle.build_ref import load_reference

            dora, _ = load_reference()
            self.kind = "reference"
        except Exception as exc:  # oracle/_ref not built: fall back to the numpy port
            self.kind = "port"
            self.why_port = f"{type(exc).__name__}: {exc}"
            self.tokens = tokens = min(tokens, CPU_PORT_TOKENS)  # numpy GEMMs: a smaller sample
        x = torch.randn(tokens, IN_F, generator=g).bfloat16()
        dy = torch.randn(tokens, OUT_F, generator=g).bfloat16()
        if self.kind == "reference":
            from torch import nn

            self.base = nn.Linear(IN_F, OUT_F, bias=False, dtype=torch.bfloat16)
            self.lora_A = nn.Linear(IN_F, RANK, bias=False, dtype=torch.bfloat16)
            self.lora_B = nn.Linear(RANK, OUT_F, bias=False, dtype=torch.bfloat16)
            with torch.no_grad():
                self.base.weight.copy_(W)
                self.lora_A.weight.copy_(A)
                self.lora_B.weight.copy_(B)
            self.base.weight.requires_grad_(False)
            self.layer = dora.DoraLinearLayer(fan_in_fan_out=False)
            self.layer.update_layer(base_layer=self.base, lora_A=self.lora_A.weight, lora_B=self.lora_B.weight,
                                    scaling=SCALE)
            self.x = x.requires_grad_(True)
            self.dy = dy
        else:
            from oracle import dora_oracle as orc

            self.orc = orc
            self.np = [t.float().numpy() for t in (W, A, B, x, dy)]
            self.m, _ = orc.weight_norm_factored(self.np[0], self.np[1], self.np[2], SCALE, "bf16")

    def step(self) -> float:
        t0 = time.perf_counter()
        if self.kind == "reference":
            for p in (self.lora_A.weight, self.lora_B.weight, self.layer.weight):
                p.grad = None
            self.x.grad = None
            result = self.base(self.x)
            delta = self.layer(self.x, lora_A=self.lora_A, lora_B=self.lora_B, scaling=SCALE,
                               base_layer=self.base, base_result=result)
            y = result + delta
            y.backward(self.dy)
        else:
            W, A, B, x, dy = self.np
            self.orc.dora_linear_forward_backward(x, W, None, A, B, self.m, SCALE, dy, "bf16")
        return time.perf_counter() - t0

    def norm(self) -> float:
        t0 = time.perf_counter()
        if self.kind == "reference":
            import torch

            with torch.no_grad():
                self.layer._get_weight_norm_linear(base_weight=self.base.weight, lora_A_w=self.lora_A.weight,
                                                   lora_B_w=self.lora_B.weight, scaling=SCALE)
        else:
            W, A, B = self.np[:3]
            self.orc.weight_norm_factored(W, A, B, SCALE, "bf16")
        return time.perf_counter() - t0

    def describe(self) -> str:
        who = ("the reference's DoraLinearLayer (dora.py / dora_fused.py byte-compiled into oracle/_ref), "
               "eager CPU path" if self.kind == "reference"
               else f"numpy oracle of the reference's eager path (oracle/_ref unavailable: {self.why_port})")
        return (f"{who}; each step: y = base(x) + DoRA delta and y.backward(dy) on {self.tokens} of the "
                f"{TOKENS} tokens over the full {OUT_F}x{IN_F} r={RANK} bf16 weight (the factored norm is "
                f"recomputed every step, as in training); {self.threads} host threads")


def cpu_baseline_sample(steps: int = 3) -> dict:
    """The CPU baseline of the native line: a few measured steps (about 10 s of host work)."""
    c = CpuLayerStep(CPU_SAMPLE_TOKENS)
    c.step()  # warm-up
    t = [c.step() for _ in range(steps)]
    t_step = sum(t) / len(t)
    t_norm = c.norm()
    full = extrapolate_full_step(t_norm, t_step, c.tokens)
    return {
        "value": c.tokens / t_step,
        "unit": "tokens/s",
        "cores": c.threads,
        "kind": c.kind,
        "sample": c.describe() + f"; mean of {steps} steps after one warm-up",
        "ms_per_sample_step": t_step * 1e3,
        "extrapolated_full_workload": {"tokens_per_s": TOKENS / full, "ms_per_step": full * 1e3,
                                       "norm_ms": t_norm * 1e3,
                                       "how": f"norm once + token part x {TOKENS}/{c.tokens}"},
    }


def run_reference(args) -> None:
    """The reference arm: the reference's own CPU implementation of the path, timed on
    the host cores with all the threads this process may use.  Rank 0 only; under
    torchrun the other ranks exit without work."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    c = CpuLayerStep(CPU_SAMPLE_TOKENS)
    for _ in range(args.warmup):
        c.step()
    times = [c.step() for _ in range(args.steps)]
    t_step = sum(times) / len(times)
    t_norm = c.norm()
    full = extrapolate_full_step(t_norm, t_step, c.tokens)
    value = c.tokens / t_step
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": t_step * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded normal / uniform weights, normal tokens)",
        "config": {**workload_config("single"), "tokens_per_step_sampled": c.tokens},
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": c.threads, "kind": c.kind,
                         "sample": c.describe()},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "step_ms": {"median": statistics.median(times) * 1e3, "min": min(times) * 1e3, "max": max(times) * 1e3},
        "extrapolated_full_workload": {"tokens_per_s": TOKENS / full, "ms_per_step": full * 1e3,
                                       "norm_ms": t_norm * 1e3,
                                       "how": (f"estimate, not a measurement: the norm once + the measured "
                                               f"token part x {TOKENS}/{c.tokens}")},
    }
    print(json.dumps(line), flush=True)


def run_rowshard(args) -> None:
    """``--mode rowshard``: only the row-sharded 70B-class layer (``--shape``), one line."""
    import datetime

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    torch.backends.cuda.matmul.allow_tf32 = False
    out_f, in_f = (int(v) for v in args.shape.split("x"))
    timer = NativeTimer()
    res = measure_rowshard(out_f, in_f, args, world, rank, device, timer)
    timer.restore()
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": res["tokens_per_s"],
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": res["ms_per_step"],
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded normal / uniform weights, normal tokens)",
            "config": {"workload": res["workload"], "out_features": out_f, "in_features": in_f,
                       "rank": ROWSHARD_RANK, "tokens": ROWSHARD_TOKENS, "parallelism": f"rowshard{world}"},
            "kernels": res["kernels"],
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


MODEL_EXTRA_WORLD = 8  # the model-level configuration runs as an extra key at this many GPUs
MODEL_EXTRA_STEPS = 5


def measure_model(layers: int, seq: int, steps: int, warmup: int, world: int, rank: int, local_rank: int,
                  device) -> dict:
    """Model-level configuration: a Llama-style decoder (hidden 4096, FFN 14336, 32
    heads / 8 KV heads, vocab 128256; ``layers`` of them) with DoRA r=128, s=2.0 on
    q, k, v, o, gate, up and down, random weights; one sequence of ``seq`` random
    tokens per GPU (weak scaling), causal-LM loss, backward, DDP all-reduce of the
    adapter gradients, fused AdamW step.  Step time is the max over ranks."""
    import torch
    import torch.distributed as dist

    from dorafactors_b200 import _native
    from dorafactors_b200.model import add_dora, build_llama, llama_config

    cfg = llama_config(layers=layers)
    model = build_llama(cfg, device)
    params = add_dora(model, r=128, scaling=2.0)
    runner = model
    if world > 1:
        runner = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local_rank])
    opt = torch.optim.AdamW(params, lr=1e-5, fused=True)
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    ids = torch.randint(0, cfg.vocab_size, (1, seq), device=device, generator=g)

    def step():
        opt.zero_grad(set_to_none=True)
        loss = runner(input_ids=ids, labels=ids).loss
        loss.backward()
        opt.step()
        return loss

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.reset_peak_memory_stats(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = _native.launch_count()
    e0.record()
    for _ in range(steps):
        loss = step()
    e1.record()
    torch.cuda.synchronize()
    launches = _native.launch_count() - launches0
    ms = e0.elapsed_time(e1) / steps
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
    out = {"workload": f"llama-style decoder x{layers} (hidden 4096, ffn 14336, 32/8 heads, vocab 128256), "
                       f"DoRA r=128 s=2 on q,k,v,o,gate,up,down, {seq} tokens per GPU",
           "metric": "DoRA model training tokens/s (Llama-style, 7 adapted projections per layer)",
           "n_gpus": world, "layers": layers, "seq_len": seq, "global_batch": world, "parallelism": f"dp{world}",
           "steps": steps, "warmup": warmup, "ms_per_step": ms, "tokens_per_s": seq * world / (ms * 1e-3),
           "trainable_params": sum(p.numel() for p in params), "loss": float(loss.detach()),
           "native_launches_per_step": launches // max(steps, 1),
           "peak_mem_gb": torch.cuda.max_memory_allocated(device) / 1e9}
    del runner, model, opt, params
    torch.cuda.empty_cache()
    return out


def run_model(args) -> None:
    """``--mode model``: only the model-level configuration, one line."""
    import datetime

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
    clocks = ClockSampler(physical_gpu_index(local_rank))
    clocks.start()
    res = measure_model(args.layers, args.seq, args.steps, args.warmup, world, rank, local_rank, device)
    clk = clocks.stop()
    if rank == 0:
        line = {
            "metric": res["metric"],
            "value": res["tokens_per_s"],
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": res["ms_per_step"],
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (random-init weights, uniform random token ids)",
            "config": {"workload": res["workload"], "layers": args.layers, "global_batch": world,
                       "seq_len": args.seq, "trainable_params": res["trainable_params"],
                       "parallelism": f"dp{world}", "l2": "activations far larger than L2, no flush needed"},
            "loss": res["loss"],
            "gpu_launches": res["native_launches_per_step"] * args.steps,
            "clocks": clk,
            "peak_mem_gb": res["peak_mem_gb"],
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the host-core reference sample")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the extra measurements (unfused drop-in wiring, row-sharded 70B-class layer, "
                         "and at 8 GPUs the model-level configuration)")
    ap.add_argument("--mode", choices=["dp", "rowshard", "model"], default="dp",
                    help="dp: token data parallelism (default); rowshard: out-feature sharding of one layer; "
                         "model: Llama-style decoder with DoRA on every projection")
    ap.add_argument("--layers", type=int, default=32, help="model mode: decoder layers")
    ap.add_argument("--seq", type=int, default=4096, help="model mode: tokens per GPU")
    ap.add_argument("--shape", default="28672x8192", help="rowshard mode: out x in of the sharded layer")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.mode == "rowshard":
        run_rowshard(args)
    elif args.mode == "model":
        run_model(args)
    else:
        run_native(args)


if __name__ == "__main__":
    main()
