"""Time one native DoRA operation at given shapes (CUDA events, device-resident inputs).

    python -m dorafactors_b200.microbench --op norm --out 8192 --in 8192 --rank 384
    python -m dorafactors_b200.microbench --op compose_fwd --rows 16384 --cols 28672
    python -m dorafactors_b200.microbench --op compose_bwd --rows 16384 --cols 28672
    python -m dorafactors_b200.microbench --op linear_output_bwd --rows 16384 --cols 28672
    python -m dorafactors_b200.microbench --op allgather:2 --rows 32768 --cols 14336
    python -m dorafactors_b200.microbench --op sweep      # rank sweep on an 8192 x 8192 layer

Each run prints one JSON line per measurement: average milliseconds per call,
the algorithmic work, achieved GB/s or TFLOP/s and the fraction of the measured
peaks (``MEASURED_PEAKS.json`` at the repository root when present).  Inputs are
seeded synthetic tensors larger than L2 at the default sizes.  ``--iters 1
--warmup 0`` gives a single launch for a profiler capture.
"""

from __future__ import annotations

import argparse
import json
import os

import torch

from . import _native

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def _peaks() -> dict:
    try:
        with open(os.path.join(_ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    except Exception:
        return {**_FALLBACK, "source": "fallback"}


def _time(fn, iters: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / max(iters, 1)


def bench_norm(out_f: int, in_f: int, r: int, iters: int, warmup: int, dtype=torch.bfloat16,
               adapter_dtype=None) -> dict:
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    adt = adapter_dtype or dtype
    W = (torch.randn(out_f, in_f, device=dev, generator=g) * 0.02).to(dtype)
    A = ((torch.rand(r, in_f, device=dev, generator=g) * 2 - 1) / in_f**0.5).to(adt)
    B = (torch.randn(out_f, r, device=dev, generator=g) * 0.01).to(adt)
    norm = torch.empty(out_f, dtype=dtype, device=dev)
    ms = _time(lambda: _native.weight_norm(W, A, B, 1.0, norm), iters, warmup)
    flops = 2 * out_f * in_f * r + 2 * r * r * in_f + 2 * out_f * r * r
    nbytes = W.element_size() * (out_f * in_f + out_f) + A.element_size() * (r * in_f + out_f * r)
    pk = _peaks()
    tf = flops / (ms * 1e-3) / 1e12
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"op": "weight_norm", "out": out_f, "in": in_f, "rank": r, "adapter_dtype": str(adt).replace("torch.", ""),
            "ms": ms, "gflop": flops / 1e9,
            "tflops": tf, "tensor_frac": tf / pk["bf16_tflops"], "bytes": nbytes, "gbs": gbs,
            "hbm_frac": gbs / pk["hbm_gbs"], "peak_source": pk["source"]}


def bench_compose(op: str, rows: int, cols: int, iters: int, warmup: int, dtype=torch.bfloat16) -> dict:
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    a = torch.randn(rows, cols, device=dev, generator=g).to(dtype)
    b = torch.randn(rows, cols, device=dev, generator=g).to(dtype)
    mag = (torch.rand(cols, device=dev, generator=g) + 0.5).to(dtype)
    e = a.element_size()
    if op == "compose_fwd":
        out = torch.empty_like(a)
        inner = torch.empty_like(a)
        ms = _time(lambda: _native.compose_fwd(a, b, mag, 1.0, out, inner), iters, warmup)
        nbytes = 4 * e * rows * cols + e * cols
    elif op == "compose_fwd_inference":
        out = torch.empty_like(a)
        ms = _time(lambda: _native.compose_fwd(a, b, mag, 1.0, out, None), iters, warmup)
        nbytes = 3 * e * rows * cols + e * cols
    elif op == "compose_bwd":
        dl = torch.empty_like(a)
        db = torch.empty_like(a)
        dg = torch.empty(cols, dtype=dtype, device=dev)
        ms = _time(lambda: _native.compose_bwd(a, b, mag, 1.0, dl, db, dg), iters, warmup)
        nbytes = 4 * e * rows * cols + 2 * e * cols
    elif op == "linear_output_fwd":
        # y = result + ((g - 1) * (result - bias) + g * (s * lora)) and inner = s * lora + (result - bias)
        bias = torch.randn(cols, device=dev, generator=g).to(dtype)
        y = torch.empty_like(a)
        inner = torch.empty_like(a)
        ms = _time(lambda: _native.linear_output_fwd(a, b, bias, mag, 1.0, y, inner), iters, warmup)
        nbytes = 4 * e * rows * cols + 2 * e * cols
    elif op.startswith("allgather"):
        # The row-sharded layer's compose with the output gather: this shard's columns
        # stored into `ranks` full-width buffers (local ones here; peers over NVLink in
        # the layer), ld = cols * ranks, the shard at column offset cols.
        ranks = int(op.split(":")[1]) if ":" in op else 1
        ld = cols * max(ranks, 2) if ranks > 1 else cols
        col0 = cols if ranks > 1 else 0
        bufs = [torch.empty(rows, ld, device=dev, dtype=dtype) for _ in range(ranks)]
        inner = torch.empty_like(a)
        ptrs = [t.data_ptr() for t in bufs]
        ms = _time(lambda: _native.linear_output_fwd_allgather(a, b, None, mag, 1.0, ptrs, 0, col0, ld, inner),
                   iters, warmup)
        nbytes = 4 * e * rows * cols + e * cols + (ranks - 1) * e * rows * cols
    elif op == "linear_output_bwd":
        # d_lora = g * s * dy, d_result = g * dy, d_g = column sums of inner * dy
        dl = torch.empty_like(a)
        dr = torch.empty_like(a)
        dg = torch.empty(cols, dtype=dtype, device=dev)
        ms = _time(lambda: _native.linear_output_bwd(a, b, mag, 1.0, dl, dr, dg), iters, warmup)
        nbytes = 4 * e * rows * cols + 2 * e * cols
    else:
        raise ValueError(op)
    pk = _peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"op": op, "rows": rows, "cols": cols, "ms": ms, "bytes": nbytes, "gbs": gbs,
            "hbm_frac": gbs / pk["hbm_gbs"], "peak_source": pk["source"]}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", required=True,
                    help="norm | compose_fwd | compose_fwd_inference | compose_bwd | linear_output_fwd | "
                         "linear_output_bwd | allgather[:ranks] | sweep")
    ap.add_argument("--out", type=int, default=28672)
    ap.add_argument("--in", dest="inp", type=int, default=8192)
    ap.add_argument("--rank", type=int, default=384)
    ap.add_argument("--rows", type=int, default=16384)
    ap.add_argument("--cols", type=int, default=28672)
    ap.add_argument("--adapter-dtype", choices=["same", "fp32"], default="same",
                    help="norm: adapters in the weight dtype or in fp32 (PEFT's default on a bf16 base)")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    if a.op == "norm":
        adt = torch.float32 if a.adapter_dtype == "fp32" else None
        print(json.dumps(bench_norm(a.out, a.inp, a.rank, a.iters, a.warmup, adapter_dtype=adt)), flush=True)
    elif a.op == "sweep":
        # Rank sweep on an 8192 x 8192 bf16 layer with 8192 tokens.
        for r in (16, 64, 128, 256, 512, 1024):
            print(json.dumps(bench_norm(8192, 8192, r, a.iters, a.warmup)), flush=True)
        for op in ("compose_fwd", "compose_bwd"):
            print(json.dumps(bench_compose(op, 8192, 8192, a.iters, a.warmup)), flush=True)
    else:
        print(json.dumps(bench_compose(a.op, a.rows, a.cols, a.iters, a.warmup)), flush=True)
    if _native.device_error(reset=True) != 0:
        raise SystemExit("device error word set")


if __name__ == "__main__":
    main()
