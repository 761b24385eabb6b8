"""The measurement side of bench.py on CPU: the algorithmic work it rates kernels
against (FLOPs of the factored norm, bytes of the compose kernels), the peak and
DRAM-traffic lookups behind `roofline`, the workload description, and the CPU
arms' thread count and full-workload estimate.  No GPU work."""

import importlib.util
import json
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_workload_is_the_high_rank_layer(bench):
    cfg = bench.workload_config("single")
    assert (cfg["out_features"], cfg["in_features"], cfg["rank"], cfg["tokens_per_rank"]) == (28672, 8192, 384, 16384)
    assert cfg["scale"] == 1.0 and cfg["parallelism"] == "single"
    assert "L2" in cfg["l2"]


def test_algorithmic_work(bench):
    # 2*out*in*r (W0 A^T) + 2*r^2*in (A A^T) + 2*out*r^2 (B G): 180.39 + 2.42 + 8.46 GFLOP.
    assert bench.norm_flops(28672, 8192, 384) == 2 * 28672 * 8192 * 384 + 2 * 384 * 384 * 8192 + 2 * 28672 * 384 * 384
    assert abs(bench.norm_flops(28672, 8192, 384) / 1e9 - 191.26) < 0.01
    # Read lora + base, write out + inner, read g: 3.758 GB at 16384 x 28672 bf16.
    assert bench.compose_fwd_bytes(16384, 28672) == 2 * 4 * 16384 * 28672 + 2 * 28672
    assert abs(bench.compose_fwd_bytes(16384, 28672) / 1e9 - 3.758) < 0.001
    assert bench.compose_bwd_bytes(16384, 28672) >= bench.compose_fwd_bytes(16384, 28672)
    # Norm bytes: W0, A, B read once and the norm written.
    assert bench.norm_bytes(8192, 8192, 16) == 2 * (8192 * 8192 + 16 * 8192 + 8192 * 16) + 2 * 8192


def test_peaks_and_traffic_lookups(bench):
    peaks, src = bench.load_peaks()
    assert src in ("measured", "fallback")
    for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained"):
        assert peaks[k] > 0
    if src == "measured":
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            assert peaks["hbm_gbs"] == float(json.load(f)["hbm_gbs"])
    # The committed one-pass ncu captures of the compose kernels back roofline.traffic.
    for k in ("linear_output_fwd", "linear_output_bwd"):
        t = bench.read_traffic(k)
        assert t is not None and 3.0e9 < t < 4.5e9
    assert bench.read_traffic("no_such_kernel") is None


def test_cpu_full_workload_extrapolation(bench):
    # A step on a token sample includes one factored norm: only the token part scales.
    t_norm, t_step, tokens = 1.0, 3.0, 4096
    est = bench.extrapolate_full_step(t_norm, t_step, tokens)
    assert abs(est - (1.0 + 2.0 * bench.TOKENS / tokens)) < 1e-12
    assert bench.extrapolate_full_step(2.0, 1.0, tokens) == 2.0  # never below the norm alone


def test_cpu_threads_follow_affinity_not_omp(bench, monkeypatch):
    # torchrun exports OMP_NUM_THREADS=1; the host-core arms use every thread they may.
    monkeypatch.setenv("OMP_NUM_THREADS", "1")
    assert bench.cpu_threads() == len(os.sched_getaffinity(0))
