"""Factored row norm (tcgen05 path for bf16/fp16, CUDA-core path otherwise)
through the C ABI, against the oracle, the reference's golden fixtures and a
PyTorch fp32 evaluation on the GPU at the full layer sizes.

Tolerance: norms within 1e-2 relative (elementwise) in bf16/fp16 and 1e-5 in
fp32.  The fp32 intermediate terms are checked tighter where the path allows.
"""

import numpy as np
import pytest
import torch

from _golden import RTOL, assert_close, load_group, to_dev, to_np
from oracle import dora_oracle as orc

pytestmark = pytest.mark.gpu

NORM = load_group("norm")
ASSEMBLY = load_group("assembly")


@pytest.fixture(autouse=True)
def _no_device_error():
    from dorafactors_b200 import _native

    yield
    assert _native.device_error(reset=True) == 0


def _native_norm(W, A, B, s, dtype, adt=None, parts=True):
    from dorafactors_b200 import _native

    adt = adt or dtype
    tW, tA, tB = to_dev(W, dtype), to_dev(A, adt), to_dev(B, adt)
    out = torch.empty(W.shape[0], dtype=tW.dtype, device="cuda")
    p = torch.empty(3 * W.shape[0], dtype=torch.float32, device="cuda") if parts else None
    _native.weight_norm(tW, tA, tB, s, out, p)
    return to_np(out), (to_np(p).reshape(3, -1) if parts else None)


def _elem_rel(a, ref):
    a = np.asarray(a, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(a - ref) / np.maximum(np.abs(ref), 1e-30)))


@pytest.mark.parametrize("case", sorted(NORM))
def test_norm_golden(case):
    from dorafactors_b200.dora import DoraLinearLayer

    st = NORM[case]
    dt = st["dtype"]
    layer = DoraLinearLayer(fan_in_fan_out=bool(st["fan_in_fan_out"]))
    n = layer._get_weight_norm_linear(
        base_weight=to_dev(st["W"], dt), lora_A_w=to_dev(st["A"], dt), lora_B_w=to_dev(st["B"], dt),
        scaling=float(st["scale"]),
    )
    assert n.dtype == to_dev(st["W"], dt).dtype
    assert _elem_rel(to_np(n), st["norm"]) <= RTOL[dt], case
    lw = to_dev(st["B"] @ st["A"], "fp32")
    nd = layer.get_weight_norm(to_dev(st["W"], dt), lw, float(st["scale"]))
    assert _elem_rel(to_np(nd), st["norm_dense"]) <= RTOL[dt], case


@pytest.mark.parametrize("case", sorted(ASSEMBLY))
def test_assembly_bitwise_vs_oracle(case):
    from dorafactors_b200.dora_fused import fused_norm_assembly

    st = ASSEMBLY[case]
    s = float(st["scale"])
    (n,) = fused_norm_assembly(to_dev(st["w"], "fp32"), to_dev(st["c"], "fp32"), to_dev(st["b"], "fp32"), s)
    np.testing.assert_array_equal(to_np(n), orc.assemble_norm(st["w"], st["c"], st["b"], s))


# (out, in, r, dtype): tensor-core shapes (in % 8 == 0), ragged M tiles, r from
# 1 to 520, and shapes that take the CUDA-core path (fp32, in % 8 != 0).
CASES = [
    (128, 64, 16, "bf16"),
    (300, 256, 8, "bf16"),
    (1000, 1024, 64, "bf16"),
    (513, 2048, 384, "bf16"),
    (256, 512, 520, "bf16"),
    (384, 768, 100, "bf16"),
    (200, 1000, 24, "fp16"),
    (640, 4096, 256, "fp16"),
    (96, 72, 1, "bf16"),
    (130, 100, 12, "bf16"),
    (257, 320, 40, "fp32"),
    (64, 4096, 128, "fp32"),
    (300, 512, 600, "bf16"),  # three N tiles of the row-dot GEMM, the last one ragged
    (700, 2048, 200, "bf16"),  # two k-blocks per stream-K stage, two stages
    (300, 1000, 176, "fp16"),  # the same with a ragged last unit (16 k-blocks, K % 64 != 0)
    (700, 4160, 256, "bf16"),  # CTA-pair stream-K, two k-blocks per stage, 65 k-blocks (last stage half past K)
    (3000, 4104, 16, "bf16"),  # low rank: Gram fused into the stream-K kernel, ragged K and M
    (1000, 2048, 8, "fp16"),  # the same in fp16, r = 8 (A's box reads zero rows past r)
    (100, 8192, 16, "bf16"),  # one partial tile: every Gram k-block on the same tile
    (20000, 512, 16, "bf16"),  # low rank, short K: two to three segments per CTA back to back
    (5000, 256, 8, "bf16"),  # one unit per tile: every unit its own segment
]


@pytest.mark.parametrize("out_f,in_f,r,dtype", CASES)
def test_norm_vs_oracle(out_f, in_f, r, dtype):
    rng = np.random.default_rng(out_f * 7 + in_f + r)
    W = orc.round_to(rng.standard_normal((out_f, in_f)) * 0.02, dtype)
    A = orc.round_to(rng.uniform(-1, 1, (r, in_f)) / np.sqrt(in_f), dtype)
    B = orc.round_to(rng.standard_normal((out_f, r)) * 0.01, dtype)
    s = 1.5
    n, parts = _native_norm(W, A, B, s, dtype)
    ref, rp = orc.weight_norm_factored(W, A, B, s, dtype)
    assert _elem_rel(n, ref) <= RTOL[dtype]
    # The fp32 intermediate terms, normwise.
    assert_close(parts[0], rp["w_norm_sq"], 1e-5, "||W||^2")
    assert_close(parts[1], rp["cross"], 1e-4 if dtype != "fp32" else 1e-5, "cross")
    assert_close(parts[2], rp["ba"], 1e-4 if dtype != "fp32" else 1e-5, "B G B^T")


def test_norm_large_lora_term():
    """A LoRA term as large as W0 exercises the cross and B G B^T terms at full weight."""
    rng = np.random.default_rng(21)
    out_f, in_f, r = 384, 1024, 64
    W = orc.round_to(rng.standard_normal((out_f, in_f)) * 0.02, "bf16")
    A = orc.round_to(rng.uniform(-1, 1, (r, in_f)) / np.sqrt(in_f), "bf16")
    B = orc.round_to(rng.standard_normal((out_f, r)) * 0.5, "bf16")
    for s in (0.5, 2.0, -1.0):
        n, _ = _native_norm(W, A, B, s, "bf16")
        dense = orc.weight_norm_dense(W, B.astype(np.float64) @ A.astype(np.float64), s, "fp32")
        assert _elem_rel(n, dense) <= 1e-2


def test_norm_scale_zero_and_rank_zero():
    rng = np.random.default_rng(2)
    W = orc.round_to(rng.standard_normal((200, 512)) * 0.02, "bf16")
    A = orc.round_to(rng.standard_normal((16, 512)), "bf16")
    B = orc.round_to(rng.standard_normal((200, 16)), "bf16")
    n, parts = _native_norm(W, A, B, 0.0, "bf16")
    ref, _ = orc.weight_norm_factored(W, A, B, 0.0, "bf16")
    assert _elem_rel(n, ref) <= 1e-2
    assert np.all(parts[1] == 0) and np.all(parts[2] == 0)


@pytest.mark.parametrize("wdt", ["bf16", "fp16"])
@pytest.mark.parametrize("out_f,in_f,r,s", [(256, 512, 32, 2.0), (1000, 2048, 384, 0.5), (3000, 4104, 200, 1.0),
                                           (512, 1000, 16, 3.0)])
def test_norm_mixed_adapter_dtype(wdt, out_f, in_f, r, s):
    """Half W0 with fp32 adapters (PEFT's default adapter dtype, dora.py:1061 computes
    in fp32): the adapters are rounded into W0's dtype and the tensor-core path runs
    (the CUDA-core path for in % 8 != 0).  Against the oracle's fp32 evaluation of
    the fp32 adapters, at the parity bar; the fp32 terms within the adapters' own
    rounding (2^-8 relative, normwise)."""
    rng = np.random.default_rng(out_f + r)
    W = orc.round_to(rng.standard_normal((out_f, in_f)) * 0.02, wdt)
    A = (rng.uniform(-1, 1, (r, in_f)) / np.sqrt(in_f)).astype(np.float32)
    B = (rng.standard_normal((out_f, r)) * 0.05).astype(np.float32)
    n, parts = _native_norm(W, A, B, s, wdt, adt="fp32")
    ref, rp = orc.weight_norm_factored(W, A, B, s, wdt)
    assert _elem_rel(n, ref) <= RTOL[wdt]
    assert_close(parts[0], rp["w_norm_sq"], 1e-5, "||W0||^2")
    assert_close(parts[1], rp["cross"], 2.0**-8, "cross")
    assert_close(parts[2], rp["ba"], 2.0**-8, "B G B^T")


def test_norm_mixed_adapter_dtype_full_size():
    """The benchmark layer (28672 x 8192, r = 384) with fp32 adapters on a bf16 W0:
    against PyTorch fp32 GEMMs of the fp32 adapters on the same GPU."""
    from dorafactors_b200 import _native

    torch.manual_seed(1)
    out_f, in_f, r = 28672, 8192, 384
    W = (torch.randn(out_f, in_f, device="cuda") * 0.02).bfloat16()
    A = (torch.rand(r, in_f, device="cuda") * 2 - 1) / in_f**0.5
    B = torch.randn(out_f, r, device="cuda") * 0.01
    norm = torch.empty(out_f, dtype=torch.bfloat16, device="cuda")
    parts = torch.empty(3 * out_f, dtype=torch.float32, device="cuda")
    _native.weight_norm(W, A, B, 1.0, norm, parts)
    w, c, b = _torch_fp32_norm_parts(W, A, B)
    p = parts.view(3, -1)
    for got, ref, tol in ((p[0], w, 1e-5), (p[1], c, 2.0**-8), (p[2], b, 2.0**-8)):
        rel = ((got.double() - ref.double()).norm() / ref.double().norm()).item()
        assert rel <= tol, rel
    ref_norm = torch.sqrt((w + 2 * c + b).clamp_min(0)).bfloat16()
    rel = ((norm.float() - ref_norm.float()).abs() / ref_norm.float()).max().item()
    assert rel <= 1e-2


def _torch_fp32_norm_parts(W, A, B):
    Wf, Af, Bf = W.float(), A.float(), B.float()
    w = (Wf * Wf).sum(1)
    U = Wf @ Af.T
    G = Af @ Af.T
    c = (Bf * U).sum(1)
    b = ((Bf @ G) * Bf).sum(1)
    return w, c, b


@pytest.mark.parametrize("out_f,in_f,r", [(28672, 8192, 384), (8192, 8192, 1024), (8192, 8192, 16),
                                         (28672, 8192, 16), (28672, 8192, 8)])
def test_norm_full_size_vs_torch_fp32(out_f, in_f, r):
    """Layer sizes of the benchmark: the tcgen05 result against PyTorch fp32 GEMMs on the same GPU."""
    from dorafactors_b200 import _native

    torch.manual_seed(0)
    W = (torch.randn(out_f, in_f, device="cuda") * 0.02).bfloat16()
    A = ((torch.rand(r, in_f, device="cuda") * 2 - 1) / in_f**0.5).bfloat16()
    B = (torch.randn(out_f, r, device="cuda") * 0.01).bfloat16()
    norm = torch.empty(out_f, dtype=torch.bfloat16, device="cuda")
    parts = torch.empty(3 * out_f, dtype=torch.float32, device="cuda")
    _native.weight_norm(W, A, B, 1.0, norm, parts)
    w, c, b = _torch_fp32_norm_parts(W, A, B)
    p = parts.view(3, -1)
    for got, ref, tol in ((p[0], w, 1e-5), (p[1], c, 1e-4), (p[2], b, 1e-4)):
        rel = ((got.double() - ref.double()).norm() / ref.double().norm()).item()
        assert rel <= tol, rel
    ref_norm = torch.sqrt((w + 2 * c + b).clamp_min(0)).bfloat16()
    rel = ((norm.float() - ref_norm.float()).abs() / ref_norm.float()).max().item()
    assert rel <= 1e-2


_PAIR_SCRIPT = r"""
import json, sys, torch
sys.path.insert(0, sys.argv[1])
from dorafactors_b200 import _native
out = {}
for out_f, in_f, r in ((28672, 8192, 384), (8192, 4096, 256), (1000, 2048, 384), (640, 1024, 64),
                      (8192, 8192, 16), (4096, 4096, 512), (257, 320, 40), (2048, 2048, 768), (640, 1024, 520),
                      (3000, 4104, 200), (1500, 4160, 256), (1024, 1024, 1024), (3000, 4104, 16)):
    g = torch.Generator(device="cuda").manual_seed(out_f + r)
    W = (torch.randn(out_f, in_f, device="cuda", generator=g) * 0.02).bfloat16()
    A = ((torch.rand(r, in_f, device="cuda", generator=g) * 2 - 1) / in_f**0.5).bfloat16()
    B = (torch.randn(out_f, r, device="cuda", generator=g) * 0.01).bfloat16()
    norm = torch.empty(out_f, dtype=torch.bfloat16, device="cuda")
    parts = torch.empty(3 * out_f, dtype=torch.float32, device="cuda")
    _native.weight_norm(W, A, B, 1.0, norm, parts)
    torch.cuda.synchronize()
    out[f"{out_f}x{in_f}r{r}"] = parts.cpu().tolist()
out["device_error"] = _native.device_error(reset=True)
json.dump(out, sys.stdout)
"""


_SWITCHES = ("DORA_B200_SK", "DORA_B200_PAIR", "DORA_B200_SK2", "DORA_B200_PAIR_NT", "DORA_B200_PAIR_WIDE",
             "DORA_B200_FUSE_G")


@pytest.mark.parametrize("env", [{"DORA_B200_SK": "0"}, {"DORA_B200_PAIR": "1"}, {"DORA_B200_SK2": "1"},
                                 {"DORA_B200_SK2": "0"}, {"DORA_B200_PAIR_NT": "128"}, {"DORA_B200_PAIR_WIDE": "0"},
                                 {"DORA_B200_FUSE_G": "0"}],
                         ids=["split_k", "cta_pair", "cta_pair_stream_k", "single_stream_k", "pair_n_tiles_128",
                              "pair_n_tiles_256", "separate_gram"])
def test_cross_term_kernels_agree(env):
    """The tcgen05 cross-term kernels give the same fp32 terms: the default choice
    (CTA-pair stream-K for r > 240, single-CTA stream-K below) against the split-K
    kernel (DORA_B200_SK=0), the CTA-pair split-K kernel (DORA_B200_PAIR=1), each
    stream-K kernel forced everywhere (DORA_B200_SK2=1 / 0), the CTA-pair stream-K
    kernel on narrower N tiles (DORA_B200_PAIR_NT=128, DORA_B200_PAIR_WIDE=0) and the
    separate Gram launches at r <= 16 (DORA_B200_FUSE_G=0), in child processes."""
    import json
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    runs = {}
    for name, extra in (("default", {}), ("other", env)):
        e = {k: v for k, v in os.environ.items() if k not in _SWITCHES}
        e.update(extra)
        res = subprocess.run([sys.executable, "-c", _PAIR_SCRIPT, root], env=e, capture_output=True, text=True,
                             timeout=300)
        assert res.returncode == 0, res.stderr[-2000:]
        runs[name] = json.loads(res.stdout)
    for name in runs:
        assert runs[name].pop("device_error") == 0
    for key, ref in runs["default"].items():
        p = np.asarray(runs["other"][key], np.float64).reshape(3, -1)
        s = np.asarray(ref, np.float64).reshape(3, -1)
        # Different K partitions sum the fp32 partials in different orders: agreement to
        # fp32 rounding (normwise 1e-5, the same bound as against PyTorch's fp32 GEMMs).
        # At r <= 16 the fused path forms B G B^T from the fp32 Gram on CUDA cores, the
        # separate launches from its two-term bf16 split (about 2^-16 relative): 1e-4 there.
        for i in range(3):
            tol = 1e-4 if (i == 2 and "DORA_B200_FUSE_G" in env) else 1e-5
            rel = np.linalg.norm(p[i] - s[i]) / max(np.linalg.norm(s[i]), 1e-30)
            assert rel <= tol, (key, i, rel)
