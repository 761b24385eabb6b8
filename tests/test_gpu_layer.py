"""The whole adapted linear (base + LoRA + DoRA) on the native path: forward and
backward against the reference's golden fixtures and the oracle.

Tolerance: 1e-2 relative (normwise) in bf16, 1e-5 in fp32, for y, the delta,
the norm and the gradients dx, dA, dB, dm.  The base and LoRA GEMMs are
PyTorch/cuBLAS (owned by the caller, as in PEFT); on fp32 they run with TF32
disabled.
"""

import numpy as np
import pytest
import torch

from _golden import RTOL, assert_close, load_group, rel_errors, to_dev, to_np
from oracle import dora_oracle as orc

pytestmark = pytest.mark.gpu

LAYER = load_group("layer")


@pytest.fixture(autouse=True)
def _no_tf32_no_device_error():
    from dorafactors_b200 import _native

    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old
    assert _native.device_error(reset=True) == 0


def _build(st, dt):
    from dorafactors_b200.dora import DoraLinearLayer

    W = to_dev(st["W"], dt)
    out_f, in_f = W.shape
    r = st["A"].shape[0]
    base = torch.nn.Linear(in_f, out_f, bias="bias" in st, device="cuda", dtype=W.dtype)
    lora_A = torch.nn.Linear(in_f, r, bias=False, device="cuda", dtype=W.dtype)
    lora_B = torch.nn.Linear(r, out_f, bias=False, device="cuda", dtype=W.dtype)
    with torch.no_grad():
        base.weight.copy_(W)
        if "bias" in st:
            base.bias.copy_(to_dev(st["bias"], dt))
        lora_A.weight.copy_(to_dev(st["A"], dt))
        lora_B.weight.copy_(to_dev(st["B"], dt))
    base.requires_grad_(False)
    layer = DoraLinearLayer(fan_in_fan_out=False)
    layer.update_layer(base_layer=base, lora_A=lora_A.weight, lora_B=lora_B.weight, scaling=float(st["scale"]))
    return base, lora_A, lora_B, layer


@pytest.mark.parametrize("case", sorted(LAYER))
def test_layer_golden(case):
    st = LAYER[case]
    dt = st["dtype"]
    base, lora_A, lora_B, layer = _build(st, dt)
    assert_close(to_np(layer.weight), st["m"], RTOL[dt], "initial magnitude")
    x = to_dev(st["x"], dt).requires_grad_(True)
    result = base(x)
    delta = layer(x, lora_A=lora_A, lora_B=lora_B, scaling=float(st["scale"]), base_layer=base, base_result=result)
    y = result + delta
    y.backward(to_dev(st["dy"], dt))
    got = {"y": y, "delta": delta, "dx": x.grad, "dA": lora_A.weight.grad, "dB": lora_B.weight.grad,
           "dm": layer.weight.grad}
    for k, v in got.items():
        assert_close(to_np(v), st[k], RTOL[dt], f"{case} {k}")


@pytest.mark.parametrize("dtype,T,in_f,out_f,r", [("bf16", 256, 512, 768, 32), ("fp32", 64, 256, 320, 16),
                                                  ("bf16", 2048, 4096, 4096, 16)])
def test_dora_linear_vs_oracle(dtype, T, in_f, out_f, r):
    """DoraLinear (PEFT wiring) forward + backward against the oracle's eager restatement."""
    from dorafactors_b200.layer import DoraLinear

    rng = np.random.default_rng(T + in_f + r)
    W = orc.round_to(rng.standard_normal((out_f, in_f)) * 0.02, dtype)
    A = orc.round_to(rng.uniform(-1, 1, (r, in_f)) / np.sqrt(in_f), dtype)
    B = orc.round_to(rng.standard_normal((out_f, r)) * 0.01, dtype)
    x = orc.round_to(rng.standard_normal((T, in_f)), dtype)
    dy = orc.round_to(rng.standard_normal((T, out_f)), dtype)
    s = 2.0
    tdt = to_dev(W, dtype).dtype
    base = torch.nn.Linear(in_f, out_f, bias=False, device="cuda", dtype=tdt)
    with torch.no_grad():
        base.weight.copy_(to_dev(W, dtype))
    mod = DoraLinear(base, r=r, scaling=s)
    with torch.no_grad():
        mod.lora_A.weight.copy_(to_dev(A, dtype))
        mod.lora_B.weight.copy_(to_dev(B, dtype))
        mod.reset_magnitude()
    m = to_np(mod.lora_magnitude_vector.weight)
    tx = to_dev(x, dtype).requires_grad_(True)
    y = mod(tx)
    y.backward(to_dev(dy, dtype))
    ref = orc.dora_linear_forward_backward(x, W, None, A, B, m, s, dy, dtype)
    assert_close(to_np(y), ref["y"], RTOL[dtype], "y")
    assert_close(to_np(tx.grad), ref["dx"], RTOL[dtype], "dx")
    assert_close(to_np(mod.lora_A.weight.grad), ref["dA"], RTOL[dtype], "dA")
    assert_close(to_np(mod.lora_B.weight.grad), ref["dB"], RTOL[dtype], "dB")
    assert_close(to_np(mod.lora_magnitude_vector.weight.grad), ref["dm"], RTOL[dtype], "dm")


def test_no_base_result_path_matches():
    """The dropout path (no precomputed base output) gives the same delta as the common path."""
    st = LAYER["layer_bias_fp32"]
    base, lora_A, lora_B, layer = _build(st, "fp32")
    x = to_dev(st["x"], "fp32")
    s = float(st["scale"])
    with torch.no_grad():
        d1 = layer(x, lora_A=lora_A, lora_B=lora_B, scaling=s, base_layer=base, base_result=base(x))
        d2 = layer(x, lora_A=lora_A, lora_B=lora_B, scaling=s, base_layer=base, base_result=None)
    assert_close(to_np(d2), to_np(d1), 1e-5, "delta")
    assert layer._last_forward_chunk_size == base.out_features


def test_inference_in_place_compose():
    """No-grad forward composes in place into the LoRA output buffer."""
    st = LAYER["layer_bf16"]
    base, lora_A, lora_B, layer = _build(st, "bf16")
    x = to_dev(st["x"], "bf16")
    with torch.no_grad():
        delta = layer(x, lora_A=lora_A, lora_B=lora_B, scaling=float(st["scale"]), base_layer=base,
                      base_result=base(x))
    assert_close(to_np(delta), st["delta"], 1e-2, "delta")


def test_dora_linear_with_bias_vs_oracle():
    """Fused layer-output path with a base bias (base = result - bias inside the kernel)."""
    from dorafactors_b200.layer import DoraLinear

    dtype, T, in_f, out_f, r, s = "bf16", 128, 256, 384, 16, 0.5
    rng = np.random.default_rng(99)
    W = orc.round_to(rng.standard_normal((out_f, in_f)) * 0.02, dtype)
    bias = orc.round_to(rng.standard_normal(out_f) * 0.1, dtype)
    A = orc.round_to(rng.uniform(-1, 1, (r, in_f)) / np.sqrt(in_f), dtype)
    B = orc.round_to(rng.standard_normal((out_f, r)) * 0.01, dtype)
    x = orc.round_to(rng.standard_normal((T, in_f)), dtype)
    dy = orc.round_to(rng.standard_normal((T, out_f)), dtype)
    base = torch.nn.Linear(in_f, out_f, bias=True, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        base.weight.copy_(to_dev(W, dtype))
        base.bias.copy_(to_dev(bias, dtype))
    mod = DoraLinear(base, r=r, scaling=s)
    with torch.no_grad():
        mod.lora_A.weight.copy_(to_dev(A, dtype))
        mod.lora_B.weight.copy_(to_dev(B, dtype))
        mod.reset_magnitude()
    m = to_np(mod.lora_magnitude_vector.weight)
    tx = to_dev(x, dtype).requires_grad_(True)
    y = mod(tx)
    y.backward(to_dev(dy, dtype))
    ref = orc.dora_linear_forward_backward(x, W, bias, A, B, m, s, dy, dtype)
    for k, v in (("y", y), ("dx", tx.grad), ("dA", mod.lora_A.weight.grad), ("dB", mod.lora_B.weight.grad),
                 ("dm", mod.lora_magnitude_vector.weight.grad)):
        assert_close(to_np(v), ref[k], RTOL[dtype], k)


def test_dora_linear_dropout_and_eval_paths():
    """Training with dropout takes the two-pass path (delta from the dropped-out input);
    eval mode takes the fused path and agrees with the two-pass composition."""
    from dorafactors_b200.layer import DoraLinear

    torch.manual_seed(3)
    base = torch.nn.Linear(256, 320, bias=False, device="cuda", dtype=torch.bfloat16)
    mod = DoraLinear(base, r=8, scaling=2.0, dropout=0.1, init_lora_B_zero=False)
    x = torch.randn(64, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    mod.train()
    y = mod(x)
    y.float().square().sum().backward()
    assert torch.isfinite(x.grad.float()).all() and mod.lora_magnitude_vector.weight.grad is not None
    mod.eval()
    with torch.no_grad():
        y_eval = mod(x)
        delta = mod.lora_magnitude_vector(x, lora_A=mod.lora_A, lora_B=mod.lora_B, scaling=2.0, base_layer=base,
                                          base_result=base(x))
        y_two = base(x) + delta
    assert_close(to_np(y_eval), to_np(y_two), 1e-2, "eval fused vs two-pass")


def test_row_sharded_single_rank_matches_dora_linear():
    """RowShardedDoraLinear on a one-rank NCCL group runs the native norm and fused
    compose on its shard; with one rank the shard is the whole layer, so it must
    match DoraLinear (the collectives are identities)."""
    import datetime
    import os
    import socket

    import torch.distributed as dist

    from dorafactors_b200.layer import DoraLinear
    from dorafactors_b200.parallel import RowShardedDoraLinear

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", 0))
    try:
        torch.manual_seed(5)
        base = torch.nn.Linear(512, 640, bias=True, device="cuda", dtype=torch.bfloat16)
        ref = DoraLinear(base, r=32, scaling=0.5, init_lora_B_zero=False)
        sh = RowShardedDoraLinear.from_full(base.weight.detach(), base.bias.detach(), ref.lora_A.weight.detach(),
                                            ref.lora_B.weight.detach(),
                                            ref.lora_magnitude_vector.weight.detach(), 0.5)
        x = torch.randn(96, 512, device="cuda", dtype=torch.bfloat16)
        dy = torch.randn(96, 640, device="cuda", dtype=torch.bfloat16)
        x1, x2 = x.clone().requires_grad_(True), x.clone().requires_grad_(True)
        y1 = ref(x1)
        y1.backward(dy)
        y2 = sh(x2)
        y2.backward(dy)
        for a, b, k in ((y2, y1, "y"), (x2.grad, x1.grad, "dx"), (sh.lora_A.grad, ref.lora_A.weight.grad, "dA"),
                        (sh.lora_B.grad, ref.lora_B.weight.grad, "dB"),
                        (sh.magnitude.grad, ref.lora_magnitude_vector.weight.grad, "dm")):
            assert_close(to_np(a), to_np(b), 1e-2, k)
    finally:
        dist.destroy_process_group()


class _FixedKeep(torch.nn.Module):
    """Dropout with a fixed mask: ``x * keep`` (keep is 0 or 1/(1-p) per element)."""

    def __init__(self, keep):
        super().__init__()
        self.keep = keep

    def forward(self, x):
        return x * self.keep


@pytest.mark.parametrize("dtype,bias", [("bf16", False), ("bf16", True), ("fp32", True)])
def test_dora_linear_dropout_path_vs_oracle(dtype, bias):
    """Training with LoRA dropout (the base_result=None path, dora.py:1155-1263 /
    1470-1484, wired as variants.py:228-232): y, dx, dA, dB and dm against the
    oracle for the same fixed dropout mask."""
    from dorafactors_b200.layer import DoraLinear

    T, in_f, out_f, r, s, p = 192, 384, 448, 16, 2.0, 0.2
    rng = np.random.default_rng(41 + bias)
    W = orc.round_to(rng.standard_normal((out_f, in_f)) * 0.02, dtype)
    bvec = orc.round_to(rng.standard_normal(out_f) * 0.1, dtype) if bias else None
    A = orc.round_to(rng.uniform(-1, 1, (r, in_f)) / np.sqrt(in_f), dtype)
    B = orc.round_to(rng.standard_normal((out_f, r)) * 0.02, dtype)
    x = orc.round_to(rng.standard_normal((T, in_f)), dtype)
    dy = orc.round_to(rng.standard_normal((T, out_f)), dtype)
    keep = orc.round_to((rng.uniform(0, 1, (T, in_f)) >= p) / (1.0 - p), dtype)
    tdt = to_dev(W, dtype).dtype
    base = torch.nn.Linear(in_f, out_f, bias=bias, device="cuda", dtype=tdt)
    with torch.no_grad():
        base.weight.copy_(to_dev(W, dtype))
        if bias:
            base.bias.copy_(to_dev(bvec, dtype))
    mod = DoraLinear(base, r=r, scaling=s, dropout=p)
    mod.lora_dropout = _FixedKeep(to_dev(keep, dtype))
    with torch.no_grad():
        mod.lora_A.weight.copy_(to_dev(A, dtype))
        mod.lora_B.weight.copy_(to_dev(B, dtype))
        mod.reset_magnitude()
        mod.lora_magnitude_vector.weight.mul_(1.0 + 0.1 * torch.randn(out_f, device="cuda").to(tdt))
    m = to_np(mod.lora_magnitude_vector.weight)
    mod.train()
    tx = to_dev(x, dtype).requires_grad_(True)
    y = mod(tx)
    y.backward(to_dev(dy, dtype))
    ref = orc.dora_linear_dropout_forward_backward(x, keep, W, bvec, A, B, m, s, dy, dtype)
    # The same bf16 values evaluated at fp32 precision: the reference's bf16 eager
    # d_mag rounds each of its two partial column sums (s*lora*dy and base*dy) to
    # bf16 before adding them, which costs up to ~1% of the largest entry where
    # they cancel; the native fp32 column sum of inner*dy does not.
    exact = orc.dora_linear_dropout_forward_backward(x, keep, W, bvec, A, B, m, s, dy, "fp32")
    for k, v in (("y", y), ("dx", tx.grad), ("dA", mod.lora_A.weight.grad), ("dB", mod.lora_B.weight.grad),
                 ("dm", mod.lora_magnitude_vector.weight.grad)):
        what = f"dropout {dtype} bias={bias} {k}"
        if dtype == "fp32":
            assert_close(to_np(v), ref[k], RTOL[dtype], what)
        else:
            l2, _ = rel_errors(to_np(v), ref[k])
            assert l2 <= RTOL[dtype], f"{what} vs the bf16 eager oracle: rel-L2 {l2:.3e}"
            assert_close(to_np(v), exact[k], RTOL[dtype], what + " vs fp32 evaluation")


def test_dora_linear_headline_shape_vs_fp32():
    """The benchmarked layer shape (W0 28672 x 8192 bf16, r = 384, s = 1.0) on 2048
    tokens: the native forward + backward against an fp32 PyTorch evaluation of the
    reference's eager formulas on the same GPU -- the dense row norm ||W0 + s B A||
    (dora.py:1012-1022), g = m / norm, the eager compose g*(s*lora) + (g-1)*base
    (dora.py:1331-1334), y = result + delta, and autograd for dx, dA, dB, dm with
    the norm held constant.  Tolerance 1e-2 (normwise), the bf16 parity bar."""
    import math

    from dorafactors_b200.layer import DoraLinear

    out_f, in_f, r, T, s = 28672, 8192, 384, 2048, 1.0
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(7)
    base = torch.nn.Linear(in_f, out_f, bias=False, device=dev, dtype=torch.bfloat16)
    with torch.no_grad():
        base.weight.copy_((torch.randn(out_f, in_f, device=dev, generator=g) * 0.02).bfloat16())
    mod = DoraLinear(base, r=r, scaling=s, init_lora_B_zero=False)
    with torch.no_grad():
        mod.lora_A.weight.copy_(((torch.rand(r, in_f, device=dev, generator=g) * 2 - 1) / math.sqrt(in_f))
                                .bfloat16())
        mod.lora_B.weight.copy_((torch.randn(out_f, r, device=dev, generator=g) * 0.01).bfloat16())
        mod.reset_magnitude()
        mod.lora_magnitude_vector.weight.mul_(1.0 + 0.05 * torch.randn(out_f, device=dev, generator=g).bfloat16())
    x = torch.randn(T, in_f, device=dev, generator=g).bfloat16().requires_grad_(True)
    dy = torch.randn(T, out_f, device=dev, generator=g).bfloat16()
    y = mod(x)
    y.backward(dy)
    got = {"y": y.float(), "dx": x.grad.float(), "dA": mod.lora_A.weight.grad.float(),
           "dB": mod.lora_B.weight.grad.float(), "dm": mod.lora_magnitude_vector.weight.grad.float()}
    del y

    # fp32 evaluation of the same step from the same bf16 values.
    W = base.weight.detach().float()
    A32 = mod.lora_A.weight.detach().float().requires_grad_(True)
    B32 = mod.lora_B.weight.detach().float().requires_grad_(True)
    m32 = mod.lora_magnitude_vector.weight.detach().float().requires_grad_(True)
    x32 = x.detach().float().requires_grad_(True)
    with torch.no_grad():
        norm = (W + s * (B32 @ A32)).norm(dim=1)
    gg = (m32 / norm.clamp_min(1e-12)).view(1, -1)
    result = x32 @ W.T
    lora = (x32 @ A32.T) @ B32.T
    y32 = result + (gg * (s * lora) + (gg - 1) * result)
    y32.backward(dy.float())
    ref = {"y": y32.detach(), "dx": x32.grad, "dA": A32.grad, "dB": B32.grad, "dm": m32.grad}
    native_norm = mod.lora_magnitude_vector._get_weight_norm_linear(
        base_weight=base.weight, lora_A_w=mod.lora_A.weight, lora_B_w=mod.lora_B.weight, scaling=s)
    assert_close(to_np(native_norm), to_np(norm), 1e-2, "headline norm")
    for k in ("y", "dx", "dA", "dB", "dm"):
        assert_close(to_np(got[k]), to_np(ref[k]), RTOL["bf16"], f"headline {k}")


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
def test_trainable_bias_gradient(dtype):
    """A trainable base bias (PEFT's bias="all") on the fused layer-output path: the
    native bias gradient (1 - g) * column sums of d_y, plus the base layer's own
    d_result sum, must equal the oracle's total d_bias = column sums of d_y."""
    from dorafactors_b200.layer import DoraLinear

    T, in_f, out_f, r, s = 300, 256, 520, 16, 1.5
    rng = np.random.default_rng(77)
    W = orc.round_to(rng.standard_normal((out_f, in_f)) * 0.02, dtype)
    bvec = orc.round_to(rng.standard_normal(out_f) * 0.1, dtype)
    x = orc.round_to(rng.standard_normal((T, in_f)), dtype)
    dy = orc.round_to(rng.standard_normal((T, out_f)), dtype)
    tdt = to_dev(W, dtype).dtype
    base = torch.nn.Linear(in_f, out_f, bias=True, device="cuda", dtype=tdt)
    with torch.no_grad():
        base.weight.copy_(to_dev(W, dtype))
        base.bias.copy_(to_dev(bvec, dtype))
    mod = DoraLinear(base, r=r, scaling=s, init_lora_B_zero=False)
    base.bias.requires_grad_(True)
    with torch.no_grad():
        mod.lora_magnitude_vector.weight.mul_(1.0 + 0.2 * torch.randn(out_f, device="cuda").to(tdt))
    y = mod(to_dev(x, dtype))
    y.backward(to_dev(dy, dtype))
    want = dy.astype(np.float64).sum(0)  # y = x W^T + b + delta(base = x W^T): dL/db = sum of d_y
    assert_close(to_np(base.bias.grad), want, RTOL[dtype], f"{dtype} bias grad")
    # The native piece alone: (1 - g) * sum_i d_y.
    from dorafactors_b200 import _native

    g = (torch.rand(out_f, device="cuda") + 0.5).to(tdt)
    d = to_dev(dy, dtype)
    got = torch.empty(out_f, dtype=tdt, device="cuda")
    _native.linear_output_bias_grad(d, g, got)
    ref = (1.0 - to_np(g).astype(np.float64)) * dy.astype(np.float64).sum(0)
    assert_close(to_np(got), ref, RTOL[dtype], "native bias grad")
    e = torch.empty(0, out_f, dtype=tdt, device="cuda")
    _native.linear_output_bias_grad(e, g, got)
    assert bool((got == 0).all())
