"""Embedding and convolution DoRA layers, the conv-layout compose kernels and the
linear merge / unmerge, against the reference's own outputs (golden fixtures made
by tests/golden/make_golden.py from dora.py:1491-1742 and variants.py:164-212)
and a PyTorch fp32 evaluation.

Tolerance: 1e-2 relative (normwise) in bf16, 1e-5 in fp32, for outputs, norms,
magnitudes and all gradients.
"""

import numpy as np
import pytest
import torch

from _golden import RTOL, assert_close, load_group, to_dev, to_np

pytestmark = pytest.mark.gpu

EMB = load_group("embedding")
CONV = load_group("conv")
MERGE = load_group("merge")


@pytest.fixture(autouse=True)
def _no_tf32_no_device_error():
    from dorafactors_b200 import _native

    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old
    assert _native.device_error(reset=True) == 0


@pytest.mark.parametrize("case", sorted(EMB))
def test_embedding_golden(case):
    """DoraEmbeddingLayer with the factored native norm (no dense V x d delta)."""
    from dorafactors_b200.dora import DoraEmbeddingLayer

    st = EMB[case]
    dt, s = st["dtype"], float(st["scale"])
    W = to_dev(st["W"], dt)
    V, d = W.shape
    base = torch.nn.Embedding(V, d, device="cuda", dtype=W.dtype)
    with torch.no_grad():
        base.weight.copy_(W)
    base.requires_grad_(False)
    A = torch.nn.Parameter(to_dev(st["A"], dt))
    B = torch.nn.Parameter(to_dev(st["B"], dt))
    layer = DoraEmbeddingLayer(fan_in_fan_out=True)
    layer.update_layer(base_layer=base, lora_A=A, lora_B=B, scaling=s)
    assert_close(to_np(layer.weight), st["m"], RTOL[dt], f"{case} initial magnitude")
    ids = torch.from_numpy(st["ids"].astype(np.int64)).cuda()
    result = base(ids)
    _, delta = layer(ids, lora_A=A.T, lora_B=B.T, scaling=s, base_layer=base,
                     embed_fn=lambda x, w: torch.nn.functional.embedding(x, w), base_result=result)
    y = result + delta.to(result.dtype)
    y.backward(to_dev(st["dy"], dt))
    for k, v in {"y": y, "dA": A.grad, "dB": B.grad, "dm": layer.weight.grad}.items():
        assert_close(to_np(v), st[k], RTOL[dt], f"{case} {k}")


@pytest.mark.parametrize("case", sorted(CONV))
def test_conv_golden(case):
    """DoraConv1d/2dLayer: factored native norm on flattened weights, native
    channel-layout compose forward and backward."""
    from dorafactors_b200.dora import DoraConv1dLayer, DoraConv2dLayer

    st = CONV[case]
    dt, s, nd, k = st["dtype"], float(st["scale"]), int(st["conv_dims"]), int(st["kernel"])
    W = to_dev(st["W"], dt)
    co, ci = W.shape[0], W.shape[1]
    r = st["A"].shape[0]
    Conv = torch.nn.Conv2d if nd == 2 else torch.nn.Conv1d
    base = Conv(ci, co, k, padding=k // 2, bias="bias" in st, device="cuda", dtype=W.dtype)
    lora_A = Conv(ci, r, k, padding=k // 2, bias=False, device="cuda", dtype=W.dtype)
    lora_B = Conv(r, co, 1, bias=False, device="cuda", dtype=W.dtype)
    with torch.no_grad():
        base.weight.copy_(W)
        if "bias" in st:
            base.bias.copy_(to_dev(st["bias"], dt))
        lora_A.weight.copy_(to_dev(st["A"], dt))
        lora_B.weight.copy_(to_dev(st["B"], dt))
    base.requires_grad_(False)
    layer = (DoraConv2dLayer if nd == 2 else DoraConv1dLayer)(fan_in_fan_out=False)
    layer.update_layer(base_layer=base, lora_A=lora_A.weight, lora_B=lora_B.weight, scaling=s)
    assert tuple(layer.weight.shape) == tuple(st["m"].shape)
    assert_close(to_np(layer.weight), st["m"], RTOL[dt], f"{case} initial magnitude")
    x = to_dev(st["x"], dt).requires_grad_(True)
    result = base(x)
    delta = layer(x, lora_A=lora_A, lora_B=lora_B, scaling=s, base_layer=base, base_result=result)
    y = result + delta.to(result.dtype)
    y.backward(to_dev(st["dy"], dt))
    got = {"y": y, "dx": x.grad, "dA": lora_A.weight.grad, "dB": lora_B.weight.grad, "dm": layer.weight.grad}
    for name, v in got.items():
        assert_close(to_np(v), st[name], RTOL[dt], f"{case} {name}")


@pytest.mark.parametrize("case", sorted(MERGE))
def test_merge_unmerge_golden(case):
    from dorafactors_b200.dora import merge_weight, unmerge_weight

    st = MERGE[case]
    dt, s = st["dtype"], float(st["scale"])
    W, A, B, m = (to_dev(st[k], dt) for k in ("W", "A", "B", "m"))
    merged, norm = merge_weight(W, A, B, m, s)
    assert_close(to_np(norm), st["norm"], RTOL[dt], f"{case} norm")
    assert_close(to_np(merged), st["merged"], RTOL[dt], f"{case} merged")
    back = unmerge_weight(to_dev(st["merged"], dt), A, B, m, to_dev(st["norm"], dt), s)
    assert_close(to_np(back), st["unmerged"], RTOL[dt], f"{case} unmerged")


def test_dora_linear_merge_roundtrip():
    """DoraLinear.merge() folds the adapter in (same output), unmerge() restores W0."""
    from dorafactors_b200.layer import DoraLinear

    torch.manual_seed(3)
    base = torch.nn.Linear(256, 192, bias=True, device="cuda", dtype=torch.float32)
    layer = DoraLinear(base, r=8, scaling=2.0, init_lora_B_zero=False)
    with torch.no_grad():
        layer.lora_magnitude_vector.weight.mul_(1.1)
    x = torch.randn(32, 256, device="cuda")
    w0 = base.weight.detach().clone()
    with torch.no_grad():
        y = layer(x)
        layer.merge()
        y_merged = layer(x)
        layer.unmerge()
    torch.testing.assert_close(y_merged, y, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(base.weight, w0, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("dtype,gdt,N,C,S", [("bf16", "fp32", 3, 24, 40), ("bf16", "bf16", 2, 8, 7),
                                             ("fp32", "fp32", 4, 16, 33), ("fp16", "fp16", 5, 12, 64),
                                             ("bf16", "fp32", 64, 256, 784)])
def test_channel_compose_kernels(dtype, gdt, N, C, S):
    """Conv-layout compose forward / backward against a PyTorch fp32 evaluation;
    d_g bitwise identical across calls."""
    from dorafactors_b200 import _native

    torch.manual_seed(N * C + S)
    td = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}
    lora = torch.randn(N, C, S, device="cuda").to(td[dtype])
    base = torch.randn(N, C, S, device="cuda").to(td[dtype])
    g = (torch.rand(C, device="cuda") + 0.5).to(td[gdt])
    s = 0.75
    out = torch.empty_like(lora)
    inner = torch.empty_like(lora)
    _native.compose_fwd_channels(lora, base, g, s, out, inner, N, C, S)
    gf = g.float().view(1, C, 1)
    ref_out = (gf - 1) * base.float() + gf * (s * lora.float())
    ref_inner = s * lora.float() + base.float()
    tol = 1e-5 if dtype == "fp32" else 1e-2
    assert_close(to_np(out), to_np(ref_out), tol, "out")
    assert_close(to_np(inner), to_np(ref_inner), tol, "inner")
    d_out = torch.randn(N, C, S, device="cuda").to(td[dtype])
    d_lora, d_base = torch.empty_like(d_out), torch.empty_like(d_out)
    d_g = torch.empty(C, device="cuda", dtype=g.dtype)
    _native.compose_bwd_channels(d_out, inner, g, s, d_lora, d_base, d_g, N, C, S)
    assert_close(to_np(d_lora), to_np(gf * s * d_out.float()), tol, "d_lora")
    assert_close(to_np(d_base), to_np((gf - 1) * d_out.float()), tol, "d_base")
    ref_dg = (inner.float() * d_out.float()).sum(dim=(0, 2))
    assert_close(to_np(d_g), to_np(ref_dg), 1e-5 if gdt == "fp32" else 1e-2, "d_g")
    d_g2 = torch.empty_like(d_g)
    _native.compose_bwd_channels(d_out, inner, g, s, None, None, d_g2, N, C, S)
    assert torch.equal(d_g, d_g2)


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
def test_reference_api_with_per_channel_magnitude(dtype):
    """The reference-facing compose functions given a convolution-layout magnitude
    ([1, C, 1, 1] on [N, C, H, W] activations; the reference evaluates that case with its
    PyTorch fallback, dora_fused.py:563-574) run the channel kernels: outputs and all
    gradients against a PyTorch fp32 evaluation."""
    from dorafactors_b200 import dora_fused as F

    td = {"bf16": torch.bfloat16, "fp32": torch.float32}[dtype]
    tol = RTOL[dtype]
    torch.manual_seed(11)
    N, C, H, W = 3, 24, 5, 7
    lora = torch.randn(N, C, H, W, device="cuda").to(td)
    base = torch.randn(N, C, H, W, device="cuda").to(td)
    mag = (torch.rand(1, C, 1, 1, device="cuda") + 0.5).to(td)
    s = 0.75
    mf, lf, bf = mag.float(), lora.float(), base.float()
    ref = (mf - 1) * bf + mf * (s * lf)
    ref_inner = s * lf + bf
    assert_close(to_np(F.fused_dora_compose(lora, base, mag, s, inplace=False)), to_np(ref), tol, "out-of-place")
    l2 = lora.clone()
    r = F.fused_dora_compose(l2, base, mag, s, inplace=True)
    assert r.data_ptr() == l2.data_ptr()
    assert_close(to_np(l2), to_np(ref), tol, "in place")
    out, inner = F.fused_dora_forward_and_inner(lora, base, mag, s)
    assert_close(to_np(out), to_np(ref), tol, "forward_and_inner out")
    assert_close(to_np(inner), to_np(ref_inner), tol, "forward_and_inner inner")
    dy = torch.randn(N, C, H, W, device="cuda").to(td)
    dyf = dy.float()
    for name, fn in (("FusedDoRAComposeFunction", F.FusedDoRAComposeFunction.apply),
                     ("fused_dora_compose_autograd", F.fused_dora_compose_autograd)):
        l = lora.clone().requires_grad_(True)
        b = base.clone().requires_grad_(True)
        m = mag.clone().requires_grad_(True)
        y = fn(l, b, m, s)
        assert_close(to_np(y), to_np(ref), tol, f"{name} out")
        y.backward(dy)
        assert m.grad.shape == mag.shape and m.grad.dtype == mag.dtype
        assert_close(to_np(l.grad), to_np(mf * s * dyf), tol, f"{name} d_lora")
        assert_close(to_np(b.grad), to_np((mf - 1) * dyf), tol, f"{name} d_base")
        assert_close(to_np(m.grad), to_np((ref_inner * dyf).sum(dim=(0, 2, 3), keepdim=True)), tol, f"{name} d_mag")
