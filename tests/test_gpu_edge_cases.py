"""Edge cases of the compose, backward and norm assembly on the native path, the
cases the reference's own suite checks on its fused module (test_dora_fused.py
TestEdgeCases and TestNumericalEdgeCasesExtended): single elements, all-zero and
large inputs, negative and extreme LoRA scales, empty tensors (no launch, correct
shapes, a zero magnitude gradient) and the magnitude gradient when one of the two
branches is zero or both are nearly equal.

Tolerances: 1e-5 (fp32) against PyTorch fp32 / fp64 evaluations of the same
formulas; exact where the arithmetic is exact.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _device_error_stays_clear():
    from dorafactors_b200 import _native

    yield
    assert _native.device_error(reset=True) == 0


def _f(*shape, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(*shape, device="cuda", generator=g)


def test_single_element_compose_and_assembly():
    from dorafactors_b200 import dora_fused as F

    lora = torch.tensor([[1.0]], device="cuda")
    base = torch.tensor([[2.0]], device="cuda")
    mag = torch.tensor([[0.5]], device="cuda")
    # (0.5 - 1) * 2 + 0.5 * (1 * 1) = -0.5, exact in fp32
    assert F.fused_dora_compose(lora.clone(), base, mag, 1.0, inplace=False).item() == -0.5
    (norm,) = F.fused_norm_assembly(torch.tensor([4.0], device="cuda"), torch.tensor([1.0], device="cuda"),
                                    torch.tensor([1.0], device="cuda"), 1.0)
    # 4 + 2*1*1 + 1*1 = 7
    assert abs(norm.item() - 7.0 ** 0.5) < 1e-6


def test_all_zero_inputs():
    from dorafactors_b200 import dora_fused as F

    z = torch.zeros(4, 16, device="cuda")
    out = F.fused_dora_compose(z.clone(), z, torch.ones(1, 16, device="cuda"), 1.0, inplace=False)
    assert torch.count_nonzero(out) == 0
    (norm,) = F.fused_norm_assembly(torch.zeros(8, device="cuda"), torch.zeros(8, device="cuda"),
                                    torch.zeros(8, device="cuda"), 0.0)
    assert torch.count_nonzero(norm) == 0


def test_negative_scale_and_large_values():
    from dorafactors_b200 import dora_fused as F

    lora, base = _f(4, 16, seed=1), _f(4, 16, seed=2)
    mag = torch.rand(1, 16, device="cuda") + 0.5
    ref = (mag - 1) * base + mag * (-0.5 * lora)
    out = F.fused_dora_compose(lora.clone(), base, mag, -0.5, inplace=False)
    assert (out - ref).abs().max().item() <= 1e-5
    big = torch.full((2, 4), 1e4, device="cuda")
    out = F.fused_dora_compose(big.clone(), big, torch.ones(1, 4, device="cuda"), 1.0, inplace=False)
    assert torch.equal(out, big)  # (1 - 1) * 1e4 + 1 * (1 * 1e4)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_empty_tensors(dtype):
    """Zero rows: nothing is launched, shapes are kept and d_mag is zero with mag's shape."""
    from dorafactors_b200 import dora_fused as F

    e = torch.empty(0, 16, device="cuda", dtype=dtype)
    mag = torch.ones(1, 16, device="cuda", dtype=dtype)
    assert F.fused_dora_compose(e.clone(), e, mag, 1.0, inplace=False).shape == (0, 16)
    assert F.fused_dora_compose(e.clone(), e, mag, 1.0, inplace=True).shape == (0, 16)
    out, inner = F.fused_dora_forward_and_inner(e, e, mag, 1.0)
    assert out.shape == (0, 16) and inner.shape == (0, 16)
    (norm,) = F.fused_norm_assembly(torch.empty(0, device="cuda"), torch.empty(0, device="cuda"),
                                    torch.empty(0, device="cuda"), 1.0)
    assert norm.shape == (0,)
    lora = e.clone().requires_grad_(True)
    base = e.clone().requires_grad_(True)
    m = mag.clone().requires_grad_(True)
    y = F.FusedDoRAComposeFunction.apply(lora, base, m, 1.0)
    assert y.shape == (0, 16)
    y.sum().backward()
    assert lora.grad.shape == (0, 16) and base.grad.shape == (0, 16)
    assert m.grad is not None and m.grad.shape == (1, 16) and torch.count_nonzero(m.grad) == 0
    # The fused layer output y = result + delta: same contract.
    lora = e.clone().requires_grad_(True)
    result = e.clone().requires_grad_(True)
    m = mag.clone().requires_grad_(True)
    y = F.fused_dora_linear_output(lora, result, m, 1.0)
    assert y.shape == (0, 16)
    y.sum().backward()
    assert lora.grad.shape == (0, 16) and result.grad.shape == (0, 16)
    assert m.grad is not None and m.grad.shape == (1, 16) and torch.count_nonzero(m.grad) == 0


def _grads(lora, base, mag, scale, d_out):
    from dorafactors_b200 import dora_fused as F

    lora = lora.clone().requires_grad_(True)
    base = base.clone().requires_grad_(True)
    mag = mag.clone().requires_grad_(True)
    out = F.FusedDoRAComposeFunction.apply(lora, base, mag, scale)
    out.backward(d_out)
    return lora.grad, base.grad, mag.grad


def test_d_mag_with_a_zero_branch():
    """lora = 0 (B initialised to zero): d_mag is the base branch alone; base = 0: it is
    scale * sum(lora * d_out)."""
    s = 0.5
    base = _f(8, 64, seed=3)
    lora = _f(8, 64, seed=4)
    mag = torch.rand(1, 64, device="cuda") + 0.5
    ones = torch.ones(8, 64, device="cuda")
    _, _, dm = _grads(torch.zeros_like(base), base, mag, s, ones)
    assert (dm - base.sum(0, keepdim=True)).abs().max().item() <= 1e-5
    _, _, dm = _grads(lora, torch.zeros_like(lora), mag, s, ones)
    assert (dm - (s * lora).sum(0, keepdim=True)).abs().max().item() <= 1e-5


def test_nearly_equal_branches_stay_finite():
    base = _f(16, 128, seed=5)
    lora = base + 0.1 * _f(16, 128, seed=6)
    mag = torch.rand(1, 128, device="cuda") + 0.5
    dl, db, dm = _grads(lora, base, mag, 1.0, _f(16, 128, seed=7))
    for t in (dl, db, dm):
        assert torch.isfinite(t).all()
    assert dm.abs().sum().item() > 0


@pytest.mark.parametrize("scale", [0.0, 0.001, 0.1, 1.0, 10.0])
def test_d_mag_across_scales_vs_fp64(scale):
    lora, base, d_out = _f(8, 64, seed=8), _f(8, 64, seed=9), _f(8, 64, seed=10)
    mag = torch.rand(1, 64, device="cuda") + 0.5
    dl, db, dm = _grads(lora, base, mag, scale, d_out)
    for t in (dl, db, dm):
        assert torch.isfinite(t).all()
    l64, b64, m64 = (t.double().requires_grad_(True) for t in (lora, base, mag))
    out64 = (m64 - 1) * b64 + m64 * (scale * l64)
    out64.backward(d_out.double())
    torch.testing.assert_close(dm.double(), m64.grad, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(dl.double(), l64.grad, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(db.double(), b64.grad, rtol=1e-5, atol=1e-6)


def test_near_zero_norm_stays_finite():
    """Norm components that cancel to ~0: the assembled norm is >= 0 and m / clamp(norm)
    is finite (test_dora_fused.py TestFusedNormAssemblyNearZero)."""
    from dorafactors_b200 import dora_fused as F

    n = 32
    w = torch.full((n,), 1e-12, device="cuda")
    (norm,) = F.fused_norm_assembly(w, -w, w, 0.5)
    assert (norm >= 0).all()
    mag = torch.rand(n, device="cuda") + 0.1
    assert torch.isfinite(mag / norm.clamp_min(1e-6)).all()


def _layer(seed=903, in_f=32, out_f=16, r=4, scaling=0.5):
    from dorafactors_b200.dora import DoraLinearLayer

    torch.manual_seed(seed)
    base = torch.nn.Linear(in_f, out_f, bias=True, device="cuda")
    base.requires_grad_(False)
    lora_A = torch.nn.Linear(in_f, r, bias=False, device="cuda")
    lora_B = torch.nn.Linear(r, out_f, bias=False, device="cuda")
    with torch.no_grad():
        lora_B.weight.normal_(0.0, 0.1)
    layer = DoraLinearLayer(fan_in_fan_out=False)
    layer.update_layer(base_layer=base, lora_A=lora_A.weight, lora_B=lora_B.weight, scaling=scaling)
    return base, lora_A, lora_B, layer


def _step(base, lora_A, lora_B, layer, x, scaling=0.5):
    out = layer(x, lora_A=lora_A, lora_B=lora_B, scaling=scaling, base_layer=base, base_result=base(x).detach())
    out.sum().backward()


def test_gradient_accumulation_equals_sum_of_passes():
    """Three passes without zeroing the gradients give the sum of the three single-pass
    gradients of A, B and the magnitude (TestGradientAccumulationCorrectness)."""
    xs = [_f(4, 32, seed=904 + i) for i in range(3)]
    acc = _layer()
    for x in xs:
        _step(*acc, x)
    ind = _layer()
    sums = [torch.zeros_like(p) for p in (ind[1].weight, ind[2].weight, ind[3].weight)]
    for x in xs:
        for p in (ind[1].weight, ind[2].weight, ind[3].weight):
            p.grad = None
        _step(*ind, x)
        for s_, p in zip(sums, (ind[1].weight, ind[2].weight, ind[3].weight)):
            s_ += p.grad
    for name, got, want in zip(("A", "B", "magnitude"), (acc[1].weight.grad, acc[2].weight.grad, acc[3].weight.grad),
                               sums):
        assert (got - want).abs().max().item() <= 1e-5, name


def test_no_device_memory_growth_across_steps():
    """Forward + backward repeated: allocated device memory does not grow after warm-up
    (workspaces are cached per device, stream and kind, not per call)."""
    import gc

    base, lora_A, lora_B, layer = _layer(seed=906, in_f=64, out_f=32, r=8)
    params = (lora_A.weight, lora_B.weight, layer.weight)

    def cycle():
        _step(base, lora_A, lora_B, layer, torch.randn(8, 64, device="cuda"))
        for p in params:
            p.grad = None

    for _ in range(10):
        cycle()
    gc.collect()
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated()
    for _ in range(40):
        cycle()
    gc.collect()
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() <= before * 1.1 + 1024
