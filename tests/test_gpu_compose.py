"""Compose forward / backward kernels (through the C ABI) against the oracle and
the reference's golden fixtures.

Tolerances: the parity bar, 1e-2 relative (normwise) for bf16/fp16 and 1e-5
for fp32.  The fp32 elementwise outputs are held to bitwise equality with the
oracle, because the kernels evaluate the reference's op order with correctly
rounded fp32 operations.
"""

import numpy as np
import pytest
import torch

from _golden import RTOL, assert_close, load_group, to_dev, to_np
from oracle import dora_oracle as orc

pytestmark = pytest.mark.gpu

COMPOSE = load_group("compose")


def _rand(rng, shape, dtype, lo=None, hi=None):
    if lo is None:
        x = rng.standard_normal(shape).astype(np.float32)
    else:
        x = rng.uniform(lo, hi, shape).astype(np.float32)
    return orc.round_to(x, dtype)


@pytest.fixture(autouse=True)
def _no_device_error():
    from dorafactors_b200 import _native

    yield
    assert _native.device_error(reset=True) == 0


@pytest.mark.parametrize("case", sorted(COMPOSE))
def test_compose_golden(case):
    from dorafactors_b200 import dora_fused as df

    st = COMPOSE[case]
    act, gdt, s = st["act_dtype"], st["g_dtype"], float(st["scale"])
    lora, base = to_dev(st["lora"], act), to_dev(st["base"], act)
    mag = to_dev(st["mag"], gdt)
    out = df.fused_dora_compose(lora.clone(), base, mag, s, inplace=False)
    assert out.dtype == lora.dtype and out.shape == lora.shape
    assert_close(to_np(out), st["eager_out"], RTOL[act], f"{case} out vs reference eager")
    inplace = lora.clone()
    res = df.fused_dora_compose(inplace, base, mag, s, inplace=True)
    assert res.data_ptr() == inplace.data_ptr()
    np.testing.assert_array_equal(to_np(res), to_np(out))
    o2, inner = df.fused_dora_forward_and_inner(lora, base, mag, s)
    np.testing.assert_array_equal(to_np(o2), to_np(out))
    if act == gdt:
        assert_close(to_np(inner), st["fwd_inner"], RTOL[act], f"{case} inner")
        d_out = to_dev(st["d_out"], act)
        dl, db, dm = df._backward(d_out, inner, mag, s, True, True, True)
        assert_close(to_np(dl), st["bwd_d_lora"], RTOL[act], f"{case} d_lora")
        assert_close(to_np(db), st["bwd_d_base"], RTOL[act], f"{case} d_base")
        assert_close(to_np(dm), st["bwd_d_mag"], RTOL[act], f"{case} d_mag")
        assert_close(to_np(dm), st["eager_d_mag"], RTOL[act], f"{case} d_mag vs eager autograd")


SHAPES = [(1, 8), (3, 24), (7, 37), (64, 4096), (513, 1000), (2048, 6144), (33, 28672)]


@pytest.mark.parametrize("dtype", ["bf16", "fp16", "fp32"])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_compose_forward_vs_oracle(dtype, rows, cols):
    from dorafactors_b200 import dora_fused as df

    rng = np.random.default_rng(rows * 131 + cols)
    lora, base = _rand(rng, (rows, cols), dtype), _rand(rng, (rows, cols), dtype)
    g = _rand(rng, (1, cols), dtype, 0.5, 1.5)
    s = 0.7
    out, inner = df.fused_dora_forward_and_inner(to_dev(lora, dtype), to_dev(base, dtype), to_dev(g, dtype), s)
    ro, ri = orc.compose_forward_and_inner(lora, base, g, s, dtype)
    if dtype == "fp32":
        np.testing.assert_array_equal(to_np(out), ro)
        np.testing.assert_array_equal(to_np(inner), ri)
    else:
        assert_close(to_np(out), ro, RTOL[dtype], "out")
        assert_close(to_np(inner), ri, RTOL[dtype], "inner")
        # One rounding of an fp32 evaluation: within half an ulp of the exact
        # value, plus the fp32 evaluation error of the two products.
        g64, l64, b64 = g.astype(np.float64), lora.astype(np.float64), base.astype(np.float64)
        terms = np.abs((g64 - 1) * b64) + np.abs(g64 * s * l64)
        exact = (g64 - 1) * b64 + g64 * (s * l64)
        # fp16 results below 2^-14 are subnormal: half their spacing is 2^-25 absolute.
        u, floor = (2.0**-8, 0.0) if dtype == "bf16" else (2.0**-11, 2.0**-25)
        assert np.all(np.abs(to_np(out) - exact) <= u * np.abs(exact) + 1e-6 * terms + floor)


@pytest.mark.parametrize("act,gdt", [("bf16", "fp32"), ("fp16", "fp32")])
def test_compose_mixed_dtype_matches_eager(act, gdt):
    """fp32 g with half activations keeps (g - 1) in fp32, like the eager reference."""
    from dorafactors_b200 import dora_fused as df

    rng = np.random.default_rng(7)
    lora, base = _rand(rng, (40, 520), act), _rand(rng, (40, 520), act)
    g = (1.0 + rng.standard_normal((1, 520)) * 1e-3).astype(np.float32)  # g close to 1
    out = df.fused_dora_compose(to_dev(lora, act), to_dev(base, act), to_dev(g, gdt), 2.0, inplace=False)
    ref = orc.compose_eager(lora, base, g, 2.0, act, gdt)
    assert_close(to_np(out), ref, RTOL[act], "mixed")


def test_compose_3d_and_noncontiguous():
    from dorafactors_b200 import dora_fused as df

    rng = np.random.default_rng(3)
    lora = _rand(rng, (4, 6, 96), "bf16")
    base = _rand(rng, (4, 6, 96), "bf16")
    g = _rand(rng, (1, 96), "bf16", 0.5, 1.5)
    tl, tb, tg = to_dev(lora, "bf16"), to_dev(base, "bf16"), to_dev(g, "bf16")
    out = df.fused_dora_compose(tl, tb, tg, 1.5, inplace=False)
    assert out.shape == (4, 6, 96)
    ref = orc.compose_fused(lora.reshape(24, 96), base.reshape(24, 96), g, 1.5, "bf16")
    assert_close(to_np(out).reshape(24, 96), ref, RTOL["bf16"], "3d")
    # A transposed (non-contiguous) base is made contiguous, not rejected.
    bt = to_dev(base.reshape(24, 96).T.copy(), "bf16").T
    out2 = df.fused_dora_compose(tl.reshape(24, 96), bt, tg, 1.5, inplace=False)
    np.testing.assert_array_equal(to_np(out2), to_np(out).reshape(24, 96))
    # In place into a non-contiguous lora writes back into the view.
    big = torch.zeros(24, 192, dtype=torch.bfloat16, device="cuda")
    view = big[:, ::2]
    view.copy_(tl.reshape(24, 96))
    df.fused_dora_compose(view, tb.reshape(24, 96), tg, 1.5, inplace=True)
    np.testing.assert_array_equal(to_np(big[:, ::2]), to_np(out).reshape(24, 96))
    assert float(big[:, 1::2].abs().sum()) == 0.0


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
@pytest.mark.parametrize("rows,cols", [(1, 8), (5, 37), (300, 1000), (2048, 6144), (4097, 2056)])
def test_backward_vs_oracle(dtype, rows, cols):
    from dorafactors_b200 import dora_fused as df

    rng = np.random.default_rng(rows + 17 * cols)
    d_out, inner = _rand(rng, (rows, cols), dtype), _rand(rng, (rows, cols), dtype)
    g = _rand(rng, (1, cols), dtype, 0.5, 1.5)
    s = 1.25
    td, ti, tg = to_dev(d_out, dtype), to_dev(inner, dtype), to_dev(g, dtype)
    dl, db, dm = df._backward(td, ti, tg, s, True, True, True)
    rl, rb, rm = orc.compose_backward(d_out, inner, g, s, dtype)
    if dtype == "fp32":
        np.testing.assert_array_equal(to_np(dl), rl)
        np.testing.assert_array_equal(to_np(db), rb)
    else:
        assert_close(to_np(dl), rl, RTOL[dtype], "d_lora")
        assert_close(to_np(db), rb, RTOL[dtype], "d_base")
    # d_g against a float64 column sum of the exact products.
    exact = (inner.astype(np.float64) * d_out.astype(np.float64)).sum(0, keepdims=True)
    assert_close(to_np(dm), exact, RTOL[dtype], "d_g")
    assert_close(to_np(dm), rm, RTOL[dtype], "d_g vs oracle")
    # Deterministic: a second call reproduces every bit (the counters reset themselves).
    dl2, db2, dm2 = df._backward(td, ti, tg, s, True, True, True)
    assert torch.equal(dm, dm2) and torch.equal(dl, dl2) and torch.equal(db, db2)
    # Each subset of outputs gives the same values.
    for nl, nb, nm in [(True, False, False), (False, True, False), (False, False, True), (True, False, True)]:
        a, b, c = df._backward(td, ti if nm else None, tg, s, nl, nb, nm)
        if nl:
            assert torch.equal(a, dl)
        if nb:
            assert torch.equal(b, db)
        if nm:
            assert torch.equal(c, dm)


def test_backward_mixed_g_fp32():
    from dorafactors_b200 import dora_fused as df

    rng = np.random.default_rng(11)
    d_out, inner = _rand(rng, (257, 640), "bf16"), _rand(rng, (257, 640), "bf16")
    g = (1 + rng.standard_normal((1, 640)) * 1e-3).astype(np.float32)
    dl, db, dm = df._backward(to_dev(d_out, "bf16"), to_dev(inner, "bf16"), to_dev(g, "fp32"), 2.0, True, True, True)
    assert dm.dtype == torch.float32 and dl.dtype == torch.bfloat16
    rl, rb, _ = orc.compose_backward(d_out, inner, g, 2.0, "bf16", "fp32")
    assert_close(to_np(dl), rl, 1e-2, "d_lora")
    assert_close(to_np(db), rb, 1e-2, "d_base")
    exact = (inner.astype(np.float64) * d_out.astype(np.float64)).sum(0, keepdims=True)
    assert_close(to_np(dm), exact, 1e-5, "d_g fp32 accumulate")


def test_autograd_function_matches_oracle():
    from dorafactors_b200 import dora_fused as df

    rng = np.random.default_rng(5)
    rows, cols, s = 96, 2048, 2.0
    lora, base = _rand(rng, (rows, cols), "bf16"), _rand(rng, (rows, cols), "bf16")
    g = _rand(rng, (1, cols), "bf16", 0.5, 1.5)
    dy = _rand(rng, (rows, cols), "bf16")
    tl = to_dev(lora, "bf16").requires_grad_(True)
    tb = to_dev(base, "bf16").requires_grad_(True)
    tg = to_dev(g, "bf16").requires_grad_(True)
    out = df.fused_dora_compose_autograd(tl, tb, tg, s)
    out.backward(to_dev(dy, "bf16"))
    _, inner = orc.compose_forward_and_inner(lora, base, g, s, "bf16")
    rl, rb, rg = orc.compose_backward(dy, inner, g, s, "bf16")
    assert_close(to_np(tl.grad), rl, 1e-2, "d_lora")
    assert_close(to_np(tb.grad), rb, 1e-2, "d_base")
    assert_close(to_np(tg.grad), rg, 1e-2, "d_g")
    # Frozen magnitude: no inner saved, no d_g.
    tg2 = to_dev(g, "bf16")
    tl2 = to_dev(lora, "bf16").requires_grad_(True)
    out2 = df.FusedDoRAComposeFunction.apply(tl2, to_dev(base, "bf16"), tg2, s)
    out2.backward(to_dev(dy, "bf16"))
    assert torch.equal(tl2.grad, tl.grad)


def test_custom_op_eager_and_opcheck():
    from dorafactors_b200 import dora_fused as df

    assert df._HAS_CUSTOM_OP
    rng = np.random.default_rng(9)
    lora, base = _rand(rng, (32, 256), "bf16"), _rand(rng, (32, 256), "bf16")
    g = _rand(rng, (1, 256), "bf16", 0.5, 1.5)
    tl = to_dev(lora, "bf16").requires_grad_(True)
    tb = to_dev(base, "bf16").requires_grad_(True)
    tg = to_dev(g, "bf16").requires_grad_(True)
    out, _ = torch.ops.dora_b200.fused_dora_compose_fwd(tl, tb, tg, 1.5, True)
    ref = df.fused_dora_compose(to_dev(lora, "bf16"), to_dev(base, "bf16"), to_dev(g, "bf16"), 1.5, inplace=False)
    assert torch.equal(out, ref)
    dy = torch.randn_like(out)
    out.backward(dy)
    dl, db, dm = df._backward(dy, df.fused_dora_forward_and_inner(tl.detach(), tb.detach(), tg.detach(), 1.5)[1],
                              tg.detach(), 1.5, True, True, True)
    assert torch.equal(tl.grad, dl) and torch.equal(tb.grad, db) and torch.equal(tg.grad, dm)


def test_peft_op_schema_eager_opcheck_and_compile():
    """The reference's op name and schema, torch.ops.peft.fused_dora_compose(lora, base,
    mag_norm_scale, scale) -> Tensor (dora_fused.py:1366-1446), served by the native
    kernels: eager forward / backward equal the autograd Function bit for bit,
    torch.library.opcheck passes, and a torch.compile'd function (Dynamo +
    AOTAutograd, fullgraph) calling the op gives the same outputs and gradients."""
    from dorafactors_b200 import dora_fused as df

    assert df._HAS_PEFT_OP
    op = torch.ops.peft.fused_dora_compose
    assert str(op.default._schema) == (
        "peft::fused_dora_compose(Tensor lora, Tensor base, Tensor mag_norm_scale, float scale) -> Tensor")
    rng = np.random.default_rng(21)
    lora, base = _rand(rng, (64, 512), "bf16"), _rand(rng, (64, 512), "bf16")
    g = _rand(rng, (1, 512), "bf16", 0.5, 1.5)
    dy = to_dev(_rand(rng, (64, 512), "bf16"), "bf16")

    def leaves():
        return (to_dev(lora, "bf16").requires_grad_(True), to_dev(base, "bf16").requires_grad_(True),
                to_dev(g, "bf16").requires_grad_(True))

    a = leaves()
    ref = df.FusedDoRAComposeFunction.apply(*a, 1.25)
    ref.backward(dy)
    b = leaves()
    out = op(*b, 1.25)
    out.backward(dy)
    assert torch.equal(out, ref)
    for x, y in zip(b, a):
        assert torch.equal(x.grad, y.grad)
    # Frozen magnitude: no d_mag, same outputs.
    with torch.no_grad():
        assert torch.equal(op(to_dev(lora, "bf16"), to_dev(base, "bf16"), to_dev(g, "bf16"), 1.25), ref)
    torch.library.opcheck(op.default, (*leaves(), 1.25))

    def f(l, b_, m):
        return torch.ops.peft.fused_dora_compose(l, b_, m, 1.25) * 2.0

    c = leaves()
    out_c = torch.compile(f, backend="aot_eager", fullgraph=True)(*c)
    out_c.backward(dy)
    assert torch.equal(out_c, ref * 2.0)
    for x, y in zip(c, a):
        assert_close(to_np(x.grad), to_np(y.grad) * 2.0, 1e-2, "compiled grad")


def test_errors_are_loud():
    from dorafactors_b200 import dora_fused as df

    x = torch.randn(4, 16, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        df.fused_dora_compose(x, x.clone(), torch.ones(1, 8, device="cuda", dtype=torch.bfloat16), 1.0)
    with pytest.raises(RuntimeError):
        df.fused_dora_compose(x.cpu(), x.cpu(), torch.ones(1, 16, dtype=torch.bfloat16), 1.0)
    e = torch.empty(0, 16, device="cuda", dtype=torch.bfloat16)
    assert df.fused_dora_compose(e, e.clone(), torch.ones(16, device="cuda", dtype=torch.bfloat16), 1.0).numel() == 0


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
@pytest.mark.parametrize("with_bias", [False, True])
@pytest.mark.parametrize("rows,cols", [(5, 37), (300, 1000), (1024, 4096)])
def test_linear_output_fused_glue(dtype, with_bias, rows, cols):
    """y = result + delta in one pass, and its backward, against the oracle's eager
    restatement of DoraLinearLayer.forward + DoraLinearVariant.forward."""
    from dorafactors_b200 import dora_fused as df

    rng = np.random.default_rng(rows * 3 + cols + with_bias)
    lora, res = _rand(rng, (rows, cols), dtype), _rand(rng, (rows, cols), dtype)
    g = _rand(rng, (1, cols), dtype, 0.5, 1.5)
    bias = _rand(rng, (cols,), dtype) if with_bias else None
    dy = _rand(rng, (rows, cols), dtype)
    s = 1.5
    tl = to_dev(lora, dtype).requires_grad_(True)
    tr = to_dev(res, dtype).requires_grad_(True)
    tg = to_dev(g, dtype).requires_grad_(True)
    tb = to_dev(bias, dtype) if with_bias else None
    y = df.fused_dora_linear_output(tl, tr, tg, s, tb)
    y.backward(to_dev(dy, dtype))
    # Oracle: base = result - bias, delta = eager compose, y = result + delta.
    base = orc._op(np.subtract, dtype, res, bias[None, :]) if with_bias else res
    delta = orc.compose_eager(lora, base, g, s, dtype, dtype)
    ry = orc._op(np.add, dtype, res, delta)
    if dtype == "fp32":
        np.testing.assert_array_equal(to_np(y), ry)
    else:
        assert_close(to_np(y), ry, RTOL[dtype], "y")
    # Gradients: d_lora = g s dy, d_result = dy + (g - 1) dy = g dy, d_g = sum inner * dy.
    g64, d64 = g.astype(np.float64), dy.astype(np.float64)
    inner64 = s * lora.astype(np.float64) + base.astype(np.float64)
    assert_close(to_np(tl.grad), g64 * s * d64, RTOL[dtype], "d_lora")
    assert_close(to_np(tr.grad), g64 * d64, RTOL[dtype], "d_result")
    assert_close(to_np(tg.grad), (inner64 * d64).sum(0, keepdims=True), RTOL[dtype], "d_g")


def test_linear_output_matches_two_pass_path():
    """The fused layer output equals delta (native compose) + result in bf16 within rounding."""
    from dorafactors_b200 import dora_fused as df

    rng = np.random.default_rng(12)
    lora, res = _rand(rng, (256, 2048), "bf16"), _rand(rng, (256, 2048), "bf16")
    g = _rand(rng, (1, 2048), "bf16", 0.5, 1.5)
    tl, tr, tg = to_dev(lora, "bf16"), to_dev(res, "bf16"), to_dev(g, "bf16")
    with torch.no_grad():
        y1 = df.fused_dora_linear_output(tl, tr, tg, 2.0)
        y2 = tr + df.fused_dora_compose(tl.clone(), tr, tg, 2.0, inplace=False)
    assert_close(to_np(y1), to_np(y2), 1e-2, "fused vs two-pass")
