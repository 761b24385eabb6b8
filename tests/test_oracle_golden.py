"""Pin the CPU oracle against fixtures made by running the reference itself.

Elementwise restatements must be bitwise equal to the reference's PyTorch
kernels (same per-op rounding); reductions and matrix products are compared
within a tolerance well inside the parity bar.
"""

import numpy as np
import pytest

from _golden import RTOL, assert_close, load_group
from oracle import dora_oracle as orc

NORM = load_group("norm")
COMPOSE = load_group("compose")
ASSEMBLY = load_group("assembly")
LAYER = load_group("layer")


@pytest.mark.parametrize("case", sorted(ASSEMBLY))
def test_assembly_within_one_ulp(case):
    """The four fp32 ops round like the reference's; only the square root may differ
    by one ulp, because PyTorch's vectorised CPU sqrt is not correctly rounded while
    the oracle (like the reference's CUDA path, ``sqrt.rn.f32`` at
    dora_fused.py:845-859) uses the IEEE square root."""
    st = ASSEMBLY[case]
    got = orc.assemble_norm(st["w"], st["c"], st["b"], float(st["scale"]))
    ref = st["norm"]
    np.testing.assert_array_equal(np.isnan(got), np.isnan(ref))
    fin = ~np.isnan(ref)
    np.testing.assert_array_max_ulp(got[fin], ref[fin], maxulp=1)
    # Squaring undoes the sqrt: the pre-sqrt sums agree bitwise where the CPU sqrt was exact.
    exact = np.sqrt(ref[fin].astype(np.float64) ** 2).astype(np.float32) == ref[fin]
    assert exact.mean() > 0.9
    if float(st["scale"]) == 1.0:
        assert got[3] == 0.0  # cancellation below zero clamps to zero
    assert np.isnan(got[7])  # NaN propagates through the clamp


@pytest.mark.parametrize("case", sorted(NORM))
def test_factored_norm(case):
    st = NORM[case]
    dt = st["dtype"]
    got, parts = orc.weight_norm_factored(
        st["W"], st["A"], st["B"], float(st["scale"]), dt, bool(st["fan_in_fan_out"])
    )
    # The factored fp32 evaluation differs from torch's only in summation order.
    tol = 1e-6 if dt == "fp32" else 0.0
    if dt == "fp32":
        np.testing.assert_allclose(got, st["norm"], rtol=tol, atol=0)
    else:
        # One ulp of the half dtype at most, from the fp32 rounding boundary.
        ulp = 2.0**-7 if dt == "bf16" else 2.0**-10
        np.testing.assert_allclose(got, st["norm"], rtol=ulp, atol=0)
    dense = orc.weight_norm_dense(
        st["W"], st["B"] @ st["A"], float(st["scale"]), dt, bool(st["fan_in_fan_out"])
    )
    assert_close(dense, st["norm_dense"], RTOL[dt], f"{case} dense")


@pytest.mark.parametrize("case", sorted(COMPOSE))
def test_compose_forward(case):
    st = COMPOSE[case]
    act, gdt, s = st["act_dtype"], st["g_dtype"], float(st["scale"])
    out = orc.compose_eager(st["lora"], st["base"], st["mag"], s, act, gdt)
    np.testing.assert_array_equal(out, st["eager_out"])
    np.testing.assert_array_equal(out, st["eager_inplace_out"])
    if act == gdt:
        fo = orc.compose_fused(st["lora"], st["base"], st["mag"], s, act)
        np.testing.assert_array_equal(fo, st["fused_oop_out"])
        o2, inner = orc.compose_forward_and_inner(st["lora"], st["base"], st["mag"], s, act)
        np.testing.assert_array_equal(o2, st["fwd_out"])
        np.testing.assert_array_equal(inner, st["fwd_inner"])


@pytest.mark.parametrize("case", sorted(COMPOSE))
def test_compose_backward(case):
    st = COMPOSE[case]
    act, gdt, s = st["act_dtype"], st["g_dtype"], float(st["scale"])
    dl, db, dg = orc.compose_backward_eager(st["d_out"], st["lora"], st["base"], st["mag"], s, act, gdt)
    np.testing.assert_array_equal(dl, st["eager_d_lora"])
    np.testing.assert_array_equal(db, st["eager_d_base"])
    assert_close(dg, st["eager_d_mag"], RTOL[gdt] / 10, f"{case} eager d_mag")
    if act == gdt:
        dl, db, dg = orc.compose_backward(st["d_out"], st["fwd_inner"], st["mag"], s, act)
        np.testing.assert_array_equal(dl, st["bwd_d_lora"])
        np.testing.assert_array_equal(db, st["bwd_d_base"])
        assert_close(dg, st["bwd_d_mag"], RTOL[act] / 10, f"{case} fused d_mag")


@pytest.mark.parametrize("case", sorted(LAYER))
def test_layer_forward_backward(case):
    st = LAYER[case]
    dt = st["dtype"]
    r = orc.dora_linear_forward_backward(
        st["x"], st["W"], st.get("bias"), st["A"], st["B"], st["m"], float(st["scale"]), st["dy"], dt
    )
    # Matrix products accumulate in a different order than oneDNN's CPU GEMMs,
    # so whole-layer results are held to the parity bar itself.
    tol = RTOL[dt]
    for k in ("y", "delta", "norm", "dx", "dA", "dB", "dm"):
        assert_close(r[k], st[k], tol, f"{case} {k}")


# ---------------------------------------------------------------------------
# Next rows: conv / embedding norms and the merge, against the reference's fixtures
# ---------------------------------------------------------------------------
def test_oracle_conv_norm_golden():
    for case, st in load_group("conv").items():
        dt = st["dtype"]
        n = orc.weight_norm_conv(st["W"], st["A"], st["B"], float(st["scale"]), dt)
        assert n.shape == st["m"].shape, case
        assert_close(n, st["m"], 1e-6 if dt == "fp32" else 8e-3, f"{case} magnitude at init")


def test_oracle_embedding_norm_golden():
    for case, st in load_group("embedding").items():
        dt = st["dtype"]
        n = orc.weight_norm_embedding(st["W"], st["A"], st["B"], float(st["scale"]), dt)
        assert_close(n, st["m"], 1e-6 if dt == "fp32" else 8e-3, f"{case} magnitude at init")


def test_oracle_merge_golden():
    for case, st in load_group("merge").items():
        dt = st["dtype"]
        merged, norm = orc.merge_weight(st["W"], st["A"], st["B"], st["m"], float(st["scale"]), dt)
        assert_close(norm, st["norm"], 1e-6 if dt == "fp32" else 8e-3, f"{case} norm")
        assert_close(merged, st["merged"], 1e-6 if dt == "fp32" else 8e-3, f"{case} merged")
