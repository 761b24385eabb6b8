"""Pin the oracle against the reference's own code, run here on fresh seeded inputs.

The reference's ``dora.py`` / ``dora_fused.py`` are byte-compiled into
``oracle/_ref`` by ``oracle/build_ref.py`` (part of ``build()`` when the
reference checkout is present).  These tests run the reference's
``DoraLinearLayer`` on its eager CPU path, wired as ``DoraLinearVariant.forward``
wires it (variants.py:214-284), and hold the numpy oracle to its outputs and
gradients, on inputs that differ from the committed fixtures -- including the
dropout path (``base_result=None``, dora.py:1470-1484) with a fixed mask, which
the fixtures do not cover.  Skipped when ``oracle/_ref`` is not built.
"""

import math

import numpy as np
import pytest
import torch
from torch import nn

from _golden import RTOL, assert_close
from oracle import build_ref
from oracle import dora_oracle as orc

pytestmark = pytest.mark.skipif(not build_ref.available(), reason="oracle/_ref not built (no reference checkout)")

_DT = {"bf16": torch.bfloat16, "fp32": torch.float32}


def _reference_layer(out_f, in_f, r, scale, dtype, bias, seed):
    dora, _ = build_ref.load_reference()
    g = torch.Generator().manual_seed(seed)
    tdt = _DT[dtype]
    base = nn.Linear(in_f, out_f, bias=bias, dtype=tdt)
    lora_A = nn.Linear(in_f, r, bias=False, dtype=tdt)
    lora_B = nn.Linear(r, out_f, bias=False, dtype=tdt)
    with torch.no_grad():
        base.weight.copy_(torch.randn(out_f, in_f, generator=g) * 0.02)
        if bias:
            base.bias.copy_(torch.randn(out_f, generator=g) * 0.1)
        lora_A.weight.copy_((torch.rand(r, in_f, generator=g) * 2 - 1) / math.sqrt(in_f))
        lora_B.weight.copy_(torch.randn(out_f, r, generator=g) * 0.05)
    base.weight.requires_grad_(False)
    if bias:
        base.bias.requires_grad_(False)
    layer = dora.DoraLinearLayer(fan_in_fan_out=False)
    layer.update_layer(base_layer=base, lora_A=lora_A.weight, lora_B=lora_B.weight, scaling=scale)
    with torch.no_grad():  # move the magnitude off its initial value so g != 1
        layer.weight.mul_(1.0 + 0.1 * torch.randn(out_f, generator=g).to(tdt))
    return base, lora_A, lora_B, layer, g


def _np(t):
    return t.detach().float().numpy()


@pytest.mark.parametrize("dtype,bias", [("bf16", False), ("bf16", True), ("fp32", False), ("fp32", True)])
def test_oracle_matches_reference_layer(dtype, bias):
    T, in_f, out_f, r, s = 48, 96, 80, 8, 1.5
    base, lora_A, lora_B, layer, g = _reference_layer(out_f, in_f, r, s, dtype, bias, seed=11 + bias)
    x = torch.randn(T, in_f, generator=g).to(_DT[dtype]).requires_grad_(True)
    dy = torch.randn(T, out_f, generator=g).to(_DT[dtype])
    result = base(x)
    delta = layer(x, lora_A=lora_A, lora_B=lora_B, scaling=s, base_layer=base, base_result=result)
    y = result + delta  # bias is not None or the base output is a fresh tensor: plain add
    y.backward(dy)
    ref = orc.dora_linear_forward_backward(
        _np(x), _np(base.weight), _np(base.bias) if bias else None, _np(lora_A.weight), _np(lora_B.weight),
        _np(layer.weight), s, _np(dy), dtype,
    )
    got = {"y": y, "delta": delta, "dx": x.grad, "dA": lora_A.weight.grad, "dB": lora_B.weight.grad,
           "dm": layer.weight.grad}
    for k, v in got.items():
        assert_close(ref[k], _np(v), RTOL[dtype], f"{dtype} bias={bias} {k}")


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
def test_oracle_matches_reference_dropout_path(dtype):
    """LoRA dropout active: the reference recomputes the base output from the
    dropped-out input inside the delta and composes it eagerly (dora.py:1155-1263)."""
    T, in_f, out_f, r, s, p = 40, 64, 72, 8, 2.0, 0.25
    base, lora_A, lora_B, layer, g = _reference_layer(out_f, in_f, r, s, dtype, True, seed=23)
    tdt = _DT[dtype]
    x = torch.randn(T, in_f, generator=g).to(tdt).requires_grad_(True)
    dy = torch.randn(T, out_f, generator=g).to(tdt)
    keep = (torch.rand(T, in_f, generator=g) >= p).to(tdt) * (1.0 / (1.0 - p))
    result = base(x)
    xd = x * keep
    delta = layer(xd, lora_A=lora_A, lora_B=lora_B, scaling=s, base_layer=base, base_result=None)
    y = result + delta
    y.backward(dy)
    ref = orc.dora_linear_dropout_forward_backward(
        _np(x), _np(keep), _np(base.weight), _np(base.bias), _np(lora_A.weight), _np(lora_B.weight),
        _np(layer.weight), s, _np(dy), dtype,
    )
    got = {"y": y, "delta": delta, "dx": x.grad, "dA": lora_A.weight.grad, "dB": lora_B.weight.grad,
           "dm": layer.weight.grad}
    for k, v in got.items():
        assert_close(ref[k], _np(v), RTOL[dtype], f"dropout {dtype} {k}")


def test_reference_norm_at_rank_above_tile():
    """The factored norm of the reference at a rank and width the fixtures do not
    reach (r = 40, 300 inputs, bf16), against the oracle."""
    base, lora_A, lora_B, layer, _ = _reference_layer(136, 300, 40, 0.75, "bf16", False, seed=5)
    with torch.no_grad():
        n = layer._get_weight_norm_linear(base_weight=base.weight, lora_A_w=lora_A.weight,
                                          lora_B_w=lora_B.weight, scaling=0.75)
    got, _ = orc.weight_norm_factored(_np(base.weight), _np(lora_A.weight), _np(lora_B.weight), 0.75, "bf16")
    np.testing.assert_allclose(got, _np(n), rtol=2.0**-7, atol=0)
