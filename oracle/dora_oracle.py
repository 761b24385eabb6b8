"""CPU oracle for the DoRA hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, what the reference (sockeye44/dorafactors, a
patched HuggingFace PEFT) computes on its eager PyTorch path for the three hot
operations: the factored row norm, the compose forward and the compose
backward.  The tests compare the CUDA kernels against it, and ``bench.py`` times it
as the CPU baseline (``--impl reference``); nothing in the product package imports it.

Numerics model.  Arrays are float32 numpy arrays whose values are exactly
representable in the logical dtype (``"bf16"``, ``"fp16"`` or ``"fp32"``).  Each
PyTorch elementwise op of the reference is restated as one numpy op in float32
followed by a round-to-nearest-even into the logical dtype, which is how
PyTorch's CPU kernels evaluate a half-precision op (upcast, compute, round).
Reductions accumulate in float64 and round once.  Matrix products run in
float32 (the reference's ``compute_dtype`` for half weights, dora.py:1061).

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here
against fixtures produced by running the reference's own code
(``tests/golden/make_golden.py``).

Reference paths below are relative to ``code/peft_patched/src/peft/tuners/lora/``.
"""

from __future__ import annotations

import numpy as np

DTYPES = ("bf16", "fp16", "fp32")


# ---------------------------------------------------------------------------
# Rounding into the logical dtype
# ---------------------------------------------------------------------------
def round_bf16(x) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), NaN kept quiet."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32)
    nan = np.isnan(x)
    if nan.any():
        r = np.where(nan, ((u.astype(np.uint32) | np.uint32(0x00400000)) & np.uint32(0xFFFF0000)), r)
    return r.view(np.float32).reshape(x.shape)


def round_to(x, dtype: str) -> np.ndarray:
    """Round float32/float64 values into ``dtype`` and return them as float32."""
    x = np.asarray(x)
    if dtype == "fp32":
        return x.astype(np.float32)
    if dtype == "bf16":
        return round_bf16(x.astype(np.float32))
    if dtype == "fp16":
        return x.astype(np.float32).astype(np.float16).astype(np.float32)
    raise ValueError(f"unsupported dtype {dtype!r}")


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    return (round_bf16(x).view(np.uint32) >> 16).astype(np.uint16)


def fp16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def promote(a: str, b: str) -> str:
    """torch.promote_types restricted to {bf16, fp16, fp32}."""
    if a == b:
        return a
    return "fp32"


def _op(fn, dt, *xs):
    return round_to(fn(*[np.asarray(x, dtype=np.float32) for x in xs]), dt)


# ---------------------------------------------------------------------------
# Factored row norm  (dora.py:1024-1153)
# ---------------------------------------------------------------------------
def weight_norm_factored(W, A, B, scale: float, dtype: str, fan_in_fan_out: bool = False):
    """||W0 + s * B @ A|| per output row without forming B @ A.

    Follows ``DoraLinearLayer._get_weight_norm_linear`` (dora.py:1024-1153):
    fp32 compute for half weights (dora.py:1061), ``||W||^2`` as a row sum of
    squares (dora.py:1115), ``U = W A^T`` and ``G = A A^T`` (dora.py:1123-1124),
    ``cross = rowsum(B * U)`` and ``ba = rowsum((B @ G) * B)``
    (dora.py:1132-1134), the norm assembly of ``assemble_norm`` and a final cast
    to the weight dtype (dora.py:1150-1151).  ``scale == 0`` takes the
    short-cut of dora.py:1125-1129.  Returns ``(norm, parts)`` where ``parts``
    holds the fp32 ``w_norm_sq``, ``cross`` and ``ba`` vectors.
    """
    Wt = np.asarray(W, dtype=np.float32)
    if fan_in_fan_out:
        Wt = Wt.T
    A = np.asarray(A, dtype=np.float32)
    B = np.asarray(B, dtype=np.float32)
    w_norm_sq = np.einsum("ij,ij->i", Wt.astype(np.float64), Wt.astype(np.float64)).astype(np.float32)
    s = float(scale)
    if s == 0.0:
        n = np.sqrt(_clamp_min0(w_norm_sq)).astype(np.float32)
        return round_to(n, dtype), {"w_norm_sq": w_norm_sq}
    U = (Wt @ A.T).astype(np.float32)
    G = (A @ A.T).astype(np.float32)
    cross = np.einsum("ij,ij->i", B.astype(np.float64), U.astype(np.float64)).astype(np.float32)
    BG = (B @ G).astype(np.float32)
    ba = np.einsum("ij,ij->i", BG.astype(np.float64), B.astype(np.float64)).astype(np.float32)
    n = assemble_norm(w_norm_sq, cross, ba, s)
    return round_to(n, dtype), {"w_norm_sq": w_norm_sq, "cross": cross, "ba": ba}


def _clamp_min0(x: np.ndarray) -> np.ndarray:
    # torch.clamp_min keeps NaN (dora_fused.py:841-844 restates the same rule).
    return np.where(np.isnan(x), x, np.maximum(x, np.float32(0))).astype(np.float32)


def assemble_norm(w_norm_sq, cross, ba, scale: float) -> np.ndarray:
    """sqrt(max(w + (2s)c + (s^2)b, 0)) in fp32 with PyTorch's per-op rounding.

    Follows ``_fused_norm_assembly_torch`` (dora_fused.py:917-934) and the eager
    branch (dora.py:1146-1148): the coefficients ``2s`` and ``s*s`` are formed
    in Python double precision and applied as fp32 scalars; the four ops round
    separately in the order ``(w + (2s)c) + (s^2)b``; the clamp keeps NaN and the
    square root is the correctly rounded IEEE one.
    """
    s = float(scale)
    two_s = np.float32(2.0 * s)
    s2 = np.float32(s * s)
    w = np.asarray(w_norm_sq, dtype=np.float32)
    t1 = (two_s * np.asarray(cross, dtype=np.float32)).astype(np.float32)
    p = (w + t1).astype(np.float32)
    t2 = (s2 * np.asarray(ba, dtype=np.float32)).astype(np.float32)
    n2 = (p + t2).astype(np.float32)
    with np.errstate(invalid="ignore"):
        return np.sqrt(_clamp_min0(n2)).astype(np.float32)


def weight_norm_dense(W, lora_weight, scale: float, dtype: str, fan_in_fan_out: bool = False):
    """Dense reference norm ``get_weight_norm`` (dora.py:1012-1022): ||W + s*BA|| in fp32."""
    Wt = np.asarray(W, dtype=np.float32)
    if fan_in_fan_out:
        Wt = Wt.T
    tot = (Wt.astype(np.float64) + float(scale) * np.asarray(lora_weight, dtype=np.float64))
    return round_to(np.sqrt((tot * tot).sum(1)), dtype)


def mag_norm_scale(m, norm, dtype: str) -> np.ndarray:
    """g = m / clamp_min(norm, eps) (dora.py:1430-1437); eps 1e-12 for fp32, 1e-6 for half."""
    eps = 1e-12 if dtype == "fp32" else 1e-6
    n = np.maximum(np.asarray(norm, np.float32), round_to(np.float32(eps), dtype))
    return _op(np.divide, dtype, m, n)


# ---------------------------------------------------------------------------
# Compose forward  (dora.py:961-1002, 1331-1334; dora_fused.py:577-604, 697-718)
# ---------------------------------------------------------------------------
def compose_eager(lora, base, g, scale: float, act: str, gdt: str) -> np.ndarray:
    """Eager training formula ``g * (s * lora) + (g - 1) * base`` (dora.py:1331-1334).

    ``s * lora`` rounds in the activation dtype; the products with ``g`` and
    the sum round in the promoted dtype (fp32 when ``g`` is fp32 and the
    activations are half, the AMP case); the result is cast back to the
    activation dtype.
    """
    pd = promote(act, gdt)
    sl = _op(lambda a: np.float32(scale) * a, act, lora)
    p = _op(np.multiply, pd, g, sl)
    g1 = _op(lambda a: a - np.float32(1), gdt, g)
    q = _op(np.multiply, pd, g1, base)
    return round_to(_op(np.add, pd, p, q), act)


def compose_fused(lora, base, g, scale: float, dtype: str) -> np.ndarray:
    """Same-dtype fused compose ``(g - 1) * base + g * (s * lora)`` (dora_fused.py:577-604);
    bitwise equal to ``compose_eager`` when every operand has one dtype."""
    sl = _op(lambda a: np.float32(scale) * a, dtype, lora)
    g1 = _op(lambda a: a - np.float32(1), dtype, g)
    q = _op(np.multiply, dtype, g1, base)
    p = _op(np.multiply, dtype, g, sl)
    return _op(np.add, dtype, q, p)


def compose_forward_and_inner(lora, base, g, scale: float, dtype: str):
    """``(out, inner)`` with ``inner = s * lora + base`` (dora_fused.py:697-718)."""
    sl = _op(lambda a: np.float32(scale) * a, dtype, lora)
    inner = _op(np.add, dtype, sl, base)
    g1 = _op(lambda a: a - np.float32(1), dtype, g)
    out = _op(np.add, dtype, _op(np.multiply, dtype, g1, base), _op(np.multiply, dtype, g, sl))
    return out, inner


# ---------------------------------------------------------------------------
# Compose backward  (dora_fused.py:1229-1261, 1137-1206)
# ---------------------------------------------------------------------------
def compose_backward(d_out, inner, g, scale: float, dtype: str, gdt: str | None = None):
    """Gradients of ``out = g * inner - base`` (the fused backward's torch restatement,
    dora_fused.py:1229-1261).

    ``d_lora = (g * s) * d_out`` with ``g * s`` rounded first; ``d_base =
    (g - 1) * d_out``; ``d_g = sum_rows(inner * d_out)`` with the product rounded
    in the activation dtype and the column sum accumulated wide and rounded
    once into ``g``'s dtype.  ``inner`` may be ``None`` (``d_g`` then ``None``).
    """
    gdt = gdt or dtype
    pd = promote(dtype, gdt)
    gs = _op(lambda a: a * np.float32(scale), gdt, g)
    d_lora = round_to(_op(np.multiply, pd, gs, d_out), dtype)
    g1 = _op(lambda a: a - np.float32(1), gdt, g)
    d_base = round_to(_op(np.multiply, pd, g1, d_out), dtype)
    d_g = None
    if inner is not None:
        prod = _op(np.multiply, dtype, inner, d_out)
        d_g = round_to(prod.astype(np.float64).sum(axis=0, keepdims=True), pd)
    return d_lora, d_base, d_g


def compose_backward_eager(d_out, lora, base, g, scale: float, act: str, gdt: str):
    """Autograd gradients of the eager formula ``g * (s * lora) + (g - 1) * base``.

    ``d_g`` gets two column sums, ``sum(d_out * s*lora)`` and ``sum(d_out * base)``,
    one per use of ``g``, added in ``g``'s dtype.
    """
    pd = promote(act, gdt)
    sl = _op(lambda a: np.float32(scale) * a, act, lora)
    d_sl = round_to(_op(np.multiply, pd, g, d_out), act)
    d_lora = _op(lambda a: np.float32(scale) * a, act, d_sl)
    g1 = _op(lambda a: a - np.float32(1), gdt, g)
    d_base = round_to(_op(np.multiply, pd, g1, d_out), act)
    c1 = round_to(_op(np.multiply, pd, d_out, sl).astype(np.float64).sum(0, keepdims=True), gdt)
    c2 = round_to(_op(np.multiply, pd, d_out, base).astype(np.float64).sum(0, keepdims=True), gdt)
    d_g = _op(np.add, gdt, c1, c2)
    return d_lora, d_base, d_g


# ---------------------------------------------------------------------------
# The whole adapted linear  (dora.py:1380-1484 + variants.py:214-284)
# ---------------------------------------------------------------------------
def _matmul(a, b, dtype):
    return round_to(a.astype(np.float32) @ b.astype(np.float32), dtype)


def dora_linear_forward_backward(x, W, bias, A, B, m, scale: float, dy, dtype: str):
    """Forward and backward of one DoRA linear, eager reference semantics.

    Forward: ``result = x W^T + bias``; the norm of ``weight_norm_factored``;
    ``g = m / clamp(norm)``; ``lora = (x A^T) B^T``; ``delta`` by
    ``compose_eager`` on ``base = result - bias``; ``y = result + delta``.
    Backward, for the upstream gradient ``dy``: the norm is a constant
    (computed under no_grad, dora.py:1404-1417), ``dm = d_g / norm``, and ``dx``
    collects the base and LoRA branches.  Returns a dict of float32 arrays.
    """
    res = _matmul(x, W.T, dtype)
    if bias is not None:
        res = _op(np.add, dtype, res, bias[None, :])
        base = _op(np.subtract, dtype, res, bias[None, :])
    else:
        base = res
    norm, _ = weight_norm_factored(W, A, B, scale, dtype)
    eps = 1e-12 if dtype == "fp32" else 1e-6
    nc = np.maximum(norm, round_to(np.float32(eps), dtype))
    g = _op(np.divide, dtype, m[None, :], nc[None, :])
    xa = _matmul(x, A.T, dtype)
    lora = _matmul(xa, B.T, dtype)
    delta = compose_eager(lora, base, g, scale, dtype, dtype)
    y = _op(np.add, dtype, res, delta)
    d_lora, d_base, d_g = compose_backward_eager(dy, lora, base, g, scale, dtype, dtype)
    dm = _op(np.divide, dtype, d_g[0], nc)
    d_res = _op(np.add, dtype, dy, d_base)
    dB = _matmul(d_lora.T, xa, dtype)
    d_xa = _matmul(d_lora, B, dtype)
    dA = _matmul(d_xa.T, x, dtype)
    dx = _op(np.add, dtype, _matmul(d_res, W, dtype), _matmul(d_xa, A, dtype))
    return {"y": y, "delta": delta, "norm": norm, "g": g, "dx": dx, "dA": dA, "dB": dB, "dm": dm}


def dora_linear_dropout_forward_backward(x, keep_scale, W, bias, A, B, m, scale: float, dy, dtype: str):
    """Forward and backward of one DoRA linear with LoRA dropout active (training).

    ``keep_scale`` is the dropout's fixed multiplier per input element (0 where
    dropped, 1/(1-p) where kept), so ``xd = x * keep_scale``.  Follows
    ``DoraLinearVariant.forward`` with a dropout (variants.py:228-232: the delta
    is computed from ``xd`` with ``base_result=None``) and the
    ``_compose_with_base_chunks`` branch of ``DoraLinearLayer.forward``
    (dora.py:1470-1484, 1155-1263): the base output inside the delta is
    recomputed as ``xd W^T`` without bias and composed eagerly
    (``_compose_eager_inplace``, dora.py:961-1002); ``y = (x W^T + bias) + delta``.
    Backward: ``dx`` gets the undropped base path ``dy W`` plus the dropped path
    ``(d_base W + d_xa A) * keep_scale``.
    """
    xd = _op(np.multiply, dtype, x, keep_scale)
    res = _matmul(x, W.T, dtype)
    if bias is not None:
        res = _op(np.add, dtype, res, bias[None, :])
    base = _matmul(xd, W.T, dtype)
    norm, _ = weight_norm_factored(W, A, B, scale, dtype)
    eps = 1e-12 if dtype == "fp32" else 1e-6
    nc = np.maximum(norm, round_to(np.float32(eps), dtype))
    g = _op(np.divide, dtype, m[None, :], nc[None, :])
    xa = _matmul(xd, A.T, dtype)
    lora = _matmul(xa, B.T, dtype)
    delta = compose_eager(lora, base, g, scale, dtype, dtype)
    y = _op(np.add, dtype, res, delta)
    d_lora, d_base, d_g = compose_backward_eager(dy, lora, base, g, scale, dtype, dtype)
    dm = _op(np.divide, dtype, d_g[0], nc)
    dB = _matmul(d_lora.T, xa, dtype)
    d_xa = _matmul(d_lora, B, dtype)
    dA = _matmul(d_xa.T, xd, dtype)
    d_xd = _op(np.add, dtype, _matmul(d_base, W, dtype), _matmul(d_xa, A, dtype))
    dx = _op(np.add, dtype, _matmul(dy, W, dtype), _op(np.multiply, dtype, d_xd, keep_scale))
    return {"y": y, "delta": delta, "norm": norm, "g": g, "dx": dx, "dA": dA, "dB": dB, "dm": dm}


# ---------------------------------------------------------------------------
# Convolution / embedding norms and merge (the next rows beside the linear path)
# ---------------------------------------------------------------------------
def weight_norm_conv(W, A, B, scale: float, dtype: str):
    """``_DoraConvNdLayer._get_weight_norm_conv_factored`` (dora.py:1594-1634): the
    linear factored norm on the flattened weights ``W [out, -1]``, ``A [r, -1]``,
    ``B [out, -1]`` (a grouped B, ``[out, r/groups]``, expanded block-diagonally),
    returned as ``[1, out, 1, ...]``."""
    W = np.asarray(W, np.float32)
    out = W.shape[0]
    r = np.asarray(A).shape[0]
    fw = W.reshape(out, -1)
    fa = np.asarray(A, np.float32).reshape(r, -1)
    fb = np.asarray(B, np.float32).reshape(out, -1)
    rpg = fb.shape[1]
    if rpg > 0 and r % rpg == 0 and r // rpg > 1 and out % (r // rpg) == 0:
        groups = r // rpg
        opg = out // groups
        e = np.zeros((out, r), np.float32)
        for gi in range(groups):
            e[gi * opg:(gi + 1) * opg, gi * rpg:(gi + 1) * rpg] = fb[gi * opg:(gi + 1) * opg]
        fb = e
    n, _ = weight_norm_factored(fw, fa, fb, scale, dtype)
    return n.reshape((1, out) + (1,) * (W.ndim - 2))


def weight_norm_embedding(table, emb_A, emb_B, scale: float, dtype: str):
    """Embedding DoRA magnitude (``DoraEmbeddingVariant.init`` -> ``update_layer`` with
    ``fan_in_fan_out=True``, variants.py:287-300, dora.py:1341-1378): one value per
    embedding dimension, ``||table[:, j] + s (emb_A^T emb_B^T)[:, j]||`` over the
    vocabulary, i.e. the factored norm of ``W0 = table^T``, ``A = emb_A``, ``B = emb_B``."""
    return weight_norm_factored(table, emb_A, emb_B, scale, dtype, fan_in_fan_out=True)[0]


def compose_channels(lora, base, g, scale: float, dtype: str) -> np.ndarray:
    """Eager compose with g per channel of ``[N, C, *spatial]`` activations
    (dora.py:1331-1334 with ``mag_norm_scale`` shaped ``[1, C, 1, ...]``)."""
    lora = np.asarray(lora, np.float32)
    gb = np.asarray(g, np.float32).reshape((1, -1) + (1,) * (lora.ndim - 2))
    sl = _op(np.multiply, dtype, np.float32(scale), lora)
    a = _op(np.multiply, dtype, gb - np.float32(1), base)
    return _op(np.add, dtype, a, _op(np.multiply, dtype, gb, sl))


def merge_weight(W, A, B, m, scale: float, dtype: str):
    """``DoraLinearVariant.merge_safe`` (variants.py:164-182): delta = s B A,
    norm = ``get_weight_norm(W, delta, 1)``, ``W' = (m / norm) (W + delta)`` in the
    weight dtype.  Returns ``(merged, norm)``."""
    delta = np.asarray(B, np.float32) @ np.asarray(A, np.float32) * np.float32(scale)
    norm = weight_norm_dense(W, delta, 1.0, dtype)
    factor = (np.asarray(m, np.float32) / norm)[:, None]
    merged = round_to(factor * (np.asarray(W, np.float32) + delta), dtype)
    return merged, norm
