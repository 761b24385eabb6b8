"""B200-native replacement of ``peft.tuners.lora.dora_fused``.

Same public surface as the reference module (``code/peft_patched/src/peft/
tuners/lora/dora_fused.py``): ``fused_dora_compose``,
``fused_dora_forward_and_inner``, ``fused_norm_assembly``,
``FusedDoRAComposeFunction``, ``fused_dora_compose_autograd`` and a
``torch.library`` custom op for ``torch.compile``.  Every function runs the
hand-written sm_100a kernels of ``libdora_b200.so``; there is no Triton, no
PyTorch-math fallback and no CPU path.  Tensors on a non-CUDA device raise.

Semantics follow the reference:
  out   = (g - 1) * base + g * (s * lora)          (dora_fused.py:32-54)
  inner = s * lora + base                          (dora_fused.py:697-718)
  d_lora = (g * s) * d_out, d_base = (g - 1) * d_out,
  d_g = sum over broadcast dims of inner * d_out   (dora_fused.py:1229-1261)
with every elementwise result computed in fp32 and rounded once into the
activation dtype.  ``g`` may be fp32 while activations are bf16/fp16 (the AMP
case); the kernels then keep ``g - 1`` in fp32, as the reference's eager path
does.
"""

from __future__ import annotations

import logging

import torch

from . import _native

logger = logging.getLogger(__name__)

try:  # pragma: no cover - torch._dynamo may not be available
    from torch._dynamo import is_compiling as dynamo_is_compiling
except Exception:  # pragma: no cover
    dynamo_is_compiling = None


def _is_dynamo_compiling() -> bool:
    return bool(dynamo_is_compiling is not None and dynamo_is_compiling())


def is_triton_available() -> bool:
    """Kept for API compatibility with the reference; this package never uses Triton."""
    return False


def is_native_available() -> bool:
    """True when ``libdora_b200.so`` is built and loadable."""
    try:
        _native.load_library()
        return True
    except (ImportError, OSError):
        return False


def _mag_broadcasts_last_dim(mag: torch.Tensor, lora: torch.Tensor) -> bool:
    """True if *mag* is a vector along the last dim of *lora* (dora_fused.py:522-536)."""
    return mag.ndim > 0 and lora.ndim > 0 and mag.numel() == lora.shape[-1] and mag.shape[-1] == lora.shape[-1]


def _mag_is_per_channel(mag: torch.Tensor, lora: torch.Tensor) -> bool:
    """True for the convolution layout: *lora* is [batch, C, *spatial] and *mag* is
    [1, C, 1, ...] of the same rank (the g of _DoraConvNdLayer.forward, dora.py:1670-1715),
    and the last-dim layout does not apply.  The reference sends this case to its
    PyTorch fallback (dora_fused.py:563-574); here it runs the channel-layout kernels."""
    if lora.ndim < 3 or mag.ndim != lora.ndim or _mag_broadcasts_last_dim(mag, lora):
        return False
    return mag.shape[1] == lora.shape[1] and all(mag.shape[i] == 1 for i in range(mag.ndim) if i != 1)


def _prepare(lora: torch.Tensor, base: torch.Tensor, mag: torch.Tensor, what: str):
    """Validate and normalise operands: 2-D contiguous activations of one dtype and a
    contiguous 1-D ``g`` in the activation dtype or fp32."""
    _native.require_cuda(lora, base, mag, what=what)
    if lora.shape != base.shape:
        raise ValueError(f"{what}: lora {tuple(lora.shape)} and base {tuple(base.shape)} differ in shape")
    if lora.ndim == 0:
        raise ValueError(f"{what}: activations must have at least one dimension")
    cols = lora.shape[-1]
    if mag.numel() != cols:
        raise ValueError(f"mag_norm_scale has {mag.numel()} elements != num_cols {cols}")
    if not _mag_broadcasts_last_dim(mag, lora):
        raise NotImplementedError(
            f"{what}: mag_norm_scale {tuple(mag.shape)} does not broadcast along the last dim of "
            f"{tuple(lora.shape)}; only the linear layout (g over out_features) is implemented"
        )
    mag_flat = mag.reshape(-1)
    if mag_flat.shape[0] != cols:
        raise ValueError(f"mag_norm_scale last dim {mag_flat.shape[0]} != num_cols {cols}")
    if base.dtype != lora.dtype:
        base = base.to(lora.dtype)
    if mag_flat.dtype not in (lora.dtype, torch.float32):
        mag_flat = mag_flat.float()
    rows = lora.numel() // cols if cols else 0
    return lora.contiguous(), base.contiguous(), mag_flat.contiguous(), rows, cols


def fused_dora_compose(
    lora: torch.Tensor,
    base: torch.Tensor,
    mag_norm_scale: torch.Tensor,
    scale: float,
    inplace: bool = True,
) -> torch.Tensor:
    """out = (mag_norm_scale - 1) * base + mag_norm_scale * (scale * lora).

    Same contract as the reference (dora_fused.py:539-574): with ``inplace`` the
    result is written into ``lora`` (the caller guarantees ``lora`` is a fresh
    buffer), otherwise a new tensor of ``lora``'s shape and dtype is returned.
    """
    orig = lora
    if _mag_is_per_channel(mag_norm_scale, lora):
        out, _ = _channels_forward(lora, base, mag_norm_scale, scale, False, "fused_dora_compose")
        if inplace:
            orig.copy_(out)
            return orig
        return out
    l, b, g, rows, cols = _prepare(lora, base, mag_norm_scale, "fused_dora_compose")
    if inplace:
        out = l  # contiguous view of lora, or a contiguous copy written back below
    else:
        out = torch.empty_like(l)
    if rows and cols:
        _native.compose_fwd(l.view(rows, cols), b.view(rows, cols), g, scale, out.view(rows, cols), None)
    if inplace:
        if out.data_ptr() != orig.data_ptr():
            orig.copy_(out.view(orig.shape))
        return orig
    return out.view(orig.shape)


def fused_dora_forward_and_inner(
    lora: torch.Tensor,
    base: torch.Tensor,
    mag_norm_scale: torch.Tensor,
    scale: float,
) -> tuple:
    """``(out, inner)`` in one pass: out as in ``fused_dora_compose``, inner = s * lora + base
    (dora_fused.py:674-772).  ``scale * lora`` never leaves registers."""
    if _mag_is_per_channel(mag_norm_scale, lora):
        return _channels_forward(lora, base, mag_norm_scale, scale, True, "fused_dora_forward_and_inner")
    l, b, g, rows, cols = _prepare(lora, base, mag_norm_scale, "fused_dora_forward_and_inner")
    out = torch.empty_like(l)
    inner = torch.empty_like(l)
    if rows and cols:
        _native.compose_fwd(l.view(rows, cols), b.view(rows, cols), g, scale, out.view(rows, cols),
                            inner.view(rows, cols))
    return out.view(lora.shape), inner.view(lora.shape)


def fused_norm_assembly(
    w_norm_sq: torch.Tensor,
    cross_term: torch.Tensor,
    ba_norm_sq: torch.Tensor,
    scale: float,
) -> tuple:
    """``(sqrt(max(w + 2s*c + s^2*b, 0)),)`` in fp32 (dora_fused.py:873-988)."""
    _native.require_cuda(w_norm_sq, cross_term, ba_norm_sq, what="fused_norm_assembly")
    w = w_norm_sq.float().contiguous().reshape(-1)
    c = cross_term.float().contiguous().reshape(-1)
    b = ba_norm_sq.float().contiguous().reshape(-1)
    if not (w.numel() == c.numel() == b.numel()):
        raise ValueError("fused_norm_assembly: inputs differ in length")
    out = torch.empty_like(w)
    if w.numel():
        _native.norm_assembly(w, c, b, scale, out)
    out = out.view(w_norm_sq.shape)
    if w_norm_sq.dtype != torch.float32:
        out = out.to(w_norm_sq.dtype)
    return (out,)


def _backward(d_out, inner, mag, scale, need_lora, need_base, need_mag):
    """Native fused backward; returns (d_lora, d_base, d_mag) shaped like the inputs."""
    if _mag_is_per_channel(mag, d_out):
        return _channels_backward(d_out, inner, mag, scale, need_lora, need_base, need_mag)
    _native.require_cuda(d_out, inner, mag, what="FusedDoRAComposeFunction.backward")
    cols = d_out.shape[-1]
    rows = d_out.numel() // cols if cols else 0
    act = d_out.dtype
    g = mag.reshape(-1)
    if g.dtype not in (act, torch.float32):
        g = g.float()
    g = g.contiguous()
    d = d_out.contiguous()
    d_lora = torch.empty_like(d) if need_lora else None
    d_base = torch.empty_like(d) if need_base else None
    d_g = None
    inn = None
    if need_mag:
        if inner is None:
            raise AssertionError("inner must be saved when mag requires grad")
        inn = inner if inner.dtype == act else inner.to(act)
        inn = inn.contiguous()
        d_g = torch.empty(cols, dtype=g.dtype, device=d.device)
    if need_lora or need_base or need_mag:
        _native.compose_bwd(
            d.view(rows, cols),
            inn.view(rows, cols) if inn is not None else None,
            g,
            scale,
            d_lora.view(rows, cols) if d_lora is not None else None,
            d_base.view(rows, cols) if d_base is not None else None,
            d_g,
        )
    if d_lora is not None:
        d_lora = d_lora.view(d_out.shape)
    if d_base is not None:
        d_base = d_base.view(d_out.shape)
    if d_g is not None:
        d_g = d_g.view(mag.shape)
        if d_g.dtype != mag.dtype:
            d_g = d_g.to(mag.dtype)
    return d_lora, d_base, d_g


class FusedDoRAComposeFunction(torch.autograd.Function):
    """Compose with a fused backward (dora_fused.py:1065-1206).

    Forward saves ``inner = scale * lora + base`` only when ``mag_norm_scale``
    requires grad (one activation-sized buffer); with a frozen magnitude
    nothing activation-sized is saved.  Backward runs one native pass over
    ``d_out`` (and ``inner``) producing ``d_lora``, ``d_base`` and the column
    sum ``d_mag`` together.
    """

    @staticmethod
    def forward(ctx, lora, base, mag_norm_scale, scale):
        with torch.no_grad():
            if mag_norm_scale.requires_grad:
                out, inner = fused_dora_forward_and_inner(lora, base, mag_norm_scale, scale)
                ctx.save_for_backward(inner, mag_norm_scale)
                ctx.needs_mag = True
            else:
                out = fused_dora_compose(lora, base, mag_norm_scale, scale, inplace=False)
                ctx.save_for_backward(mag_norm_scale)
                ctx.needs_mag = False
        ctx.scale = scale
        return out

    @staticmethod
    def backward(ctx, d_out):
        if ctx.needs_mag:
            inner, mag = ctx.saved_tensors
        else:
            (mag,) = ctx.saved_tensors
            inner = None
        d_lora, d_base, d_mag = _backward(
            d_out, inner, mag, ctx.scale, ctx.needs_input_grad[0], ctx.needs_input_grad[1], ctx.needs_input_grad[2]
        )
        return d_lora, d_base, d_mag, None


class FusedDoRALinearOutputFunction(torch.autograd.Function):
    """The adapted linear's output ``y = result + delta`` in one pass.

    Forward: ``base = result - bias``, ``y = result + ((g - 1) * base + g * (s * lora))``
    (what ``DoraLinearLayer.forward`` followed by ``DoraLinearVariant.forward``'s
    ``result + delta`` computes, variants.py:244-283), plus ``inner = s * lora + base``
    when ``g`` needs a gradient.  Backward: one pass giving ``d_lora = (g * s) * d_y``,
    ``d_result = g * d_y`` (the direct path and the base path of ``result`` summed) and
    ``d_g = sum_rows inner * d_y``.  The separate ``result + delta`` pass and
    autograd's ``d_y + d_base`` accumulation disappear.
    """

    @staticmethod
    def forward(ctx, lora, result, mag_norm_scale, scale, bias):
        l, r, g, rows, cols = _prepare(lora, result, mag_norm_scale, "fused_dora_linear_output")
        bvec = None
        if bias is not None:
            bvec = bias.detach().reshape(-1).to(device=l.device, dtype=l.dtype).contiguous()
            if bvec.numel() != cols:
                raise ValueError(f"bias has {bvec.numel()} elements != num_cols {cols}")
        needs_mag = mag_norm_scale.requires_grad
        with torch.no_grad():
            y = torch.empty_like(l)
            inner = torch.empty_like(l) if needs_mag else None
            if rows and cols:
                _native.linear_output_fwd(l.view(rows, cols), r.view(rows, cols), bvec, g, scale,
                                          y.view(rows, cols), inner.view(rows, cols) if inner is not None else None)
        ctx.needs_mag = needs_mag
        ctx.scale = scale
        ctx.has_bias = bias is not None
        ctx.bias_meta = (bias.shape, bias.dtype) if bias is not None else None
        if needs_mag:
            ctx.save_for_backward(inner, mag_norm_scale)
        else:
            ctx.save_for_backward(mag_norm_scale)
        return y.view(lora.shape)

    @staticmethod
    def backward(ctx, d_y):
        if ctx.needs_mag:
            inner, mag = ctx.saved_tensors
        else:
            (mag,) = ctx.saved_tensors
            inner = None
        need_lora, need_result, need_mag = ctx.needs_input_grad[0], ctx.needs_input_grad[1], ctx.needs_input_grad[2]
        _native.require_cuda(d_y, inner, mag, what="FusedDoRALinearOutputFunction.backward")
        cols = d_y.shape[-1]
        rows = d_y.numel() // cols if cols else 0
        act = d_y.dtype
        g = mag.reshape(-1)
        if g.dtype not in (act, torch.float32):
            g = g.float()
        g = g.contiguous()
        d = d_y.contiguous()
        d_lora = torch.empty_like(d) if need_lora else None
        d_result = torch.empty_like(d) if need_result else None
        d_g = None
        inn = None
        if need_mag:
            inn = (inner if inner.dtype == act else inner.to(act)).contiguous()
            d_g = torch.empty(cols, dtype=g.dtype, device=d.device)
        if (need_lora or need_result or need_mag) and rows and cols:
            _native.linear_output_bwd(
                d.view(rows, cols), inn.view(rows, cols) if inn is not None else None, g, ctx.scale,
                d_lora.view(rows, cols) if d_lora is not None else None,
                d_result.view(rows, cols) if d_result is not None else None, d_g,
            )
        elif need_mag:
            d_g.zero_()
        d_bias = None
        if ctx.has_bias and ctx.needs_input_grad[4]:
            # y depends on the bias directly through base = result - bias:
            # d_bias = (1 - g) * column sums of d_y, one native pass over d_y.
            d_bias = torch.empty(cols, dtype=d.dtype, device=d.device)
            _native.linear_output_bias_grad(d.view(rows, cols), g, d_bias)
            shape, dtype = ctx.bias_meta
            d_bias = d_bias.view(shape).to(dtype)
        if d_lora is not None:
            d_lora = d_lora.view(d_y.shape)
        if d_result is not None:
            d_result = d_result.view(d_y.shape)
        if d_g is not None:
            d_g = d_g.view(mag.shape)
            if d_g.dtype != mag.dtype:
                d_g = d_g.to(mag.dtype)
        return d_lora, d_result, d_g, None, d_bias


def fused_dora_linear_output(lora, result, mag_norm_scale, scale, bias=None):
    """``result + DoRA delta`` in one native pass, with the fused backward.

    ``result`` is the base layer's output including ``bias``; the delta uses
    ``base = result - bias`` exactly as ``DoraLinearLayer.forward`` does
    (dora.py:1443-1459).
    """
    return FusedDoRALinearOutputFunction.apply(lora, result, mag_norm_scale, scale, bias)


def _broadcast_reduce_dims(out_shape: torch.Size, mag_shape: torch.Size) -> list:
    """Dims of *out_shape* broadcast from *mag_shape* (dora_fused.py:1209-1226)."""
    ndim_out, ndim_mag = len(out_shape), len(mag_shape)
    dims = []
    for i in range(ndim_out):
        j = i - (ndim_out - ndim_mag)
        if j < 0 or (mag_shape[j] == 1 and out_shape[i] != 1):
            dims.append(i)
    return dims


# ---------------------------------------------------------------------------
# torch.library custom ops: the opaque node torch.compile traces through.  The
# real implementations call the native kernels (the reference's custom op
# had to use PyTorch math, dora_fused.py:1360-1446).
# ---------------------------------------------------------------------------
_HAS_CUSTOM_OP = False
try:

    @torch.library.custom_op("dora_b200::fused_dora_compose_fwd", mutates_args=())
    def _compose_fwd_op(lora: torch.Tensor, base: torch.Tensor, mag_norm_scale: torch.Tensor, scale: float,
                        save_inner: bool) -> tuple[torch.Tensor, torch.Tensor]:
        if save_inner:
            out, inner = fused_dora_forward_and_inner(lora, base, mag_norm_scale, scale)
            return out, inner
        out = fused_dora_compose(lora, base, mag_norm_scale, scale, inplace=False)
        return out, lora.new_empty(0)

    @_compose_fwd_op.register_fake
    def _(lora, base, mag_norm_scale, scale, save_inner):
        return torch.empty_like(lora), (torch.empty_like(lora) if save_inner else lora.new_empty(0))

    @torch.library.custom_op("dora_b200::fused_dora_compose_bwd", mutates_args=())
    def _compose_bwd_op(d_out: torch.Tensor, inner: torch.Tensor, mag_norm_scale: torch.Tensor, scale: float,
                        need_lora: bool, need_base: bool, need_mag: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        dl, db, dm = _backward(d_out, inner if need_mag else None, mag_norm_scale, scale, need_lora, need_base,
                               need_mag)
        empty = d_out.new_empty(0)
        return (dl if dl is not None else empty, db if db is not None else empty,
                dm if dm is not None else mag_norm_scale.new_empty(0))

    @_compose_bwd_op.register_fake
    def _(d_out, inner, mag_norm_scale, scale, need_lora, need_base, need_mag):
        e = d_out.new_empty(0)
        return (torch.empty_like(d_out) if need_lora else e, torch.empty_like(d_out) if need_base else e,
                torch.empty_like(mag_norm_scale) if need_mag else mag_norm_scale.new_empty(0))

    def _setup_context(ctx, inputs, output):
        lora, base, mag, scale, save_inner = inputs
        _, inner = output
        ctx.save_for_backward(inner, mag)
        ctx.scale = scale
        ctx.save_inner = save_inner

    def _op_backward(ctx, d_out, _d_inner):
        inner, mag = ctx.saved_tensors
        nl, nb, nm = ctx.needs_input_grad[0], ctx.needs_input_grad[1], ctx.needs_input_grad[2] and ctx.save_inner
        dl, db, dm = torch.ops.dora_b200.fused_dora_compose_bwd(d_out.contiguous(), inner, mag, ctx.scale, nl, nb, nm)
        return (dl if nl else None, db if nb else None, dm if nm else None, None, None)

    _compose_fwd_op.register_autograd(_op_backward, setup_context=_setup_context)
    _HAS_CUSTOM_OP = True
except Exception:  # pragma: no cover - very old torch
    logger.debug("dora_b200: custom op registration failed", exc_info=True)
    _HAS_CUSTOM_OP = False


# ---------------------------------------------------------------------------
# The reference's op name and schema, peft::fused_dora_compose(Tensor lora,
# Tensor base, Tensor mag_norm_scale, float scale) -> Tensor
# (dora_fused.py:1366-1446), so code and compiled graphs that call
# torch.ops.peft.fused_dora_compose keep working.  It is registered as a
# CompositeImplicitAutograd kernel over the dora_b200 ops above: it runs above
# autograd, so it can see whether the magnitude needs a gradient and save
# ``inner`` only then (the reference's setup_context rule, dora_fused.py:1380-1397),
# while forward and backward are the native kernels with their own autograd
# and fake implementations.  When the reference's own module registered the
# name first in this process, that registration is left in place.
# ---------------------------------------------------------------------------
_HAS_PEFT_OP = False
_peft_lib = None


def _peft_compose_impl(lora: torch.Tensor, base: torch.Tensor, mag_norm_scale: torch.Tensor,
                       scale: float) -> torch.Tensor:
    save_inner = bool(mag_norm_scale.requires_grad and torch.is_grad_enabled())
    out, _ = torch.ops.dora_b200.fused_dora_compose_fwd(lora, base, mag_norm_scale, scale, save_inner)
    return out


def _register_peft_op() -> bool:
    global _peft_lib
    if not _HAS_CUSTOM_OP:
        return False
    try:
        if hasattr(torch.ops.peft, "fused_dora_compose"):
            return False
    except Exception:  # pragma: no cover - namespace lookup failure means "absent"
        pass
    try:
        lib = torch.library.Library("peft", "FRAGMENT")
        lib.define("fused_dora_compose(Tensor lora, Tensor base, Tensor mag_norm_scale, float scale) -> Tensor")
        lib.impl("fused_dora_compose", _peft_compose_impl, "CompositeImplicitAutograd")
    except Exception:  # pragma: no cover - defined concurrently by another module
        logger.debug("dora_b200: peft::fused_dora_compose registration failed", exc_info=True)
        return False
    _peft_lib = lib  # the registration lives as long as this Library object
    return True


_HAS_PEFT_OP = _register_peft_op()


def fused_dora_compose_autograd(
    lora: torch.Tensor,
    base: torch.Tensor,
    mag_norm_scale: torch.Tensor,
    scale: float,
) -> torch.Tensor:
    """Training-time compose with the fused backward (dora_fused.py:1449-1480).

    Eager mode uses ``FusedDoRAComposeFunction``; under ``torch.compile`` the
    reference's op ``peft::fused_dora_compose`` (native kernels underneath) is
    the graph node, or ``dora_b200::fused_dora_compose_fwd`` when that name
    belongs to another registration.
    """
    if _is_dynamo_compiling() and _HAS_CUSTOM_OP:
        if _HAS_PEFT_OP:
            return torch.ops.peft.fused_dora_compose(lora, base, mag_norm_scale, scale)
        out, _ = torch.ops.dora_b200.fused_dora_compose_fwd(lora, base, mag_norm_scale, scale,
                                                            mag_norm_scale.requires_grad)
        return out
    return FusedDoRAComposeFunction.apply(lora, base, mag_norm_scale, scale)


# ---------------------------------------------------------------------------
# Convolution layout: activations [batch, channels, *spatial], g per channel
# (the compose of _DoraConvNdLayer.forward, dora.py:1670-1715; the reference
# evaluates it eagerly, dora.py:1331-1334).
# ---------------------------------------------------------------------------
def _prepare_channels(lora: torch.Tensor, base: torch.Tensor, mag: torch.Tensor, what: str):
    _native.require_cuda(lora, base, mag, what=what)
    if lora.shape != base.shape:
        raise ValueError(f"{what}: lora {tuple(lora.shape)} and base {tuple(base.shape)} differ in shape")
    if lora.ndim < 2:
        raise ValueError(f"{what}: expected [batch, channels, *spatial] activations, got {tuple(lora.shape)}")
    channels = lora.shape[1]
    if mag.numel() != channels or (mag.ndim >= 2 and mag.shape[1] != channels):
        raise ValueError(f"mag_norm_scale {tuple(mag.shape)} does not hold one value per channel ({channels})")
    batch = lora.shape[0]
    spatial = lora.numel() // (batch * channels) if batch and channels else 0
    if base.dtype != lora.dtype:
        base = base.to(lora.dtype)
    g = mag.reshape(-1)
    if g.dtype not in (lora.dtype, torch.float32):
        g = g.float()
    return lora.contiguous(), base.contiguous(), g.contiguous(), batch, channels, spatial


def _channels_forward(lora, base, mag, scale, with_inner: bool, what: str):
    """Conv-layout ``(out, inner or None)``: new tensors shaped like ``lora``."""
    l, b, g, n, c, sp = _prepare_channels(lora, base, mag, what)
    out = torch.empty_like(l)
    inner = torch.empty_like(l) if with_inner else None
    if out.numel():
        _native.compose_fwd_channels(l, b, g, scale, out, inner, n, c, sp)
    return out, inner


def _channels_backward(d_out, inner, mag, scale, need_lora, need_base, need_mag):
    """Conv-layout backward: (d_lora, d_base, d_mag) with d_mag shaped and typed like ``mag``."""
    _native.require_cuda(d_out, inner, mag, what="fused_dora_compose_channels backward")
    if d_out.ndim < 2:
        raise ValueError(f"expected [batch, channels, *spatial] gradients, got {tuple(d_out.shape)}")
    n, c = d_out.shape[0], d_out.shape[1]
    sp = d_out.numel() // (n * c) if n and c else 0
    if mag.numel() != c:
        raise ValueError(f"mag_norm_scale {tuple(mag.shape)} does not hold one value per channel ({c})")
    act = d_out.dtype
    g = mag.reshape(-1)
    if g.dtype not in (act, torch.float32):
        g = g.float()
    g = g.contiguous()
    d = d_out.contiguous()
    if need_mag and inner is None:
        raise AssertionError("mag_norm_scale needs a gradient but inner was not saved")
    inn = None
    if need_mag:
        inn = (inner if inner.dtype == act else inner.to(act)).contiguous()
    d_lora = torch.empty_like(d) if need_lora else None
    d_base = torch.empty_like(d) if need_base else None
    d_g = torch.empty(c, dtype=g.dtype, device=d.device) if need_mag else None
    if d.numel() and (need_lora or need_base or need_mag):
        _native.compose_bwd_channels(d, inn, g, scale, d_lora, d_base, d_g, n, c, sp)
    elif d_g is not None:
        d_g.zero_()
    d_mag = d_g.view(mag.shape).to(mag.dtype) if d_g is not None else None
    return d_lora, d_base, d_mag


class FusedDoRAComposeChannelsFunction(torch.autograd.Function):
    """Conv-layout compose with the native fused backward; saves ``inner`` only when
    the magnitude needs a gradient, like ``FusedDoRAComposeFunction``."""

    @staticmethod
    def forward(ctx, lora, base, mag_norm_scale, scale):
        needs_mag = mag_norm_scale.requires_grad
        out, inner = _channels_forward(lora, base, mag_norm_scale, scale, needs_mag, "fused_dora_compose_channels")
        ctx.save_for_backward(*((inner, mag_norm_scale) if needs_mag else (mag_norm_scale,)))
        ctx.needs_mag = needs_mag
        ctx.scale = scale
        return out

    @staticmethod
    def backward(ctx, d_out):
        if ctx.needs_mag:
            inner, mag = ctx.saved_tensors
        else:
            (mag,) = ctx.saved_tensors
            inner = None
        d_lora, d_base, d_mag = _channels_backward(d_out, inner, mag, ctx.scale, ctx.needs_input_grad[0],
                                                   ctx.needs_input_grad[1], ctx.needs_input_grad[2])
        return d_lora, d_base, d_mag, None


def fused_dora_compose_channels(lora: torch.Tensor, base: torch.Tensor, mag_norm_scale: torch.Tensor,
                                scale: float) -> torch.Tensor:
    """out = (g - 1) * base + g * (scale * lora) with g per channel of [batch, channels, *spatial]
    activations; differentiable in all three tensors."""
    return FusedDoRAComposeChannelsFunction.apply(lora, base, mag_norm_scale, scale)
