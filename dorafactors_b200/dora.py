"""B200-native replacement of ``peft.tuners.lora.dora`` for linear layers.

``DoraLinearLayer`` keeps the reference's interface (``code/peft_patched/src/
peft/tuners/lora/dora.py:1005-1489``): ``update_layer``, ``forward`` returning
the DoRA *delta* ``(g - 1) * base + g * s * lora``, ``get_weight_norm``,
``_get_weight_norm_linear`` and the ``weight`` magnitude parameter, so PEFT's
``DoraLinearVariant`` (variants.py:132-284) drives it unchanged.

What changed underneath:
  * the row norm runs natively in one call: tcgen05 tensor-core GEMMs with the
    ``||W0||^2`` and row-sum reductions fused in (bf16/fp16), an fp32 CUDA-core
    path otherwise;
  * compose forward / backward are the fused sm_100a kernels of
    ``dora_fused``, always (no eager/Triton dispatch, no shape heuristics);
  * the chunking knobs ``PEFT_DORA_NORM_CHUNK_MB`` / ``PEFT_DORA_FWD_CHUNK_MB``
    are read for compatibility and ignored: the norm's working set is
    O(out + r^2) floats regardless of ``in``, and the no-``base_result`` path
    forms the base output in one GEMM, which 180 GB of HBM holds for any
    practical layer.
Convolution and embedding layers (``DoraConv1d/2d/3dLayer``,
``DoraEmbeddingLayer``, dora.py:1491-1742) reuse the native factored norm on
flattened (conv) or transposed (embedding) weights; the embedding norm no longer
forms the dense [num_embeddings x embedding_dim] delta the reference builds.
ZeRO-3 / FSDP parameter gathering and quantized base weights are outside this
package.
"""

from __future__ import annotations

import logging
import os
import threading
from contextlib import contextmanager
from typing import Optional

import torch
import torch.nn.functional as F
from torch import nn

from . import _native
from .dora_fused import (
    fused_dora_compose,
    fused_dora_compose_autograd,
    fused_norm_assembly,
    is_triton_available,
)

logger = logging.getLogger(__name__)

__all__ = [
    "DoraConv1dLayer",
    "DoraConv2dLayer",
    "DoraConv3dLayer",
    "DoraEmbeddingLayer",
    "DoraLinearLayer",
    "fused_dora_compose",
    "fused_dora_compose_autograd",
    "fused_norm_assembly",
    "is_triton_available",
    "set_dora_norm_threshold_mb",
]

_DTYPE_TO_ELEMENT_SIZE = {torch.float32: 4, torch.float64: 8, torch.float16: 2, torch.bfloat16: 2}

# ---------------------------------------------------------------------------
# Compatibility knobs (dora.py:192-628).  They select nothing here: there is a
# single native path.  They are parsed and cached the same way so that code
# which sets them keeps working, and the chunk sizes are logged as ignored.
# ---------------------------------------------------------------------------
_cache_lock = threading.Lock()
_cached_thresholds: dict = {}


def _read_mb(name: str, default_mb: int = 256) -> int:
    env = os.environ.get(name)
    mb = default_mb
    if env is not None:
        try:
            mb = max(16, int(env))
        except (ValueError, TypeError):
            mb = default_mb
    return mb * 1024 * 1024


def _get_norm_memory_threshold_bytes() -> int:
    with _cache_lock:
        if "norm" not in _cached_thresholds:
            _cached_thresholds["norm"] = _read_mb("PEFT_DORA_NORM_CHUNK_MB")
        return _cached_thresholds["norm"]


def _get_forward_chunk_threshold_bytes() -> int:
    with _cache_lock:
        if "fwd" not in _cached_thresholds:
            _cached_thresholds["fwd"] = _read_mb("PEFT_DORA_FWD_CHUNK_MB")
        return _cached_thresholds["fwd"]


def _invalidate_threshold_cache() -> None:
    with _cache_lock:
        _cached_thresholds.clear()


def _invalidate_fused_cache() -> None:
    """Reset cached environment reads (kept for test-suite compatibility)."""
    _invalidate_threshold_cache()


def set_dora_norm_threshold_mb(mb: int) -> None:
    """Set ``PEFT_DORA_NORM_CHUNK_MB`` (16..65536), as the reference does (dora.py:614-627).

    The native norm does not chunk, so the value has no effect on results or memory.
    """
    if not isinstance(mb, int):
        raise ValueError(f"mb must be an integer, got {type(mb).__name__}")
    if not (16 <= mb <= 65536):
        raise ValueError(f"mb must be between 16 and 65536 (got {mb})")
    os.environ["PEFT_DORA_NORM_CHUNK_MB"] = str(mb)
    _invalidate_threshold_cache()


@contextmanager
def _disable_autocast(device_type: str):
    """Disable autocast for the scope; body exceptions propagate (dora.py:871-892)."""
    try:
        ctx = torch.autocast(device_type=device_type, enabled=False)
    except (TypeError, RuntimeError, ValueError):
        yield
        return
    with ctx:
        yield


def _transpose(w: torch.Tensor, fan_in_fan_out: bool) -> torch.Tensor:
    return w.T if fan_in_fan_out else w


class DoraLinearLayer(nn.Module):
    """DoRA magnitude module for one linear layer (dora.py:1005-1489)."""

    def __init__(self, fan_in_fan_out):
        super().__init__()
        self.fan_in_fan_out = fan_in_fan_out
        self._last_chunk_size: Optional[int] = None
        self._last_forward_chunk_size: Optional[int] = None

    # ------------------------------------------------------------------ norms
    @torch.no_grad()
    def get_weight_norm(self, weight, lora_weight, scaling) -> torch.Tensor:
        """Dense ``||W + s * lora_weight||`` per row, fp32 compute, weight dtype out (dora.py:1012-1022)."""
        W = _transpose(weight, self.fan_in_fan_out)
        _native.require_cuda(W, what="get_weight_norm")
        if W.dtype not in _native.DTYPE_CODE:
            raise ValueError(f"Unsupported weight dtype {W.dtype} for DoRA norm computation.")
        W = W.contiguous()
        L = lora_weight.to(device=W.device)
        if L.dtype not in _native.DTYPE_CODE:
            L = L.float()
        L = L.contiguous()
        if L.shape != W.shape:
            raise ValueError(f"lora_weight shape {tuple(L.shape)} != weight shape {tuple(W.shape)}")
        out = torch.empty(W.shape[0], dtype=W.dtype, device=W.device)
        _native.weight_norm_dense(W, L, float(scaling), out)
        return out

    @torch.no_grad()
    def _get_weight_norm_linear(
        self,
        *,
        base_weight: torch.Tensor,
        lora_A_w: torch.Tensor,
        lora_B_w: torch.Tensor,
        scaling: float,
        chunk_size: Optional[int] = None,
    ):
        """``||W + s * (B A)||`` per row without forming ``B A`` (dora.py:1024-1153).

        One native call: tensor-core GEMMs for ``W A^T`` and ``A A^T`` with the
        ``||W||^2`` and row-sum contractions fused in, then the norm assembly
        and the cast to the weight dtype.  ``chunk_size`` is accepted for
        compatibility; the computation is never chunked, so ``_last_chunk_size``
        records ``in_features``.
        """
        W = _transpose(base_weight, self.fan_in_fan_out)
        dtype = W.dtype
        if dtype not in _native.DTYPE_CODE:
            raise ValueError(
                f"Unsupported compute_dtype {dtype} for DoRA norm computation. "
                f"Expected one of {set(_native.DTYPE_CODE.keys())}."
            )
        _native.require_cuda(W, what="_get_weight_norm_linear")
        out_features, in_features = W.shape
        A = lora_A_w.to(device=W.device)
        B = lora_B_w.to(device=W.device)
        if A.dtype not in _native.DTYPE_CODE:
            A = A.float()
        if B.dtype not in _native.DTYPE_CODE:
            B = B.float()
        if A.shape[1] != in_features or B.shape[0] != out_features or B.shape[1] != A.shape[0]:
            raise ValueError(
                f"shape mismatch: W {tuple(W.shape)}, A {tuple(A.shape)}, B {tuple(B.shape)}"
            )
        self._last_chunk_size = in_features if chunk_size is None else max(1, min(in_features, chunk_size))
        if chunk_size is None and _get_norm_memory_threshold_bytes() and logger.isEnabledFor(logging.DEBUG):
            logger.debug("DoRA: PEFT_DORA_NORM_CHUNK_MB is ignored; the native norm does not chunk")
        norm = torch.empty(out_features, dtype=dtype, device=W.device)
        _native.weight_norm(W.contiguous(), A.contiguous(), B.contiguous(), float(scaling), norm)
        return norm

    # ------------------------------------------------------------------ init
    def update_layer(self, *, base_layer, lora_A, lora_B, scaling, place_on_cpu=False) -> None:
        """Create the magnitude parameter m = ||W0 + s B A|| (dora.py:1341-1378)."""
        dtype_is_fp16 = lora_A.dtype == torch.float16
        if dtype_is_fp16:
            lora_A = lora_A.float()
            lora_B = lora_B.float()
        weight = base_layer.weight.to(lora_A.device)
        if weight.data.ndim >= 3:  # convolution weights (dora.py:1358-1364)
            if not hasattr(self, "_get_weight_norm_conv_factored"):
                raise NotImplementedError("a convolution weight needs a DoraConvNdLayer")
            weight_norm = self._get_weight_norm_conv_factored(
                base_weight=weight, lora_A_w=lora_A, lora_B_w=lora_B, scaling=scaling
            )
        else:
            weight_norm = self._get_weight_norm_linear(
                base_weight=weight, lora_A_w=lora_A, lora_B_w=lora_B, scaling=scaling
            )
        if dtype_is_fp16:
            weight_norm = weight_norm.half()
        if place_on_cpu:
            weight_norm = weight_norm.to("cpu")
        self.weight = nn.Parameter(weight_norm, requires_grad=True)

    # ------------------------------------------------------------------ forward
    def _compose_with_dispatch(self, *, lora_out, base_result, mag_norm_scale, scale):
        """Native compose: fused autograd when anything needs grad, in-place otherwise
        (dora.py:1265-1339 without the eager branches)."""
        needs_grad = lora_out.requires_grad or base_result.requires_grad or mag_norm_scale.requires_grad
        g = mag_norm_scale
        if g.dtype not in (lora_out.dtype, torch.float32):
            g = g.float()
        if needs_grad:
            return fused_dora_compose_autograd(lora_out, base_result, g, scale)
        return fused_dora_compose(lora_out, base_result, g, scale, inplace=True)

    def forward(self, x, *, lora_A, lora_B, scaling, base_layer, base_result=None):
        """DoRA delta ``(g - 1) * base + g * s * lora`` to add to the base output (dora.py:1380-1484).

        The norm is computed under ``no_grad`` (DoRA section 4.3) and detached;
        ``g = m / clamp_min(norm, eps)`` stays differentiable in ``m``.
        """
        magnitude = self.weight
        device_type = base_layer.weight.device.type
        with torch.no_grad(), _disable_autocast(device_type):
            base_weight = base_layer.weight
            weight_norm = self._get_weight_norm_linear(
                base_weight=base_weight,
                lora_A_w=lora_A.weight,
                lora_B_w=lora_B.weight,
                scaling=scaling,
            )
        if weight_norm.device != magnitude.device:
            weight_norm = weight_norm.to(device=magnitude.device)
        eps = 1e-12 if weight_norm.dtype in (torch.float32, torch.float64) else 1e-6
        weight_norm = weight_norm.clamp_min(eps)
        mag_norm_scale = (magnitude / weight_norm).view(1, -1)

        lora_result = lora_B(lora_A(x))
        scale = scaling

        if base_result is not None:
            bias = base_layer.bias
            if bias is not None:
                if bias.device != base_result.device or bias.dtype != base_result.dtype:
                    bias = bias.to(device=base_result.device, dtype=base_result.dtype)
                base_result = base_result - bias
            self._last_forward_chunk_size = None
            return self._compose_with_dispatch(
                lora_out=lora_result, base_result=base_result, mag_norm_scale=mag_norm_scale, scale=scale
            )

        # Dropout path (dora.py:1155-1263): the base output is not given, so it is
        # recomputed from the (dropped-out) input in one GEMM and composed natively.
        W = base_layer.weight
        if W.device != x.device or W.dtype != x.dtype:
            W = W.to(device=x.device, dtype=x.dtype)
        W = _transpose(W, self.fan_in_fan_out)
        if _get_forward_chunk_threshold_bytes() and logger.isEnabledFor(logging.DEBUG):
            logger.debug("DoRA: PEFT_DORA_FWD_CHUNK_MB is ignored; base output formed in one GEMM")
        self._last_forward_chunk_size = W.shape[0]
        base_full = F.linear(x, W)
        return self._compose_with_dispatch(
            lora_out=lora_result, base_result=base_full, mag_norm_scale=mag_norm_scale, scale=scale
        )

    def forward_output(self, x, *, lora_A, lora_B, scaling, base_layer, result):
        """The layer output ``result + delta`` in one fused pass.

        Equivalent to ``result + self.forward(x, ..., base_result=result)``, the
        composition ``DoraLinearVariant.forward`` performs (variants.py:214-284), with
        the add folded into the compose kernel and its backward.  ``result`` is the
        base layer's output on ``x`` (bias included).
        """
        from .dora_fused import fused_dora_linear_output

        magnitude = self.weight
        with torch.no_grad(), _disable_autocast(base_layer.weight.device.type):
            weight_norm = self._get_weight_norm_linear(
                base_weight=base_layer.weight,
                lora_A_w=lora_A.weight,
                lora_B_w=lora_B.weight,
                scaling=scaling,
            )
        if weight_norm.device != magnitude.device:
            weight_norm = weight_norm.to(device=magnitude.device)
        eps = 1e-12 if weight_norm.dtype in (torch.float32, torch.float64) else 1e-6
        mag_norm_scale = (magnitude / weight_norm.clamp_min(eps)).view(1, -1)
        lora_result = lora_B(lora_A(x))
        g = mag_norm_scale
        if g.dtype not in (lora_result.dtype, torch.float32):
            g = g.float()
        bias = base_layer.bias
        self._last_forward_chunk_size = None
        if result.dtype != lora_result.dtype:
            result = result.to(lora_result.dtype)
        return fused_dora_linear_output(lora_result, result, g, scaling, bias)

    def __repr__(self) -> str:
        return "lora.dora." + super().__repr__()


class DoraEmbeddingLayer(DoraLinearLayer):
    """DoRA magnitude module for an embedding (dora.py:1491-1590), built with
    ``fan_in_fan_out=True`` by PEFT's ``DoraEmbeddingVariant`` (variants.py:287-300).

    The magnitude holds one value per embedding dimension: the norm is taken over
    the vocabulary, ``||W[:, j] + s (lora_A lora_B)[:, j]||``.  With ``W0 = W^T``,
    ``A = lora_A^T`` and ``B = lora_B^T`` that is the factored row norm of the linear
    layer, so it runs natively without forming the [V x d] delta.
    """

    def forward(self, x, *, lora_A, lora_B, scaling, base_layer, embed_fn, base_result=None):
        """Return ``(mag_norm_scale, delta)``; ``lora_A`` [V x r] and ``lora_B`` [r x d] are
        the transposed adapter tensors, as ``DoraEmbeddingVariant.forward`` passes them."""
        magnitude = self.weight
        with torch.no_grad(), _disable_autocast(base_layer.weight.device.type):
            weight_norm = self._get_weight_norm_linear(
                base_weight=base_layer.weight, lora_A_w=lora_A.T, lora_B_w=lora_B.T, scaling=scaling
            )
        if weight_norm.device != magnitude.device:
            weight_norm = weight_norm.to(device=magnitude.device)
        eps = 1e-12 if weight_norm.dtype in (torch.float32, torch.float64) else 1e-6
        mag_norm_scale = magnitude / weight_norm.clamp_min(eps)
        if base_result is None:
            weight = base_layer.weight
            if weight.device != x.device:
                weight = weight.to(device=x.device)
            base_result = embed_fn(x, weight)
        lora_out = embed_fn(x, lora_A) @ lora_B
        if base_result.dtype != lora_out.dtype:
            base_result = base_result.to(lora_out.dtype)
        result_dora = self._compose_with_dispatch(
            lora_out=lora_out, base_result=base_result, mag_norm_scale=mag_norm_scale, scale=scaling
        )
        return mag_norm_scale, result_dora


class _DoraConvNdLayer(DoraLinearLayer):
    """DoRA magnitude module for Conv1d/2d/3d (dora.py:1593-1724).

    The norm is the linear factored norm on the flattened weights
    ``W [out, in/groups * k...]``, ``A [r, in/groups * k...]``, ``B [out, r]`` (grouped
    adapters expand B block-diagonally, dora.py:1612-1624); the compose runs on the
    native channel-layout kernels (g per output channel of [N, C, *spatial]).
    The magnitude has shape [1, out, 1, ...].
    """

    conv_fn = None

    @torch.no_grad()
    def _get_weight_norm_conv_factored(self, *, base_weight, lora_A_w, lora_B_w, scaling, chunk_size=None):
        out_channels = base_weight.shape[0]
        flat_weight = base_weight.reshape(out_channels, -1)
        rank = lora_A_w.shape[0]
        flat_A = lora_A_w.reshape(rank, -1)
        flat_B = lora_B_w.reshape(out_channels, -1)
        rank_per_group = flat_B.shape[1]
        if rank_per_group > 0 and rank % rank_per_group == 0:
            groups = rank // rank_per_group
            if groups > 1 and out_channels % groups == 0:
                out_per_group = out_channels // groups
                expanded = flat_B.new_zeros((out_channels, rank))
                for gi in range(groups):
                    rows = slice(gi * out_per_group, (gi + 1) * out_per_group)
                    cols = slice(gi * rank_per_group, (gi + 1) * rank_per_group)
                    expanded[rows, cols] = flat_B[rows, :]
                flat_B = expanded
        saved = self.fan_in_fan_out
        self.fan_in_fan_out = False  # conv weights are never stored transposed
        try:
            norms = self._get_weight_norm_linear(
                base_weight=flat_weight, lora_A_w=flat_A, lora_B_w=flat_B, scaling=scaling, chunk_size=chunk_size
            )
        finally:
            self.fan_in_fan_out = saved
        return norms.view((1, out_channels) + (1,) * max(0, base_weight.dim() - 2))

    @torch.no_grad()
    def get_weight_norm(self, weight, lora_weight, scaling) -> torch.Tensor:
        """Dense ``||W + s * lora_weight||`` per output channel, shaped [1, out, 1, ...] (dora.py:1636-1646)."""
        out_channels = weight.shape[0]
        W = weight.reshape(out_channels, -1)
        _native.require_cuda(W, what="get_weight_norm")
        if W.dtype not in _native.DTYPE_CODE:
            raise ValueError(f"Unsupported weight dtype {W.dtype} for DoRA norm computation.")
        L = lora_weight.to(device=W.device).reshape(out_channels, -1)
        if L.dtype not in _native.DTYPE_CODE:
            L = L.float()
        out = torch.empty(out_channels, dtype=W.dtype, device=W.device)
        _native.weight_norm_dense(W.contiguous(), L.contiguous(), float(scaling), out)
        return out.view((1, out_channels) + (1,) * max(0, weight.dim() - 2))

    def _compose_with_dispatch(self, *, lora_out, base_result, mag_norm_scale, scale):
        from .dora_fused import fused_dora_compose_channels

        return fused_dora_compose_channels(lora_out, base_result, mag_norm_scale, scale)

    def forward(self, x, *, lora_A, lora_B, scaling, base_layer, base_result=None):
        """DoRA delta of a convolution (dora.py:1648-1715): norm under ``no_grad`` and
        detached, ``g = m / clamp_min(norm, eps)``, compose on the native kernels."""
        magnitude = self.weight
        with torch.no_grad(), _disable_autocast(base_layer.weight.device.type):
            weight = base_layer.weight
            weight_norm = self._get_weight_norm_conv_factored(
                base_weight=weight, lora_A_w=lora_A.weight, lora_B_w=lora_B.weight, scaling=scaling
            )
        if weight_norm.device != magnitude.device:
            weight_norm = weight_norm.to(device=magnitude.device)
        eps = 1e-12 if weight_norm.dtype in (torch.float32, torch.float64) else 1e-6
        mag_norm_scale = magnitude / weight_norm.clamp_min(eps)
        if base_result is None:
            w = base_layer.weight
            if w.device != x.device or w.dtype != x.dtype:
                w = w.to(device=x.device, dtype=x.dtype)
            base_result = self.conv_fn(
                x, w, bias=None, stride=base_layer.stride, padding=base_layer.padding,
                dilation=base_layer.dilation, groups=base_layer.groups,
            )
        else:
            bias = base_layer.bias
            if bias is not None:
                if bias.device != base_result.device or bias.dtype != base_result.dtype:
                    bias = bias.to(device=base_result.device, dtype=base_result.dtype)
                base_result = base_result - bias.view((1, -1) + (1,) * (base_result.dim() - 2))
        lora_out = lora_B(lora_A(x))
        if base_result.dtype != lora_out.dtype:
            base_result = base_result.to(lora_out.dtype)
        return self._compose_with_dispatch(
            lora_out=lora_out, base_result=base_result, mag_norm_scale=mag_norm_scale, scale=scaling
        )


class DoraConv1dLayer(_DoraConvNdLayer):
    conv_fn = staticmethod(F.conv1d)


class DoraConv2dLayer(_DoraConvNdLayer):
    conv_fn = staticmethod(F.conv2d)


class DoraConv3dLayer(_DoraConvNdLayer):
    conv_fn = staticmethod(F.conv3d)


# ---------------------------------------------------------------------------
# Merge / unmerge of a linear DoRA adapter into the base weight
# (DoraLinearVariant.merge_safe / merge_unsafe / unmerge, variants.py:164-212).
# ---------------------------------------------------------------------------
@torch.no_grad()
def merge_weight(base_weight, lora_A_w, lora_B_w, magnitude, scaling, fan_in_fan_out=False):
    """Return ``(merged_weight, weight_norm)`` with
    ``merged = (m / ||W + s B A||) * (W + s B A)`` in the weight's dtype and layout.

    The norm is the native factored norm (the reference forms it densely from the
    delta, variants.py:168-173; same value within fp32 rounding).  Keep
    ``weight_norm`` for ``unmerge_weight``: it must be the norm of the original
    weight, as the reference caches it."""
    layer = DoraLinearLayer(fan_in_fan_out=fan_in_fan_out)
    norm = layer._get_weight_norm_linear(base_weight=base_weight, lora_A_w=lora_A_w, lora_B_w=lora_B_w,
                                         scaling=scaling)
    delta = _transpose((lora_B_w.float() @ lora_A_w.float()) * scaling, fan_in_fan_out)
    factor = _transpose((magnitude.detach().float() / norm.float()).view(-1, 1), fan_in_fan_out)
    merged = (factor * (base_weight.float() + delta)).to(base_weight.dtype)
    return merged, norm


@torch.no_grad()
def unmerge_weight(merged_weight, lora_A_w, lora_B_w, magnitude, weight_norm, scaling, fan_in_fan_out=False):
    """Invert ``merge_weight``: ``W = merged / (m / norm) - s B A`` (variants.py:202-212)."""
    delta = _transpose((lora_B_w.float() @ lora_A_w.float()) * scaling, fan_in_fan_out)
    factor = _transpose((magnitude.detach().float() / weight_norm.float()).view(-1, 1), fan_in_fan_out)
    return (merged_weight.float() / factor - delta).to(merged_weight.dtype)
