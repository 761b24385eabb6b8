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
ZeRO-3 / FSDP parameter gathering, quantized base weights, conv and embedding
DoRA are outside this package.
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
        weight = base_layer.weight
        if weight.data.ndim >= 3:
            raise NotImplementedError("convolutional DoRA layers are not implemented by dorafactors_b200")
        weight = weight.to(lora_A.device)
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
