"""A self-contained DoRA linear layer wired the way PEFT wires it.

``DoraLinear`` stands in for ``peft.tuners.lora.layer.Linear`` with
``use_dora=True`` (layer.py:653-878) plus ``DoraLinearVariant.forward``
(variants.py:214-284): a frozen base ``nn.Linear``, ``lora_A`` / ``lora_B``
adapters, and the magnitude module ``DoraLinearLayer`` that returns the DoRA
delta.  It exists so the hot path can be exercised and benchmarked without the
rest of PEFT; inside PEFT the same ``DoraLinearLayer`` is driven by PEFT's own
variant code.
"""

from __future__ import annotations

import math

import torch
from torch import nn

from .dora import DoraLinearLayer


class DoraLinear(nn.Module):
    """y = base(x) + DoRA delta.  ``scaling`` is lora_alpha / r (layer.py:254-257)."""

    def __init__(self, base_layer: nn.Linear, r: int, scaling: float, dropout: float = 0.0,
                 init_lora_B_zero: bool = True):
        super().__init__()
        self.base_layer = base_layer
        self.base_layer.weight.requires_grad_(False)
        if self.base_layer.bias is not None:
            self.base_layer.bias.requires_grad_(False)
        w = base_layer.weight
        self.lora_A = nn.Linear(base_layer.in_features, r, bias=False, device=w.device, dtype=w.dtype)
        self.lora_B = nn.Linear(r, base_layer.out_features, bias=False, device=w.device, dtype=w.dtype)
        nn.init.kaiming_uniform_(self.lora_A.weight, a=math.sqrt(5))
        if init_lora_B_zero:
            nn.init.zeros_(self.lora_B.weight)
        self.scaling = float(scaling)
        self.lora_dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()
        self.lora_magnitude_vector = DoraLinearLayer(fan_in_fan_out=False)
        self.reset_magnitude()

    @torch.no_grad()
    def reset_magnitude(self) -> None:
        """m = ||W0 + s B A|| per output row (DoraLinearVariant.init, variants.py:133-161)."""
        self.lora_magnitude_vector.update_layer(
            base_layer=self.base_layer, lora_A=self.lora_A.weight, lora_B=self.lora_B.weight, scaling=self.scaling
        )

    @torch.no_grad()
    def merge(self) -> None:
        """Fold the adapter into the base weight (DoraLinearVariant.merge_unsafe,
        variants.py:184-200); the forward is then the base layer alone."""
        if getattr(self, "_merged_norm", None) is not None:
            return
        from .dora import merge_weight

        merged, norm = merge_weight(self.base_layer.weight, self.lora_A.weight, self.lora_B.weight,
                                    self.lora_magnitude_vector.weight, self.scaling)
        self.base_layer.weight.copy_(merged)
        self._merged_norm = norm

    @torch.no_grad()
    def unmerge(self) -> None:
        """Restore the base weight (DoraLinearVariant.unmerge, variants.py:202-212)."""
        norm = getattr(self, "_merged_norm", None)
        if norm is None:
            return
        from .dora import unmerge_weight

        self.base_layer.weight.copy_(unmerge_weight(self.base_layer.weight, self.lora_A.weight, self.lora_B.weight,
                                                    self.lora_magnitude_vector.weight, norm, self.scaling))
        self._merged_norm = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if getattr(self, "_merged_norm", None) is not None:
            return self.base_layer(x)
        result = self.base_layer(x)
        if isinstance(self.lora_dropout, nn.Identity) or not self.training:
            # The common path: the DoRA delta and the add to the base output are one
            # native pass (forward) and one native pass (backward).
            return self.lora_magnitude_vector.forward_output(
                x, lora_A=self.lora_A, lora_B=self.lora_B, scaling=self.scaling, base_layer=self.base_layer,
                result=result,
            )
        # Dropout active: the delta is formed from the dropped-out input, with the base
        # output recomputed from it (dora.py:1155-1263), and added to the undropped
        # result (variants.py:244-283).
        xd = self.lora_dropout(x)
        delta = self.lora_magnitude_vector(
            xd, lora_A=self.lora_A, lora_B=self.lora_B, scaling=self.scaling, base_layer=self.base_layer,
            base_result=None,
        )
        if delta.dtype != result.dtype:
            delta = delta.to(result.dtype)
        return result + delta
