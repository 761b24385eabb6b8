"""DoRA on a whole (small) Llama-style decoder: every q/k/v/o/gate/up/down
projection adapted by ``dorafactors_b200.model.add_dora``, one training step
(causal-LM loss, backward) against the same model adapted with an eager PyTorch
fp32 restatement of the reference DoRA layer (dense norm ||W + s B A|| per row,
delta = (g - 1) * base + g * (s * lora), dora.py:1012-1022, 1331-1334).

Tolerance: fp32, 1e-5 relative for the loss, 1e-4 (normwise) for the adapter and
magnitude gradients after two decoder layers.
"""

import copy

import pytest
import torch
from torch import nn

pytestmark = pytest.mark.gpu


class _EagerDora(nn.Module):
    def __init__(self, dora_linear):
        super().__init__()
        self.base = dora_linear.base_layer
        self.A = dora_linear.lora_A
        self.B = dora_linear.lora_B
        self.m = dora_linear.lora_magnitude_vector.weight
        self.s = dora_linear.scaling

    def forward(self, x):
        result = self.base(x)
        with torch.no_grad():
            norm = (self.base.weight + self.s * (self.B.weight @ self.A.weight)).norm(dim=1)
        g = (self.m / norm.clamp_min(1e-12)).view(1, -1)
        lora = self.B(self.A(x))
        base = result - self.base.bias if self.base.bias is not None else result
        return result + ((g - 1) * base + g * (self.s * lora))


def _swap_eager(model):
    from dorafactors_b200.layer import DoraLinear

    for module in list(model.modules()):
        for name, child in list(module.named_children()):
            if isinstance(child, DoraLinear):
                setattr(module, name, _EagerDora(child))


def test_llama_dora_step_matches_eager():
    from dorafactors_b200 import _native
    from dorafactors_b200.model import add_dora, build_llama, llama_config

    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        cfg = llama_config(layers=2, hidden=256, ffn=512, heads=4, kv_heads=2, vocab=1000, max_pos=256)
        cfg._attn_implementation = "eager"
        model = build_llama(cfg, "cuda", dtype=torch.float32, seed=1)
        params = add_dora(model, r=8, scaling=2.0, seed=2)
        ref = copy.deepcopy(model)
        _swap_eager(ref)
        ids = torch.randint(0, cfg.vocab_size, (2, 64), device="cuda", generator=torch.Generator("cuda").manual_seed(3))
        loss = model(input_ids=ids, labels=ids).loss
        loss.backward()
        ref_loss = ref(input_ids=ids, labels=ids).loss
        ref_loss.backward()
        torch.testing.assert_close(loss, ref_loss, rtol=1e-5, atol=0)
        ours = {n: p for n, p in model.named_parameters() if p.requires_grad}
        rename = {"lora_A.weight": "A.weight", "lora_B.weight": "B.weight", "lora_magnitude_vector.weight": "m"}
        theirs = {n: p for n, p in ref.named_parameters() if p.requires_grad}
        assert len(ours) == len(theirs) == len(params) == 2 * 7 * 3
        for n, p in ours.items():
            key = next(n[: -len(a)] + b for a, b in rename.items() if n.endswith(a))
            q = theirs[key]
            num = (p.grad.double() - q.grad.double()).norm()
            den = q.grad.double().norm().clamp_min(1e-30)
            assert float(num / den) <= 1e-4, (n, float(num / den))
        assert _native.device_error(reset=True) == 0
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
