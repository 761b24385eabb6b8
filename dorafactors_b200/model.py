"""DoRA on a whole decoder model: the Llama-style training step of the
model-level configuration (7 projections per layer adapted, token data
parallelism across GPUs).

``add_dora(model, r, scaling)`` swaps every ``q/k/v/o_proj`` and
``gate/up/down_proj`` ``nn.Linear`` of a ``transformers`` Llama model for
``DoraLinear`` (the PEFT wiring of ``DoraLinearLayer``), freezing the base
weights, the way ``LoraConfig(use_dora=True, target_modules=[...])`` adapts them
(code/peft_patched/src/peft/tuners/lora/layer.py:653-878,
variants.py:132-284).  Weights are random (seeded); no checkpoint is read.

    python bench.py --mode model [--layers 32] [--gpus N]
"""

from __future__ import annotations

import torch
from torch import nn

from .layer import DoraLinear

TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def llama_config(layers: int = 32, hidden: int = 4096, ffn: int = 14336, heads: int = 32, kv_heads: int = 8,
                 vocab: int = 128256, max_pos: int = 4096):
    from transformers import LlamaConfig

    return LlamaConfig(hidden_size=hidden, intermediate_size=ffn, num_attention_heads=heads,
                       num_key_value_heads=kv_heads, num_hidden_layers=layers, vocab_size=vocab,
                       max_position_embeddings=max_pos, rms_norm_eps=1e-5, tie_word_embeddings=False)


def build_llama(config, device, dtype=torch.bfloat16, seed: int = 0):
    """A randomly initialised ``LlamaForCausalLM`` built directly on ``device``."""
    from transformers import LlamaForCausalLM

    torch.manual_seed(seed)
    with torch.device(device):
        model = LlamaForCausalLM(config).to(dtype)
    model.config.use_cache = False
    return model


def add_dora(model: nn.Module, r: int, scaling: float, targets=TARGETS, seed: int = 0) -> list:
    """Replace the target linears by ``DoraLinear`` (base frozen; lora_A kaiming-uniform,
    lora_B small random so the DoRA path is exercised from step one).  Returns the
    trainable parameters."""
    gen = torch.Generator(device="cpu").manual_seed(seed)
    for p in model.parameters():
        p.requires_grad_(False)
    trainable = []
    for name, module in list(model.named_modules()):
        for child_name, child in list(module.named_children()):
            if child_name in targets and isinstance(child, nn.Linear):
                layer = DoraLinear(child, r=r, scaling=scaling, init_lora_B_zero=False)
                with torch.no_grad():
                    b = torch.randn(layer.lora_B.weight.shape, generator=gen) * 1e-3
                    layer.lora_B.weight.copy_(b.to(layer.lora_B.weight))
                    layer.reset_magnitude()
                setattr(module, child_name, layer)
                trainable += [layer.lora_A.weight, layer.lora_B.weight, layer.lora_magnitude_vector.weight]
    return trainable
