"""Generate the golden fixtures for the DoRA hot path by running the reference itself.

The reference (sockeye44/dorafactors, a patched subset of HuggingFace PEFT) is
pure Python.  Its DoRA modules import four helpers from ``peft.utils`` that the
patched subset does not ship (``code/peft_patched/src/peft/tuners/lora/dora.py:57-62``),
so this script writes a four-function stub package into a temporary directory,
puts it beside ``code/peft_patched/src`` on ``sys.path`` (both halves of the
``peft`` namespace package merge), imports ``peft.tuners.lora.dora`` and
``peft.tuners.lora.dora_fused`` and records what they compute on seeded CPU
inputs.  On CPU the reference always takes its eager PyTorch path
(``dora.py:928-958`` gates the fused paths on ``is_cuda``), which is the path the
parity contract names.

Output: ``tests/golden/*.npz``.  Half-precision tensors are stored as their raw
``uint16`` bit patterns under ``<name>__bf16`` / ``<name>__fp16`` keys, fp32 as
float32.  Run from the repository root::

    python tests/golden/make_golden.py --reference <reference checkout>

The fixtures are small (a few hundred KB in total) and committed; the reference
is never read at test time.
"""

from __future__ import annotations

import argparse
import importlib
import os
import sys
import tempfile
import textwrap

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

_STUB_INTEGRATIONS = textwrap.dedent(
    """
    from contextlib import nullcontext


    def dequantize_module_weight(module):
        return module.weight


    def gather_params_ctx(*args, **kwargs):
        return nullcontext()


    def check_deepspeed_zero3_enabled():
        return False
    """
)

_STUB_OTHER = textwrap.dedent(
    """
    def transpose(weight, fan_in_fan_out):
        return weight.T if fan_in_fan_out else weight
    """
)


def import_reference(reference_root: str):
    """Import the reference's dora / dora_fused modules through the stub package."""
    stub_root = tempfile.mkdtemp(prefix="peft_stub_")
    os.makedirs(os.path.join(stub_root, "peft", "utils"))
    with open(os.path.join(stub_root, "peft", "utils", "integrations.py"), "w") as f:
        f.write(_STUB_INTEGRATIONS)
    with open(os.path.join(stub_root, "peft", "utils", "other.py"), "w") as f:
        f.write(_STUB_OTHER)
    src = os.path.join(reference_root, "code", "peft_patched", "src")
    sys.path.insert(0, src)
    sys.path.insert(0, stub_root)
    dora = importlib.import_module("peft.tuners.lora.dora")
    dora_fused = importlib.import_module("peft.tuners.lora.dora_fused")
    return dora, dora_fused


_TORCH_DT = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}


def _put(store: dict, name: str, t: torch.Tensor) -> None:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        store[name + "__bf16"] = t.view(torch.int16).numpy().view(np.uint16)
    elif t.dtype == torch.float16:
        store[name + "__fp16"] = t.view(torch.int16).numpy().view(np.uint16)
    elif t.dtype == torch.float32:
        store[name] = t.numpy().astype(np.float32)
    else:
        raise TypeError(t.dtype)


def _meta(store: dict, **kw) -> None:
    for k, v in kw.items():
        store["meta_" + k] = np.asarray(v)


def gen_norm_cases(dora) -> dict:
    """Factored row norm, ``DoraLinearLayer._get_weight_norm_linear`` (dora.py:1024-1153),
    and the dense ``get_weight_norm`` (dora.py:1012-1022) for the same inputs."""
    cases = {
        # name: (out, in, r, scale, dtype, fan_in_fan_out)
        "norm_fp32": (96, 64, 8, 2.0, "fp32", False),
        "norm_bf16": (96, 64, 8, 2.0, "bf16", False),
        "norm_fp16": (64, 48, 16, 0.5, "fp16", False),
        "norm_ragged_bf16": (130, 72, 12, 0.5, "bf16", False),
        "norm_s0_fp32": (64, 48, 4, 0.0, "fp32", False),
        "norm_fifo_fp32": (80, 56, 8, 1.5, "fp32", True),
        "norm_rank1_fp32": (40, 24, 1, 3.0, "fp32", False),
    }
    out = {}
    for name, (o, i, r, s, dt, fifo) in cases.items():
        g = torch.Generator().manual_seed(1000 + o + i + r)
        tdt = _TORCH_DT[dt]
        W = (torch.randn(o, i, generator=g) * 0.02).to(tdt)
        if fifo:
            W = W.T.contiguous()  # stored [in, out] like a GPT-2 Conv1D weight
        A = (torch.rand(r, i, generator=g) * 2 - 1).mul(1.0 / i**0.5).to(tdt)
        B = (torch.randn(o, r, generator=g) * 0.01).to(tdt)
        layer = dora.DoraLinearLayer(fan_in_fan_out=fifo)
        norm = layer._get_weight_norm_linear(base_weight=W, lora_A_w=A, lora_B_w=B, scaling=s)
        dense = layer.get_weight_norm(W, B.float() @ A.float() if dt != "fp32" else B @ A, s)
        st = {}
        _put(st, "W", W)
        _put(st, "A", A)
        _put(st, "B", B)
        _put(st, "norm", norm)
        _put(st, "norm_dense", dense)
        _meta(st, scale=s, dtype=dt, fan_in_fan_out=int(fifo))
        out[name] = st
    return out


def gen_compose_cases(dora, dora_fused) -> dict:
    """Compose forward (eager formula dora.py:1331 and in-place helper dora.py:961-1002),
    the fused module's torch restatements (dora_fused.py:577-604, 697-718) and the
    fused backward's torch restatement (dora_fused.py:1229-1261)."""
    cases = {
        # name: (rows, cols, scale, act dtype, g dtype)
        "compose_bf16": (33, 96, 2.0, "bf16", "bf16"),
        "compose_fp16": (8, 24, 0.5, "fp16", "fp16"),
        "compose_fp32": (17, 100, 1.0, "fp32", "fp32"),
        "compose_ragged_bf16": (5, 37, 0.7, "bf16", "bf16"),
        "compose_mixed_bf16_g32": (12, 64, 2.0, "bf16", "fp32"),
        "compose_3d_bf16": (24, 40, 1.0, "bf16", "bf16"),
    }
    out = {}
    for name, (rows, cols, s, adt, gdt) in cases.items():
        g = torch.Generator().manual_seed(2000 + rows * 7 + cols)
        at, gt = _TORCH_DT[adt], _TORCH_DT[gdt]
        lora = torch.randn(rows, cols, generator=g).to(at)
        base = torch.randn(rows, cols, generator=g).to(at)
        mag = (torch.rand(1, cols, generator=g) + 0.5).to(gt)
        d_out = torch.randn(rows, cols, generator=g).to(at)
        st = {}
        _put(st, "lora", lora)
        _put(st, "base", base)
        _put(st, "mag", mag)
        _put(st, "d_out", d_out)
        # Eager training formula (dora.py:1331-1334): promoted dtype, cast back.
        eager = mag * (s * lora) + (mag - 1) * base
        if eager.dtype != lora.dtype:
            eager = eager.to(lora.dtype)
        _put(st, "eager_out", eager)
        # Eager in-place helper (dora.py:961-1002).
        _put(st, "eager_inplace_out", dora._compose_eager_inplace(lora.clone(), base, mag, s))
        if adt == gdt:
            _put(st, "fused_oop_out", dora_fused._fused_dora_compose_torch(lora, base, mag, s, inplace=False))
            o2, inner = dora_fused._fused_dora_forward_and_inner_torch(lora, base, mag, s)
            _put(st, "fwd_out", o2)
            _put(st, "fwd_inner", inner)
            dl, db, dm = dora_fused._fused_backward_torch(d_out, inner, mag, s, True, True, True)
            _put(st, "bwd_d_lora", dl)
            _put(st, "bwd_d_base", db)
            _put(st, "bwd_d_mag", dm)
        # Eager autograd gradients of the training formula.
        lr = lora.clone().requires_grad_(True)
        bs = base.clone().requires_grad_(True)
        mg = mag.clone().requires_grad_(True)
        y = mg * (s * lr) + (mg - 1) * bs
        if y.dtype != lr.dtype:
            y = y.to(lr.dtype)
        y.backward(d_out)
        _put(st, "eager_d_lora", lr.grad)
        _put(st, "eager_d_base", bs.grad)
        _put(st, "eager_d_mag", mg.grad)
        _meta(st, scale=s, act_dtype=adt, g_dtype=gdt)
        out[name] = st
    return out


def gen_assembly_cases(dora_fused) -> dict:
    """Norm assembly torch restatement (dora_fused.py:917-934), including
    cancellation to a negative sum (clamped to 0) and NaN propagation."""
    g = torch.Generator().manual_seed(3000)
    w = torch.rand(257, generator=g) * 10
    c = torch.randn(257, generator=g)
    b = torch.rand(257, generator=g) * 5
    w[3], c[3], b[3] = 1.0, -1.0, 0.25  # 1 - 2 + 0.25 < 0 -> clamped to 0 at s=1
    w[7] = float("nan")
    out = {}
    for s in (0.0, 1.0, 0.3, 2.0):
        st = {}
        _put(st, "w", w)
        _put(st, "c", c)
        _put(st, "b", b)
        (n,) = dora_fused._fused_norm_assembly_torch(w, c, b, s)
        _put(st, "norm", n)
        _meta(st, scale=s)
        out[f"assembly_s{str(s).replace('.', 'p')}"] = st
    return out


def gen_layer_cases(dora) -> dict:
    """Full ``DoraLinearLayer.forward`` (dora.py:1380-1484) on the eager path with
    ``base_result`` given, the way ``DoraLinearVariant.forward`` calls it
    (variants.py:214-284): y = base(x) + delta, then backward with a seeded
    upstream gradient.  Records y, delta, the norm, dx, dA, dB, dm."""
    cases = {
        # name: (tokens, in, out, r, scale, dtype, bias)
        "layer_fp32": (24, 64, 96, 8, 2.0, "fp32", False),
        "layer_bf16": (24, 64, 96, 8, 2.0, "bf16", False),
        "layer_bias_fp32": (16, 48, 40, 4, 0.5, "fp32", True),
        "layer_ragged_bf16": (9, 40, 52, 6, 1.0, "bf16", True),
    }
    out = {}
    for name, (T, i, o, r, s, dt, has_bias) in cases.items():
        g = torch.Generator().manual_seed(4000 + T + i + o + r)
        tdt = _TORCH_DT[dt]
        base = torch.nn.Linear(i, o, bias=has_bias).to(tdt)
        lora_A = torch.nn.Linear(i, r, bias=False).to(tdt)
        lora_B = torch.nn.Linear(r, o, bias=False).to(tdt)
        with torch.no_grad():
            base.weight.copy_((torch.randn(o, i, generator=g) * 0.02).to(tdt))
            if has_bias:
                base.bias.copy_((torch.randn(o, generator=g) * 0.1).to(tdt))
            lora_A.weight.copy_(((torch.rand(r, i, generator=g) * 2 - 1) / i**0.5).to(tdt))
            lora_B.weight.copy_((torch.randn(o, r, generator=g) * 0.01).to(tdt))
        base.weight.requires_grad_(False)
        if has_bias:
            base.bias.requires_grad_(False)
        layer = dora.DoraLinearLayer(fan_in_fan_out=False)
        layer.update_layer(base_layer=base, lora_A=lora_A.weight, lora_B=lora_B.weight, scaling=s)
        x = torch.randn(T, i, generator=g).to(tdt).requires_grad_(True)
        dy = torch.randn(T, o, generator=g).to(tdt)
        result = base(x)
        delta = layer(x, lora_A=lora_A, lora_B=lora_B, scaling=s, base_layer=base, base_result=result)
        y = result + delta
        y.backward(dy)
        with torch.no_grad():
            norm = layer._get_weight_norm_linear(
                base_weight=base.weight, lora_A_w=lora_A.weight, lora_B_w=lora_B.weight, scaling=s
            )
        st = {}
        _put(st, "x", x)
        _put(st, "W", base.weight)
        if has_bias:
            _put(st, "bias", base.bias)
        _put(st, "A", lora_A.weight)
        _put(st, "B", lora_B.weight)
        _put(st, "m", layer.weight)
        _put(st, "dy", dy)
        _put(st, "y", y)
        _put(st, "delta", delta)
        _put(st, "norm", norm)
        _put(st, "dx", x.grad)
        _put(st, "dA", lora_A.weight.grad)
        _put(st, "dB", lora_B.weight.grad)
        _put(st, "dm", layer.weight.grad)
        _meta(st, scale=s, dtype=dt, has_bias=int(has_bias))
        out[name] = st
    return out


def gen_embedding_cases(dora) -> dict:
    """``DoraEmbeddingLayer`` (dora.py:1491-1590) as ``DoraEmbeddingVariant`` drives it
    (variants.py:287-379): init through ``update_layer`` with ``fan_in_fan_out=True``,
    forward with the transposed adapter tensors and ``base_result = embedding(x)``,
    y = result + delta, backward with a seeded upstream gradient."""
    cases = {
        # name: (tokens, vocab, dim, r, scale, dtype)
        "emb_fp32": (20, 50, 64, 8, 2.0, "fp32"),
        "emb_bf16": (24, 77, 96, 8, 0.5, "bf16"),
    }
    out = {}
    for name, (T, V, d, r, s, dt) in cases.items():
        g = torch.Generator().manual_seed(5000 + T + V + d + r)
        tdt = _TORCH_DT[dt]
        base = torch.nn.Embedding(V, d).to(tdt)
        with torch.no_grad():
            base.weight.copy_((torch.randn(V, d, generator=g) * 0.5).to(tdt))
        base.weight.requires_grad_(False)
        emb_A = torch.nn.Parameter((torch.randn(r, V, generator=g) * 0.3).to(tdt))  # lora_embedding_A [r, V]
        emb_B = torch.nn.Parameter((torch.randn(d, r, generator=g) * 0.3).to(tdt))  # lora_embedding_B [d, r]
        layer = dora.DoraEmbeddingLayer(fan_in_fan_out=True)
        layer.update_layer(base_layer=base, lora_A=emb_A, lora_B=emb_B, scaling=s)
        x = torch.randint(0, V, (T,), generator=g)
        dy = torch.randn(T, d, generator=g).to(tdt)
        embed_fn = lambda ids, w: torch.nn.functional.embedding(ids, w)  # noqa: E731
        result = base(x)
        _, delta = layer(x, lora_A=emb_A.T, lora_B=emb_B.T, scaling=s, base_layer=base, embed_fn=embed_fn,
                         base_result=result)
        if delta.dtype != result.dtype:
            delta = delta.to(result.dtype)
        y = result + delta
        y.backward(dy)
        st = {}
        store_ids = x.to(torch.float32)  # token ids are small integers, exact in fp32
        _put(st, "ids", store_ids)
        _put(st, "W", base.weight)
        _put(st, "A", emb_A)
        _put(st, "B", emb_B)
        _put(st, "m", layer.weight)
        _put(st, "dy", dy)
        _put(st, "y", y)
        _put(st, "dA", emb_A.grad)
        _put(st, "dB", emb_B.grad)
        _put(st, "dm", layer.weight.grad)
        _meta(st, scale=s, dtype=dt)
        out[name] = st
    return out


def gen_conv_cases(dora) -> dict:
    """``DoraConv1dLayer`` / ``DoraConv2dLayer`` (dora.py:1593-1742) the way PEFT's conv
    LoRA wires them: lora_A = Conv(in, r, kernel, stride, padding), lora_B = Conv(r, out, 1),
    ``base_result = base(x)`` (bias included; the layer subtracts it), y = result + delta,
    backward with a seeded upstream gradient."""
    cases = {
        # name: (conv dims, batch, in, out, r, kernel, spatial, scale, dtype, bias)
        "conv2d_fp32": (2, 3, 8, 12, 4, 3, 9, 2.0, "fp32", True),
        "conv2d_bf16": (2, 2, 16, 24, 8, 3, 16, 0.5, "bf16", False),
        "conv1d_fp32": (1, 4, 6, 10, 3, 5, 21, 1.0, "fp32", True),
    }
    out = {}
    for name, (nd, N, ci, co, r, k, sp, s, dt, has_bias) in cases.items():
        g = torch.Generator().manual_seed(6000 + N + ci + co + r + k + sp)
        tdt = _TORCH_DT[dt]
        Conv = torch.nn.Conv2d if nd == 2 else torch.nn.Conv1d
        base = Conv(ci, co, k, padding=k // 2, bias=has_bias).to(tdt)
        lora_A = Conv(ci, r, k, padding=k // 2, bias=False).to(tdt)
        lora_B = Conv(r, co, 1, bias=False).to(tdt)
        with torch.no_grad():
            base.weight.copy_((torch.randn(base.weight.shape, generator=g) * 0.1).to(tdt))
            if has_bias:
                base.bias.copy_((torch.randn(co, generator=g) * 0.1).to(tdt))
            lora_A.weight.copy_((torch.randn(lora_A.weight.shape, generator=g) * 0.1).to(tdt))
            lora_B.weight.copy_((torch.randn(lora_B.weight.shape, generator=g) * 0.1).to(tdt))
        base.weight.requires_grad_(False)
        if has_bias:
            base.bias.requires_grad_(False)
        layer = (dora.DoraConv2dLayer if nd == 2 else dora.DoraConv1dLayer)(fan_in_fan_out=False)
        layer.update_layer(base_layer=base, lora_A=lora_A.weight, lora_B=lora_B.weight, scaling=s)
        shape = (N, ci) + (sp,) * nd
        x = torch.randn(shape, generator=g).to(tdt).requires_grad_(True)
        result = base(x)
        dy = torch.randn(result.shape, generator=g).to(tdt)
        delta = layer(x, lora_A=lora_A, lora_B=lora_B, scaling=s, base_layer=base, base_result=result)
        if delta.dtype != result.dtype:
            delta = delta.to(result.dtype)
        y = result + delta
        y.backward(dy)
        st = {}
        _put(st, "x", x)
        _put(st, "W", base.weight)
        if has_bias:
            _put(st, "bias", base.bias)
        _put(st, "A", lora_A.weight)
        _put(st, "B", lora_B.weight)
        _put(st, "m", layer.weight)
        _put(st, "dy", dy)
        _put(st, "y", y)
        _put(st, "dx", x.grad)
        _put(st, "dA", lora_A.weight.grad)
        _put(st, "dB", lora_B.weight.grad)
        _put(st, "dm", layer.weight.grad)
        _meta(st, scale=s, dtype=dt, has_bias=int(has_bias), conv_dims=nd, kernel=k)
        out[name] = st
    return out


def gen_merge_cases(dora) -> dict:
    """DoRA merge / unmerge of a linear layer (variants.py:164-212): the dense
    ``get_weight_norm(W, delta, 1)`` of the reference with delta = s * B A, then
    W' = (m / norm) * (W + delta) and back W = W' / (m / norm) - delta.  The two
    variant formulas are restated here (the variants module needs the rest of PEFT);
    the norm is the reference's own ``get_weight_norm``."""
    cases = {
        # name: (out, in, r, scale, dtype)
        "merge_fp32": (48, 40, 4, 2.0, "fp32"),
        "merge_bf16": (64, 96, 8, 0.5, "bf16"),
    }
    out = {}
    for name, (o, i, r, s, dt) in cases.items():
        g = torch.Generator().manual_seed(7000 + o + i + r)
        tdt = _TORCH_DT[dt]
        W = (torch.randn(o, i, generator=g) * 0.05).to(tdt)
        A = (torch.randn(r, i, generator=g) * 0.2).to(tdt)
        B = (torch.randn(o, r, generator=g) * 0.2).to(tdt)
        layer = dora.DoraLinearLayer(fan_in_fan_out=False)
        base = torch.nn.Linear(i, o, bias=False).to(tdt)
        with torch.no_grad():
            base.weight.copy_(W)
        layer.update_layer(base_layer=base, lora_A=A, lora_B=B, scaling=s)
        with torch.no_grad():
            layer.weight.mul_(1.05)  # a trained-looking magnitude
            delta = (B @ A) * s
            norm = layer.get_weight_norm(W, delta, scaling=1).detach()
            factor = (layer.weight / norm).view(-1, 1)
            merged = (factor * (W + delta)).to(tdt)
            unmerged = (merged / factor - delta).to(tdt)
        st = {}
        _put(st, "W", W)
        _put(st, "A", A)
        _put(st, "B", B)
        _put(st, "m", layer.weight.detach())
        _put(st, "norm", norm)
        _put(st, "merged", merged)
        _put(st, "unmerged", unmerged)
        _meta(st, scale=s, dtype=dt)
        out[name] = st
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DORA_REFERENCE_ROOT"),
                    required="DORA_REFERENCE_ROOT" not in os.environ,
                    help="reference checkout (default: $DORA_REFERENCE_ROOT)")
    ap.add_argument("--groups", default="", help="comma-separated subset of groups to (re)write")
    args = ap.parse_args()
    torch.manual_seed(0)
    dora, dora_fused = import_reference(args.reference)
    makers = {
        "norm": lambda: gen_norm_cases(dora),
        "compose": lambda: gen_compose_cases(dora, dora_fused),
        "assembly": lambda: gen_assembly_cases(dora_fused),
        "layer": lambda: gen_layer_cases(dora),
        "embedding": lambda: gen_embedding_cases(dora),
        "conv": lambda: gen_conv_cases(dora),
        "merge": lambda: gen_merge_cases(dora),
    }
    wanted = [g for g in args.groups.split(",") if g] or list(makers)
    groups = {name: makers[name]() for name in wanted}
    for group, cases in groups.items():
        flat = {}
        for case, st in cases.items():
            for k, v in st.items():
                flat[f"{case}/{k}"] = v
        path = os.path.join(HERE, f"{group}.npz")
        np.savez_compressed(path, **flat)
        print(f"wrote {path}: {len(cases)} cases, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
