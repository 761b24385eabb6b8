"""Multi-GPU layouts of the DoRA linear: out-feature row sharding and token data parallelism.

Row sharding (tensor parallel over out_features).  Rank p of P owns rows
``[p*out/P, (p+1)*out/P)`` of W0, B, the magnitude and the bias, and a replica
of A.  Every row of the factored norm depends only on its own W0 / B rows and
on A (A A^T is recomputed per rank, 2 r^2 in FLOPs), and every output column
of the compose depends only on its own g, so the norm and the compose run
locally on each shard.  The layer then needs exactly one collective in the
forward pass -- an all-gather of the [T x out/P] output shards over NCCL -- and
two in the backward pass: the all-reduce of dX (every shard used the whole
input) and of dA (every shard used the whole of A).  dB, dm and the bias
gradient stay local.

Token data parallelism.  Every rank runs the whole layer on its own tokens;
the LoRA A / B and magnitude gradients are all-reduced after backward
(``allreduce_grads``).

The collective pieces are plain ``torch.distributed`` calls wrapped in autograd
Functions, so the sharding logic runs (and is tested) on CPU ``gloo`` ranks
with any local layer; the DoRA compute itself is the native CUDA path.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Rows owned by ``rank`` when ``total`` rows are split into ``world`` near-equal blocks."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class _ReplicatedInput(torch.autograd.Function):
    """Identity forward; all-reduce (sum) of the gradient in backward.

    Marks a tensor every rank holds in full and uses to compute a different
    output shard (the layer input x, the replicated LoRA A)."""

    @staticmethod
    def forward(ctx, t, group):
        ctx.group = group
        return t.view_as(t)

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous()
        dist.all_reduce(g, group=ctx.group)
        return g, None


class _GatherColumns(torch.autograd.Function):
    """All-gather of [..., cols_p] shards into [..., sum cols_p]; backward keeps this rank's slice."""

    @staticmethod
    def forward(ctx, shard, group, sizes):
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        ctx.rank, ctx.sizes = rank, sizes
        lead = shard.shape[:-1]
        flat = shard.reshape(-1, shard.shape[-1]).contiguous()
        width = max(sizes)
        if flat.shape[1] < width:  # collectives move equal-sized blocks: pad the short shards
            flat = F.pad(flat, (0, width - flat.shape[1]))
        out = torch.empty((world * flat.shape[0], flat.shape[1]), dtype=flat.dtype, device=flat.device)
        dist.all_gather_into_tensor(out, flat, group=group)
        out = out.view(world, flat.shape[0], flat.shape[1])
        if len(set(sizes)) == 1:
            # [P, rows, cols_p] -> [rows, P * cols_p]
            y = out.permute(1, 0, 2).reshape(flat.shape[0], -1)
        else:
            y = torch.cat([out[p, :, : sizes[p]] for p in range(world)], dim=1)
        return y.reshape(*lead, y.shape[-1])

    @staticmethod
    def backward(ctx, g):
        start = sum(ctx.sizes[: ctx.rank])
        return g[..., start : start + ctx.sizes[ctx.rank]].contiguous(), None, None


def replicated_input(t: torch.Tensor, group=None) -> torch.Tensor:
    return _ReplicatedInput.apply(t, group)


def gather_columns(shard: torch.Tensor, sizes: list[int], group=None) -> torch.Tensor:
    return _GatherColumns.apply(shard, group, list(sizes))


class RowShardedDoraLinear(nn.Module):
    """One DoRA linear split over out_features across the ranks of ``group``.

    ``from_full`` slices a full layer's tensors; every rank must pass the same
    full tensors (or at least the same A).  ``forward(x)`` takes the full input
    on every rank and returns the full output on every rank.
    """

    def __init__(self, W_shard, bias_shard, A, B_shard, magnitude_shard, scaling: float, out_sizes, group=None):
        super().__init__()
        self.group = group
        self.out_sizes = list(out_sizes)
        self.scaling = float(scaling)
        self.weight = nn.Parameter(W_shard.contiguous(), requires_grad=False)
        self.bias = None if bias_shard is None else nn.Parameter(bias_shard.contiguous(), requires_grad=False)
        self.lora_A = nn.Parameter(A.contiguous())
        self.lora_B = nn.Parameter(B_shard.contiguous())
        self.magnitude = nn.Parameter(magnitude_shard.contiguous())

    @classmethod
    def from_full(cls, W, bias, A, B, magnitude, scaling, group=None):
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        out = W.shape[0]
        sizes = [shard_range(out, world, p)[1] - shard_range(out, world, p)[0] for p in range(world)]
        a, b = shard_range(out, world, rank)
        return cls(W[a:b], None if bias is None else bias[a:b], A, B[a:b], magnitude[a:b], scaling, sizes, group)

    def local_output(self, x: torch.Tensor, A: torch.Tensor) -> torch.Tensor:
        """This shard's [T x out_p] output of the DoRA linear (native norm + fused compose)."""
        from . import _native
        from .dora_fused import fused_dora_linear_output

        with torch.no_grad():
            norm = torch.empty(self.weight.shape[0], dtype=self.weight.dtype, device=self.weight.device)
            _native.weight_norm(self.weight, self.lora_A.detach(), self.lora_B.detach(), self.scaling, norm)
        eps = 1e-12 if norm.dtype in (torch.float32, torch.float64) else 1e-6
        g = (self.magnitude / norm.clamp_min(eps)).view(1, -1)
        result = F.linear(x, self.weight, self.bias)
        lora = F.linear(F.linear(x, A), self.lora_B)
        if g.dtype not in (lora.dtype, torch.float32):
            g = g.float()
        return fused_dora_linear_output(lora, result, g, self.scaling, self.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x_rep = replicated_input(x, self.group)
        A_rep = replicated_input(self.lora_A, self.group)
        y_shard = self.local_output(x_rep, A_rep)
        return gather_columns(y_shard, self.out_sizes, self.group)


def allreduce_grads(params, group=None, average: bool = False) -> None:
    """Token data parallelism: sum (or average) the gradients of ``params`` over the group."""
    world = dist.get_world_size(group)
    for p in params:
        if p.grad is None:
            continue
        dist.all_reduce(p.grad, group=group)
        if average:
            p.grad.div_(world)
