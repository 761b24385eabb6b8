"""Multi-GPU layouts of the DoRA linear: out-feature row sharding and token data parallelism.

Row sharding (tensor parallel over out_features).  Rank p of P owns rows
``[p*out/P, (p+1)*out/P)`` of W0, B, the magnitude and the bias, and a replica
of A.  Every row of the factored norm depends only on its own W0 / B rows and
on A (A A^T is recomputed per rank, 2 r^2 in FLOPs), and every output column
of the compose depends only on its own g, so the norm and the compose run
locally on each shard (the row independence of the reference's factored norm,
dora.py:1024-1153).  The layer then needs one exchange forward -- every rank
needs every shard of the [T x out] output -- and two backward: the
all-reduce of dX (every shard used the whole input) and of dA (every shard
used the whole of A).  dB, dm and the bias gradient stay local.

On CUDA with NCCL the forward exchange is fused into the compose: the
``dora_linear_output_fwd_allgather`` kernel stores each output value straight
into every rank's output buffer over NVLink (CUDA IPC peer mappings),
at its final column, so there is no separate all-gather pass and no
rank-major-to-column-major copy.  The backward reads this rank's columns of
the full output gradient in place (``dora_linear_output_bwd_strided``) and
overlaps the dX all-reduce with the dX GEMMs, chunk by chunk.

Token data parallelism.  Every rank runs the whole layer on its own tokens;
``GradAllReducer`` all-reduces each LoRA A / B and magnitude gradient
asynchronously as soon as autograd has accumulated it, so the exchange runs
under the rest of the backward pass.

The collective pieces of the generic path are plain ``torch.distributed``
calls wrapped in autograd Functions, so the sharding logic runs (and is
tested) on CPU ``gloo`` ranks with any local layer.
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


# ---------------------------------------------------------------------------
# Output buffers every rank can store into (CUDA IPC peer mappings over NVLink)
# ---------------------------------------------------------------------------
def _storage_users(t: torch.Tensor) -> int:
    return torch._C._storage_Use_Count(t.untyped_storage()._cdata)


class PeerOutputPool:
    """Full-size [rows x ld] output buffers, one per rank, that every rank of the
    group can write through a peer pointer.

    Each rank allocates its buffer with the library's ``dora_peer_buffer_alloc``
    (cudaMalloc + CUDA IPC handle), the handles are exchanged over the process
    group, and every rank maps the others' buffers (``dora_peer_buffer_open``):
    plain NVLink peer mappings, no multicast object.  A buffer is handed out
    again only when no tensor outside the pool refers to its storage (the
    previous output and every autograd-saved copy of it are gone).  Allocation
    is collective, so all ranks must make the same acquire calls in the same
    order -- which SPMD code does, since every rank holds the same references.
    With one rank the buffers are ordinary device tensors and nothing is mapped.
    ``close()`` (collective) unmaps and frees everything.
    """

    def __init__(self, group=None):
        self.group = group
        self.entries: list[dict] = []
        self._flag = None

    def _world(self) -> int:
        return dist.get_world_size(self.group) if dist.is_initialized() else 1

    def acquire(self, rows: int, ld: int, dtype: torch.dtype, device: torch.device) -> dict:
        from . import _native

        key = (rows, ld, dtype, device)
        for e in self.entries:
            if e["key"] == key and _storage_users(e["buf"]) <= e["idle_users"]:
                return e
        world = self._world()
        if world == 1:
            buf = torch.empty(rows, ld, dtype=dtype, device=device)
            e = {"key": key, "buf": buf, "ptrs": [buf.data_ptr()], "addr": None, "opened": []}
        else:
            rank = dist.get_rank(self.group)
            nbytes = rows * ld * torch.empty(0, dtype=dtype).element_size()
            with torch.cuda.device(device):
                addr, handle = _native.peer_buffer_alloc(max(nbytes, 1))
            handles: list = [None] * world
            dist.all_gather_object(handles, handle, group=self.group)
            ptrs, opened = [], []
            with torch.cuda.device(device):
                for p in range(world):
                    if p == rank:
                        ptrs.append(addr)
                    else:
                        a = _native.peer_buffer_open(handles[p])
                        ptrs.append(a)
                        opened.append(a)
            buf = _native.tensor_from_device_ptr(addr, (rows, ld), dtype, device)
            e = {"key": key, "buf": buf, "ptrs": ptrs, "addr": addr, "opened": opened}
        e["idle_users"] = _storage_users(e["buf"])
        self.entries.append(e)
        return e

    def barrier(self, device: torch.device) -> None:
        """Order the current stream with every rank's: a one-element NCCL all-reduce
        that cannot finish before every rank's earlier work on its stream has."""
        if self._world() == 1:
            return
        if self._flag is None or self._flag.device != device:
            self._flag = torch.zeros(1, dtype=torch.int32, device=device)
        dist.all_reduce(self._flag, group=self.group)

    def close(self) -> None:
        """Unmap and free every buffer (collective).  No output may still be in use."""
        from . import _native

        for e in self.entries:
            if _storage_users(e["buf"]) > e["idle_users"]:
                raise RuntimeError("PeerOutputPool.close: an output buffer is still referenced")
        if self._world() > 1:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            for e in self.entries:
                for a in e["opened"]:
                    _native.peer_buffer_close(a)
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
        for e in self.entries:
            if e["addr"] is not None:
                e["buf"] = None
                _native.peer_buffer_free(e["addr"])
        self.entries.clear()


class _RowShardedDoraFn(torch.autograd.Function):
    """The row-sharded DoRA linear on CUDA: native norm, fused compose + all-gather
    forward; strided fused backward, dX all-reduce overlapped with its GEMMs."""

    @staticmethod
    def forward(ctx, x, A, B, m, layer):
        from . import _native

        W, bias, s = layer.weight, layer.bias, layer.scaling
        group = layer.group
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        in_f = W.shape[1]
        ld = sum(layer.out_sizes)
        col0 = sum(layer.out_sizes[:rank])
        with torch.no_grad():
            norm = torch.empty(W.shape[0], dtype=W.dtype, device=W.device)
            _native.weight_norm(W, A.detach(), B.detach(), s, norm)
            eps = 1e-12 if norm.dtype in (torch.float32, torch.float64) else 1e-6
            nc = norm.clamp_min(eps)
            g = m.detach() / nc
            x2 = x.detach().reshape(-1, in_f)
            result = F.linear(x2, W, bias)
            xa = F.linear(x2, A.detach())
            lora = F.linear(xa, B.detach())
            gk = g if g.dtype in (lora.dtype, torch.float32) else g.float()
            if result.dtype != lora.dtype:
                result = result.to(lora.dtype)
            needs_m = m.requires_grad
            inner = torch.empty_like(lora) if needs_m else None
            entry = layer.pool.acquire(x2.shape[0], ld, lora.dtype, lora.device)
            bvec = None if bias is None else bias.detach().to(lora.dtype).contiguous()
            if world == 1:
                # One shard holds every column: nothing to gather.
                _native.linear_output_fwd(lora, result, bvec, gk.contiguous(), s, entry["buf"], inner)
            else:
                layer.pool.barrier(lora.device)  # every rank is done reading its buffer
                _native.linear_output_fwd_allgather(lora, result, bvec, gk.contiguous(), s, entry["ptrs"], rank,
                                                    col0, ld, inner)
                layer.pool.barrier(lora.device)  # every rank's columns have landed in every buffer
            y = entry["buf"].view(*x.shape[:-1], ld)
        ctx.layer, ctx.col0, ctx.world, ctx.x_shape = layer, col0, world, x.shape
        ctx.m_dtype = m.dtype
        ctx.save_for_backward(x2, xa, inner, gk, nc, A.detach(), B.detach())
        return y

    @staticmethod
    def backward(ctx, dy):
        from . import _native

        x2, xa, inner, gk, nc, A, B = ctx.saved_tensors
        layer = ctx.layer
        W, s, group = layer.weight, layer.scaling, layer.group
        need_x, need_A, need_B, need_m = ctx.needs_input_grad[:4]
        ld = sum(layer.out_sizes)
        w = B.shape[0]
        dy2 = dy.reshape(-1, ld)
        if dy2.stride(1) != 1 or dy2.stride(0) != ld:
            dy2 = dy2.contiguous()
        if dy2.dtype != xa.dtype:
            dy2 = dy2.to(xa.dtype)
        T = dy2.shape[0]
        d_lora = torch.empty(T, w, dtype=dy2.dtype, device=dy2.device)
        d_result = torch.empty(T, w, dtype=dy2.dtype, device=dy2.device) if need_x else None
        d_g = torch.empty(w, dtype=gk.dtype, device=dy2.device) if need_m else None
        _native.linear_output_bwd_strided(dy2, ctx.col0, w, inner if need_m else None, gk, s, d_lora, d_result, d_g)
        dm = (d_g / nc).to(ctx.m_dtype) if need_m else None
        dB = d_lora.t().mm(xa) if need_B else None
        d_xa = d_lora.mm(B) if (need_A or need_x) else None
        dx = None
        works = []
        comm = ctx.world > 1
        if need_x:
            # dX = d_result W + d_xa A, summed over ranks.  Rows are produced in chunks
            # and each chunk's all-reduce starts as soon as its GEMMs are done, so the
            # exchange of chunk c runs under the GEMMs of chunk c + 1.
            dx = torch.empty(T, W.shape[1], dtype=dy2.dtype, device=dy2.device)
            n_chunks = 4 if comm and T >= 4096 else 1
            step = (T + n_chunks - 1) // n_chunks
            for r0 in range(0, T, step):
                r1 = min(T, r0 + step)
                torch.mm(d_xa[r0:r1], A, out=dx[r0:r1])
                dx[r0:r1].addmm_(d_result[r0:r1], W)
                if comm:
                    works.append(dist.all_reduce(dx[r0:r1], group=group, async_op=True))
        dA = None
        if need_A:
            dA = d_xa.t().mm(x2)
            if comm:
                works.append(dist.all_reduce(dA, group=group, async_op=True))
        for wk in works:
            wk.wait()
        if dx is not None:
            dx = dx.view(ctx.x_shape)
        return dx, dA, dB, dm, None


class RowShardedDoraLinear(nn.Module):
    """One DoRA linear split over out_features across the ranks of ``group``.

    ``from_full`` slices a full layer's tensors; every rank must pass the same
    full tensors (or at least the same A).  ``forward(x)`` takes the full input
    on every rank and returns the full output on every rank.  On CUDA with the
    NCCL backend the fused native path runs (the returned output lives in a
    peer-writable buffer that is reused once nothing refers to it); otherwise
    the generic path composes locally (``local_output``) and all-gathers.
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
        self.pool = PeerOutputPool(group)

    @classmethod
    def from_full(cls, W, bias, A, B, magnitude, scaling, group=None):
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        out = W.shape[0]
        sizes = [shard_range(out, world, p)[1] - shard_range(out, world, p)[0] for p in range(world)]
        a, b = shard_range(out, world, rank)
        return cls(W[a:b], None if bias is None else bias[a:b], A, B[a:b], magnitude[a:b], scaling, sizes, group)

    def fused_path(self, x: torch.Tensor) -> bool:
        """True when the native fused compose + all-gather path serves ``x``."""
        if not x.is_cuda:
            return False
        if not dist.is_initialized():
            return True
        return dist.get_backend(self.group) == "nccl" and dist.get_world_size(self.group) <= 8

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
        if self.fused_path(x):
            return _RowShardedDoraFn.apply(x, self.lora_A, self.lora_B, self.magnitude, self)
        x_rep = replicated_input(x, self.group)
        A_rep = replicated_input(self.lora_A, self.group)
        y_shard = self.local_output(x_rep, A_rep)
        return gather_columns(y_shard, self.out_sizes, self.group)


# ---------------------------------------------------------------------------
# Token data parallelism
# ---------------------------------------------------------------------------
def allreduce_grads(params, group=None, average: bool = False) -> None:
    """Sum (or average) the gradients of ``params`` over the group, blocking."""
    world = dist.get_world_size(group)
    for p in params:
        if p.grad is None:
            continue
        dist.all_reduce(p.grad, group=group)
        if average:
            p.grad.div_(world)


class GradAllReducer:
    """Asynchronous gradient all-reduce for token data parallelism.

    Each parameter's gradient is all-reduced as soon as autograd has finished
    accumulating it (a post-accumulate-grad hook), without blocking, so the
    exchange overlaps whatever backward work is still to come (for the DoRA
    linear: the base layer's dX GEMM).  ``wait()`` joins every pending
    exchange into the current stream; call it after ``backward()`` and before
    the gradients are read.  Hooks fire in the same order on every rank, so the
    collectives match.
    """

    def __init__(self, params, group=None, average: bool = False):
        self.group = group
        self.average = average
        self.pending: list = []
        self.handles = [p.register_post_accumulate_grad_hook(self._ready) for p in params]

    def _ready(self, p: torch.Tensor) -> None:
        self.pending.append((p, dist.all_reduce(p.grad, group=self.group, async_op=True)))

    def wait(self) -> None:
        world = dist.get_world_size(self.group) if self.average else 1
        for p, work in self.pending:
            work.wait()
            if self.average:
                p.grad.div_(world)
        self.pending.clear()

    def remove(self) -> None:
        for h in self.handles:
            h.remove()
        self.handles.clear()
