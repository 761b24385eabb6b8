"""Multi-rank host logic on CPU: gloo ranks run the row-sharded DoRA linear
(out-feature shards, one all-gather forward, dX / dA all-reduces backward) and
token data parallelism, and must reproduce a single-process computation.

The local per-shard math here is an eager PyTorch restatement of the DoRA
linear, because the native kernels need a GPU; the GPU path is exercised by
the gpu-marked tests.  What is under test is the sharding: row ranges, the
all-gather layout (including uneven shards), and which gradients are reduced.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _eager_dora(x, W, bias, A, B, m, s):
    with torch.no_grad():
        norm = (W + s * (B @ A)).norm(dim=1)
    g = (m / norm).view(1, -1)
    result = F.linear(x, W, bias)
    lora = F.linear(F.linear(x, A), B)
    base = result - bias if bias is not None else result
    return result + ((g - 1) * base + g * (s * lora))


def _make(seed=0, T=6, inp=10, out=7, r=3):
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(out, inp, generator=g, dtype=torch.float64) * 0.3
    bias = torch.randn(out, generator=g, dtype=torch.float64) * 0.1
    A = torch.randn(r, inp, generator=g, dtype=torch.float64) * 0.3
    B = torch.randn(out, r, generator=g, dtype=torch.float64) * 0.3
    m = torch.rand(out, generator=g, dtype=torch.float64) + 0.5
    x = torch.randn(T, inp, generator=g, dtype=torch.float64)
    dy = torch.randn(T, out, generator=g, dtype=torch.float64)
    return x, W, bias, A, B, m, dy


def _worker(rank, world, port, q):
    try:
        _run_worker(rank, world, port, q)
    except BaseException as e:  # report instead of leaving the parent waiting
        q.put((rank, repr(e)))
        raise


def _run_worker(rank, world, port, q):
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from dorafactors_b200 import parallel

        class EagerShard(parallel.RowShardedDoraLinear):
            def local_output(self, x, A):
                return _eager_dora(x, self.weight, self.bias, A, self.lora_B, self.magnitude, self.scaling)

        x, W, bias, A, B, m, dy = _make()
        s = 0.7
        layer = EagerShard.from_full(W, bias, A, B, m, s)
        xr = x.clone().requires_grad_(True)
        y = layer(xr)
        y.backward(dy)
        a, b = parallel.shard_range(W.shape[0], world, rank)
        # numpy copies travel through the queue by value (shared tensors would need
        # this process to stay alive until the parent has read them).
        out = {
            "y": y.detach().numpy().copy(),
            "dx": xr.grad.numpy().copy(),
            "dA": layer.lora_A.grad.numpy().copy(),
            "dB": (a, b, layer.lora_B.grad.numpy().copy()),
            "dm": (a, b, layer.magnitude.grad.numpy().copy()),
            "sizes": layer.out_sizes,
        }
        # Token data parallelism: each rank a different batch, gradients summed.
        xs = torch.randn(4, W.shape[1], generator=torch.Generator().manual_seed(10 + rank), dtype=torch.float64)
        Ad = A.clone().requires_grad_(True)
        _eager_dora(xs, W, bias, Ad, B, m, s).sum().backward()
        parallel.allreduce_grads([Ad])
        out["dp_dA"] = Ad.grad.numpy().copy()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_row_sharded_and_data_parallel_match_single_process(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for rank, r in results.items():
        assert not isinstance(r, str), f"rank {rank} failed: {r}"
    assert all(p.exitcode == 0 for p in procs)

    x, W, bias, A, B, m, dy = _make()
    s = 0.7
    xr, Ar, Br, mr = (t.clone().requires_grad_(True) for t in (x, A, B, m))
    y = _eager_dora(xr, W, bias, Ar, Br, mr, s)
    y.backward(dy)

    def close(a, b, tol=1e-12):
        torch.testing.assert_close(torch.from_numpy(a), b, rtol=tol, atol=tol)

    for rank in range(world):
        r = results[rank]
        assert sum(r["sizes"]) == W.shape[0]
        close(r["y"], y.detach())
        close(r["dx"], xr.grad)
        close(r["dA"], Ar.grad)
        a, b, dB = r["dB"]
        close(dB, Br.grad[a:b])
        a, b, dm = r["dm"]
        close(dm, mr.grad[a:b])
    # Data parallel: the summed gradient equals the gradient of the concatenated batch.
    Ad = A.clone().requires_grad_(True)
    xs = torch.cat([torch.randn(4, W.shape[1], generator=torch.Generator().manual_seed(10 + k),
                                dtype=torch.float64) for k in range(world)])
    _eager_dora(xs, W, bias, Ad, B, m, s).sum().backward()
    for rank in range(world):
        close(results[rank]["dp_dA"], Ad.grad, 1e-10)


def test_shard_range_covers_rows():
    from dorafactors_b200.parallel import shard_range

    for total in (1, 7, 8, 28672):
        for world in (1, 2, 3, 8):
            spans = [shard_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)
