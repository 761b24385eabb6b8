"""Multi-GPU paths on two GPUs (NCCL, one process per GPU).

Row sharding: each rank owns half the out-features, runs the native norm and
the fused compose + all-gather (its output columns stored into both ranks'
buffers over NVLink), and the strided fused backward with the dX all-reduce.
The gathered output and every gradient must match the single-GPU DoraLinear
within the bf16 parity bar, for an even split (16-byte vectors) and an odd one
(scalar stores at an unaligned column offset), across two steps (the second
reuses the output buffers).  Token data parallelism: the asynchronous
gradient all-reduce equals the gradient of the concatenated batch.  Skipped
when fewer than two GPUs are visible.
"""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rel(u, v):
    u, v = u.double(), v.double()
    return float((u - v).norm() / v.norm().clamp_min(1e-30))


def _rank_main(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    from dorafactors_b200.layer import DoraLinear
    from dorafactors_b200.parallel import GradAllReducer, RowShardedDoraLinear, shard_range

    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        errs = {}
        for out_f in (1536, 1538):
            torch.manual_seed(11)  # same full layer on every rank
            base = torch.nn.Linear(1024, out_f, bias=True, device=dev, dtype=torch.bfloat16)
            ref = DoraLinear(base, r=64, scaling=0.5, init_lora_B_zero=False)
            sh = RowShardedDoraLinear.from_full(base.weight.detach(), base.bias.detach(),
                                                ref.lora_A.weight.detach(), ref.lora_B.weight.detach(),
                                                ref.lora_magnitude_vector.weight.detach(), 0.5)
            assert sh.fused_path(torch.empty(1, device=dev))
            a, b = shard_range(out_f, world, rank)
            for it in range(2):
                x = torch.randn(256, 1024, device=dev, dtype=torch.bfloat16)
                dy = torch.randn(256, out_f, device=dev, dtype=torch.bfloat16)
                for p in (ref.lora_A.weight, ref.lora_B.weight, ref.lora_magnitude_vector.weight, sh.lora_A,
                          sh.lora_B, sh.magnitude):
                    p.grad = None
                x1, x2 = x.clone().requires_grad_(True), x.clone().requires_grad_(True)
                y1 = ref(x1)
                y1.backward(dy)
                y2 = sh(x2)
                y2.backward(dy)
                tag = f"out{out_f}/step{it}"
                errs.update({f"{tag} y": _rel(y2, y1), f"{tag} dx": _rel(x2.grad, x1.grad),
                             f"{tag} dA": _rel(sh.lora_A.grad, ref.lora_A.weight.grad),
                             f"{tag} dB": _rel(sh.lora_B.grad, ref.lora_B.weight.grad[a:b]),
                             f"{tag} dm": _rel(sh.magnitude.grad, ref.lora_magnitude_vector.weight.grad[a:b])})
                del y2
            sh.pool.close()
        # Token data parallelism with the asynchronous reducer.
        torch.manual_seed(5)
        base = torch.nn.Linear(512, 768, bias=False, device=dev, dtype=torch.float32)
        mod = DoraLinear(base, r=16, scaling=2.0, init_lora_B_zero=False)
        params = [mod.lora_A.weight, mod.lora_B.weight, mod.lora_magnitude_vector.weight]
        xs = [torch.randn(64, 512, device=dev, generator=torch.Generator(device=dev).manual_seed(100 + k))
              for k in range(world)]
        red = GradAllReducer(params)
        mod(xs[rank]).square().sum().backward()
        red.wait()
        got = [p.grad.clone() for p in params]
        red.remove()
        for p in params:
            p.grad = None
        mod(torch.cat(xs)).square().sum().backward()
        for name, g1, p in zip(("dA", "dB", "dm"), got, params):
            errs[f"dp {name}"] = _rel(g1, p.grad)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, errs))
    except BaseException as e:
        q.put((rank, repr(e)))
        raise


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_row_sharded_and_data_parallel_two_gpus():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    for rank, errs in res.items():
        assert not isinstance(errs, str), f"rank {rank}: {errs}"
        for k, e in errs.items():
            tol = 1e-5 if k.startswith("dp") else 1e-2
            assert e <= tol, f"rank {rank} {k}: rel-L2 {e:.3e}"
