"""Row-sharded DoRA linear on two GPUs (NCCL): each rank owns half the out-features,
runs the native norm and fused compose on its shard and all-gathers the output.
The gathered output and every gradient must match the single-GPU DoraLinear
within the bf16 parity bar.  Skipped when fewer than two GPUs are visible."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import datetime

    import numpy as np
    import torch.distributed as dist

    from dorafactors_b200.layer import DoraLinear
    from dorafactors_b200.parallel import RowShardedDoraLinear, shard_range

    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        torch.manual_seed(11)  # same full layer on every rank
        base = torch.nn.Linear(1024, 1536, bias=True, device=dev, dtype=torch.bfloat16)
        ref = DoraLinear(base, r=64, scaling=0.5, init_lora_B_zero=False)
        x = torch.randn(256, 1024, device=dev, dtype=torch.bfloat16)
        dy = torch.randn(256, 1536, device=dev, dtype=torch.bfloat16)
        sh = RowShardedDoraLinear.from_full(base.weight.detach(), base.bias.detach(), ref.lora_A.weight.detach(),
                                            ref.lora_B.weight.detach(), ref.lora_magnitude_vector.weight.detach(),
                                            0.5)
        x1, x2 = x.clone().requires_grad_(True), x.clone().requires_grad_(True)
        y1 = ref(x1)
        y1.backward(dy)
        y2 = sh(x2)
        y2.backward(dy)
        a, b = shard_range(1536, world, rank)

        def rel(u, v):
            u, v = u.double(), v.double()
            return float((u - v).norm() / v.norm().clamp_min(1e-30))

        errs = {"y": rel(y2, y1), "dx": rel(x2.grad, x1.grad), "dA": rel(sh.lora_A.grad, ref.lora_A.weight.grad),
                "dB": rel(sh.lora_B.grad, ref.lora_B.weight.grad[a:b]),
                "dm": rel(sh.magnitude.grad, ref.lora_magnitude_vector.weight.grad[a:b])}
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, errs))
    except BaseException as e:
        q.put((rank, repr(e)))
        raise


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_row_sharded_two_gpus_matches_single_gpu():
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
            assert e <= 1e-2, f"rank {rank} {k}: rel-L2 {e:.3e}"
