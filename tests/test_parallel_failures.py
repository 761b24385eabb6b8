"""Collective failures on the host: a rank that leaves between steps, and a rank
that never joins a collective, end the other ranks' next collective with a
Python exception within the process group's timeout instead of hanging.

Run as two gloo ranks on CPU (spawned processes).  The row-sharded layer's
generic path all-gathers its output shards in forward and all-reduces dX / dA
in backward; the token-data-parallel reducer all-reduces gradients
asynchronously and joins them in ``wait()``.  The reference's own loud
failures of the distributed paths are Python exceptions too (dora.py:517-524,
842-858).  Nothing here touches a GPU.
"""

import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

TIMEOUT_S = 4


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _eager(x, W, bias, A, B, m, s):
    with torch.no_grad():
        norm = (W + s * (B @ A)).norm(dim=1)
    g = (m / norm).view(1, -1)
    result = F.linear(x, W, bias)
    lora = F.linear(F.linear(x, A), B)
    return result + ((g - 1) * result + g * (s * lora))


def _layer():
    from dorafactors_b200 import parallel

    class EagerShard(parallel.RowShardedDoraLinear):
        def local_output(self, x, A):
            return _eager(x, self.weight, self.bias, A, self.lora_B, self.magnitude, self.scaling)

    g = torch.Generator().manual_seed(0)
    W = torch.randn(8, 6, generator=g, dtype=torch.float64)
    A = torch.randn(2, 6, generator=g, dtype=torch.float64)
    B = torch.randn(8, 2, generator=g, dtype=torch.float64)
    m = torch.rand(8, generator=g, dtype=torch.float64) + 0.5
    return EagerShard.from_full(W, None, A, B, m, 0.5)


def _step(layer):
    x = torch.randn(4, 6, dtype=torch.float64, requires_grad=True)
    layer(x).sum().backward()


def _report(q, item):
    """Put and flush: the queue's feeder thread must finish before os._exit."""
    q.put(item)
    q.close()
    q.join_thread()


def _worker(rank, world, port, scenario, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=TIMEOUT_S))
    try:
        if scenario in ("rowshard_exit", "rowshard_absent"):
            layer = _layer()
            _step(layer)  # a healthy step on every rank
            dist.barrier()
            if rank == 1:
                if scenario == "rowshard_exit":
                    _report(q, (rank, "left"))
                    os._exit(0)  # leaves between steps, no goodbye
                time.sleep(3 * TIMEOUT_S)  # alive, but never joins the next collective
                _report(q, (rank, "slept"))
                os._exit(0)
            t0 = time.monotonic()
            try:
                _step(layer)
                _report(q, (rank, "no error"))
            except Exception as e:  # noqa: BLE001 - the type is what the test reports
                _report(q, (rank, (type(e).__name__, time.monotonic() - t0)))
        elif scenario == "dp_exit":
            from dorafactors_b200.parallel import GradAllReducer

            w = torch.randn(16, dtype=torch.float64, requires_grad=True)
            red = GradAllReducer([w])
            (w * w).sum().backward()
            red.wait()
            dist.barrier()
            if rank == 1:
                _report(q, (rank, "left"))
                os._exit(0)
            t0 = time.monotonic()
            w.grad = None
            try:
                (w * w).sum().backward()
                red.wait()
                _report(q, (rank, "no error"))
            except Exception as e:  # noqa: BLE001
                _report(q, (rank, (type(e).__name__, time.monotonic() - t0)))
    finally:
        if rank == 0:
            os._exit(0)  # the group is broken: skip the collective teardown


@pytest.mark.parametrize("scenario", ["rowshard_exit", "rowshard_absent", "dp_exit"])
def test_collective_failure_raises(scenario):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, scenario, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    outcome = got[0]
    assert outcome != "no error", f"{scenario}: the surviving rank's collective did not fail"
    name, waited = outcome
    assert waited < 10 * TIMEOUT_S, f"{scenario}: failure took {waited:.1f} s"
    assert name in ("RuntimeError", "DistBackendError", "DistNetworkError", "DistError"), name
