"""Host-side collectives of the query-sharded step, on 2 gloo ranks (CPU).

The GPU path uses the same functions over NCCL (bench.py under torchrun)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from flashlog_b200 import multigpu as MG
        ids = torch.arange(4, dtype=torch.int64) + 100 * rank
        hidden = MG.gather_hidden_triples(ids)
        grad = torch.full((3, 2), float(rank + 1))
        MG.allreduce_mean_(grad)
        ms, work = MG.max_time_sum_work(10.0 + rank, 7 * (rank + 1), torch.device("cpu"))
        out.put((rank, hidden.tolist(), grad.tolist(), ms, work))
    finally:
        dist.destroy_process_group()


def test_collectives_on_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, hidden, grad, ms, work in res:
        assert hidden == [0, 1, 2, 3, 100, 101, 102, 103]  # every replica hides the union
        assert grad == [[1.5, 1.5]] * 3                       # mean of the ranks' gradients
        assert ms == 11.0 and work == 21.0                    # max time, summed work


def test_single_process_is_identity():
    from flashlog_b200 import multigpu as MG
    if dist.is_initialized():
        pytest.skip("a process group is already set up")
    port = _free_port()
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        ids = torch.arange(5)
        assert MG.gather_hidden_triples(ids) is ids
        g = torch.ones(2)
        assert MG.allreduce_mean_(g) is g and g.tolist() == [1.0, 1.0]
        assert MG.max_time_sum_work(3.0, 4, torch.device("cpu")) == (3.0, 4)
    finally:
        dist.destroy_process_group()
