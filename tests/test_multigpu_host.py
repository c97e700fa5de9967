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
        # sharded evaluation: 5 queries over 2 ranks, per-query results gathered in rank order
        lo, hi = MG.shard_bounds(5, rank, world)
        ranks_all = MG.gather_varlen(torch.arange(lo, hi, dtype=torch.float32) * 10)
        out.put((rank, hidden.tolist(), grad.tolist(), ms, work, (lo, hi), ranks_all.tolist()))
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
    for rank, hidden, grad, ms, work, bounds, ranks_all in res:
        assert hidden == [0, 1, 2, 3, 100, 101, 102, 103]  # every replica hides the union
        assert grad == [[1.5, 1.5]] * 3                       # mean of the ranks' gradients
        assert ms == 11.0 and work == 21.0                    # max time, summed work
        assert bounds == ((0, 3) if rank == 0 else (3, 5))    # contiguous shards
        assert ranks_all == [0.0, 10.0, 20.0, 30.0, 40.0]     # unsharded order


def _parts_worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from flashlog_b200 import multigpu as MG
        T = 3
        grad_hop = torch.zeros(T, 4, 2)           # [T, rows, cols], as DrumTrainStep.grad_hop
        table = torch.ones(4, T, 2)                # [rows, T, cols]
        order = []

        def part(hop):
            def run():
                order.append(hop)
                if hop >= 0:  # the part completes hop `hop`'s gradient
                    grad_hop[hop].fill_(float((rank + 1) * (hop + 1)))
            return run
        parts = [part(2), part(1), part(0), part(-1)]  # forward + last hop, hops T-2..0, the update part
        MG.run_parts_with_overlapped_allreduce(parts, grad_hop, grad_hop.permute(1, 0, 2), table, lr=0.5)
        out.put((rank, order, table.tolist(), grad_hop.tolist()))
    finally:
        dist.destroy_process_group()


def _parts_rows_worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from flashlog_b200 import multigpu as MG
        T = 3
        rels = torch.tensor([0, 2, 2] if rank == 0 else [3, 2])  # the batch's query relations
        rows = MG.union_rows(rels, 4)
        grad_hop = torch.zeros(T, 4, 2)
        table = torch.ones(4, T, 2)

        def part(hop):
            def run():
                if hop >= 0:  # only the batch's rows are written, as DrumTrainStep does
                    grad_hop[hop].zero_()
                    grad_hop[hop][rels.unique()] = float((rank + 1) * (hop + 1))
            return run
        parts = [part(2), part(1), part(0), part(-1)]
        MG.run_parts_with_overlapped_allreduce(parts, grad_hop, grad_hop.permute(1, 0, 2), table, lr=0.5,
                                               rows=rows)
        out.put((rank, rows.tolist(), table.tolist(), grad_hop.tolist()))
    finally:
        dist.destroy_process_group()


def test_compact_allreduce_of_the_union_rows_on_two_gloo_ranks():
    """Rank 0's batch writes rows {0, 2}, rank 1's rows {2, 3}: the union
    [0, 2, 3] is all-reduced and updated; row 1 stays untouched, and every
    row gets what the dense all-reduce would give."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_parts_rows_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    per_row = {0: 1.0, 1: 0.0, 2: 3.0, 3: 2.0}  # sum over ranks of (rank + 1) for the rows each rank writes
    for rank, rows, table, grad in res:
        assert rows == [0, 2, 3]
        for hop in range(3):
            for row in range(4):
                assert grad[hop][row] == [per_row[row] * (hop + 1)] * 2
                assert table[row][hop] == [1.0 - 0.25 * per_row[row] * (hop + 1)] * 2


def test_overlapped_allreduce_parts_on_two_gloo_ranks():
    """Each hop's gradient is summed over the ranks once its part has run, and
    the update applies lr / world times the sums: here table = 1 - 0.25 *
    (1 + 2) * (hop + 1) on both ranks."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_parts_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, order, table, grad in res:
        assert order == [2, 1, 0, -1]
        for hop in range(3):
            assert grad[hop] == [[3.0 * (hop + 1)] * 2] * 4
            for row in range(4):
                assert table[row][hop] == [1.0 - 0.25 * 3.0 * (hop + 1)] * 2


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
        assert MG.union_rows(torch.tensor([3, 1, 3]), 5).tolist() == [1, 3]
    finally:
        dist.destroy_process_group()


def test_shard_bounds_cover_every_query_once():
    from flashlog_b200 import multigpu as MG
    for n in (0, 1, 7, 64, 1001):
        for world in (1, 2, 3, 8):
            spans = [MG.shard_bounds(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        MG.shard_bounds(4, 2, 2)


def _rank_worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import numpy as np
        from flashlog_b200 import multigpu as MG
        from oracle import oracle as O
        rng = np.random.default_rng(5)
        B, E = 9, 40
        keys = np.unique(rng.integers(0, B * E, 150))
        vals = (rng.integers(0, 6, keys.size) / 5.0).astype(np.float32)
        targets = rng.integers(0, E, B)
        filt = np.unique(rng.integers(0, B * E, 60))

        def oracle_ranks(ib, ie, v, t, fk, b, e, eql):
            return torch.from_numpy(O.filtered_ranks(ib.numpy(), ie.numpy(), v.numpy(), t.numpy(), fk.numpy(), b, e,
                                                     eql))
        got = MG.sharded_filtered_ranks(torch.from_numpy(keys // E), torch.from_numpy(keys % E),
                                        torch.from_numpy(vals), torch.from_numpy(targets), torch.from_numpy(filt),
                                        B, E, True, rank_fn=oracle_ranks)
        want = O.filtered_ranks(keys // E, keys % E, vals, targets, filt, B, E, True)
        out.put((rank, got.tolist(), want.tolist()))
    finally:
        dist.destroy_process_group()


def test_sharded_filtered_ranks_on_two_gloo_ranks():
    """Each rank ranks its query shard; the gathered ranks equal the unsharded ones."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, got, want in res:
        assert got == want
