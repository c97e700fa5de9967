"""Query-sharded multi-GPU training step: the host-side collectives.

Queries are independent (c1 is per (query, channel), c2 per (entry,
direction)), so every rank keeps a full CSR replica and propagates its own
queries with no exchange inside a hop.  Per step:

  * the batch triple ids of all ranks are gathered, so every replica hides
    the union, as one global batch would (src/main.py:888);
  * the attention gradients are averaged with one all-reduce;
  * timing is the maximum over ranks, work counts the sum.

Evaluation (filtered ranks, rule-bank scores) shards the queries the same
way: shard_bounds gives each rank a contiguous query range and
gather_varlen concatenates the per-rank results in rank order, so the
gathered ranks equal an unsharded run (a query's rank does not depend on the
others).

Each function takes the process group (default: the global group); NCCL on
GPUs, gloo on CPU for tests.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def gather_hidden_triples(ids: torch.Tensor, group=None) -> torch.Tensor:
    """Triple ids of every rank's batch, concatenated in rank order."""
    world = dist.get_world_size(group)
    if world == 1:
        return ids
    gathered = [torch.empty_like(ids) for _ in range(world)]
    dist.all_gather(gathered, ids.contiguous(), group=group)
    return torch.cat(gathered)


def allreduce_mean_(grad: torch.Tensor, group=None) -> torch.Tensor:
    """grad <- mean over ranks, in place."""
    world = dist.get_world_size(group)
    if world > 1:
        dist.all_reduce(grad, group=group)
        grad.div_(world)
    return grad


def union_rows(rels: torch.Tensor, n_rows: int, group=None) -> torch.Tensor:
    """The table rows any rank's step can write: the sorted distinct values of
    every rank's `rels` (the batch's query relations; the ranks' batches may
    differ in size), from an all-reduced row mask.  The step's gradient is
    zero outside them on every rank (DrumTrainStep zeroes grad_hop and adds
    only the batch's rows).  One host read (the count)."""
    mask = torch.zeros(n_rows, dtype=torch.int32, device=rels.device)
    mask[rels.to(torch.int64)] = 1
    if dist.get_world_size(group) > 1:
        dist.all_reduce(mask, group=group)
    return torch.nonzero(mask).flatten()


def run_parts_with_overlapped_allreduce(parts, grad_hop, table_grad, table, lr: float, comm_stream=None,
                                        group=None, rows=None):
    """One training step given as parts (DrumTrainStep.parts(), or replays of
    their CUDA graphs): after part j < T has been issued, hop T-1-j's table
    gradient grad_hop[T-1-j] is complete and its all-reduce (sum) is issued
    on comm_stream (a CUDA stream; None: in order, e.g. gloo on CPU), so it
    overlaps the parts that follow.  Then the update waits for all of them:
    table -= lr / world * table_grad (a view of the summed hop gradients).
    rows (union_rows of the step): only those rows of each hop's gradient are
    all-reduced, gathered into a compact buffer and written back, and only
    those rows of the table are updated; the other rows are zero on every
    rank, so the result is the same."""
    world = dist.get_world_size(group)
    T = len(grad_hop)

    def reduce(hop):
        if rows is None:
            dist.all_reduce(grad_hop[hop], group=group)
            return
        buf = grad_hop[hop].index_select(0, rows)
        dist.all_reduce(buf, group=group)
        grad_hop[hop].index_copy_(0, rows, buf)

    for j, part in enumerate(parts):
        part()
        if world > 1 and j < T:
            hop = T - 1 - j
            if comm_stream is not None:
                comm_stream.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(comm_stream):
                    reduce(hop)
            else:
                reduce(hop)
    if world > 1:
        if comm_stream is not None:
            torch.cuda.current_stream().wait_stream(comm_stream)
        if rows is None:
            table.sub_(table_grad, alpha=lr / world)
        else:
            table.index_add_(0, rows, table_grad.index_select(0, rows), alpha=-lr / world)


def max_time_sum_work(ms: float, work: float, device, group=None):
    """(max over ranks of ms, sum over ranks of work)."""
    if dist.get_world_size(group) == 1:
        return ms, work
    t = torch.tensor([ms, float(work)], dtype=torch.float64, device=device)
    mx = t.clone()
    dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
    sm = t.clone()
    dist.all_reduce(sm, op=dist.ReduceOp.SUM, group=group)
    return float(mx[0].item()), float(sm[1].item())


def shard_bounds(n: int, rank: int, world: int):
    """[lo, hi) of this rank's share of n queries: contiguous, sizes differ by at most one."""
    if world < 1 or not (0 <= rank < world) or n < 0:
        raise ValueError("bad shard arguments")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def gather_varlen(t: torch.Tensor, group=None) -> torch.Tensor:
    """Concatenation in rank order of every rank's 1-D tensor t (lengths may differ)."""
    world = dist.get_world_size(group)
    if world == 1:
        return t
    t = t.contiguous().reshape(-1)
    n = torch.tensor([t.numel()], dtype=torch.int64, device=t.device)
    sizes = [torch.empty_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    sizes = [int(x.item()) for x in sizes]
    cap = max(sizes)
    padded = torch.zeros(cap, dtype=t.dtype, device=t.device)
    padded[:t.numel()] = t
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    return torch.cat([p[:k] for p, k in zip(parts, sizes)])


def sharded_filtered_ranks(idx_b, idx_e, values, targets, filter_keys, B: int, E: int, use_eql: bool = False,
                           group=None, rank_fn=None):
    """Filtered ranks of B queries with each rank scoring its query shard
    (sparse2d_filtered_ranks_cuda on the shard's slice of the scores and of
    the sorted filter keys), gathered in query order.  The scores are a
    coalesced [B, E] COO (idx_b sorted); rank_fn defaults to the library's
    kernel."""
    if rank_fn is None:
        from .flashlog_kernel import sparse2d_filtered_ranks_cuda as rank_fn
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    lo, hi = shard_bounds(int(B), rank, world)
    dev = idx_b.device
    a, b = (int(x) for x in torch.searchsorted(idx_b, torch.tensor([lo, hi], dtype=idx_b.dtype, device=dev)))
    keys = torch.tensor([lo * int(E), hi * int(E)], dtype=filter_keys.dtype, device=filter_keys.device)
    ka, kb = (int(x) for x in torch.searchsorted(filter_keys, keys))
    local = rank_fn(idx_b[a:b] - lo, idx_e[a:b], values[a:b], targets[lo:hi], filter_keys[ka:kb] - lo * int(E),
                    hi - lo, int(E), use_eql)
    local = torch.as_tensor(local, device=values.device, dtype=torch.float32)
    return gather_varlen(local, group) if world > 1 else local
