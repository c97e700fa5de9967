"""Query-sharded multi-GPU training step: the host-side collectives.

Queries are independent (c1 is per (query, channel), c2 per (entry,
direction)), so every rank keeps a full CSR replica and propagates its own
queries with no exchange inside a hop.  Per step:

  * the batch triple ids of all ranks are gathered, so every replica hides
    the union, as one global batch would (src/main.py:888);
  * the attention gradients are averaged with one all-reduce;
  * timing is the maximum over ranks, work counts the sum.

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
