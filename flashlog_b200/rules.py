"""Max-product rule-bank evaluation (smDRUM / mmDRUM rule inference).

Restates rules/max_inference.py:4-8 -> rules/shared_inference.py:12-245 with
reduction 'max' (Boolean paths):

  for every query q and rule k (body: directed relations, 2R = identity), the
  rule's state starts at the query's source entity and advances one body
  operator at a time (flashlog.cu:1561-1741, the fixed-relation step), made
  Boolean after every step (shared_inference.py:123-126);
  score_r[q, e] = max over the rules reaching e of rank_weight[k, r]
  (the dense accumulator of shared_inference.py:200-206);
  each rank row is divided by its sum (normalize_sparse_rows,
  rules/evaluate.py:366-378, clamped at 1e-30), and the ranks are combined by
  sum (smDRUM) or by max (mmDRUM, final_max).

The grounding runs in the library's fixed-relation kernels and the reduction
in fl_rule_max_reduce (an exact, order-independent atomic max of the weights'
fp32 bit patterns).  Rules are processed in chunks of chunk_size; queries in
batches whose [ranks, batch, E] accumulator fits `accumulator_bytes`.
"""
from __future__ import annotations

import torch

from . import ops
from .ops import Graph, _p, _stream, check, lib


def _graph(csr_struct):
    c = tuple(csr_struct)
    dev = c[1].device
    z = torch.empty(0, dtype=torch.int32, device=dev)
    return Graph.of((c[8], c[1], z.to(torch.int16), z, c[12], c[5], z.to(torch.int16), z,
                     c[8], c[9], c[10], c[11], c[12], c[13], c[14], c[15]))


def _empty(B, E, device):
    return torch.sparse_coo_tensor(torch.empty((2, 0), dtype=torch.long, device=device),
                                   torch.empty(0, device=device), (B, E), is_coalesced=True)


def _ground(sources, ops_chunk, graph, relations, E):
    """Boolean end states of C rules for every query: rows q * C + c."""
    B = sources.numel()
    C, steps = ops_chunk.shape
    dev = sources.device
    b = torch.arange(B, device=dev).repeat_interleave(C)
    l = torch.arange(C, device=dev).repeat(B)
    e = sources.to(torch.int64).repeat_interleave(C)
    v = torch.ones(B * C, dtype=torch.float32, device=dev)
    for step in range(steps):
        if v.numel() == 0:
            break
        step_ops = ops_chunk[:, step].unsqueeze(0).expand(B, C).contiguous()
        row_ptr, ent, val = ops.fixed_relation(b, l, e, v, step_ops, graph, relations, B, C)
        v = (val > 0).to(torch.float32)  # several paths are one Boolean proof
        idx = ops.rows_to_coo(row_ptr, ent, C)
        b, l, e = idx[0], idx[1], idx[2]
    row_ptr, ent, _ = ops.coo_to_rows(b, l, e, B, C, E)
    return row_ptr, ent, v


def max_product_scores(sources, rules, csr_struct, relations: int, entities: int, chunk_size: int = 16,
                       final_max: bool = False, accumulator_bytes: int = 4 << 30):
    """Rule-bank scores [len(sources), entities] (sparse COO, coalesced).

    rules: sequence of {'body': tuple of operators, 'rank_weights': list}
    (rules/evaluate.py:94-119), all with the same number of ranks.
    """
    if chunk_size < 1:
        raise ValueError("chunk_size must be positive")
    ops._require_cuda(sources)
    dev = sources.device
    B, E = sources.numel(), int(entities)
    if not rules:
        return _empty(B, E, dev)
    widths = {len(r["rank_weights"]) for r in rules}
    if len(widths) != 1 or next(iter(widths)) < 1:
        raise ValueError("nonempty rank_weights must have matching widths")
    ranks = next(iter(widths))
    weights = torch.tensor([list(r["rank_weights"]) for r in rules], dtype=torch.float32, device=dev)
    if not bool(torch.isfinite(weights).all()) or bool((weights < 0).any()):
        raise ValueError("MAX rule weights must be finite and nonnegative")
    identity = 2 * relations
    for r in rules:
        if any(not (0 <= int(o) <= identity) for o in r["body"]):
            raise ValueError("rule operators must lie in [0, 2R]")
    graph = _graph(csr_struct)
    qb = max(1, min(B, accumulator_bytes // max(1, ranks * E * 4)))
    keys_out, vals_out = [], []
    for q0 in range(0, B, qb):
        src = sources[q0:q0 + qb]
        Bq = src.numel()
        acc = torch.zeros(ranks * Bq * E, dtype=torch.int32, device=dev)
        for off in range(0, len(rules), chunk_size):
            chunk = rules[off:off + chunk_size]
            C = len(chunk)
            steps = max(len(r["body"]) for r in chunk)
            if steps == 0:
                ops_chunk = torch.full((C, 1), identity, dtype=torch.int64, device=dev)
            else:
                ops_chunk = torch.tensor([tuple(int(o) for o in r["body"]) + (identity,) * (steps - len(r["body"]))
                                          for r in chunk], dtype=torch.int64, device=dev)
            row_ptr, ent, val = _ground(src, ops_chunk, graph, relations, E)
            w = weights[off:off + C].contiguous()
            check(lib().fl_rule_max_reduce(_p(row_ptr), Bq * C, _p(ent), _p(val), C, _p(w), ranks, Bq, E, _p(acc),
                                           _stream()), "rule_max_reduce")
        scores = acc.view(torch.float32).view(ranks, Bq, E)
        totals = scores.sum(-1, keepdim=True)
        norm = scores / totals.clamp_min(1e-30)
        combined = (norm.amax(0) if final_max else norm.sum(0)).reshape(-1)
        keys = combined.nonzero().flatten()
        keys_out.append(keys + q0 * E)
        vals_out.append(combined[keys])
    keys = torch.cat(keys_out)
    return torch.sparse_coo_tensor(torch.stack((keys // E, keys % E)), torch.cat(vals_out), (B, E),
                                   is_coalesced=True)


def score(ev, sources, rules, csr, relations, entities, chunk_size, final_max=False, dense_budget_bytes=None,
          prefix_budget_bytes=128 * 1024 ** 2, stats=None):
    """Drop-in for rules/max_inference.py:4-8 (the evaluator module `ev` and
    the prefix-cache budget are not needed; dense_budget_bytes bounds the
    [ranks, queries, E] accumulator)."""
    if stats is not None:
        stats.setdefault("rules_before", len(rules))
    return max_product_scores(sources, rules, csr, relations, entities, chunk_size=chunk_size, final_max=final_max,
                              accumulator_bytes=dense_budget_bytes or (4 << 30))
