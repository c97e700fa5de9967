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


def available_first_operators(sources, csr_struct, relations: int):
    """Operators with at least one edge at some source (rules/shared_inference.py:34-47):
    r for a forward group of relation r, r + R for an inverse group, and the
    identity 2R.  Returns a bool tensor [2R + 1] on the sources' device."""
    c = tuple(csr_struct)
    s = sources.to(torch.int64)
    avail = torch.zeros(2 * relations + 1, dtype=torch.bool, device=s.device)
    for gptr, grel, off in ((c[8], c[9], 0), (c[12], c[13], relations)):
        a, b = gptr[s].to(torch.int64), gptr[s + 1].to(torch.int64)
        n = b - a
        total = int(n.sum().item())
        if total:
            start = torch.repeat_interleave(a - torch.cumsum(n, 0) + n, n, output_size=total)
            idx = start + torch.arange(total, device=s.device)
            avail[grel[idx].to(torch.int64) + off] = True
    avail[2 * relations] = True
    return avail


def _weights_and_ops(rules, relations, dev):
    ranks = len(rules[0]["rank_weights"])
    weights = torch.tensor([list(r["rank_weights"]) for r in rules], dtype=torch.float32, device=dev)
    identity = 2 * relations
    steps = max(1, max(len(r["body"]) for r in rules))
    ops_all = torch.tensor([tuple(int(o) for o in r["body"]) + (identity,) * (steps - len(r["body"])) for r in rules],
                           dtype=torch.int64, device=dev)
    return ranks, weights, ops_all


def _sparse_scores(src, ops_all, weights, ranks, graph, relations, E, chunk_size, final_max):
    """Rank rows of maxima accumulated chunk by chunk, normalized per (query,
    rank) row (clamped at 1e-30, rules/evaluate.py:366-378) and combined by
    sum (in rank order) or max; returns the row layout over the queries."""
    Bq = src.numel()
    running = None
    for off in range(0, ops_all.shape[0], chunk_size):
        ops_chunk = ops_all[off:off + chunk_size]
        C = ops_chunk.shape[0]
        row_ptr, ent, val = _ground(src, ops_chunk, graph, relations, E)
        running = ops.rule_rank_maxima(row_ptr, ent, val, Bq, C, weights[off:off + C], ranks, E, running)
    rp, ent, x = running
    y, _ = ops.normalize_forward(rp, x, eps=1e-30)
    if final_max:
        return ops.row_max(rp[::ranks].contiguous(), ent, y, Bq, E)
    out_rp, out_ent, out_x, _ = ops.channel_merge(rp, ent, y, Bq, ranks, E)
    return out_rp, out_ent, out_x


def max_product_scores(sources, rules, csr_struct, relations: int, entities: int, chunk_size: int = 16,
                       final_max: bool = False, accumulator_bytes: int = 4 << 30, query_batch: int = 256,
                       stats=None):
    """Rule-bank scores [len(sources), entities] (sparse COO, coalesced).

    rules: sequence of {'body': tuple of operators, 'rank_weights': list}
    (rules/evaluate.py:94-119), all with the same number of ranks.  Rules whose
    first operator has no edge at any source are dropped first
    (rules/shared_inference.py:34-47).  When the [ranks, queries, E]
    accumulator of a query batch fits accumulator_bytes, the maxima go
    through the dense exact atomic max (fl_rule_max_reduce); otherwise (86M
    entities) through sparse rank rows reduced by the MAX row reduction, in
    batches of query_batch queries, with no dense buffer.
    """
    if chunk_size < 1:
        raise ValueError("chunk_size must be positive")
    ops._require_cuda(sources)
    dev = sources.device
    B, E = sources.numel(), int(entities)
    stats = {} if stats is None else stats
    stats["rules_before"] = len(rules)
    if not rules:
        return _empty(B, E, dev)
    widths = {len(r["rank_weights"]) for r in rules}
    if len(widths) != 1 or next(iter(widths)) < 1:
        raise ValueError("nonempty rank_weights must have matching widths")
    identity = 2 * relations
    for r in rules:
        if any(not (0 <= int(o) <= identity) for o in r["body"]):
            raise ValueError("rule operators must lie in [0, 2R]")
    w_all = torch.tensor([list(r["rank_weights"]) for r in rules], dtype=torch.float32)
    if not bool(torch.isfinite(w_all).all()) or bool((w_all < 0).any()):
        raise ValueError("MAX rule weights must be finite and nonnegative")
    if B:
        avail = available_first_operators(sources, csr_struct, relations).cpu().tolist()
        rules = [r for r in rules if not r["body"] or avail[int(r["body"][0])]]
    stats["rules_after"] = len(rules)
    if not rules:
        return _empty(B, E, dev)
    ranks, weights, ops_all = _weights_and_ops(rules, relations, dev)
    graph = _graph(csr_struct)
    dense_qb = accumulator_bytes // max(1, ranks * E * 4)
    stats["dense_accumulation"] = dense_qb >= min(B, 1)
    qb = max(1, min(B, dense_qb)) if dense_qb >= 1 else max(1, min(B, query_batch))
    keys_out, vals_out = [], []
    for q0 in range(0, B, qb):
        src = sources[q0:q0 + qb]
        Bq = src.numel()
        if dense_qb >= 1:
            acc = torch.zeros(ranks * Bq * E, dtype=torch.int32, device=dev)
            for off in range(0, len(rules), chunk_size):
                ops_chunk = ops_all[off:off + chunk_size]
                C = ops_chunk.shape[0]
                row_ptr, ent, val = _ground(src, ops_chunk, graph, relations, E)
                w = weights[off:off + C].contiguous()
                check(lib().fl_rule_max_reduce(_p(row_ptr), Bq * C, _p(ent), _p(val), C, _p(w), ranks, Bq, E,
                                               _p(acc), _stream()), "rule_max_reduce")
            scores = acc.view(torch.float32).view(ranks, Bq, E)
            totals = scores.sum(-1, keepdim=True)
            norm = scores / totals.clamp_min(1e-30)
            combined = (norm.amax(0) if final_max else norm.sum(0)).reshape(-1)
            keys = combined.nonzero().flatten()
            keys_out.append(keys + q0 * E)
            vals_out.append(combined[keys])
        else:
            rp, ent, x = _sparse_scores(src, ops_all, weights, ranks, graph, relations, E, chunk_size, final_max)
            counts = rp[1:] - rp[:-1]
            q = torch.repeat_interleave(torch.arange(Bq, device=dev), counts, output_size=ent.numel())
            keys_out.append((q + q0) * E + ent.to(torch.int64))
            vals_out.append(x)
    keys = torch.cat(keys_out)
    return torch.sparse_coo_tensor(torch.stack((keys // E, keys % E)), torch.cat(vals_out), (B, E),
                                   is_coalesced=True)


def compact_routed_rules(rules):
    """Rules with the same (head, body) share one grounding; their group
    weights become one rank_weights vector (rules/evaluate.py:94-119)."""
    if any(r.get("group_id") is None for r in rules):
        raise ValueError("routed_normalized requires a group_id column")
    groups = max(r["group_id"] for r in rules) + 1
    compact = {}
    for r in rules:
        key = (r["head"], tuple(r["body"]))
        if key not in compact:
            compact[key] = {**r, "weight": 1.0, "rank_weights": [0.0] * groups, "group_id": None}
        rw = compact[key]["rank_weights"]
        if rw[r["group_id"]] != 0:
            raise ValueError("duplicate Horn rule/group instance")
        rw[r["group_id"]] = r["weight"]
    return [{**r, "rank_weights": tuple(r["rank_weights"])} for r in compact.values()]


def evaluate_rule_bank(sources, query_relations, targets, rules, csr_struct, relations: int, entities: int,
                       final_max: bool = False, chunk_size: int = 16, query_batch: int = 64,
                       accumulator_bytes: int = 4 << 30, filter_keys=None, stats=None):
    """Filtered, tie-averaged ranks of the targets under the rule bank's
    max-product scores (rules/evaluate.py:1015-1095 with --aggregations
    routed_normalized and reduction 'max': smDRUM sums the normalized ranks,
    mmDRUM takes their max).  Queries are routed by relation to the rules
    whose head is that relation (compacted per (head, body)), scored in
    batches of query_batch, and ranked with fl_filtered_ranks against
    filter_keys (sorted keys q * E + e of known answers; the targets are
    added).  Returns float32 ranks in query order."""
    dev = sources.device
    E = int(entities)
    Q = sources.numel()
    compact = compact_routed_rules(rules) if rules else []
    by_head = {}
    for r in compact:
        by_head.setdefault(int(r["head"]), []).append(r)
    rel_h = query_relations.cpu().numpy()
    ranks_out = torch.empty(Q, dtype=torch.float32, device=dev)
    import numpy as np
    order = np.argsort(rel_h, kind="stable")
    bounds = np.flatnonzero(np.diff(rel_h[order])) + 1
    for group in np.split(order, bounds):
        if group.size == 0:
            continue
        rel = int(rel_h[group[0]])
        head_rules = by_head.get(rel, [])
        for g0 in range(0, group.size, query_batch):
            idx = torch.from_numpy(group[g0:g0 + query_batch]).to(dev)
            src, tgt = sources[idx], targets[idx]
            Bq = idx.numel()
            if head_rules:
                sc = max_product_scores(src, head_rules, csr_struct, relations, E, chunk_size=chunk_size,
                                        final_max=final_max, accumulator_bytes=accumulator_bytes,
                                        query_batch=query_batch, stats=stats)
                si, sv = sc.indices(), sc.values()
            else:
                si = torch.empty((2, 0), dtype=torch.int64, device=dev)
                sv = torch.empty(0, dtype=torch.float32, device=dev)
            fk = torch.arange(Bq, device=dev) * E + tgt
            if filter_keys is not None:
                fk = torch.cat([fk, filter_keys(idx) if callable(filter_keys) else filter_keys[idx]])
            fk = torch.unique(fk)
            ranks_out[idx] = ops.filtered_ranks(si[0], si[1], sv, tgt, fk, Bq, E, True)
    return ranks_out


def score(ev, sources, rules, csr, relations, entities, chunk_size, final_max=False, dense_budget_bytes=None,
          prefix_budget_bytes=128 * 1024 ** 2, stats=None):
    """Drop-in for rules/max_inference.py:4-8 (the evaluator module `ev` and
    the prefix-cache budget are not needed; dense_budget_bytes bounds the
    [ranks, queries, E] accumulator)."""
    if stats is not None:
        stats.setdefault("rules_before", len(rules))
    return max_product_scores(sources, rules, csr, relations, entities, chunk_size=chunk_size, final_max=final_max,
                              accumulator_bytes=dense_budget_bytes or (4 << 30))
