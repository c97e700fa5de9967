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

Both entry points ground whole batches of (query, rule) instances at once,
one state row per instance, in the library's fixed-relation kernels (or
entity bitmaps for instances with many facts).  The maxima go through dense
per-query accumulators (fl_rule_instance_max: an exact, order-independent
atomic max of the weights' fp32 bit patterns) or through rank facts and the
MAX row reduction; both give the same scores.  max_product_scores gives
every query the same rule list; evaluate_rule_bank gives each query the rules
of its own relation.
"""
from __future__ import annotations

import ctypes
import time

import numpy as np
import torch

from . import ops
from .ops import EPS, Graph, _p, _stream, _ws, check, lib


def _graph(csr_struct):
    c = tuple(csr_struct)
    dev = c[1].device
    z = torch.empty(0, dtype=torch.int32, device=dev)
    return Graph.of((c[8], c[1], z.to(torch.int16), z, c[12], c[5], z.to(torch.int16), z,
                     c[8], c[9], c[10], c[11], c[12], c[13], c[14], c[15]))


def _empty(B, E, device):
    return torch.sparse_coo_tensor(torch.empty((2, 0), dtype=torch.long, device=device),
                                   torch.empty(0, device=device), (B, E), is_coalesced=True)


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


def max_product_scores(sources, rules, csr_struct, relations: int, entities: int, chunk_size: int = 16,
                       final_max: bool = False, accumulator_bytes: int = 4 << 30, query_batch: int = 256,
                       stats=None):
    """Rule-bank scores [len(sources), entities] (sparse COO, coalesced).

    rules: sequence of {'body': tuple of operators, 'rank_weights': list}
    (rules/evaluate.py:94-119), all with the same number of ranks.  Rules whose
    first operator has no edge at any source are dropped first
    (rules/shared_inference.py:34-47).  Every query gets every remaining
    rule: batches of at most query_batch queries (and 2^20 (query, rule)
    instances) are grounded as one instance state each (_ground_instances).
    When one query's [ranks, E] accumulator fits accumulator_bytes, the
    maxima go through dense per-query accumulators (fl_rule_instance_max);
    otherwise (86M entities) through rank facts and the MAX row reduction,
    with no dense buffer.  chunk_size is the reference's knob, kept for the
    signature: the scores do not depend on it.
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
    K = len(rules)
    dense = accumulator_bytes >= ranks * E * 4  # one query's [ranks, E] accumulator fits
    stats["dense_accumulation"] = dense
    qb = max(1, min(B, query_batch, (1 << 20) // K))  # at most 2^20 (query, rule) instances per batch
    keys_out, vals_out = [], []
    for q0 in range(0, B, qb):
        src = sources[q0:q0 + qb].to(torch.int64)
        Bq = src.numel()
        inst_rule = torch.arange(K, device=dev).repeat(Bq)
        row_ptr, ent, _ = _ground_instances(src.repeat_interleave(K), inst_rule, ops_all, graph, relations, E,
                                            1 << 29, stats, None)
        q_inst = torch.arange(Bq + 1, dtype=torch.int64, device=dev) * K
        for qa, qz, (s_rp, s_ent, s_x) in _instance_scores(
                row_ptr, ent, q_inst, weights[inst_rule].contiguous(), ranks, E, final_max, 1 << 29, stats,
                0 if dense else 1 << 62, accumulator_bytes if dense else 4 << 30):
            q = torch.repeat_interleave(torch.arange(qz - qa, device=dev), s_rp[1:] - s_rp[:-1],
                                        output_size=s_ent.numel())
            keys_out.append((q + q0 + qa) * E + s_ent.to(torch.int64))
            vals_out.append(s_x)
    keys = torch.cat(keys_out) if keys_out else torch.empty(0, dtype=torch.int64, device=dev)
    vals = torch.cat(vals_out) if vals_out else torch.empty(0, dtype=torch.float32, device=dev)
    return torch.sparse_coo_tensor(torch.stack((keys // E, keys % E)), vals, (B, E), is_coalesced=True)


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


def _reduce_rows(row_ptr, rows: int, E: int, slot_base, entry_count, fact_dst, fact_val, T: int):
    """The sorted distinct destinations of every row's facts (the row
    reduction; the sums are not needed by a Boolean state).  One host read
    sizes the outputs."""
    dev = fact_dst.device
    out_row_ptr = torch.empty(rows + 1, dtype=torch.int64, device=dev)
    out_ent = torch.empty(max(T, 1), dtype=torch.int32, device=dev)
    out_x = torch.empty(max(T, 1), dtype=torch.float32, device=dev)
    out_denom = torch.empty(max(rows, 1), dtype=torch.float32, device=dev)
    ws = _ws(lib().fl_reduce_workspace(rows, max(T, 1)), dev)
    check(lib().fl_row_reduce(_p(row_ptr), rows, E, _p(slot_base), _p(entry_count), _p(fact_dst), _p(fact_val),
                              max(T, 1), None, ctypes.c_float(EPS), _p(out_row_ptr), _p(out_ent), _p(out_x), None,
                              _p(out_denom), None, None, _p(ws), ws.numel(), None, _stream()), "row_reduce")
    return out_row_ptr, out_ent[:int(out_row_ptr[rows].item())]


# Entries above which a query's maxima always go through the dense
# accumulator: the sparse path ends in one row-reduction CTA per query.
_DENSE_QUERY_ENTRIES = 1 << 16

# Facts above which a row always goes through a bitmap: the row reduction
# runs one CTA per row and re-reads a row once per 12,288-fact chunk, so rows
# far above a chunk are cheaper as bitmaps even when E is large.
_BITMAP_ROW_FACTS = 1 << 16


def _bitmap_words(E: int) -> int:
    """u32 words of one entity bitmap, rounded up to the 256-word chunks of fl_bitmap_rows_*."""
    return ((E + 31) // 32 + 255) // 256 * 256


def _merge_rows(rows: int, parts):
    """Concatenate per-row results of disjoint row sets: parts are (row_ptr
    over all rows, entities) whose rows are empty outside their set."""
    dev = parts[0][1].device
    counts = sum(rp[1:] - rp[:-1] for rp, _ in parts)
    out_rp = torch.zeros(rows + 1, dtype=torch.int64, device=dev)
    torch.cumsum(counts, 0, out=out_rp[1:])
    total = int(out_rp[rows].item())
    out = torch.empty(max(total, 1), dtype=torch.int32, device=dev)
    for rp, e in parts:
        if e.numel():
            check(lib().fl_rows_copy(_p(rp), _p(e), rows, _p(out_rp), _p(out), _stream()), "rows_copy")
    return out_rp, out[:total]


def _plan_step(ent, b, ops_col, graph, relations: int):
    """Facts of every entry of a fixed step: slot_base i64[nnz + 1] (its
    exclusive prefix) and the total (one host read)."""
    nnz = ent.numel()
    slot_base = torch.empty(nnz + 1, dtype=torch.int64, device=ent.device)
    ws = _ws(lib().fl_fixed_relation_workspace(nnz), ent.device)
    total = ctypes.c_int64(0)
    check(lib().fl_fixed_relation_plan(_p(b), None, _p(ent), nnz, _p(ops_col), 1, relations, graph.ori, graph.inv,
                                       _p(slot_base), ctypes.byref(total), _p(ws), ws.numel(), _stream()),
          "fixed_relation_plan")
    return slot_base, total


def _sorted_step(row_ptr, ent, b, ops_col, graph, relations: int, E: int, fact_budget: int, stats, plan=None):
    """The fixed step by the row reduction (sorted distinct destinations per
    row), over ranges of rows of at most fact_budget facts.  plan: the
    entries' _plan_step, when already computed."""
    dev = ent.device
    rows = row_ptr.numel() - 1
    nnz = ent.numel()
    if nnz == 0:
        return torch.zeros(rows + 1, dtype=torch.int64, device=dev), ent
    slot_base, total = plan if plan is not None else _plan_step(ent, b, ops_col, graph, relations)
    if total.value <= fact_budget:
        ranges = [(0, rows, 0, nnz)]
    else:
        rp_h = row_ptr.cpu().numpy()
        starts = slot_base[row_ptr].cpu().numpy()  # facts before each row
        ranges = []
        r0 = 0
        while r0 < rows:
            r1 = min(int(np.searchsorted(starts, starts[r0] + fact_budget, side="right")) - 1, rows)
            r1 = max(r1, r0 + 1)  # one instance above the budget still runs alone
            ranges.append((r0, r1, int(rp_h[r0]), int(rp_h[r1])))
            r0 = r1
    stats["step_ranges"] = stats.get("step_ranges", 0) + len(ranges)
    out_rp, out_ent, offset = [], [], 0
    for r0, r1, e0, e1 in ranges:
        sb = slot_base if len(ranges) == 1 else slot_base[e0:e1 + 1] - slot_base[e0]
        T = int(total.value) if len(ranges) == 1 else int((slot_base[e1] - slot_base[e0]).item())
        fact_dst = torch.empty(max(T, 1), dtype=torch.int32, device=dev)
        fact_val = torch.empty(max(T, 1), dtype=torch.float32, device=dev)
        entry_count = torch.empty(max(e1 - e0, 1), dtype=torch.int32, device=dev)
        check(lib().fl_fixed_relation_fill(_p(b[e0:e1]), None, _p(ent[e0:e1]), None, e1 - e0, _p(ops_col), 1,
                                           relations, graph.ori, graph.inv, _p(sb), _p(fact_dst), _p(fact_val),
                                           _p(entry_count), _stream()), "fixed_relation_fill")
        rp = row_ptr if len(ranges) == 1 else row_ptr[r0:r1 + 1] - e0
        o_rp, o_ent = _reduce_rows(rp, r1 - r0, E, sb, entry_count, fact_dst, fact_val, T)
        out_rp.append(o_rp[:-1] + offset)
        out_ent.append(o_ent)
        offset += o_ent.numel()
    out_rp.append(torch.tensor([offset], dtype=torch.int64, device=dev))
    return torch.cat(out_rp), (out_ent[0] if len(out_ent) == 1 else torch.cat(out_ent))


def _bitmap_step(row_ptr, ent, b, ops_col, big_rows, graph, relations: int, E: int, bitmap_bytes: int, stats):
    """The fixed step of the rows big_rows (host array, ascending) through
    entity bitmaps, in groups of rows whose bitmaps fit bitmap_bytes.
    Returns (row_ptr over all rows, empty outside big_rows; entities)."""
    dev = ent.device
    rows = row_ptr.numel() - 1
    words = _bitmap_words(E)
    per = max(1, bitmap_bytes // (4 * words))
    counts = row_ptr[1:] - row_ptr[:-1]
    out_cnt = torch.zeros(rows, dtype=torch.int64, device=dev)
    ents = []
    for g0 in range(0, big_rows.size, per):
        grp = torch.from_numpy(big_rows[g0:g0 + per]).to(dev)
        nb = grp.numel()
        lens = counts[grp]
        n = int(lens.sum().item())
        row_slot = torch.full((rows,), -1, dtype=torch.int32, device=dev)
        row_slot[grp] = torch.arange(nb, dtype=torch.int32, device=dev)
        first = row_ptr[grp] - (torch.cumsum(lens, 0) - lens)
        entries = torch.repeat_interleave(first, lens, output_size=n) + torch.arange(n, device=dev)
        bitmap = torch.zeros(nb * words, dtype=torch.int32, device=dev)
        check(lib().fl_fixed_relation_bitmap(_p(entries), n, _p(b), _p(row_slot), _p(ent), _p(ops_col), relations,
                                             graph.ori, graph.inv, _p(bitmap), words, _stream()),
              "fixed_relation_bitmap")
        chunk_off = torch.empty(nb * (words // 256) + 1, dtype=torch.int64, device=dev)
        g_rp = torch.empty(nb + 1, dtype=torch.int64, device=dev)
        ws = _ws(lib().fl_bitmap_rows_workspace(nb, words), dev)
        check(lib().fl_bitmap_rows_count(_p(bitmap), nb, words, _p(chunk_off), _p(g_rp), _p(ws), ws.numel(),
                                         _stream()), "bitmap_rows_count")
        g_ent = torch.empty(max(int(g_rp[nb].item()), 1), dtype=torch.int32, device=dev)
        check(lib().fl_bitmap_rows_emit(_p(bitmap), nb, words, _p(chunk_off), _p(g_ent), _stream()),
              "bitmap_rows_emit")
        out_cnt[grp] = g_rp[1:] - g_rp[:-1]
        ents.append(g_ent[:int(g_rp[nb].item())])
    stats["bitmap_rows"] = stats.get("bitmap_rows", 0) + int(big_rows.size)
    out_rp = torch.zeros(rows + 1, dtype=torch.int64, device=dev)
    torch.cumsum(out_cnt, 0, out=out_rp[1:])
    return out_rp, (ents[0] if len(ents) == 1 else torch.cat(ents))


def _fixed_step_rows(row_ptr, ent, ops_col, graph, relations: int, E: int, fact_budget: int, stats,
                     bitmap_min_facts=None, bitmap_bytes: int = 4 << 30):
    """One fixed-operator step of a Boolean state whose rows are rule
    instances: row i moves along operator ops_col[i] (flashlog.cu:1561-1741),
    and every reached entity is kept once (the step's Boolean projection,
    rules/shared_inference.py:123-126).  A row with more facts than
    bitmap_min_facts (default: twice its entity bitmap's words, at most
    65,536) is reduced
    through the bitmap (fl_fixed_relation_bitmap); the others through the row
    reduction, over ranges of rows of at most
    fact_budget facts (or a single row).  stats counts the ranges
    ("step_ranges") and the bitmap rows ("bitmap_rows").  Returns the next
    state (row_ptr, ent), each row's entities ascending."""
    dev = ent.device
    rows = row_ptr.numel() - 1
    nnz = ent.numel()
    if nnz == 0:
        return torch.zeros(rows + 1, dtype=torch.int64, device=dev), ent
    counts = row_ptr[1:] - row_ptr[:-1]
    b = torch.repeat_interleave(torch.arange(rows, device=dev), counts, output_size=nnz)
    ops_col = ops_col.to(torch.int64).contiguous()
    plan = _plan_step(ent, b, ops_col, graph, relations)
    row_facts = plan[0][row_ptr[1:]] - plan[0][row_ptr[:-1]]
    limit = min(2 * _bitmap_words(E), _BITMAP_ROW_FACTS) if bitmap_min_facts is None else bitmap_min_facts
    big = torch.nonzero(row_facts > limit).flatten().cpu().numpy()
    if big.size == 0:
        return _sorted_step(row_ptr, ent, b, ops_col, graph, relations, E, fact_budget, stats, plan)
    bm = _bitmap_step(row_ptr, ent, b, ops_col, big, graph, relations, E, bitmap_bytes, stats)
    if big.size == rows:
        return bm
    small = torch.ones(rows, dtype=torch.bool, device=dev)
    small[torch.from_numpy(big).to(dev)] = False
    keep = small[b]
    s_counts = torch.where(small, counts, torch.zeros_like(counts))
    s_rp = torch.zeros(rows + 1, dtype=torch.int64, device=dev)
    torch.cumsum(s_counts, 0, out=s_rp[1:])
    s_ent = ent[keep]
    srt = _sorted_step(s_rp, s_ent, b[keep], ops_col, graph, relations, E, fact_budget, stats)
    return _merge_rows(rows, [srt, bm])


def _combine_ranks(rp, r_ent, x, nq: int, ranks: int, E: int, final_max: bool):
    """Rank rows (q, r) of maxima: each divided by its sum (clamped at 1e-30,
    rules/evaluate.py:366-378), then per query the ranks summed in rank order
    or, with final_max, maximised.  Returns the row layout over the queries."""
    y, _ = ops.normalize_forward(rp, x, eps=1e-30)
    if final_max:
        return ops.row_max(rp[::ranks].contiguous(), r_ent, y, nq, E)
    out_rp, out_ent, out_x, _ = ops.channel_merge(rp, r_ent, y, nq, ranks, E)
    return out_rp, out_ent, out_x


def _dense_scores(acc, nq: int, ranks: int, E: int, final_max: bool):
    """Scores of nq queries from their dense rank maxima acc (u32 fp32 bits,
    [nq, ranks, E], consumed): the rank rows read back sorted, normalized in
    the row layout (the same sums as the sparse path), written back and
    combined densely, where the absent entries are +0.0 and leave the
    rank-order sum and the max of the present ones exact.  Returns the row
    layout over the queries."""
    dev = acc.device
    nz = torch.nonzero(acc.view(nq * ranks, E))
    row, r_ent = nz[:, 0], nz[:, 1]
    rp = torch.zeros(nq * ranks + 1, dtype=torch.int64, device=dev)
    torch.cumsum(torch.bincount(row, minlength=nq * ranks), 0, out=rp[1:])
    dense = acc.view(torch.float32).view(nq * ranks, E)
    y, _ = ops.normalize_forward(rp, dense[row, r_ent].contiguous(), eps=1e-30)
    dense[row, r_ent] = y
    del nz, row, r_ent, y
    dense = dense.view(nq, ranks, E)
    if final_max:
        comb = dense.amax(1)
    else:
        comb = dense[:, 0].clone()
        for r in range(1, ranks):
            comb += dense[:, r]
    del dense
    nz = torch.nonzero(comb)
    s_rp = torch.zeros(nq + 1, dtype=torch.int64, device=dev)
    torch.cumsum(torch.bincount(nz[:, 0], minlength=nq), 0, out=s_rp[1:])
    return s_rp, nz[:, 1].to(torch.int32), comb[nz[:, 0], nz[:, 1]].contiguous()


def _instance_scores(row_ptr, ent, q_inst, w_inst, ranks: int, E: int, final_max: bool, fact_budget: int, stats,
                     dense_min_entries=None, dense_bytes: int = 4 << 30):
    """Scores of the queries of an instance-grouped Boolean state (query q
    owns the instance rows [q_inst[q], q_inst[q + 1])): per rank r the largest
    weight of the instances reaching each entity, then _combine_ranks.  A
    query whose instances hold more than dense_min_entries entries (default
    E / 8 or 65,536, whichever is smaller) starts a run that accumulates, with
    the queries after it (as many as dense_bytes holds), in dense [ranks, E]
    buffers (fl_rule_instance_max), normalized in the rank-row layout and
    combined densely; the other runs go through rank facts and the exact MAX
    row reduction, with at most fact_budget facts each (a single query above
    it runs alone).  Both give the same scores, bit for bit.  stats counts the runs
    ("score_ranges", "dense_queries").  Yields, run by run, (qa, qb, row
    layout over the queries qa..qb-1 of the state)."""
    dev = ent.device
    Bq = q_inst.numel() - 1
    before = row_ptr[q_inst].cpu().numpy().astype(np.int64)  # entries before each query
    entries = np.diff(before)
    dense = entries > (min(E // 8, _DENSE_QUERY_ENTRIES) if dense_min_entries is None else dense_min_entries)
    per_dense = max(1, dense_bytes // (4 * ranks * E))
    runs, qa = [], 0
    while qa < Bq:
        if dense[qa]:
            # a dense run takes the queries after it whatever their size (the
            # dense accumulator gives every query the same rank rows), up to
            # its memory: fewer, longer runs
            qb = min(qa + per_dense, Bq)
        else:
            qb = qa + 1
            while qb < Bq and not dense[qb] and ranks * (before[qb + 1] - before[qa]) <= fact_budget:
                qb += 1
        runs.append((qa, qb, bool(dense[qa])))
        qa = qb
    stats["score_ranges"] = stats.get("score_ranges", 0) + len(runs)
    stats["dense_queries"] = stats.get("dense_queries", 0) + sum(qb - qa for qa, qb, d in runs if d)
    for qa, qb, is_dense in runs:
        nq = qb - qa
        if is_dense:
            acc = torch.zeros(nq * ranks * E, dtype=torch.int32, device=dev)
            check(lib().fl_rule_instance_max(_p(row_ptr), _p(ent), _p(q_inst[qa:]), nq, _p(w_inst), ranks, E,
                                             _p(acc), _stream()), "rule_instance_max")
            yield qa, qb, _dense_scores(acc, nq, ranks, E, final_max)
            continue
        else:
            T = int(ranks * (before[qb] - before[qa]))
            slot_base = torch.empty(nq * ranks + 1, dtype=torch.int64, device=dev)
            fact_dst = torch.empty(max(T, 1), dtype=torch.int32, device=dev)
            fact_val = torch.empty(max(T, 1), dtype=torch.float32, device=dev)
            check(lib().fl_rule_instance_facts(_p(row_ptr), _p(ent), _p(q_inst[qa:]), nq, _p(w_inst), ranks,
                                               _p(slot_base), _p(fact_dst), _p(fact_val), _stream()),
                  "rule_instance_facts")
            rp, r_ent, x = ops.row_max(slot_base, fact_dst, fact_val, nq * ranks, E)
        yield qa, qb, _combine_ranks(rp, r_ent, x, nq, ranks, E, final_max)


def _ground_instances(inst_src, inst_rule, ops_all, graph, relations: int, E: int, fact_budget: int, stats,
                      bitmap_min_facts=None):
    """Boolean end states of rule instances: row i starts at entity
    inst_src[i] and follows the body of rule inst_rule[i] (ops_all, padded
    with the identity) one fixed step at a time (_fixed_step_rows).  Returns
    (row_ptr, ent, the largest state of a step in entries)."""
    dev = inst_src.device
    row_ptr = torch.arange(inst_src.numel() + 1, dtype=torch.int64, device=dev)
    ent = inst_src.to(torch.int32)
    peak = 1
    for step in range(ops_all.shape[1]):
        row_ptr, ent = _fixed_step_rows(row_ptr, ent, ops_all[inst_rule, step], graph, relations, E, fact_budget,
                                        stats, bitmap_min_facts)
        peak = max(peak, ent.numel())
    return row_ptr, ent, peak


class _PhaseClock:
    """Host time per phase of evaluate_rule_bank, accumulated in stats[name]
    when stats["timing"] is set (the device is synchronized at each tick);
    nothing otherwise."""

    def __init__(self, stats):
        self.stats = stats if stats.get("timing") else None
        if self.stats is not None:
            torch.cuda.synchronize()
            self.t = time.perf_counter()

    def tick(self, name):
        if self.stats is not None:
            torch.cuda.synchronize()
            now = time.perf_counter()
            self.stats[name] = self.stats.get(name, 0.0) + now - self.t
            self.t = now


def route_instances(rel_h, heads, query_batch: int, instance_budget):
    """Batches of the routed evaluation (host side): the queries in relation
    order (stable), cut into batches of consecutive queries with at most
    query_batch queries and instance_budget instances (a query whose rules
    alone exceed the budget forms its own batch).  instance_budget may be a
    callable, read before every batch.  heads: the head relation
    of every compacted rule, ascending.  Yields (queries i64[Bq] in batch
    order, q_inst i64[Bq + 1] (query q owns instances q_inst[q]..q_inst[q+1]),
    inst_rule i64[instances] (the rule of every instance, in the order of
    its query's rules))."""
    rel_h = np.asarray(rel_h, dtype=np.int64)
    heads = np.asarray(heads, dtype=np.int64)
    lo = np.searchsorted(heads, rel_h, side="left")
    n_inst = np.searchsorted(heads, rel_h, side="right") - lo
    order = np.argsort(rel_h, kind="stable")
    q0 = 0
    while q0 < rel_h.size:
        budget = instance_budget() if callable(instance_budget) else instance_budget
        cum = np.cumsum(n_inst[order[q0:q0 + query_batch]])
        q1 = q0 + max(1, int(np.searchsorted(cum, budget, side="right")))
        bq = order[q0:q1]
        counts = n_inst[bq]
        q_inst = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
        inst_rule = (np.repeat(lo[bq] - q_inst[:-1], counts) + np.arange(int(q_inst[-1]))).astype(np.int64)
        yield bq.astype(np.int64), q_inst, inst_rule
        q0 = q1


def evaluate_rule_bank(sources, query_relations, targets, rules, csr_struct, relations: int, entities: int,
                       final_max: bool = False, chunk_size: int = 16, query_batch: int = 4096,
                       accumulator_bytes: int = 4 << 30, filter_keys=None, stats=None,
                       instance_budget: int = 1 << 20, fact_budget: int = 1 << 29, bitmap_min_facts=None,
                       dense_min_entries=None, entry_budget: int = 1 << 27):
    """Filtered, tie-averaged ranks of the targets under the rule bank's
    max-product scores (rules/evaluate.py:1015-1095 with --aggregations
    routed_normalized and reduction 'max': smDRUM sums the normalized ranks,
    mmDRUM takes their max).  Every query is routed to the rules whose head
    is its relation (compacted per (head, body), rules/evaluate.py:94-119).

    The queries, ordered by relation, run in batches of at most query_batch
    queries and instance_budget rule instances (query, rule), fewer when the
    instances reach many entities: after each batch the instance budget is
    set so that the largest state of a step (entities over all instances)
    would stay near entry_budget, from the batch's entities per instance (the
    first batch takes at most 2^12 instances); a single query with more
    instances than that is grounded in parts whose maxima meet in the query's
    dense accumulator.  One batch is
    one Boolean state whose rows are its instances, advanced one body
    operator per step for all instances at once, so the number of launches
    and host reads grows with the batches, not with the rules or the
    relations.  Instances whose step has many facts are reduced through entity
    bitmaps (more than bitmap_min_facts, default twice the bitmap's words or
    65,536, whichever is smaller),
    the others through the row reduction; a step with more than fact_budget
    facts runs over ranges of instances, which is the reference's per-source split
    (rules/shared_inference.py:60-76); an instance whose first operator has no
    edge at its source ends empty in the first step, as the reference's
    first-operator pruning (rules/shared_inference.py:34-47) drops it.  A
    query's rank maxima accumulate in a dense [ranks, E] buffer when its
    instances hold more than dense_min_entries entries (default E / 8 or
    65,536, whichever is smaller), else
    sparsely through the MAX row reduction (no [ranks, queries, E] buffer);
    both give the same scores.  Ranks come
    from fl_filtered_ranks against filter_keys (sorted keys q * E + e of known
    answers, numbered within the batch; the targets are added).  chunk_size
    and accumulator_bytes are the reference's knobs, kept for the signature:
    the scores do not depend on them.  Returns float32 ranks in query order."""
    dev = sources.device
    E = int(entities)
    Q = sources.numel()
    stats = {} if stats is None else stats
    ranks_out = torch.empty(Q, dtype=torch.float32, device=dev)
    if Q == 0:
        return ranks_out
    compact = sorted(compact_routed_rules(rules), key=lambda r: int(r["head"])) if rules else []
    for r in compact:
        if any(not (0 <= int(o) <= 2 * relations) for o in r["body"]):
            raise ValueError("rule operators must lie in [0, 2R]")
        if not all(np.isfinite(x) and x >= 0 for x in r["rank_weights"]):
            raise ValueError("MAX rule weights must be finite and nonnegative")
    heads = np.array([int(r["head"]) for r in compact], dtype=np.int64)
    rel_h = query_relations.cpu().numpy().astype(np.int64)
    n_inst = np.searchsorted(heads, rel_h, side="right") - np.searchsorted(heads, rel_h, side="left")
    if compact:
        ranks, weights, ops_all = _weights_and_ops(compact, relations, dev)
        graph = _graph(csr_struct)
    src_h = sources.to(torch.int64).cpu().numpy()
    stats.update(instances=int(n_inst.sum()), batches=0, rules_after=len(compact))
    budget = {"instances": min(instance_budget, 1 << 12)}
    for bq, q_inst_h, inst_rule_h in route_instances(rel_h, heads, query_batch, lambda: budget["instances"]):
        Bq = bq.size
        idx = torch.from_numpy(bq).to(dev)
        tgt = targets[idx]
        counts = np.diff(q_inst_h)
        I = int(q_inst_h[-1])
        clock = _PhaseClock(stats)
        if I > budget["instances"] and Bq == 1:
            # one query with more instances than a batch holds: its instances
            # are grounded in parts, each part's maxima raised into the
            # query's dense accumulator (the same maxima, in any part order)
            acc = torch.zeros(ranks * E, dtype=torch.int32, device=dev)
            c0 = 0
            while c0 < I:
                c1 = min(I, c0 + budget["instances"])
                part_rule = torch.from_numpy(inst_rule_h[c0:c1]).to(dev)
                part_src = torch.full((c1 - c0,), int(src_h[bq[0]]), dtype=torch.int32, device=dev)
                row_ptr, ent, peak = _ground_instances(part_src, part_rule, ops_all, graph, relations, E,
                                                       fact_budget, stats, bitmap_min_facts)
                stats["entries"] = stats.get("entries", 0) + ent.numel()
                q_part = torch.tensor([0, c1 - c0], dtype=torch.int64, device=dev)
                check(lib().fl_rule_instance_max(_p(row_ptr), _p(ent), _p(q_part), 1,
                                                 _p(weights[part_rule].contiguous()), ranks, E, _p(acc), _stream()),
                      "rule_instance_max")
                del row_ptr, ent
                budget["instances"] = int(min(instance_budget, max(256, entry_budget * (c1 - c0) // peak)))
                c0 = c1
            stats["split_queries"] = stats.get("split_queries", 0) + 1
            stats["dense_queries"] = stats.get("dense_queries", 0) + 1
            clock.tick("ground_s")
            scored = [(0, 1, _dense_scores(acc, 1, ranks, E, final_max))]
            del acc
        elif I:
            inst_rule = torch.from_numpy(inst_rule_h).to(dev)
            inst_src = torch.from_numpy(np.repeat(src_h[bq], counts).astype(np.int32)).to(dev)
            row_ptr, ent, peak = _ground_instances(inst_src, inst_rule, ops_all, graph, relations, E, fact_budget,
                                                   stats, bitmap_min_facts)
            stats["entries"] = stats.get("entries", 0) + ent.numel()
            budget["instances"] = int(min(instance_budget, max(256, entry_budget * I // peak)))
            clock.tick("ground_s")
            scored = _instance_scores(row_ptr, ent, torch.from_numpy(q_inst_h).to(dev),
                                      weights[inst_rule].contiguous(), ranks, E, final_max, fact_budget, stats,
                                      dense_min_entries)
        else:
            scored = [(0, Bq, None)]
        fk = torch.arange(Bq, device=dev) * E + tgt
        if filter_keys is not None:
            fk = torch.cat([fk, filter_keys(idx) if callable(filter_keys) else filter_keys[idx]])
        fk = torch.unique(fk)  # sorted: each run's keys are a contiguous range
        bounds = torch.searchsorted(fk, torch.arange(Bq + 1, device=dev) * E).cpu().tolist()
        # each run's queries are ranked as soon as they are scored (their scores are then dropped)
        for qa, qb, sc in scored:
            n = qb - qa
            if sc is None:
                si_b = si_e = torch.empty(0, dtype=torch.int64, device=dev)
                sv = torch.empty(0, dtype=torch.float32, device=dev)
            else:
                s_rp, s_ent, s_x = sc
                si_b = torch.repeat_interleave(torch.arange(n, device=dev), s_rp[1:] - s_rp[:-1],
                                               output_size=s_ent.numel())
                si_e, sv = s_ent.to(torch.int64), s_x
            fk_run = fk[bounds[qa]:bounds[qb]] - qa * E
            ranks_out[idx[qa:qb]] = ops.filtered_ranks(si_b, si_e, sv, tgt[qa:qb], fk_run, n, E, True)
        clock.tick("score_s")
        stats["batches"] += 1
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
