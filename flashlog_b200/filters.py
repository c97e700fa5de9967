"""Filter keys for filtered ranking, on the GPU.

Restates the known-answer lookups of the reference's evaluation drivers:

* build_filter_indices_csr (src/main.py:281-318): for every query (x, r),
  the entities t with (x, r, t) in a split's triples -- the relation-r group
  of x on the forward side for r < R, the group of relation r - R on the
  inverse side otherwise.  The reference binary-searches sorted group keys
  on the host (src/main.py:196-278) and expands with repeat_interleave; here
  every query is one entry of the fixed-relation step (flashlog.cu:1561-1741),
  so the whole batch is one search-and-copy launch.
* create_eval_filter_csr (src/main.py:136-151): the per-split lookups (train,
  then valid+test), here built as device CSR structures.
* filter_keys_for_batch_flashlog (rules/evaluate.py:746-780): keys
  b * E + t of a rule-evaluation batch, plus the split's known answers and
  the targets; the reference expands one query per launch, here one launch
  covers the batch.

Output order: the reference returns each lookup's pairs grouped by side, and
within a group in the order of an unstable host argsort; its consumers only
use the sorted unique keys (src/main.py:401-407).  The pairs here come sorted
by (query, entity) per lookup, the same multiset.
"""
from __future__ import annotations

import torch

from .flashlog_kernel import build_csr_structure, vectorized_operation_sparse3d_fixed_relation


def _empty(device):
    e = torch.empty(0, dtype=torch.long, device=device)
    return e, e


def _filter_from_csr(input_x, input_r, relation_size: int, csr):
    dev = csr[1].device
    if dev.type != "cuda":
        raise ValueError("filter lookups run on CUDA: the CSR structure must be on the device")
    x = input_x.detach().to(dev, torch.int64).reshape(-1)
    r = input_r.detach().to(dev, torch.int64).reshape(-1)
    if x.numel() != r.numel():
        raise ValueError("input_x and input_r must have the same length")
    R = int(relation_size)
    E = csr[0].numel() - 1
    if r.numel() and bool(((r < 0) | (r >= 2 * R)).any()):
        raise ValueError(f"query relations must lie in [0, {2 * R})")
    B = x.numel()
    if B == 0:
        return _empty(dev)
    # a head outside [0, E) has no group (as the reference's key search finds none)
    ok = (x >= 0) & (x < E)
    b = torch.arange(B, device=dev)[ok]
    e = x[ok]
    if b.numel() == 0:
        return _empty(dev)
    state = torch.sparse_coo_tensor(torch.stack([b, torch.zeros_like(b), e]),
                                    torch.ones(b.numel(), device=dev), (B, 1, E), is_coalesced=True)
    out = vectorized_operation_sparse3d_fixed_relation(state, r.view(B, 1), csr, R)
    idx = out.indices()
    return idx[0], idx[2]


def _filter_from_reference_lookup(input_x, input_r, relation_size: int, lookup, device):
    """A lookup in the reference's own format ((group_keys, starts, counts,
    columns) per side, src/main.py:154-169), searched on the device."""
    x = input_x.detach().to(device, torch.int64).reshape(-1)
    r = input_r.detach().to(device, torch.int64).reshape(-1)
    R = int(relation_size)
    pos_all = torch.arange(x.numel(), device=device)
    batches, ents = [], []
    for side, sel in ((lookup[0], r < R), (lookup[1], r >= R)):
        keys, starts, counts, cols = (t.to(device) for t in side)
        if keys.numel() == 0 or not bool(sel.any()):
            continue
        q = x[sel] * R + (r[sel] - (0 if side is lookup[0] else R))
        p = torch.searchsorted(keys, q)
        safe = p.clamp(max=keys.numel() - 1)
        hit = (p < keys.numel()) & (keys[safe] == q)
        cnt = torch.where(hit, counts[safe].long(), torch.zeros_like(q))
        total = int(cnt.sum())
        if total == 0:
            continue
        bq = pos_all[sel]
        ob = torch.repeat_interleave(bq, cnt)
        first = torch.cumsum(cnt, 0) - cnt
        local = torch.arange(total, device=device) - torch.repeat_interleave(first, cnt)
        edge = torch.repeat_interleave(starts[safe].long(), cnt) + local
        batches.append(ob)
        ents.append(cols[edge].long())
    if not batches:
        return _empty(device)
    return torch.cat(batches), torch.cat(ents)


def build_filter_indices_csr(input_x, input_r, relation_size, csr_struct):
    """(batch ids, entity ids) of the known answers of each query (src/main.py:281-288).

    csr_struct: the training CSR 16-tuple of build_csr_structure, or
    {"filter_lookups": [...]} whose items are CSR tuples (create_eval_filter_csr
    here) or the reference's own lookup pairs.
    """
    if isinstance(csr_struct, dict) and "filter_lookups" in csr_struct:
        results = []
        for lookup in csr_struct["filter_lookups"]:
            if isinstance(lookup, (tuple, list)) and len(lookup) == 16:
                results.append(_filter_from_csr(input_x, input_r, relation_size, lookup))
            else:
                dev = input_x.device if input_x.is_cuda else torch.device("cuda")
                results.append(_filter_from_reference_lookup(input_x, input_r, relation_size, lookup, dev))
        if not results:
            return _empty(input_x.device)
        return tuple(torch.cat([res[i] for res in results]) for i in range(2))
    return _filter_from_csr(input_x, input_r, relation_size, tuple(csr_struct))


def create_eval_filter_csr(splits, relation_size, entity_size, device):
    """{"filter_lookups": [CSR per split]} for build_filter_indices_csr
    (src/main.py:136-151 builds one lookup for train and one for valid+test).
    splits: sequence of (heads, relations, tails) integer tensors or arrays."""
    lookups = []
    for h, r, t in splits:
        h, r, t = (torch.as_tensor(a, dtype=torch.int64).to(device) for a in (h, r, t))
        if r.numel() and bool(((r < 0) | (r >= int(relation_size))).any()):
            raise ValueError(f"split relations must lie in [0, {int(relation_size)})")
        lookups.append(build_csr_structure(h, t, r, int(entity_size)))
    return {"filter_lookups": lookups}, None, None


def filter_keys_for_batch_flashlog(csr, batch, sources, split_known, num_relations, num_entities,
                                   include_targets=True):
    """Sorted unique keys b * E + t of known answers for a rule-evaluation
    batch of (source, relation, target) triples (rules/evaluate.py:746-780):
    the CSR's own answers, those in split_known[(source, relation)], and the
    targets when include_targets."""
    dev = sources.device
    B = len(batch)
    if B == 0:
        return torch.empty(0, dtype=torch.long, device=dev)
    rels = torch.tensor([int(rel) for _, rel, _ in batch], dtype=torch.int64, device=dev)
    qb, qe = _filter_from_csr(sources.reshape(-1)[:B], rels, num_relations, tuple(csr))
    parts = [qb * int(num_entities) + qe]
    extra = []
    for bi, (source, relation, target) in enumerate(batch):
        answers = set(split_known.get((source, relation), set()))
        if include_targets:
            answers.add(target)
        extra.extend(bi * int(num_entities) + int(a) for a in answers)
    if extra:
        parts.append(torch.tensor(extra, dtype=torch.long, device=dev))
    return torch.unique(torch.cat(parts), sorted=True)
