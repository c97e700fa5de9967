"""numpy front end of the C oracle (flashlog_oracle.c).

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's CPU
baseline / reference legs use it as the checker.  The product package never
imports this module.

Conventions follow the reference operator API (flashlog_kernel/flashlog_kernel.py):
a state is a coalesced COO over [B, L, E] given as row = b * L + l (int64),
entity (int64) and value (float32), sorted by (row, entity); w is [B, L, n].
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build as _build

_lib = None

SKIP_NONPOS_W = 1
DROP_MASKED = 2
MASK_BY_TRIPLE = 4
WOT_I = 8
SAMPLED = 16
EDGE_SCORE = 32

# Flag sets of the three reference expansion paths.
MODE_TOPK = SKIP_NONPOS_W | DROP_MASKED | MASK_BY_TRIPLE   # flashlog.cu:1402-1559 + flashlog_kernel.py:1217-1228
MODE_CPU = SKIP_NONPOS_W | DROP_MASKED                     # flashlog.cpp:506-578
MODE_ALL_EDGES = 0                                         # flashlog.cu:1743-1829
# The MAX path keeps hidden facts (value 0): flashlog_kernel.py:1450-1518 has no visibility filter.
MODE_TOPK_MAX = SKIP_NONPOS_W | MASK_BY_TRIPLE


def lib():
    global _lib
    if _lib is None:
        path = _build.ORACLE_SO
        if not os.path.exists(path):
            _build.build_oracle()
        _lib = ctypes.CDLL(path)
        _lib.flo_group_threshold.restype = ctypes.c_float
        _lib.flo_sampling_phase.restype = ctypes.c_double
        for name in ("flo_build_side", "flo_topc", "flo_hop_forward", "flo_hop_forward_edges", "flo_fact_bound",
                     "flo_fixed_relation", "flo_coalesce_sum"):
            getattr(_lib, name).restype = ctypes.c_int64
    return _lib


def _p(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else ctypes.c_void_p(0)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def build_side(src, dst, rel, nodes):
    """One CSR side: (row_ptr, columns, edge_rel, order, group_ptr, group_rel, group_start, group_count)."""
    src, dst, rel = _c(src, np.int64), _c(dst, np.int64), _c(rel, np.int64)
    m = src.size
    row_ptr = np.empty(nodes + 1, np.int32)
    cols = np.empty(m, np.int32)
    erel = np.empty(m, np.int16)
    order = np.empty(m, np.int32)
    gptr = np.empty(nodes + 1, np.int32)
    grel = np.empty(max(m, 1), np.int16)
    gstart = np.empty(max(m, 1), np.int32)
    gcount = np.empty(max(m, 1), np.int32)
    g = lib().flo_build_side(ctypes.c_int64(m), _p(src), _p(dst), _p(rel), ctypes.c_int64(nodes),
                             _p(row_ptr), _p(cols), _p(erel), _p(order), _p(gptr), _p(grel),
                             _p(gstart), _p(gcount))
    if g < 0:
        raise ValueError("CSR requires equal 1D arrays and int32-sized graph")
    return row_ptr, cols, erel, order, gptr, grel[:g].copy(), gstart[:g].copy(), gcount[:g].copy()


def build_csr(head, tail, rel, nodes):
    """The reference's 16-tuple layout (flashlog_kernel.py:678-697)."""
    ori = build_side(head, tail, rel, nodes)
    inv = build_side(tail, head, rel, nodes)
    return (*ori[:4], *inv[:4], *ori[4:], *inv[4:])


def filter_indices(x, r, relation_size, csr):
    """Known answers of each query (x, r) from a 16-tuple CSR
    (src/main.py:196-278): the forward-side group of relation r of x for
    r < R, the inverse-side group of relation r - R otherwise; a head
    outside [0, E) has none.  Returns (batch, entity) sorted by (batch,
    entity) -- the reference's pairs up to order."""
    x, r = _c(x, np.int64), _c(r, np.int64)
    R = int(relation_size)
    E = csr[0].size - 1
    out_b, out_e = [], []
    for j in range(x.size):
        if not (0 <= x[j] < E):
            continue
        inv = r[j] >= R
        rel = r[j] - R if inv else r[j]
        gptr, grel, gstart, gcount = (csr[12], csr[13], csr[14], csr[15]) if inv else (csr[8], csr[9], csr[10], csr[11])
        col = csr[5] if inv else csr[1]
        g0, g1 = int(gptr[x[j]]), int(gptr[x[j] + 1])
        k = g0 + int(np.searchsorted(grel[g0:g1], rel))
        if k < g1 and grel[k] == rel:
            ents = np.sort(col[gstart[k]:gstart[k] + gcount[k]].astype(np.int64))
            out_b.append(np.full(ents.size, j, np.int64))
            out_e.append(ents)
    if not out_b:
        return np.empty(0, np.int64), np.empty(0, np.int64)
    return np.concatenate(out_b), np.concatenate(out_e)


def topc(row, val, c1):
    """c1 kept-entry indices, or None when no row exceeds c1 nonzeros."""
    row, val = _c(row, np.int64), _c(val, np.float32)
    keep = np.zeros(row.size, np.uint8)
    k = lib().flo_topc(ctypes.c_int64(row.size), _p(row), _p(val), ctypes.c_int64(c1), _p(keep))
    if k < 0:
        return None
    return np.flatnonzero(keep).astype(np.int64)


def csr_masks(csr, mask, edge_weight=None):
    """CSR-ordered float masks per side (prepare_csr_masks, flashlog_kernel.py:232-255)."""
    m = _c(mask, np.float32).reshape(-1)
    if edge_weight is not None:
        m = (m * (1.0 / (1.0 + np.exp(-_c(edge_weight, np.float32).reshape(-1))))).astype(np.float32)
    return m[csr[3].astype(np.int64)], m[csr[7].astype(np.int64)]


def hop_forward(row, ent, val, w, csr, r_size, E, topk_edges=1 << 60, mode=MODE_TOPK,
                mask=None, edge_weight=None, wot_i=False, sampling_seed=-1, record=True, record_edges=False):
    """One propagation hop with coalesce-sum; returns a dict of numpy arrays.

    out_key = row * E + e (sorted), out_val = pre-normalization sums, and the
    per-fact provenance (entry, relation column, m, output position; with
    record_edges also the triple id, fact_edge).
    """
    row, ent, val = _c(row, np.int64), _c(ent, np.int64), _c(val, np.float32)
    w = _c(w, np.float32)
    B, L, n = w.shape
    nnz = row.size
    ori_rp, ori_col, _, ori_order, inv_rp, inv_col, _, inv_order = csr[:8]
    ori_gptr, ori_grel, ori_gstart, ori_gcount, inv_gptr, inv_grel, inv_gstart, inv_gcount = csr[8:]
    flags = mode | (WOT_I if wot_i else 0)
    if sampling_seed >= 0:
        flags |= SAMPLED
    if edge_weight is not None and not (flags & MASK_BY_TRIPLE):
        raise ValueError("edge weights are applied through the triple-indexed mask")
    if mask is None:
        mask = np.ones(ori_col.size, np.uint8)
    if flags & MASK_BY_TRIPLE:
        mask_triple = _c(np.asarray(mask).reshape(-1) != 0, np.uint8)
        mo = mi = None
    else:
        mask_triple = None
        mo, mi = csr_masks(csr, mask, None)
    ew = _c(edge_weight, np.float32).reshape(-1) if edge_weight is not None else None
    cap = lib().flo_fact_bound(ctypes.c_int64(nnz), _p(ent), _p(_c(ori_rp, np.int32)), _p(_c(inv_rp, np.int32)))
    cap = max(int(cap), 1)
    out_key = np.empty(cap, np.int64)
    out_val = np.empty(cap, np.float32)
    if record:
        f_entry = np.empty(cap, np.int64)
        f_rel = np.empty(cap, np.int32)
        f_m = np.empty(cap, np.float32)
        f_out = np.empty(cap, np.int64)
    else:
        f_entry = f_rel = f_m = f_out = None
    f_edge = np.empty(cap, np.int64) if (record and record_edges) else None
    nf = ctypes.c_int64(0)
    arrs = [_c(a, t) for a, t in ((ori_col, np.int32), (ori_order, np.int32), (ori_gptr, np.int32),
                                   (ori_grel, np.int16), (ori_gstart, np.int32), (ori_gcount, np.int32),
                                   (inv_col, np.int32), (inv_order, np.int32), (inv_gptr, np.int32),
                                   (inv_grel, np.int16), (inv_gstart, np.int32), (inv_gcount, np.int32))]
    u = lib().flo_hop_forward_edges(
        ctypes.c_int64(nnz), _p(row), _p(ent), _p(val), _p(w), ctypes.c_int64(L), ctypes.c_int64(n),
        ctypes.c_int64(E), ctypes.c_int64(r_size), *[_p(a) for a in arrs],
        _p(mo), _p(mi), _p(mask_triple), _p(ew), ctypes.c_int64(int(min(topk_edges, 1 << 62))),
        ctypes.c_int64(flags), ctypes.c_int64(sampling_seed),
        _p(out_key), _p(out_val), _p(f_entry), _p(f_rel), _p(f_m), _p(f_out), _p(f_edge), ctypes.byref(nf))
    nf = nf.value
    res = dict(out_key=out_key[:u].copy(), out_val=out_val[:u].copy(), n_facts=nf)
    if record:
        res.update(fact_entry=f_entry[:nf].copy(), fact_rel=f_rel[:nf].copy(),
                   fact_m=f_m[:nf].copy(), fact_out=f_out[:nf].copy())
        if f_edge is not None:
            res["fact_edge"] = f_edge[:nf].copy()
    return res


def edge_weight_grad(fw, g_out, row, val, w, edge_weight):
    """Gradient of learnable edge weights (flashlog_kernel.py:1306-1336 for
    SUM, 1590-1614 for MAX): every edge fact that reached an output
    (fact_out >= 0; MAX records -1 for the facts that lost) adds
    g_out[fact_out] * v * w[row, rel] * m * (1 - sigmoid(ew[edge])), the
    product in fp32 in the reference's order, summed in float64 per triple.
    fw: a forward recorded with record_edges (hop_forward_max records them)."""
    row, val, w = _c(row, np.int64), _c(val, np.float32), _c(w, np.float32)
    n = w.shape[-1]
    ew = np.asarray(edge_weight, np.float32).reshape(-1)
    f = (np.asarray(fw["fact_rel"]) < n - 1) & (np.asarray(fw["fact_out"]) >= 0)
    e = fw["fact_entry"][f]
    rel = fw["fact_rel"][f].astype(np.int64)
    edge = fw["fact_edge"][f].astype(np.int64)
    score = (np.float32(1) / (np.float32(1) + np.exp(-ew[edge]))).astype(np.float32)
    wv = w.reshape(-1, n)[row[e], rel]
    g = np.asarray(g_out, np.float32)[fw["fact_out"][f]]
    c = (g * val[e]).astype(np.float32)
    c = (c * wv).astype(np.float32)
    c = (c * fw["fact_m"][f]).astype(np.float32)
    c = (c * (np.float32(1) - score)).astype(np.float32)
    grad = np.zeros(ew.size, np.float64)
    np.add.at(grad, edge, c.astype(np.float64))
    return grad


def max_coalesce(keys, values, source, tie):
    """MAX coalesce with an exact winner (flashlog_kernel.py:399-478).

    Per key: the largest value; among equal values the smallest source (0 ori,
    1 inv, 2 identity), then the smallest tie key (triple id, 0 for identity),
    then the earliest fact.  Returns (unique_keys, max_values, winner_index).
    """
    keys = np.asarray(keys, np.int64)
    values = np.asarray(values, np.float32)
    if keys.size == 0:
        return keys[:0], values[:0], np.zeros(0, np.int64)
    pos = np.arange(keys.size)
    order = np.lexsort((pos, np.asarray(tie, np.int64), np.asarray(source, np.int64), -values, keys))
    sk = keys[order]
    first = np.ones(sk.size, bool)
    first[1:] = sk[1:] != sk[:-1]
    win = order[first]
    return keys[win], values[win], win


def hop_forward_max(row, ent, val, w, csr, r_size, E, topk_edges=1 << 60, mask=None, wot_i=False, edge_weight=None,
                    edge_score=False):
    """One hop of FlashLogFunctionSparse3DTopKMax (flashlog_kernel.py:1450-1518):
    the top-k fill without the visibility filter (hidden edges give facts of
    value 0), then the MAX coalesce with exact winners.

    Returns a dict with out_key, out_val and the recorded facts (entry, rel,
    m, edge, value, source) in emission order, fact_out = output index of a
    winning fact and -1 for the others.
    """
    row, ent, val = _c(row, np.int64), _c(ent, np.int64), _c(val, np.float32)
    w = _c(w, np.float32)
    B, L, n = w.shape
    nnz = row.size
    ori_rp, ori_col, _, ori_order, inv_rp, inv_col, _, inv_order = csr[:8]
    ori_gptr, ori_grel, ori_gstart, ori_gcount, inv_gptr, inv_grel, inv_gstart, inv_gcount = csr[8:]
    flags = MODE_TOPK_MAX | (WOT_I if wot_i else 0) | (EDGE_SCORE if edge_score else 0)
    if mask is None:
        mask = np.ones(ori_col.size, np.uint8)
    mask_triple = _c(np.asarray(mask).reshape(-1) != 0, np.uint8)
    ew = _c(edge_weight, np.float32).reshape(-1) if edge_weight is not None else None
    cap = max(int(lib().flo_fact_bound(ctypes.c_int64(nnz), _p(ent), _p(_c(ori_rp, np.int32)),
                                        _p(_c(inv_rp, np.int32)))), 1)
    out_key = np.empty(cap, np.int64)
    out_val = np.empty(cap, np.float32)
    f_entry = np.empty(cap, np.int64)
    f_rel = np.empty(cap, np.int32)
    f_m = np.empty(cap, np.float32)
    f_out = np.empty(cap, np.int64)
    f_edge = np.empty(cap, np.int64)
    nf = ctypes.c_int64(0)
    arrs = [_c(a, t) for a, t in ((ori_col, np.int32), (ori_order, np.int32), (ori_gptr, np.int32),
                                   (ori_grel, np.int16), (ori_gstart, np.int32), (ori_gcount, np.int32),
                                   (inv_col, np.int32), (inv_order, np.int32), (inv_gptr, np.int32),
                                   (inv_grel, np.int16), (inv_gstart, np.int32), (inv_gcount, np.int32))]
    u = lib().flo_hop_forward_edges(
        ctypes.c_int64(nnz), _p(row), _p(ent), _p(val), _p(w), ctypes.c_int64(L), ctypes.c_int64(n),
        ctypes.c_int64(E), ctypes.c_int64(r_size), *[_p(a) for a in arrs],
        None, None, _p(mask_triple), _p(ew), ctypes.c_int64(int(min(topk_edges, 1 << 62))),
        ctypes.c_int64(flags), ctypes.c_int64(-1),
        _p(out_key), _p(out_val), _p(f_entry), _p(f_rel), _p(f_m), _p(f_out), _p(f_edge), ctypes.byref(nf))
    nf = nf.value
    sum_keys = out_key[:u]
    f_entry, f_rel, f_m, f_edge = f_entry[:nf], f_rel[:nf], f_m[:nf], f_edge[:nf]
    keys = sum_keys[f_out[:nf]]
    # fact values as the fill writes them: (v * w) * m in fp32
    prod = (val[f_entry] * w.reshape(B * L, n)[row[f_entry], f_rel]).astype(np.float32)
    values = (prod * f_m).astype(np.float32)
    source = np.where(f_rel == n - 1, 2, np.where(f_rel >= r_size, 1, 0))
    ukeys, uvals, win = max_coalesce(keys, values, source, f_edge)
    fact_out = np.full(nf, -1, np.int64)
    fact_out[win] = np.arange(win.size)
    return dict(out_key=ukeys, out_val=uvals, n_facts=nf, fact_entry=f_entry, fact_rel=f_rel, fact_m=f_m,
                fact_edge=f_edge, fact_value=values, fact_source=source, fact_out=fact_out)


def dense_forward(A, w, csr, mask, r_size, topk_edges=1 << 60, wot_i=False, mode="sum", active=None):
    """Dense propagation of A [B, L, E] (flashlog.cpp:151-393 for SUM; the
    packed CAS-max of flashlog.cu:103-121, 523-637 for MAX): the outputs
    (out_ind, out_ori, out_inv) and the per-side facts.

    Sources are the nonzero entries of A over the active entities (those with a
    nonzero sum over the channels, flashlog_kernel.py:617-623); hidden edges
    (CSR mask 0) emit nothing.  SUM adds a side's facts per (row, destination)
    in source-entity, group and edge order; MAX keeps the fact whose fp32 bit
    pattern is largest, ties to the lower CSR position.
    """
    A = _c(A, np.float32)
    B, L, E = A.shape
    n = w.shape[-1]
    act = (A.sum(1) != 0).any(0) if active is None else np.isin(np.arange(E), active)
    Af = A.reshape(B * L, E)
    rows, ents = np.nonzero((Af != 0) & act[None, :])
    vals = Af[rows, ents]
    ori_rp, ori_col, _, ori_order, inv_rp, inv_col, _, inv_order = csr[:8]
    ori_gptr, ori_grel, ori_gstart, ori_gcount, inv_gptr, inv_grel, inv_gstart, inv_gcount = csr[8:]
    mo, mi = csr_masks(csr, mask, None)
    flags = SKIP_NONPOS_W | DROP_MASKED | WOT_I | (1024 if mode == "max" else 0)
    nnz = rows.size
    ent64 = _c(ents, np.int64)
    cap = max(int(lib().flo_fact_bound(ctypes.c_int64(nnz), _p(ent64), _p(_c(ori_rp, np.int32)),
                                        _p(_c(inv_rp, np.int32)))), 1)
    out_key = np.empty(cap, np.int64)
    out_val = np.empty(cap, np.float32)
    f_entry = np.empty(cap, np.int64)
    f_rel = np.empty(cap, np.int32)
    f_m = np.empty(cap, np.float32)
    f_out = np.empty(cap, np.int64)
    f_edge = np.empty(cap, np.int64)
    nf = ctypes.c_int64(0)
    arrs = [_c(a, t) for a, t in ((ori_col, np.int32), (ori_order, np.int32), (ori_gptr, np.int32),
                                   (ori_grel, np.int16), (ori_gstart, np.int32), (ori_gcount, np.int32),
                                   (inv_col, np.int32), (inv_order, np.int32), (inv_gptr, np.int32),
                                   (inv_grel, np.int16), (inv_gstart, np.int32), (inv_gcount, np.int32))]
    wr = _c(w.reshape(B, L, n), np.float32)
    u = lib().flo_hop_forward_edges(
        ctypes.c_int64(nnz), _p(_c(rows, np.int64)), _p(ent64), _p(_c(vals, np.float32)), _p(wr),
        ctypes.c_int64(L), ctypes.c_int64(n), ctypes.c_int64(E), ctypes.c_int64(r_size), *[_p(a) for a in arrs],
        _p(mo), _p(mi), None, None, ctypes.c_int64(int(min(topk_edges, 1 << 62))), ctypes.c_int64(flags),
        ctypes.c_int64(-1), _p(out_key), _p(out_val), _p(f_entry), _p(f_rel), _p(f_m), _p(f_out), _p(f_edge),
        ctypes.byref(nf))
    nf = nf.value
    f_entry, f_rel, f_m, f_edge = f_entry[:nf], f_rel[:nf], f_m[:nf], f_edge[:nf]
    keys = out_key[:u][f_out[:nf]]  # row * E + destination of every fact
    prod = (vals[f_entry] * wr.reshape(B * L, n)[rows[f_entry], f_rel]).astype(np.float32)
    fval = (prod * f_m).astype(np.float32)
    outs, side_facts = [], []
    for lo, hi in ((0, r_size), (r_size, 2 * r_size)):
        sel = np.nonzero((f_rel >= lo) & (f_rel < hi))[0]
        dense = np.zeros(B * L * E, np.float32)
        fout = np.full(nf, -1, np.int64)
        if mode == "max":
            bits = fval[sel].view(np.uint32).astype(np.int64)
            order = np.lexsort((f_edge[sel], -bits, keys[sel]))
            sk = keys[sel][order]
            first = np.ones(sk.size, bool)
            first[1:] = sk[1:] != sk[:-1]
            win = sel[order[first]]
            dense[keys[win]] = fval[win]
            fout[win] = keys[win]
        else:
            np.add.at(dense, keys[sel], fval[sel])  # in fact order
            fout[sel] = keys[sel]
        outs.append(dense.reshape(B, L, E))
        side_facts.append(fout)
    out_ind = np.zeros_like(A) if wot_i else (A * w.reshape(B, L, n)[..., n - 1:n]).astype(np.float32)
    return dict(out_ind=out_ind, out_ori=outs[0], out_inv=outs[1], rows=rows, ents=ents, vals=vals,
                fact_entry=f_entry, fact_rel=f_rel, fact_m=f_m, fact_dense=side_facts, n_facts=nf)


def dense_backward(fw, A, w, grad_ind, grad_ori, grad_inv, r_size, wot_i=False):
    """Gradients of the dense propagation (flashlog.cpp:222-283 for SUM; winning
    edges only for MAX, flashlog.cu:639-726)."""
    A = _c(A, np.float32)
    B, L, E = A.shape
    n = w.shape[-1]
    wr = w.reshape(B * L, n).astype(np.float32)
    gA = np.zeros(B * L * E, np.float64)
    gw = np.zeros((B * L, n), np.float64)
    if not wot_i:
        gi = np.asarray(grad_ind, np.float64).reshape(B * L, E)
        gA += (gi * wr[:, n - 1:n]).reshape(-1)
        gw[:, n - 1] += (gi * A.reshape(B * L, E)).sum(1)
    rows, ents, vals = fw["rows"], fw["ents"], fw["vals"]
    for side, g in ((0, grad_ori), (1, grad_inv)):
        gf = np.asarray(g, np.float64).reshape(-1)
        fo = fw["fact_dense"][side]
        sel = np.nonzero(fo >= 0)[0]
        e = fw["fact_entry"][sel]
        go = gf[fo[sel]]
        rel = fw["fact_rel"][sel]
        m = fw["fact_m"][sel].astype(np.float64)
        r = rows[e]
        np.add.at(gA, r * E + ents[e], go * wr[r, rel] * m)
        np.add.at(gw, (r, rel), go * vals[e] * m)
    return gA.reshape(B, L, E).astype(np.float32), gw.reshape(B, L, n).astype(np.float32)


def hop_backward(fw, g_out, row, val, w, r_size):
    """grad of the entry values and of w from a recorded forward (flashlog.cpp:991-1134)."""
    row, val, w = _c(row, np.int64), _c(val, np.float32), _c(w, np.float32)
    g_out = _c(g_out, np.float32)
    grad_v = np.empty(row.size, np.float32)
    grad_w = np.zeros(w.shape, np.float32)
    lib().flo_hop_backward(ctypes.c_int64(fw["n_facts"]), _p(fw["fact_entry"]), _p(fw["fact_rel"]),
                           _p(fw["fact_m"]), _p(fw["fact_out"]), _p(g_out), ctypes.c_int64(row.size),
                           _p(row), _p(val), _p(w), ctypes.c_int64(w.shape[-1]), ctypes.c_int64(r_size),
                           _p(grad_v), _p(grad_w))
    return grad_v, grad_w


def normalize_forward(out_row, x, rows, eps=1e-7):
    out_row, x = _c(out_row, np.int64), _c(x, np.float32)
    denom = np.empty(rows, np.float32)
    y = np.empty(x.size, np.float32)
    lib().flo_normalize_forward(ctypes.c_int64(x.size), _p(out_row), _p(x), ctypes.c_int64(rows),
                                ctypes.c_float(eps), _p(denom), _p(y))
    return y, denom


def normalize_backward(out_row, x, denom, g, eps=1e-7):
    out_row, x, denom, g = _c(out_row, np.int64), _c(x, np.float32), _c(denom, np.float32), _c(g, np.float32)
    gx = np.empty(x.size, np.float32)
    lib().flo_normalize_backward(ctypes.c_int64(x.size), _p(out_row), _p(x), _p(denom), _p(g),
                                 ctypes.c_int64(denom.size), ctypes.c_float(eps), _p(gx))
    return gx


def fixed_relation(b, l, e, v, ops, csr, r_size, E):
    """Rule step + coalesce-sum (flashlog.cu:1561-1741, flashlog_kernel.py:182-210)."""
    b, l, e, v = _c(b, np.int64), _c(l, np.int64), _c(e, np.int64), _c(v, np.float32)
    ops = _c(ops, np.int64)
    Bq, L = ops.shape
    arrs = [_c(csr[1], np.int32), _c(csr[8], np.int32), _c(csr[9], np.int16), _c(csr[10], np.int32),
            _c(csr[11], np.int32), _c(csr[5], np.int32), _c(csr[12], np.int32), _c(csr[13], np.int16),
            _c(csr[14], np.int32), _c(csr[15], np.int32)]
    args = [ctypes.c_int64(v.size), _p(b), _p(l), _p(e), _p(v), _p(ops), ctypes.c_int64(L),
            ctypes.c_int64(r_size), *[_p(a) for a in arrs]]
    nf = lib().flo_fixed_relation(*args, ctypes.c_int64(0), None, None, None, None)
    nf = int(nf)
    ob, ol, oe, ov = (np.empty(max(nf, 1), np.int64) for _ in range(3)), None, None, None
    ob = np.empty(max(nf, 1), np.int64)
    ol = np.empty(max(nf, 1), np.int64)
    oe = np.empty(max(nf, 1), np.int64)
    ov = np.empty(max(nf, 1), np.float32)
    lib().flo_fixed_relation(*args, ctypes.c_int64(nf), _p(ob), _p(ol), _p(oe), _p(ov))
    keys = (ob[:nf] * L + ol[:nf]) * E + oe[:nf]
    return coalesce_sum(keys, ov[:nf])


def max_product(sources, bodies, weights, csr, r_size, E, final_max=False):
    """Max-product rule scores (rules/shared_inference.py:12-245, reduction
    'max'): Boolean fixed-relation grounding of every (source, rule), per rank
    the largest weight of the rules reaching an entity, rows normalized by
    their sums, ranks combined by sum or max.  Returns (keys q * E + e, values)."""
    sources = np.asarray(sources, np.int64)
    weights = np.asarray(weights, np.float32)
    B, K, ranks = sources.size, len(bodies), weights.shape[1]
    acc = np.zeros((ranks, B * E), np.float32)
    for k, body in enumerate(bodies):
        keys = np.arange(B, dtype=np.int64) * E + sources
        for op in body:
            if keys.size == 0:
                break
            b, e = keys // E, keys % E
            ops_ = np.full((B, 1), int(op), np.int64)
            out, vals = fixed_relation(b, np.zeros_like(b), e, np.ones(b.size, np.float32), ops_, csr, r_size, E)
            keys = out[vals > 0]
        for r in range(ranks):
            np.maximum.at(acc[r], keys, weights[k, r])
    totals = acc.reshape(ranks, B, E).sum(-1, keepdims=True, dtype=np.float64).astype(np.float32)
    norm = (acc.reshape(ranks, B, E) / np.maximum(totals, np.float32(1e-30))).astype(np.float32)
    combined = (norm.max(0) if final_max else norm.sum(0)).reshape(-1)
    keys = np.nonzero(combined)[0]
    return keys, combined[keys]


def max_product_sparse(sources, bodies, weights, csr, r_size, E, final_max=False):
    """max_product without the dense [ranks, B, E] accumulator, for graphs
    with tens of millions of entities: the same Boolean grounding
    (flashlog.cu:1561-1741 then values > 0), per rank the largest weight of
    the rules reaching an entity (zero weights contribute nothing, as the
    dense accumulator's nonzero() drops them), rows normalized by their
    float64 sums clamped at 1e-30 (rules/evaluate.py:366-378), ranks combined
    by sum or max (rules/shared_inference.py:209-225).  Returns (keys, values)."""
    sources = np.asarray(sources, np.int64)
    weights = np.asarray(weights, np.float32)
    B, ranks = sources.size, weights.shape[1]
    reach_keys, reach_rule = [], []
    for k, body in enumerate(bodies):
        keys = np.arange(B, dtype=np.int64) * E + sources
        for op in body:
            if keys.size == 0:
                break
            b, e = keys // E, keys % E
            ops_ = np.full((B, 1), int(op), np.int64)
            out, vals = fixed_relation(b, np.zeros_like(b), e, np.ones(b.size, np.float32), ops_, csr, r_size, E)
            keys = out[vals > 0]
        reach_keys.append(keys)
        reach_rule.append(np.full(keys.size, k, np.int64))
    keys = np.concatenate(reach_keys) if reach_keys else np.zeros(0, np.int64)
    rule = np.concatenate(reach_rule) if reach_rule else np.zeros(0, np.int64)
    parts_k, parts_v = [], []
    for r in range(ranks):
        w = weights[rule, r]
        m = w > 0
        uk, inv = np.unique(keys[m], return_inverse=True)
        mx = np.zeros(uk.size, np.float32)
        np.maximum.at(mx, inv, w[m])
        tot = np.zeros(B, np.float64)
        np.add.at(tot, uk // E, mx.astype(np.float64))
        norm = (mx / np.maximum(tot.astype(np.float32), np.float32(1e-30))[uk // E]).astype(np.float32)
        parts_k.append(uk)
        parts_v.append(norm)
    allk = np.concatenate(parts_k)
    allv = np.concatenate(parts_v)
    uk, inv = np.unique(allk, return_inverse=True)
    out = np.zeros(uk.size, np.float32)
    if final_max:
        np.maximum.at(out, inv, allv)
    else:
        for pk, pv in zip(parts_k, parts_v):  # rank order, as the dense accumulation
            out[np.searchsorted(uk, pk)] += pv
    nz = out != 0
    return uk[nz], out[nz]


def coalesce_sum(keys, vals):
    keys, vals = _c(keys, np.int64), _c(vals, np.float32)
    ok = np.empty(max(keys.size, 1), np.int64)
    ov = np.empty(max(keys.size, 1), np.float32)
    u = lib().flo_coalesce_sum(ctypes.c_int64(keys.size), _p(keys), _p(vals), _p(ok), _p(ov))
    return ok[:u].copy(), ov[:u].copy()


def filtered_ranks(idx_b, idx_e, values, targets, filter_keys, B, E, use_eql=False):
    idx_b, idx_e = _c(idx_b, np.int64), _c(idx_e, np.int64)
    values, targets = _c(values, np.float32), _c(targets, np.int64)
    fk = _c(np.sort(np.asarray(filter_keys, np.int64)), np.int64)
    ranks = np.empty(B, np.float32)
    lib().flo_filtered_ranks(ctypes.c_int64(values.size), _p(idx_b), _p(idx_e), _p(values), _p(targets),
                             ctypes.c_int64(fk.size), _p(fk), ctypes.c_int64(B), ctypes.c_int64(E),
                             ctypes.c_int(int(bool(use_eql))), _p(ranks))
    return ranks


def sampled_takes(w_dir, grel, gcount, budget, seed, b, l, src, is_inv):
    """Per-group quotas of the sampled c2 path for one (entry, direction)."""
    w_dir, grel, gcount = _c(w_dir, np.float32), _c(grel, np.int16), _c(gcount, np.int32)
    take = np.empty(max(grel.size, 1), np.int32)
    lib().flo_sampled_takes(_p(w_dir), _p(grel), _p(gcount), ctypes.c_int64(0), ctypes.c_int64(grel.size),
                            ctypes.c_int64(budget), ctypes.c_int64(seed), ctypes.c_int64(b), ctypes.c_int64(l),
                            ctypes.c_int64(src), ctypes.c_int(int(bool(is_inv))), _p(take))
    return take[:grel.size]


def _splitmix64(z):
    """SplitMix64 output function (Steele, Lea and Flood, OOPSLA 2014) on uint64 arrays."""
    z = np.asarray(z, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def value_dropout(x, p, seed, counter=0, subseq=0):
    """nn.Dropout(p) on hop values (src/model_DRUM_kernel_sp.py:189-192) with
    the library's counter-based keep bits; returns (y, keep).

    key = splitmix64(seed ^ splitmix64((counter << 16) | subseq)); entry i is
    kept iff (splitmix64(key + i) >> 32) >= floor(p * 2^32); kept entries are
    x * float32(1 / float32(1 - p)) (torch's rounding of the scale), dropped
    ones x * 0.  The
    reference draws its mask from torch's generator, so parity with it is in
    distribution (keep rate 1 - p, the scale, the gradient through the same
    mask), and bit-exact against this restatement."""
    x = np.asarray(x, dtype=np.float32).reshape(-1)
    p = float(p)
    m64 = (1 << 64) - 1
    off = _splitmix64(np.array([((int(counter) << 16) | int(subseq)) & m64], dtype=np.uint64))
    key = _splitmix64(np.array([int(seed) & m64], dtype=np.uint64) ^ off)
    with np.errstate(over="ignore"):
        h = _splitmix64(key + np.arange(x.size, dtype=np.uint64))
    cut = (1 << 32) if p >= 1.0 else int(p * 4294967296.0)
    keep = (h >> np.uint64(32)) >= np.uint64(cut)
    scale = np.float32(0.0) if p >= 1.0 else np.float32(1.0 / float(np.float32(1.0 - p)))
    y = (x * np.where(keep, scale, np.float32(0.0))).astype(np.float32)  # dropped: x * 0, as in torch
    return y, keep
