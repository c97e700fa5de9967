"""The reference's OpenMP CPU path of one DRUM fwd+bwd step, timed on host cores.

TEST / BASELINE INFRASTRUCTURE ONLY: bench.py's cpu_baseline leg and its
--impl reference arm call this; the product never does.

The expansion, coalesce-sum, normalization and their backward run in the
reference's own CPU extension (flashlog_kernel/source/flashlog.cpp:1231-1933,
flashlog_forward_sparse3d_sum_norm_cpu / flashlog_backward_sparse3d_sum_norm_cpu,
compiled from its sources into oracle/_ref).  The c1 selection, which the
reference performs in Python/torch (flashlog_kernel.py:1092-1137), comes from
the C oracle's restatement of it.  When the reference build is missing, the
whole step runs in the C oracle (kind "port").
"""
from __future__ import annotations

import time

import numpy as np

from . import oracle as O
from . import reference as R


def _softmax(x):
    x = x - x.max(-1, keepdims=True)
    e = np.exp(x)
    return (e / e.sum(-1, keepdims=True)).astype(np.float32)


def drum_step(csr_np, heads, tails, w_all, mask, r_size, E, c1, c2, eps=1e-7, dropout=0.0, seed=0):
    """One 3-hop fwd+bwd step; returns (facts, loss, kind).

    dropout > 0 applies the models' training dropout to every hop's values
    (src/model_DRUM_kernel_sp.py:189-192: keep with probability 1 - p,
    scale kept values by 1 / (1 - p), the indices stay), with keep bits from
    numpy's generator seeded by `seed`; the backward applies the same mask."""
    import torch

    Q, T, N, n = w_all.shape
    topk = c2 // 2 if c2 > 0 else (1 << 60)
    use_ref = R.available()
    kind = "reference" if use_ref else "port"
    t = lambda a, d=torch.long: torch.from_numpy(np.ascontiguousarray(a)).to(d)
    mo, mi = O.csr_masks(csr_np, mask.astype(np.float32))
    row = np.arange(Q * N, dtype=np.int64)
    ent = np.repeat(heads, N).astype(np.int64)
    val = np.ones(row.size, np.float32)
    tape = []
    drops = []
    drop_rng = np.random.default_rng(seed)
    facts = 0
    for hop in range(T):
        w = np.ascontiguousarray(_softmax(w_all[:, hop]))
        kept = O.topc(row, val, c1) if c1 else None
        sel = np.arange(row.size) if kept is None else kept
        srow, sent, sval = row[sel], ent[sel], val[sel]
        if use_ref:
            M = R.module()
            c = csr_np
            res = M.flashlog_forward_sparse3d_sum_norm_cpu(
                t(srow // N), t(srow % N), t(sent), t(sval, torch.float32), t(w, torch.float32),
                t(c[1], torch.int32), t(mo, torch.float32), t(c[8], torch.int32), t(c[9], torch.int16),
                t(c[10], torch.int32), t(c[11], torch.int32),
                t(c[5], torch.int32), t(mi, torch.float32), t(c[12], torch.int32), t(c[13], torch.int16),
                t(c[14], torch.int32), t(c[15], torch.int32),
                Q, N, E, r_size, False, topk, float(eps), True)
            out_b, out_l, out_e, out_v = (x.numpy() for x in res[:4])
            facts += int(res[7].numel() + res[14].numel())
            tape.append((res, srow, sent, sval, w, sel, row.size))
            row = out_b * N + out_l
            ent, val = out_e, out_v
        else:
            fw = O.hop_forward(srow, sent, sval, w, csr_np, r_size, E, topk_edges=topk, mode=O.MODE_CPU, mask=mask)
            facts += int(fw["n_facts"] - srow.size)
            out_row = fw["out_key"] // E
            y, denom = O.normalize_forward(out_row, fw["out_val"], Q * N, eps)
            tape.append(((fw, out_row, denom), srow, sent, sval, w, sel, row.size))
            row, ent, val = out_row, fw["out_key"] % E, y
        if dropout > 0:
            keep = (drop_rng.random(val.size) >= dropout).astype(np.float32) * np.float32(1.0 / (1.0 - dropout))
            val = (val * keep).astype(np.float32)
            drops.append(keep)
        else:
            drops.append(None)
    # readout + loss (src/utils.py:36-47) and its gradient
    q = row // N
    hit = ent == tails[q]
    score = np.zeros(Q, np.float32)
    np.add.at(score, q[hit], val[hit])
    loss = float(-np.mean(np.log(np.maximum(score, 1e-7))))
    gscore = np.where(score > 1e-7, -1.0 / (Q * np.maximum(score, 1e-7)), 0.0).astype(np.float32)
    g = np.where(hit, gscore[q], 0.0).astype(np.float32)
    for (rec, srow, sent, sval, w, sel, n_in), keep in zip(reversed(tape), reversed(drops)):
        if keep is not None:
            g = (g * keep).astype(np.float32)
        if use_ref:
            res = rec
            M = R.module()
            ob, ol, oe = res[0], res[1], res[2]
            gv, gw = M.flashlog_backward_sparse3d_sum_norm_cpu(
                ob, ol, oe, t(g, torch.float32), res[4], res[5], res[6],
                t(srow // N), t(srow % N), t(sent), t(sval, torch.float32), t(w, torch.float32),
                *res[7:14], *res[14:21], res[21], Q, N, E, r_size, False, float(eps))
            gv = gv.numpy()
        else:
            fw, out_row, denom = rec
            gx = O.normalize_backward(out_row, fw["out_val"], denom, g, eps)
            gv, gw = O.hop_backward(fw, gx, srow, sval, w, r_size)
        full = np.zeros(n_in, np.float32)
        full[sel] = gv
        g = full
    return facts, loss, kind


def drum_step_trace(csr_np, heads, tails, w_hops, mask, r_size, E, c1, c2, eps=1e-7):
    """One 3-hop fwd+bwd step like drum_step, recording every hop for parity tests.

    w_hops[t] is hop t's attention [Q, N, n] as given (already a softmax), so a
    test can feed the exact fp32 weights its device step used.  Per hop the
    record holds the c1 selection (indices into the hop's input state), the
    output state (row, entity, normalized value), the gradient w.r.t. w and
    the gradient w.r.t. the hop's output values.  Forward and backward run in
    the reference's compiled CPU extension
    (flashlog.cpp:1231-1933), on one thread; c1 is the oracle's restatement
    of flashlog_kernel.py:1092-1137, itself pinned to that function's outputs.
    """
    import torch

    if not R.available():
        raise FileNotFoundError("the reference CPU extension (oracle/_ref) is not built")
    M = R.module()
    # one thread: the extension's parallel loops merge per-thread partial sums,
    # so its summation order (and last bits) would depend on the core count
    threads = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        return _trace(M, csr_np, heads, tails, w_hops, mask, r_size, E, c1, c2, eps)
    finally:
        torch.set_num_threads(threads)


def _trace(M, csr_np, heads, tails, w_hops, mask, r_size, E, c1, c2, eps):
    import torch

    Q, N, n = w_hops[0].shape
    T = len(w_hops)
    topk = c2 // 2 if c2 > 0 else (1 << 60)
    t = lambda a, d=torch.long: torch.from_numpy(np.ascontiguousarray(a)).to(d)
    mo, mi = O.csr_masks(csr_np, mask.astype(np.float32))
    c = csr_np
    row = np.arange(Q * N, dtype=np.int64)
    ent = np.repeat(np.asarray(heads, np.int64), N)
    val = np.ones(row.size, np.float32)
    hops = []
    for hop in range(T):
        w = np.ascontiguousarray(w_hops[hop], dtype=np.float32)
        kept = O.topc(row, val, c1) if c1 else None
        sel = np.arange(row.size) if kept is None else kept
        srow, sent, sval = row[sel], ent[sel], val[sel]
        res = M.flashlog_forward_sparse3d_sum_norm_cpu(
            t(srow // N), t(srow % N), t(sent), t(sval, torch.float32), t(w, torch.float32),
            t(c[1], torch.int32), t(mo, torch.float32), t(c[8], torch.int32), t(c[9], torch.int16),
            t(c[10], torch.int32), t(c[11], torch.int32),
            t(c[5], torch.int32), t(mi, torch.float32), t(c[12], torch.int32), t(c[13], torch.int16),
            t(c[14], torch.int32), t(c[15], torch.int32),
            Q, N, E, r_size, False, topk, float(eps), True)
        out_b, out_l, out_e, out_v = (x.numpy() for x in res[:4])
        hops.append(dict(sel=sel, n_in=row.size, res=res, srow=srow, sent=sent, sval=sval, w=w,
                         out_row=out_b * N + out_l, out_ent=out_e.astype(np.int64), y=out_v.copy(),
                         facts=int(res[7].numel() + res[14].numel())))
        row, ent, val = out_b * N + out_l, out_e.astype(np.int64), out_v
    q = row // N
    hit = ent == np.asarray(tails, np.int64)[q]
    score = np.zeros(Q, np.float32)
    np.add.at(score, q[hit], val[hit])
    loss = float(-np.mean(np.log(np.maximum(score, 1e-7))))
    gscore = np.where(score > 1e-7, -1.0 / (Q * np.maximum(score, 1e-7)), 0.0).astype(np.float32)
    g = np.where(hit, gscore[q], 0.0).astype(np.float32)
    for h in reversed(hops):
        res = h["res"]
        h["g_out"] = g
        gv, gw = M.flashlog_backward_sparse3d_sum_norm_cpu(
            res[0], res[1], res[2], t(g, torch.float32), res[4], res[5], res[6],
            t(h["srow"] // N), t(h["srow"] % N), t(h["sent"]), t(h["sval"], torch.float32),
            t(h["w"], torch.float32), *res[7:14], *res[14:21], res[21], Q, N, E, r_size, False, float(eps))
        h["gw"] = gw.numpy().reshape(Q, N, n)
        full = np.zeros(h["n_in"], np.float32)
        full[h["sel"]] = gv.numpy()
        g = full
    for h in hops:
        for k in ("res", "srow", "sent", "sval"):
            del h[k]
    return dict(hops=hops, loss=loss, score=score)


def time_sample(csr_np, batches, r_size, E, c1, c2, min_seconds=10.0, max_seconds=30.0, dropout=0.0):
    """Run whole steps over `batches` until min_seconds of CPU work; returns (facts/s, facts, seconds, steps, kind)."""
    facts = 0
    steps = 0
    t0 = time.perf_counter()
    kind = "port"
    while True:
        for heads, tails, w_all, mask in batches:
            f, _, kind = drum_step(csr_np, heads, tails, w_all, mask, r_size, E, c1, c2, dropout=dropout, seed=steps)
            facts += f
            steps += 1
            if time.perf_counter() - t0 >= max_seconds:
                break
        el = time.perf_counter() - t0
        if el >= min_seconds or el >= max_seconds:
            break
    el = time.perf_counter() - t0
    return facts / el, facts, el, steps, kind
