"""Generate golden vectors by running the reference's own code (build container only).

The reference's Python operator glue (flashlog_kernel/flashlog_kernel.py) and
the evaluation helper of src/main.py are imported read-only from the reference
checkout; their native module is the reference's CPU extension compiled from
its own sources by oracle/build.py (oracle/_ref), so no JIT build runs.  The
fixtures are small .npz files committed beside this script; the GPU box and the
CPU test suite read only the fixtures.

Usage:  python tests/golden/make_golden.py [--reference /path/to/reference]
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)


def _import_reference(ref_root):
    import torch  # noqa: F401
    from oracle import reference as R
    sys.path.insert(0, ref_root)
    sys.path.insert(0, os.path.join(ref_root, "src"))
    import flashlog_kernel.flashlog_kernel as fk
    fk._module = R.module("flashlog_ref_cpu")
    fk._csr_builder = R.module("flashlog_ref_csr")
    return fk


def _graph(E, R, m, seed):
    rng = np.random.default_rng(seed)
    h = rng.integers(0, E, m)
    t = np.minimum((rng.pareto(1.2, m) * E / 20).astype(np.int64), E - 1)
    r = rng.integers(0, R, m)
    tri = np.unique(np.stack([h, r, t], 1), axis=0)
    tri = tri[rng.permutation(tri.shape[0])]
    return tri


def _state(rng, B, L, E, per_row, zero_frac=0.1, ties=False, neg=False):
    rows, ents = [], []
    for r in range(B * L):
        k = int(rng.integers(1, per_row + 1))
        rows.append(np.full(k, r))
        ents.append(np.sort(rng.choice(E, k, replace=False)))
    row = np.concatenate(rows)
    ent = np.concatenate(ents)
    if ties:
        val = (rng.integers(0, 5, row.size) / 4.0).astype(np.float32)
    else:
        val = rng.random(row.size).astype(np.float32)
    if neg:
        val = np.where(rng.random(row.size) < 0.3, -val, val).astype(np.float32)
    val[rng.random(row.size) < zero_frac] = 0
    return row.astype(np.int64), ent.astype(np.int64), val


def _w(rng, B, L, n, ties):
    if ties:
        return (rng.integers(0, 4, size=(B, L, n)) / 4.0).astype(np.float32)
    x = rng.standard_normal((B, L, n)).astype(np.float32)
    e = np.exp(x - x.max(-1, keepdims=True))
    return (e / e.sum(-1, keepdims=True)).astype(np.float32)


def main():
    ap = argparse.ArgumentParser()
    from oracle.build import reference_root
    ap.add_argument("--reference", default=reference_root(),
                    help="reference checkout (default: $FLASHLOG_REFERENCE, else BASELINE.json reference_path)")
    ap.add_argument("--only", choices=["filter", "readout", "model"], help="write only this fixture")
    args = ap.parse_args()
    import torch
    torch.set_num_threads(1)
    fk = _import_reference(args.reference)
    if args.only == "filter":
        from flashlog_b200.synthetic import CONFIGS, load_or_generate
        import main as ref_main
        cfg = CONFIGS[1]
        train, valid, test = load_or_generate(cfg)
        csr1 = fk.build_csr_structure(torch.from_numpy(train[:, 0]), torch.from_numpy(train[:, 2]),
                                      torch.from_numpy(train[:, 1]), cfg.entities)
        filter_fixture(ref_main, cfg, train, valid, test, tuple(csr1))
        return
    if args.only == "readout":
        readout_fixture()
        return
    if args.only == "model":
        model_fixture()
        return
    out = {}

    # --- CSR: a tiny graph in full, the config-1 graph by digest -------------
    tri = _graph(60, 4, 400, 11)
    csr = fk.build_csr_structure(torch.from_numpy(tri[:, 0]), torch.from_numpy(tri[:, 2]),
                                 torch.from_numpy(tri[:, 1]), 60)
    np.savez_compressed(os.path.join(HERE, "csr_tiny.npz"), triples=tri, E=60,
                        **{f"f{i}": c.numpy() for i, c in enumerate(csr)})
    from flashlog_b200.synthetic import CONFIGS, load_or_generate
    cfg = CONFIGS[1]
    train, valid, test = load_or_generate(cfg)
    csr1 = fk.build_csr_structure(torch.from_numpy(train[:, 0]), torch.from_numpy(train[:, 2]),
                                  torch.from_numpy(train[:, 1]), cfg.entities)
    digests = np.array([hashlib.sha256(c.numpy().tobytes()).hexdigest() for c in csr1])
    train_digest = hashlib.sha256(np.ascontiguousarray(train).tobytes()).hexdigest()
    np.savez_compressed(os.path.join(HERE, "csr_config1.npz"), digests=digests,
                        train_digest=np.array(train_digest))

    # --- c1 selection (flashlog_kernel.py:1092-1137) ------------------------
    rng = np.random.default_rng(21)
    cases = {}
    for ci, (c1, ties, neg, per_row) in enumerate([(5, False, False, 12), (5, True, False, 12),
                                                   (3, True, True, 9), (0, False, False, 6),
                                                   (20, False, False, 12), (1, True, False, 4)]):
        row, ent, val = _state(rng, 4, 3, 500, per_row, ties=ties, neg=neg)
        t = lambda a: torch.from_numpy(a)
        kept = fk._sparse_topc_entries(t(row // 3), t(row % 3), t(ent), t(val), c1, 3)
        cases[f"c{ci}_row"] = row
        cases[f"c{ci}_ent"] = ent
        cases[f"c{ci}_val"] = val
        cases[f"c{ci}_c1"] = np.array(c1)
        cases[f"c{ci}_kept"] = np.array([-1]) if kept is None else kept.numpy()
    np.savez_compressed(os.path.join(HERE, "topc.npz"), n=np.array(6), **cases)

    # --- one hop forward + backward through the reference CPU operators -----
    E, Rr = cfg.entities, cfg.relations
    n = 2 * Rr + 1
    ctuple = tuple(c for c in csr1)
    rng = np.random.default_rng(31)
    hop = {}
    specs = [("topk3_ties", 3, True, 4, True, False), ("topk200", 200, False, 30, True, False),
             ("notopk", 0, False, 25, False, False), ("topk5_c1", 5, False, 40, True, True),
             ("wot_i", 4, True, 10, True, False)]
    for name, topk, ties, per_row, use_topk, with_c1 in specs:
        B, L = 4, 3
        row, ent, val = _state(rng, B, L, E, per_row, zero_frac=0.05)
        w = _w(rng, B, L, n, ties)
        mask = rng.random(train.shape[0]) > 0.15
        idx = torch.from_numpy(np.stack([row // L, row % L, ent]))
        v = torch.from_numpy(val).requires_grad_(True)
        wt = torch.from_numpy(w).requires_grad_(True)
        sp = torch.sparse_coo_tensor(idx, v, (B, L, E)).coalesce()
        c1 = 6 if with_c1 else None
        wot_i = name == "wot_i"
        y = fk.vectorized_operation_sparse3d_csr_sum_norm(
            sp, wt, ctuple, torch.from_numpy(mask), Rr, wot_i=wot_i, use_topk=use_topk,
            topk_edges=topk, topk_nodes=c1)
        yc = y.coalesce()
        g = torch.from_numpy(rng.standard_normal(yc.values().shape[0]).astype(np.float32))
        (yc.values() * g).sum().backward()
        x = fk.vectorized_operation_sparse3d_csr_sum(
            torch.sparse_coo_tensor(idx, torch.from_numpy(val), (B, L, E)).coalesce(),
            torch.from_numpy(w), ctuple, torch.from_numpy(mask), Rr, wot_i=wot_i,
            use_topk=use_topk, topk_edges=topk, topk_nodes=c1).coalesce()
        yi = yc.indices().numpy()
        hop.update({f"{name}_row": row, f"{name}_ent": ent, f"{name}_val": val, f"{name}_w": w,
                    f"{name}_mask": mask.astype(np.uint8), f"{name}_topk": np.array(topk),
                    f"{name}_use_topk": np.array(use_topk), f"{name}_c1": np.array(-1 if c1 is None else c1),
                    f"{name}_wot_i": np.array(wot_i),
                    f"{name}_out_key": (yi[0] * L + yi[1]) * E + yi[2],
                    f"{name}_out_y": yc.values().detach().numpy(),
                    f"{name}_out_x": x.values().numpy(),
                    f"{name}_g": g.numpy(), f"{name}_grad_v": v.grad.numpy(),
                    f"{name}_grad_w": wt.grad.numpy()})
    np.savez_compressed(os.path.join(HERE, "hop_config1.npz"), names=np.array([s[0] for s in specs]), **hop)

    # --- MAX coalesce (FlashLogFunctionSparse3DTopKMax, flashlog_kernel.py:1450-1518):
    # raw facts as the top-k fill emits them (hidden edges kept at value 0, the
    # triple id as tie key), from the C oracle, reduced by the reference's own
    # _coalesce_sparse3d_max_raw_parts (flashlog_kernel.py:399-478).
    from oracle import oracle as O
    csr_np = tuple(c.numpy() for c in csr1)
    rng = np.random.default_rng(35)
    mx = {}
    mspecs = [("max_ties", 3, True, 6, False), ("max_topk200", 200, False, 30, False),
              ("max_wot_i", 4, True, 10, True), ("max_notopk", 1 << 60, True, 8, False)]
    for name, topk, ties, per_row, wot_i in mspecs:
        B, L = 4, 3
        row, ent, val = _state(rng, B, L, E, per_row, zero_frac=0.05, ties=ties)
        w = _w(rng, B, L, n, ties)
        mask = (rng.random(train.shape[0]) > 0.2).astype(np.uint8)
        fw = O.hop_forward_max(row, ent, val, w, csr_np, Rr, E, topk_edges=topk, mask=mask, wot_i=wot_i)
        fb, fl_ = row[fw["fact_entry"]] // L, row[fw["fact_entry"]] % L
        # destination of every fact: the output it belongs to in the SUM coalesce of the same facts
        dst = np.empty(fw["n_facts"], np.int64)
        sfw = O.hop_forward(row, ent, val, w, csr_np, Rr, E, topk_edges=topk,
                            mode=O.SKIP_NONPOS_W | O.MASK_BY_TRIPLE, mask=mask, wot_i=wot_i)
        dst[:] = sfw["out_key"][sfw["fact_out"]] % E
        parts = []
        for src_id in range(3):
            sel = np.nonzero(fw["fact_source"] == src_id)[0]
            t = lambda a, d=torch.long: torch.from_numpy(np.ascontiguousarray(a)).to(d)
            parts.append((src_id, t(fb[sel]), t(fl_[sel]), t(dst[sel]), t(fw["fact_value"][sel], torch.float32),
                          t(fw["fact_edge"][sel])))
        sp, ukeys, win_source, win_raw, out_vals = fk._coalesce_sparse3d_max_raw_parts(tuple(parts), B, L, E)
        mx.update({f"{name}_row": row, f"{name}_ent": ent, f"{name}_val": val, f"{name}_w": w,
                   f"{name}_mask": mask, f"{name}_topk": np.array(min(topk, 1 << 62)),
                   f"{name}_wot_i": np.array(wot_i), f"{name}_out_key": ukeys.numpy(),
                   f"{name}_out_val": out_vals.numpy(), f"{name}_win_source": win_source.numpy(),
                   f"{name}_win_raw": win_raw.numpy()})
    np.savez_compressed(os.path.join(HERE, "max_config1.npz"), names=np.array([s[0] for s in mspecs]), **mx)

    # --- dense propagation (FlashLogFunction on the reference CPU path,
    # flashlog.cpp:151-393, with the dense c1 of flashlog_kernel.py:814-842)
    rng = np.random.default_rng(37)
    dn = {}
    dspecs = [("dense_plain", False, 0, 0, False), ("dense_topk", True, 6, 3, False),
              ("dense_wot_i", True, 4, 5, True), ("dense_ties", True, 3, 2, False)]
    for name, use_topk, c1, c2, wot_i in dspecs:
        B, L = 3, 3
        A = np.zeros((B, L, E), np.float32)
        for b in range(B):
            for l in range(L):
                k = int(rng.integers(4, 14))
                e = rng.choice(E, k, replace=False)
                A[b, l, e] = (rng.integers(1, 5, k) / 4.0) if name == "dense_ties" else rng.random(k)
        w = _w(rng, B, L, n, name == "dense_ties")
        mask = rng.random(train.shape[0]) > 0.15
        At = torch.from_numpy(A).requires_grad_(True)
        wt = torch.from_numpy(w).requires_grad_(True)
        s_i, s_h, s_t = fk.vectorized_operation_csr(At, wt, ctuple, torch.from_numpy(mask), Rr, wot_i=wot_i,
                                                    use_topk=use_topk, topk_nodes=c1, topk_edges=c2)
        gi = rng.standard_normal(A.shape).astype(np.float32)
        gh = rng.standard_normal(A.shape).astype(np.float32)
        gt = rng.standard_normal(A.shape).astype(np.float32)
        ((s_i * torch.from_numpy(gi)).sum() + (s_h * torch.from_numpy(gh)).sum() +
         (s_t * torch.from_numpy(gt)).sum()).backward()
        dn.update({f"{name}_A": A, f"{name}_w": w, f"{name}_mask": mask.astype(np.uint8),
                   f"{name}_use_topk": np.array(use_topk), f"{name}_c1": np.array(c1), f"{name}_c2": np.array(c2),
                   f"{name}_wot_i": np.array(wot_i), f"{name}_s_i": s_i.detach().numpy(),
                   f"{name}_s_h": s_h.detach().numpy(), f"{name}_s_t": s_t.detach().numpy(),
                   f"{name}_gi": gi, f"{name}_gh": gh, f"{name}_gt": gt, f"{name}_grad_A": At.grad.numpy(),
                   f"{name}_grad_w": wt.grad.numpy()})
    np.savez_compressed(os.path.join(HERE, "dense_config1.npz"), names=np.array([s[0] for s in dspecs]), **dn)

    # --- max-product rule-bank scores: the reference's own rules/shared_inference.py
    # score(reduction='max') on CPU; its CUDA-only fixed-relation step is the C
    # oracle's restatement of flashlog.cu:1561-1741.
    import types
    sys.path.insert(0, args.reference)
    import rules.evaluate as ref_ev
    from rules.max_inference import score as ref_max_score

    def cpu_fixed_relation(sp_state, operators, csr_struct, r_size):
        st = sp_state.coalesce()
        ix = st.indices().numpy()
        Bq, Lq, Eq = st.shape
        keys, vals = O.fixed_relation(ix[0], ix[1], ix[2], st.values().numpy(), operators.numpy(), csr_np, r_size,
                                      Eq)
        kk = torch.from_numpy(keys)
        return torch.sparse_coo_tensor(torch.stack([kk // (Lq * Eq), (kk // Eq) % Lq, kk % Eq]),
                                       torch.from_numpy(vals), (Bq, Lq, Eq), is_coalesced=True)

    ev = types.SimpleNamespace(**{k: getattr(ref_ev, k) for k in dir(ref_ev) if not k.startswith("__")})
    ev.vectorized_operation_sparse3d_fixed_relation = cpu_fixed_relation
    rng = np.random.default_rng(71)
    rb = {}
    for ci, (nrules, final_max, chunk) in enumerate([(40, False, 16), (40, True, 7), (25, False, 25)]):
        rules_ = []
        for k in range(nrules):
            blen = int(rng.integers(1, 4))
            body = tuple(int(x) for x in rng.integers(0, 2 * Rr, blen))
            if k % 9 == 0:
                body = body + (2 * Rr,)
            wts = rng.random(3).astype(np.float32)
            if k % 7 == 0:
                wts[int(rng.integers(0, 3))] = 0.0
            if k % 5 == 0:
                wts = np.round(wts * 4) / 4
            rules_.append({"body": body, "rank_weights": [float(x) for x in wts]})
        sources = torch.from_numpy(rng.choice(E, 10, replace=False).astype(np.int64))
        out = ref_max_score(ev, sources, rules_, ctuple, Rr, E, chunk, final_max=final_max,
                            dense_budget_bytes=1 << 28).coalesce()
        oi = out.indices().numpy()
        lens = np.array([len(r["body"]) for r in rules_])
        rb.update({f"r{ci}_sources": sources.numpy(), f"r{ci}_body_len": lens,
                   f"r{ci}_body": np.concatenate([np.array(r["body"], np.int64) for r in rules_]),
                   f"r{ci}_weights": np.array([r["rank_weights"] for r in rules_], np.float32),
                   f"r{ci}_final_max": np.array(final_max), f"r{ci}_chunk": np.array(chunk),
                   f"r{ci}_key": oi[0] * E + oi[1], f"r{ci}_val": out.values().numpy()})
    np.savez_compressed(os.path.join(HERE, "maxproduct_config1.npz"), n=np.array(3), **rb)

    # --- three-hop DRUM propagation + readout + loss (src/model_DRUM_kernel_sp.py:92-204)
    rng = np.random.default_rng(41)
    from flashlog_b200.synthetic import training_queries
    ids, qh, qr, qt = training_queries(train, cfg)
    qh, qr, qt = qh[:8], qr[:8], qt[:8]
    B, L, T = 8, 3, 3
    logits = rng.standard_normal((B, T, L, n)).astype(np.float32)
    mask = np.ones(train.shape[0], bool)
    mask[ids[:4]] = False
    lg = torch.from_numpy(logits).requires_grad_(True)
    sb = torch.arange(B).repeat_interleave(L)
    sl = torch.arange(L).repeat(B)
    se = torch.from_numpy(qh).repeat_interleave(L)
    state = torch.sparse_coo_tensor(torch.stack([sb, sl, se]), torch.ones(B * L), (B, L, E)).coalesce()
    c1, c2 = 30, 16
    for t in range(T):
        w_t = torch.softmax(lg[:, t], dim=-1)
        state = fk.vectorized_operation_sparse3d_csr_sum_norm(
            state, w_t, ctuple, torch.from_numpy(mask), Rr, use_topk=True, topk_edges=c2 // 2,
            topk_nodes=c1).coalesce()
    sidx = state.indices()
    final = torch.sparse_coo_tensor(torch.stack([sidx[0], sidx[2]]), state.values(), (B, E)).coalesce()
    from utils import log_loss_common_sp
    loss = log_loss_common_sp(final, torch.from_numpy(qt), E, 1.0)
    loss.backward()
    fi = final.indices().numpy()
    np.savez_compressed(os.path.join(HERE, "drum3_config1.npz"), heads=qh, rels=qr, tails=qt,
                        logits=logits, mask=mask.astype(np.uint8), c1=np.array(c1), c2=np.array(c2),
                        final_key=fi[0] * E + fi[1], final_val=final.values().detach().numpy(),
                        loss=np.array(loss.item(), np.float32), grad_logits=lg.grad.numpy())

    # --- normalize forward/backward (flashlog_kernel.py:536-607) ------------
    rng = np.random.default_rng(51)
    row, ent, val = _state(rng, 5, 3, 400, 30, zero_frac=0.0)
    val[:3] = 0.0
    idx = torch.from_numpy(np.stack([row // 3, row % 3, ent]))
    v = torch.from_numpy(val).requires_grad_(True)
    y = fk.normalize_sparse3d(torch.sparse_coo_tensor(idx, v, (5, 3, 400)).coalesce())
    g = torch.from_numpy(rng.standard_normal(val.size).astype(np.float32))
    (y.coalesce().values() * g).sum().backward()
    np.savez_compressed(os.path.join(HERE, "normalize.npz"), row=row, ent=ent, val=val,
                        y=y.coalesce().values().detach().numpy(), g=g.numpy(), grad=v.grad.numpy())

    # --- filtered ranks: MRR / hits of the CPU twin (src/main.py:391-466) ---
    import main as ref_main
    rng = np.random.default_rng(61)
    rk = {}
    for ci, use_eql in enumerate([False, True, True]):
        Bq, Eq = 16, 300
        keys = np.unique(rng.integers(0, Bq * Eq, 1200))
        vals = (rng.integers(0, 6, keys.size) / 5.0).astype(np.float32) if ci else rng.random(keys.size).astype(np.float32)
        targets = rng.integers(0, Eq, Bq)
        fb = rng.integers(0, Bq, 200)
        fe = rng.integers(0, Eq, 200)
        state = torch.sparse_coo_tensor(torch.from_numpy(np.stack([keys // Eq, keys % Eq])),
                                        torch.from_numpy(vals), (Bq, Eq)).coalesce()
        hits = np.zeros(10)
        mrr = ref_main.calculate_hits_full_sparse(state, [{"t": int(x)} for x in targets],
                                                  (torch.from_numpy(fb), torch.from_numpy(fe)), hits,
                                                  use_eql=use_eql)
        rk.update({f"r{ci}_keys": keys, f"r{ci}_vals": vals, f"r{ci}_targets": targets,
                   f"r{ci}_fb": fb, f"r{ci}_fe": fe, f"r{ci}_eql": np.array(use_eql),
                   f"r{ci}_mrr": np.array(mrr), f"r{ci}_hits": hits, f"r{ci}_B": np.array(Bq),
                   f"r{ci}_E": np.array(Eq)})
    np.savez_compressed(os.path.join(HERE, "ranks.npz"), n=np.array(3), **rk)

    filter_fixture(ref_main, cfg, train, valid, test, ctuple)
    print("golden fixtures written to", HERE)


def filter_fixture(ref_main, cfg, train, valid, test, ctuple):
    """Filter indices for filtered ranking (src/main.py:136-318): queries are
    every test triple in both directions (r and r + R) plus two heads outside
    the graph; the training-CSR path and the per-split lookup path (train,
    valid+test) of the reference itself."""
    import pandas as pd
    import torch
    E, R0 = cfg.entities, cfg.relations
    qx = np.concatenate([test[:, 0], test[:, 2], np.array([E + 3, E + 9])]).astype(np.int64)
    qr = np.concatenate([test[:, 1], test[:, 1] + R0, np.array([1, R0 + 2])]).astype(np.int64)
    fb, fe = ref_main.build_filter_indices_csr(torch.from_numpy(qx), torch.from_numpy(qr), R0, ctuple)

    class _Split:
        kg = pd.DataFrame(train)
        valid_data = pd.DataFrame(valid)
        test_data = pd.DataFrame(test)
        relation_size = R0
    lk, _, _ = ref_main.create_eval_filter_csr(_Split, E, "cpu")
    lb, le = ref_main.build_filter_indices_csr(torch.from_numpy(qx), torch.from_numpy(qr), R0, lk)
    np.savez_compressed(os.path.join(HERE, "filter_config1.npz"), qx=qx, qr=qr, csr_batch=fb.numpy(),
                        csr_entity=fe.numpy(), lookup_batch=lb.numpy(), lookup_entity=le.numpy())


def readout_fixture():
    """Channel readouts of the model files (src/model_DRUM_kernel_sp.py:22-28,
    src/model_mmDRUM_kernel_sp.py:17-32): outputs and the gradient of the
    values for a fixed upstream gradient, on states with channel ties."""
    import torch
    from model_DRUM_kernel_sp import sum_sp_3d
    from model_mmDRUM_kernel_sp import max_sp_3d
    out = {}
    for ci, (B, L, E, per_row, ties) in enumerate([(6, 3, 500, 60, False), (5, 3, 300, 120, True),
                                                  (4, 2, 2000, 400, True)]):
        rng = np.random.default_rng(81 + ci)
        row, ent, val = _state(rng, B, L, E, per_row, zero_frac=0.05, ties=ties)
        idx = torch.from_numpy(np.stack([row // L, row % L, ent]))
        for name, fn in (("sum", sum_sp_3d), ("max", max_sp_3d)):
            v = torch.from_numpy(val.copy()).requires_grad_(True)
            y = fn(torch.sparse_coo_tensor(idx, v, (B, L, E)).coalesce())
            g = torch.from_numpy(rng.standard_normal(y.values().numel()).astype(np.float32))
            (y.values() * g).sum().backward()
            yi = y.indices().numpy()
            out.update({f"c{ci}_{name}_key": yi[0] * E + yi[1], f"c{ci}_{name}_val": y.values().detach().numpy(),
                        f"c{ci}_{name}_g": g.numpy(), f"c{ci}_{name}_grad": v.grad.numpy()})
        out.update({f"c{ci}_row": row, f"c{ci}_ent": ent, f"c{ci}_val": val, f"c{ci}_shape": np.array([B, L, E])})
    np.savez_compressed(os.path.join(HERE, "readout.npz"), n=np.array(3), **out)


def model_fixture():
    """The reference's sparse DRUM model file (src/model_DRUM_kernel_sp.py,
    unmodified) on its CPU path with the reference's own operators: one
    forward (is_training=False, use_topk with c1 = 40, c2 = 16) and the
    log loss on a config-1 batch, then backward.  Records the attention
    logits the model's linear layer produced for each channel (hooked), the
    final [B, E] scores, the loss and the gradient of every logits tensor, so
    a test can drive the hops of the same forward through the drop-in."""
    import torch
    import model_DRUM_kernel_sp as M
    from flashlog_b200.synthetic import CONFIGS, load_or_generate, training_queries
    cfg = CONFIGS[1]
    train, _, _ = load_or_generate(cfg)
    E, R = cfg.entities, cfg.relations
    n = 2 * R + 1
    torch.manual_seed(1234)
    model = M.Model(n, 3, 3, E, train.shape[0], 32, use_gpu=False, dropout=0.0, c1=40, use_topk=True, c2=16)
    csr = M.build_csr_structure(torch.from_numpy(train[:, 0]), torch.from_numpy(train[:, 2]),
                                torch.from_numpy(train[:, 1]), E)
    ids, h, r, t = training_queries(train, cfg, step=5)
    h, r, t, ids = h[:24], r[:24], t[:24], ids[:12]
    mask = torch.ones(train.shape[0], dtype=torch.bool)
    mask[torch.from_numpy(ids)] = False
    logits = []

    def keep(_m, _i, o):
        o.retain_grad()
        logits.append(o)
    handle = model.linear.register_forward_hook(keep)
    final = model(torch.from_numpy(h), torch.from_numpy(r), None, None, None, is_training=False,
                  csr_struct=tuple(csr), mask_values=mask)
    loss = model.log_loss(final, torch.from_numpy(t))
    loss.backward()
    handle.remove()
    final = final.coalesce()
    fi = final.indices().numpy()
    out = {"heads": h, "rels": r, "tails": t, "hidden": ids, "loss": np.array(float(loss)),
           "final_key": fi[0] * E + fi[1], "final_val": final.values().detach().numpy(),
           "tau_1": np.array(float(model.tau_1)), "tau_2": np.array(float(model.tau_2)),
           "c1": np.array(40), "c2": np.array(16)}
    for l, o in enumerate(logits):
        out[f"logits{l}"] = o.detach().numpy()
        out[f"grad{l}"] = o.grad.numpy()
    np.savez_compressed(os.path.join(HERE, "model_drum_sp.npz"), **out)


if __name__ == "__main__":
    main()
