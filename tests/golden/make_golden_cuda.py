"""Record fixtures of the reference's CUDA-only paths by running its own CUDA code.

The reference's sampled c2 quotas (flashlog.cu:1458-1528), its deterministic
top-k fill (flashlog.cu:1368-1559), the fixed-relation rule step
(flashlog.cu:1561-1741), the dense MAX forward/backward (flashlog.cu:523-726,
997-1255) and the CSR-ordered mask gather (apply_mask_cuda,
flashlog.cu:1286-1340) have no CPU twin.  This script calls them through the
reference's extension compiled from its sources by oracle/build.py
(oracle/_ref/flashlog_ref_cuda*.so), with the argument preparation of the
reference's own Python glue (flashlog_kernel/flashlog_kernel.py, cited per
case), and saves inputs and raw outputs as one .npz fixture.

It runs on a GPU box (the extension needs a device).  The reference checkout
is not read at run time: the extension and the reference's CSR builder
(oracle/_ref/flashlog_ref_csr*.so) are prebuilt files.

Usage:  python tests/golden/make_golden_cuda.py --out tests/golden/ref_cuda.npz
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)


def load_reference_cuda():
    import torch  # noqa: F401  (the extension links against libtorch)
    from oracle import build as B
    path = B.ref_module_path("flashlog_ref_cuda")
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is not built (oracle/build.py build_reference_cuda)")
    spec = importlib.util.spec_from_file_location("flashlog_ref_cuda", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def hub_triples(seed=77, E=3000, R=300, m=60000, hubs=24):
    """A graph whose hub heads have hundreds of relation groups per side, so
    c2 thresholds go through more than 32 groups (the rank select)."""
    rng = np.random.default_rng(seed)
    h = np.where(rng.random(m) < 0.5, rng.integers(0, hubs, m), rng.integers(0, E, m))
    t = np.where(rng.random(m) < 0.3, rng.integers(0, hubs, m), rng.integers(0, E, m))
    r = rng.integers(0, R, m)
    tri = np.unique(np.stack([h, r, t], 1), axis=0)
    return tri[rng.permutation(tri.shape[0])].astype(np.int64), E, R


def config1_triples():
    from flashlog_b200.synthetic import CONFIGS, load_or_generate
    cfg = CONFIGS[1]
    train, _, _ = load_or_generate(cfg)
    return train.astype(np.int64), cfg.entities, cfg.relations


def state(rng, B, L, E, per_row, ties=False, hubs=None):
    rows, ents = [], []
    for r in range(B * L):
        k = int(rng.integers(1, per_row + 1))
        pool = E if hubs is None else hubs
        k = min(k, pool)
        rows.append(np.full(k, r))
        ents.append(np.sort(rng.choice(pool, k, replace=False)))
    row = np.concatenate(rows).astype(np.int64)
    ent = np.concatenate(ents).astype(np.int64)
    val = ((rng.integers(1, 5, row.size) / 4.0) if ties else rng.random(row.size) + 0.05).astype(np.float32)
    return row, ent, val


def attention(rng, B, L, n, ties):
    if ties:
        w = (rng.integers(0, 4, size=(B, L, n)) / 4.0).astype(np.float32)
        return w
    x = rng.standard_normal((B, L, n)).astype(np.float32)
    e = np.exp(x - x.max(-1, keepdims=True))
    return (e / e.sum(-1, keepdims=True)).astype(np.float32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(HERE, "ref_cuda.npz"))
    args = ap.parse_args()
    import torch
    from oracle import reference as Rf
    M = load_reference_cuda()
    dev = torch.device("cuda")
    out = {}

    def cu(a, dt=None):
        t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        return t if dt is None else t.to(dt)

    graphs = {"c1": config1_triples(), "hub": hub_triples()}
    csrs = {}
    for gname, (tri, E, R) in graphs.items():
        csr = Rf.build_csr(tri[:, 0], tri[:, 2], tri[:, 1], E)  # the reference's csr.cpp
        csrs[gname] = tuple(cu(c) for c in csr)
        if gname == "hub":
            out["hub_triples"] = tri.astype(np.int32)
            out["hub_E"], out["hub_R"] = np.int64(E), np.int64(R)

    # --- top-k fill, deterministic and sampled (flashlog_kernel.py:1158-1228 prepares
    # int64 COO coordinates, fp32 values and w, a bool mask and no edge weight) ---
    cases = []
    k = 0
    for gname, per_row, hubs in (("c1", 30, None), ("hub", 12, 24)):
        tri, E, R = graphs[gname]
        n = 2 * R + 1
        for topk in (2, 5, 40, 150):
            for ties in (False, True):
                for seed in (-1, 987654321123 + topk):
                    for wot_i in (False, True):
                        if gname == "hub" and wot_i:
                            continue
                        rng = np.random.default_rng(1000 + k)
                        B, L = 4, 3
                        row, ent, val = state(rng, B, L, E, per_row, ties=ties, hubs=hubs)
                        w = attention(rng, B, L, n, ties)
                        mask = rng.random(tri.shape[0]) > 0.1
                        c = csrs[gname]
                        res = M.flashlog_forward_sparse3d_topk_cuda(
                            cu(row // L), cu(row % L), cu(ent), cu(val), cu(w),
                            c[1], c[3], c[8], c[9], c[10], c[11],
                            c[5], c[7], c[12], c[13], c[14], c[15],
                            cu(mask), torch.empty(0, device=dev), B, L, E, R, wot_i, topk, False, seed)
                        torch.cuda.synchronize()
                        (ob, ol, oe, ov, ib, il, ie, iv, db, dl, de, dv, o_ent, o_rel, o_m, i_ent, i_rel, i_m,
                         o_off, i_off, o_edge, i_edge) = [x.cpu().numpy() for x in res]
                        p = f"t{k}_"
                        out.update({p + "graph": np.array(gname), p + "B": np.int64(B), p + "L": np.int64(L),
                                    p + "topk": np.int64(topk), p + "seed": np.int64(seed),
                                    p + "wot_i": np.int64(wot_i), p + "row": row, p + "ent": ent, p + "val": val,
                                    p + "w": w, p + "mask": mask.astype(np.uint8),
                                    p + "ori_e": oe, p + "ori_v": ov, p + "ori_entry": o_ent, p + "ori_rel": o_rel,
                                    p + "ori_m": o_m, p + "ori_edge": o_edge, p + "ori_off": o_off,
                                    p + "inv_e": ie, p + "inv_v": iv, p + "inv_entry": i_ent, p + "inv_rel": i_rel,
                                    p + "inv_m": i_m, p + "inv_edge": i_edge, p + "inv_off": i_off,
                                    p + "ind_e": de, p + "ind_v": dv})
                        cases.append(k)
                        k += 1
    out["topk_cases"] = np.array(cases, np.int64)

    # --- fixed-relation rule step (flashlog_kernel.py:182-210: COO coordinates of the
    # coalesced state, fp32 values, int64 operators) ---
    tri, E, R = graphs["c1"]
    c = csrs["c1"]
    fcases = []
    for j in range(3):
        rng = np.random.default_rng(500 + j)
        Bq, Lr = 5, 7
        row, ent, val = state(rng, Bq, Lr, E, 20)
        val = np.round(val * 4).astype(np.float32)
        ops_ = rng.integers(0, 2 * R + 1, size=(Bq, Lr))
        ops_[0, 0] = 2 * R
        res = M.flashlog_forward_sparse3d_fixed_relation_cuda(
            cu(row // Lr), cu(row % Lr), cu(ent), cu(val), cu(ops_),
            c[1], c[8], c[9], c[10], c[11], c[5], c[12], c[13], c[14], c[15], Bq, Lr, E, R)
        torch.cuda.synchronize()
        fb, fl, fe, fv = (x.cpu().numpy() for x in res)
        p = f"f{j}_"
        out.update({p + "B": np.int64(Bq), p + "L": np.int64(Lr), p + "row": row, p + "ent": ent, p + "val": val,
                    p + "ops": ops_, p + "out_b": fb, p + "out_l": fl, p + "out_e": fe, p + "out_v": fv})
        fcases.append(j)
    out["fixed_cases"] = np.array(fcases, np.int64)

    # --- dense MAX (FlashLogDenseMaxFunction, flashlog_kernel.py:992-1089): the
    # pruned A (the test's own dense c1 of the golden inputs), active nodes,
    # CSR-ordered masks from apply_mask_cuda, then forward and backward ---
    g = np.load(os.path.join(HERE, "dense_config1.npz"))
    sys.path.insert(0, os.path.dirname(HERE))
    from test_oracle_golden import _dense_keep
    for name in ("dense_plain", "dense_topk", "dense_ties"):
        q = lambda s: g[f"{name}_{s}"]
        use_topk, c1, c2, wot_i = bool(q("use_topk")), int(q("c1")), int(q("c2")), bool(q("wot_i"))
        A_np, w_np, mask = q("A"), q("w"), q("mask")
        keep = _dense_keep(A_np, c1) if use_topk else np.ones(A_np.shape, bool)
        Ap = (A_np * keep).astype(np.float32)
        Bd, Ld, Ed = Ap.shape
        A_flat = cu(Ap.reshape(Bd * Ld, Ed))
        w_flat = cu(w_np.reshape(Bd * Ld, -1))
        active = M.compute_active_nodes_cuda(A_flat)
        mask_f = cu(mask).bool()
        ori_mask = M.apply_mask_cuda(mask_f, c[3], torch.empty(0, device=dev))
        inv_mask = M.apply_mask_cuda(mask_f, c[7], torch.empty(0, device=dev))
        topk_edges = c2
        fwd = M.flashlog_forward_max_cuda(
            A_flat, w_flat, active, c[0], c[1], c[2], ori_mask, c[4], c[5], c[6], inv_mask,
            c[8], c[9], c[10], c[11], c[12], c[13], c[14], c[15], R, wot_i, use_topk, topk_edges)
        out_ind, out_ori, out_inv, ori_arg, inv_arg = fwd
        gi, gh, gt = (cu(q(s)) for s in ("gi", "gh", "gt"))
        gA, gw = M.flashlog_backward_max_cuda(
            gi.reshape(Bd * Ld, Ed), gh.reshape(Bd * Ld, Ed), gt.reshape(Bd * Ld, Ed), ori_arg, inv_arg,
            A_flat, w_flat, active, c[0], c[1], c[2], ori_mask, c[4], c[5], c[6], inv_mask,
            c[8], c[9], c[10], c[11], c[12], c[13], c[14], c[15], R, wot_i, use_topk, topk_edges)
        torch.cuda.synchronize()
        p = f"{name}_"
        out.update({p + "out_ind": out_ind.cpu().numpy().reshape(Bd, Ld, Ed),
                    p + "out_ori": out_ori.cpu().numpy().reshape(Bd, Ld, Ed),
                    p + "out_inv": out_inv.cpu().numpy().reshape(Bd, Ld, Ed),
                    p + "gA": gA.cpu().numpy().reshape(Bd, Ld, Ed), p + "gw": gw.cpu().numpy().reshape(Bd, Ld, -1)})

    # --- CSR-ordered masks with learnable edge weights (prepare_csr_masks with
    # --use_soft, flashlog_kernel.py:225-255 -> apply_mask_cuda) ---
    rng = np.random.default_rng(9)
    m = tri.shape[0]
    mask = rng.random(m) > 0.2
    ew = rng.standard_normal(m).astype(np.float32) * 2
    out["mask_mask"] = mask.astype(np.uint8)
    out["mask_weight"] = ew
    for label, wt in (("plain", torch.empty(0, device=dev)), ("soft", cu(ew))):
        mo = M.apply_mask_cuda(cu(mask).bool(), c[3], wt)
        mi = M.apply_mask_cuda(cu(mask).bool(), c[7], wt)
        torch.cuda.synchronize()
        out[f"mask_{label}_ori"] = mo.cpu().numpy()
        out[f"mask_{label}_inv"] = mi.cpu().numpy()

    os.makedirs(os.path.dirname(os.path.abspath(args.out)), exist_ok=True)
    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out}: {len(cases)} top-k cases, {len(fcases)} fixed-relation cases, 3 dense MAX cases, "
          f"2 mask cases; {os.path.getsize(args.out)} bytes")


if __name__ == "__main__":
    main()
