"""Shared helpers for the parity tests (the oracle is the checker here)."""
import functools
import os
import sys

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

from flashlog_b200.synthetic import CONFIGS, load_or_generate  # noqa: E402
from oracle import oracle as O  # noqa: E402


@functools.lru_cache(maxsize=None)
def config1_graph():
    cfg = CONFIGS[1]
    train, valid, test = load_or_generate(cfg)
    csr = O.build_csr(train[:, 0], train[:, 2], train[:, 1], cfg.entities)
    return cfg, train, csr


def oracle_hop_norm(row, ent, val, w, csr, r_size, E, topk, use_topk, c1, mask, wot_i, mode=None,
                    eps=1e-7):
    """c1 -> expansion -> coalesce-sum -> row normalize, as the reference CPU path."""
    L = w.shape[1]
    rows = w.shape[0] * L
    kept = O.topc(row, val, c1) if (use_topk and c1 is not None and c1 >= 0) else None
    sel = np.arange(row.size) if kept is None else kept
    eff = topk if (use_topk and topk > 0) else (1 << 60)
    fw = O.hop_forward(row[sel], ent[sel], val[sel], w, csr, r_size, E, topk_edges=eff,
                       mode=O.MODE_CPU if mode is None else mode, mask=mask, wot_i=wot_i)
    out_row = fw["out_key"] // E
    y, denom = O.normalize_forward(out_row, fw["out_val"], rows, eps)
    return dict(sel=sel, fw=fw, out_row=out_row, y=y, denom=denom)


def oracle_hop_norm_backward(h, g, row, val, w, r_size, eps=1e-7):
    gx = O.normalize_backward(h["out_row"], h["fw"]["out_val"], h["denom"], g, eps)
    sel = h["sel"]
    gv_sel, gw = O.hop_backward(h["fw"], gx, row[sel], val[sel], w, r_size)
    gv = np.zeros(row.size, np.float32)
    gv[sel] = gv_sel
    return gv, gw
