"""The C oracle against golden vectors produced by the reference's own code.

These run on CPU.  They pin the checker that the GPU parity tests rely on.
"""
import hashlib

import numpy as np
import pytest

from helpers import O, config1_graph, oracle_hop_norm, oracle_hop_norm_backward


def test_csr_tiny_matches_reference(golden):
    d = golden("csr_tiny.npz")
    tri = d["triples"]
    csr = O.build_csr(tri[:, 0], tri[:, 2], tri[:, 1], int(d["E"]))
    for i, c in enumerate(csr):
        ref = d[f"f{i}"]
        assert c.dtype == ref.dtype, i
        assert np.array_equal(c, ref), i


def test_csr_config1_digests(golden):
    d = golden("csr_config1.npz")
    cfg, train, csr = config1_graph()
    assert hashlib.sha256(np.ascontiguousarray(train).tobytes()).hexdigest() == str(d["train_digest"])
    for i, c in enumerate(csr):
        assert hashlib.sha256(c.tobytes()).hexdigest() == str(d["digests"][i]), i


def test_csr_rejects_out_of_range():
    with pytest.raises(ValueError):
        O.build_side(np.array([0, 5]), np.array([1, 2]), np.array([0, 0]), 3)


def test_topc_matches_reference(golden):
    d = golden("topc.npz")
    for ci in range(int(d["n"])):
        kept = O.topc(d[f"c{ci}_row"], d[f"c{ci}_val"], int(d[f"c{ci}_c1"]))
        ref = d[f"c{ci}_kept"]
        if ref.size == 1 and ref[0] == -1:
            assert kept is None, ci
        else:
            assert kept is not None and np.array_equal(kept, ref), ci


@pytest.mark.parametrize("name", ["topk3_ties", "topk200", "notopk", "topk5_c1", "wot_i"])
def test_hop_forward_backward_matches_reference(golden, name):
    d = golden("hop_config1.npz")
    cfg, train, csr = config1_graph()
    E, R = cfg.entities, cfg.relations
    row, ent, val, w = d[f"{name}_row"], d[f"{name}_ent"], d[f"{name}_val"], d[f"{name}_w"]
    c1 = int(d[f"{name}_c1"])
    h = oracle_hop_norm(row, ent, val, w, csr, R, E, int(d[f"{name}_topk"]), bool(d[f"{name}_use_topk"]),
                        None if c1 < 0 else c1, d[f"{name}_mask"], bool(d[f"{name}_wot_i"]))
    assert np.array_equal(h["fw"]["out_key"], d[f"{name}_out_key"])
    # Expansion sums follow the reference's order exactly.
    assert np.array_equal(h["fw"]["out_val"], d[f"{name}_out_x"])
    np.testing.assert_allclose(h["y"], d[f"{name}_out_y"], rtol=1e-6, atol=0)
    gv, gw = oracle_hop_norm_backward(h, d[f"{name}_g"], row, val, w, R)
    np.testing.assert_allclose(gv, d[f"{name}_grad_v"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(gw, d[f"{name}_grad_w"], rtol=1e-5, atol=1e-6)


def test_normalize_matches_reference(golden):
    d = golden("normalize.npz")
    row = d["row"]
    y, denom = O.normalize_forward(row, d["val"], 15)
    np.testing.assert_array_equal(y, d["y"])
    gx = O.normalize_backward(row, d["val"], denom, d["g"])
    np.testing.assert_allclose(gx, d["grad"], rtol=1e-5, atol=1e-6)


def test_filtered_ranks_match_reference(golden):
    d = golden("ranks.npz")
    for ci in range(int(d["n"])):
        keys, B, E = d[f"r{ci}_keys"], int(d[f"r{ci}_B"]), int(d[f"r{ci}_E"])
        targets = d[f"r{ci}_targets"]
        filt = np.unique(np.concatenate([d[f"r{ci}_fb"] * E + d[f"r{ci}_fe"], np.arange(B) * E + targets]))
        ranks = O.filtered_ranks(keys // E, keys % E, d[f"r{ci}_vals"], targets, filt, B, E,
                                 bool(d[f"r{ci}_eql"]))
        hits = np.zeros(10)
        for r in ranks:
            hits += (float(r) <= np.arange(1, 11))
        np.testing.assert_allclose((1.0 / ranks.astype(np.float64)).sum(), float(d[f"r{ci}_mrr"]), rtol=1e-6)
        np.testing.assert_array_equal(hits, d[f"r{ci}_hits"])


def test_drum3_matches_reference(golden):
    """Three hops of the DRUM sparse model with deterministic c1/c2, readout and loss."""
    import torch
    d = golden("drum3_config1.npz")
    cfg, train, csr = config1_graph()
    E, R = cfg.entities, cfg.relations
    heads, tails = d["heads"], d["tails"]
    B, T, L, n = d["logits"].shape
    logits = torch.from_numpy(d["logits"]).requires_grad_(True)
    ws = [torch.softmax(logits[:, t], dim=-1) for t in range(T)]
    row = np.repeat(np.arange(B) * L, L) + np.tile(np.arange(L), B)
    ent = np.repeat(heads, L).astype(np.int64)
    val = np.ones(row.size, np.float32)
    states, hops = [], []
    c1, c2 = int(d["c1"]), int(d["c2"])
    for t in range(T):
        w = ws[t].detach().numpy()
        h = oracle_hop_norm(row, ent, val, w, csr, R, E, c2 // 2, True, c1, d["mask"], False)
        hops.append((h, row, val, w))
        row, ent, val = h["out_row"], h["fw"]["out_key"] % E, h["y"]
    b = row // L
    key = b * E + ent
    fk, fv = O.coalesce_sum(key, val)
    np.testing.assert_array_equal(fk, d["final_key"])
    np.testing.assert_allclose(fv, d["final_val"], rtol=1e-5, atol=1e-9)
    # loss = -mean(log(max(score(b, tail_b), 1e-7)))
    score = np.zeros(B, np.float32)
    for k, v in zip(fk, fv):
        if k % E == tails[k // E]:
            score[k // E] = v
    loss = -np.mean(np.log(np.maximum(score, 1e-7)))
    np.testing.assert_allclose(loss, float(d["loss"]), rtol=1e-5)
    # backward: dloss/dscore, through the three hops
    gscore = np.where(score > 1e-7, -1.0 / (B * np.maximum(score, 1e-7)), 0.0).astype(np.float32)
    g = np.array([gscore[r // L] if e == tails[r // L] else 0.0 for r, e in zip(row, ent)], np.float32)
    gws = []
    for h, hrow, hval, w in reversed(hops):
        gv, gw = oracle_hop_norm_backward(h, g, hrow, hval, w, R)
        gws.append(gw)
        g = gv
    gws = gws[::-1]
    total = sum((ws[t] * torch.from_numpy(gws[t])).sum() for t in range(T))
    total.backward()
    np.testing.assert_allclose(logits.grad.numpy(), d["grad_logits"], rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("name", ["max_ties", "max_topk200", "max_wot_i", "max_notopk"])
def test_max_coalesce_matches_reference(golden, name):
    """The MAX hop (FlashLogFunctionSparse3DTopKMax): outputs and exact winners
    (source, position within that source's raw facts) equal what the
    reference's _coalesce_sparse3d_max_raw_parts (flashlog_kernel.py:399-478)
    computed from the same raw facts."""
    g = golden("max_config1.npz")
    cfg, train, csr = config1_graph()
    E, R = cfg.entities, cfg.relations
    p = lambda k: g[f"{name}_{k}"]
    fw = O.hop_forward_max(p("row"), p("ent"), p("val"), p("w"), csr, R, E, topk_edges=int(p("topk")),
                           mask=p("mask"), wot_i=bool(p("wot_i")))
    assert np.array_equal(fw["out_key"], p("out_key"))
    assert np.array_equal(fw["out_val"], p("out_val"))
    win = np.nonzero(fw["fact_out"] >= 0)[0]
    win = win[np.argsort(fw["fact_out"][win])]
    src = fw["fact_source"]
    within = np.empty(src.size, np.int64)
    for s in range(3):
        sel = src == s
        within[sel] = np.arange(int(sel.sum()))
    assert np.array_equal(src[win], p("win_source"))
    assert np.array_equal(within[win], p("win_raw"))


def _dense_keep(A, c1):
    """Keep mask of the dense c1 of flashlog_kernel.py:814-842, through the oracle's c1."""
    B, L, E = A.shape
    Af = A.reshape(B * L, E)
    rows, ents = np.nonzero(Af != 0)
    kept = O.topc(rows, Af[rows, ents], c1)
    keep = np.ones(B * L * E, bool)
    if kept is None:
        return keep.reshape(A.shape)
    counts = np.bincount(rows, minlength=B * L)
    keep[np.repeat(counts > c1, E)] = False
    keep[rows[kept] * E + ents[kept]] = True
    return keep.reshape(A.shape)


@pytest.mark.parametrize("name", ["dense_plain", "dense_topk", "dense_wot_i", "dense_ties"])
def test_dense_sum_matches_reference(golden, name):
    """Dense propagation (FlashLogFunction): the oracle reproduces the reference
    CPU outputs bit for bit and its gradients to rounding."""
    g = golden("dense_config1.npz")
    cfg, train, csr = config1_graph()
    R = cfg.relations
    p = lambda k: g[f"{name}_{k}"]
    A = p("A")
    use_topk, c1, c2, wot_i = bool(p("use_topk")), int(p("c1")), int(p("c2")), bool(p("wot_i"))
    keep = _dense_keep(A, c1) if use_topk else np.ones(A.shape, bool)
    Ap = (A * keep).astype(np.float32)
    topk = c2 if (use_topk and c2 > 0) else 1 << 60
    fw = O.dense_forward(Ap, p("w"), csr, p("mask"), R, topk_edges=topk, wot_i=wot_i)
    assert np.array_equal(fw["out_ind"], p("s_i"))
    assert np.array_equal(fw["out_ori"], p("s_h"))
    assert np.array_equal(fw["out_inv"], p("s_t"))
    gA, gw = O.dense_backward(fw, Ap, p("w"), p("gi"), p("gh"), p("gt"), R, wot_i=wot_i)
    np.testing.assert_allclose(np.where(keep, gA, 0), p("grad_A"), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(gw, p("grad_w"), rtol=1e-5, atol=1e-6)


def _rule_bank(g, ci):
    lens = g[f"r{ci}_body_len"]
    flat = g[f"r{ci}_body"]
    bodies, k = [], 0
    for n in lens:
        bodies.append(tuple(int(x) for x in flat[k:k + n]))
        k += n
    return bodies, g[f"r{ci}_weights"]


@pytest.mark.parametrize("ci", [0, 1, 2])
def test_max_product_matches_reference(golden, ci):
    """Max-product rule scores: the oracle gives the entries and values of the
    reference's rules/shared_inference.py score(reduction='max')."""
    g = golden("maxproduct_config1.npz")
    cfg, train, csr = config1_graph()
    bodies, weights = _rule_bank(g, ci)
    keys, vals = O.max_product(g[f"r{ci}_sources"], bodies, weights, csr, cfg.relations, cfg.entities,
                               final_max=bool(g[f"r{ci}_final_max"]))
    assert np.array_equal(keys, g[f"r{ci}_key"])
    np.testing.assert_allclose(vals, g[f"r{ci}_val"], rtol=1e-5, atol=1e-9)


@pytest.mark.parametrize("ci", [0, 1, 2])
def test_sparse_max_product_oracle_matches_reference(golden, ci):
    """The oracle's sparse max-product (no dense accumulator, for 86M
    entities) gives the reference's score() entries and values too."""
    g = golden("maxproduct_config1.npz")
    cfg, train, csr = config1_graph()
    bodies, weights = _rule_bank(g, ci)
    keys, vals = O.max_product_sparse(g[f"r{ci}_sources"], bodies, weights, csr, cfg.relations, cfg.entities,
                                      final_max=bool(g[f"r{ci}_final_max"]))
    assert np.array_equal(keys, g[f"r{ci}_key"])
    np.testing.assert_allclose(vals, g[f"r{ci}_val"], rtol=1e-5, atol=1e-9)


def test_rule_bank_generator_shape():
    """The seeded rule bank: heads among the query relations, bodies of 1-3
    directed operators, weights in [0, 1), three groups; deterministic."""
    from flashlog_b200.synthetic import CONFIGS, evaluation_queries, load_or_generate, rule_bank
    cfg = CONFIGS[1]
    train, valid, test = load_or_generate(cfg)
    src, rel, dst = evaluation_queries(test, cfg.relations, 200)
    assert src.size == rel.size == dst.size == 400
    rb = rule_bank(train, rel, cfg.relations, 3000)
    assert rb == rule_bank(train, rel, cfg.relations, 3000)
    assert set(r["head"] for r in rb) <= set(rel.tolist())
    assert {len(r["body"]) for r in rb} == {1, 2, 3}
    assert all(0 <= o < 2 * cfg.relations for r in rb for o in r["body"])
    assert all(0.0 <= r["weight"] < 1.0 for r in rb) and {r["group_id"] for r in rb} == {0, 1, 2}


def test_filter_indices_oracle_matches_reference_golden(golden):
    """The oracle's known-answer lookup against the reference's own
    build_filter_indices_csr (training-CSR path): the same (query, entity)
    multiset."""
    d = golden("filter_config1.npz")
    cfg, train, csr_np = config1_graph()
    E = cfg.entities
    b, e = O.filter_indices(d["qx"], d["qr"], cfg.relations, csr_np)
    assert np.array_equal(np.sort(b * E + e), np.sort(d["csr_batch"] * E + d["csr_entity"]))


def test_dropout_oracle_keep_bits_and_torch_semantics():
    """The oracle's SplitMix64 against the published seed-0 sequence, and the
    dropout restatement against nn.Dropout's semantics (keep rate, torch's
    scale, x * 0 for dropped entries)."""
    import torch
    g = 0x9E3779B97F4A7C15
    seq = [int(O._splitmix64(np.array([(k * g) % (1 << 64)], np.uint64))[0]) for k in range(4)]
    assert seq == [0xE220A8397B1DCDAF, 0x6E789E6AA1B965F4, 0x06C45D188009454F, 0xF88BB8A8724C81EC]
    x = np.random.default_rng(5).standard_normal(200_000).astype(np.float32)
    for p in (0.1, 0.123, 0.5, 0.9):
        y, keep = O.value_dropout(x, p, seed=3, counter=1, subseq=2)
        n = x.size
        assert abs(keep.mean() - (1 - p)) < 5 * np.sqrt(p * (1 - p) / n)
        t = torch.nn.functional.dropout(torch.ones(4096), p, training=True)
        scale = float(t[t != 0][0])
        assert np.array_equal(y[keep], x[keep] * np.float32(scale))
        assert np.array_equal(np.signbit(y[~keep]), np.signbit(x[~keep])) and not y[~keep].any()
    assert np.array_equal(O.value_dropout(x, 0.0, 1)[0], x)
    assert not O.value_dropout(x, 1.0, 1)[0].any()
    # masks differ across counters and sub-sequences, and repeat for the same arguments
    k0 = O.value_dropout(x, 0.5, 9, 1, 0)[1]
    assert np.array_equal(k0, O.value_dropout(x, 0.5, 9, 1, 0)[1])
    assert not np.array_equal(k0, O.value_dropout(x, 0.5, 9, 2, 0)[1])
    assert not np.array_equal(k0, O.value_dropout(x, 0.5, 9, 1, 1)[1])


def test_edge_weight_grad_oracle_is_the_derivative_of_its_forward():
    """The oracle's edge-weight gradient (the formula of
    flashlog_kernel.py:1306-1336) against central differences of the oracle's
    own forward, whose facts the golden vectors pin: d/d ew of
    sum(g * out) = sum over facts of g * v * w * mask * sigmoid' (ew)."""
    cfg, train, csr = config1_graph()
    E, R = cfg.entities, cfg.relations
    n = 2 * R + 1
    rng = np.random.default_rng(17)
    B, L = 3, 2
    rows, ents = [], []
    for r in range(B * L):
        k = int(rng.integers(5, 25))
        rows.append(np.full(k, r))
        ents.append(np.sort(rng.choice(E, k, replace=False)))
    row = np.concatenate(rows).astype(np.int64)
    ent = np.concatenate(ents).astype(np.int64)
    val = rng.random(row.size).astype(np.float32)
    x = rng.standard_normal((B, L, n))
    w = (np.exp(x) / np.exp(x).sum(-1, keepdims=True)).astype(np.float32)
    mask = rng.random(train.shape[0]) > 0.1
    ew = rng.standard_normal(train.shape[0]).astype(np.float32)
    kw = dict(topk_edges=6, mode=O.MODE_TOPK, mask=mask)
    fw = O.hop_forward(row, ent, val, w, csr, R, E, edge_weight=ew, record_edges=True, **kw)
    g = rng.standard_normal(fw["out_key"].size)
    grad = O.edge_weight_grad(fw, g.astype(np.float32), row, val, w, ew)
    edges = np.unique(fw["fact_edge"][(fw["fact_rel"] < n - 1)])
    assert edges.size > 20
    delta = 1e-2
    for e in rng.choice(edges, 20, replace=False):
        lo, hi = ew.copy(), ew.copy()
        lo[e] -= delta
        hi[e] += delta
        f_lo = O.hop_forward(row, ent, val, w, csr, R, E, edge_weight=lo, **kw)
        f_hi = O.hop_forward(row, ent, val, w, csr, R, E, edge_weight=hi, **kw)
        assert np.array_equal(f_lo["out_key"], fw["out_key"]) and np.array_equal(f_hi["out_key"], fw["out_key"])
        fd = (np.dot(g, f_hi["out_val"].astype(np.float64)) - np.dot(g, f_lo["out_val"].astype(np.float64))) / (2 * delta)
        assert abs(fd - grad[e]) <= 2e-3 * abs(grad[e]) + 1e-5, (e, fd, grad[e])


def test_edge_weight_grad_oracle_max_winners_only():
    """MAX: only each destination's winning fact passes gradient
    (flashlog_kernel.py:1590-1614); central differences of the oracle's MAX
    forward agree wherever the perturbation leaves the winners unchanged."""
    cfg, train, csr = config1_graph()
    E, R = cfg.entities, cfg.relations
    n = 2 * R + 1
    rng = np.random.default_rng(23)
    B, L = 2, 2
    rows, ents = [], []
    for r in range(B * L):
        k = int(rng.integers(5, 20))
        rows.append(np.full(k, r))
        ents.append(np.sort(rng.choice(E, k, replace=False)))
    row = np.concatenate(rows).astype(np.int64)
    ent = np.concatenate(ents).astype(np.int64)
    val = rng.random(row.size).astype(np.float32)
    x = rng.standard_normal((B, L, n))
    w = (np.exp(x) / np.exp(x).sum(-1, keepdims=True)).astype(np.float32)
    mask = rng.random(train.shape[0]) > 0.1
    ew = rng.standard_normal(train.shape[0]).astype(np.float32)
    kw = dict(topk_edges=6, mask=mask)
    fw = O.hop_forward_max(row, ent, val, w, csr, R, E, edge_weight=ew, **kw)
    g = rng.standard_normal(fw["out_key"].size)
    grad = O.edge_weight_grad(fw, g.astype(np.float32), row, val, w, ew)
    won = (fw["fact_out"] >= 0) & (fw["fact_rel"] < n - 1)
    edges = np.unique(fw["fact_edge"][won])
    assert edges.size > 10
    delta, checked = 1e-3, 0
    for e in rng.choice(edges, min(20, edges.size), replace=False):
        lo, hi = ew.copy(), ew.copy()
        lo[e] -= delta
        hi[e] += delta
        f_lo = O.hop_forward_max(row, ent, val, w, csr, R, E, edge_weight=lo, **kw)
        f_hi = O.hop_forward_max(row, ent, val, w, csr, R, E, edge_weight=hi, **kw)
        if not (np.array_equal(f_lo["fact_out"], fw["fact_out"]) and np.array_equal(f_hi["fact_out"], fw["fact_out"])):
            continue  # a winner changed: the max is not differentiable across that step
        fd = (np.dot(g, f_hi["out_val"].astype(np.float64)) - np.dot(g, f_lo["out_val"].astype(np.float64))) / (2 * delta)
        assert abs(fd - grad[e]) <= 1e-2 * abs(grad[e]) + 1e-4, (e, fd, grad[e])
        checked += 1
    assert checked >= 10
    lost = np.setdiff1d(np.unique(fw["fact_edge"][(fw["fact_out"] < 0) & (fw["fact_rel"] < n - 1)]), edges)
    assert lost.size == 0 or not grad[lost].any()  # edges whose facts all lost get nothing
