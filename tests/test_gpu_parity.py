"""Parity of the CUDA path (through the C ABI) with the oracle and the golden vectors.

Integer and index results (CSR, c1/c2 selections, output coordinates, ranks)
are compared bit for bit.  Expansion sums follow the reference CPU order and
are compared bit for bit as well; normalized values and gradients use the
north-star tolerance rel 1e-5.
"""
import numpy as np
import pytest

from helpers import O, config1_graph, oracle_hop_norm, oracle_hop_norm_backward

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

RTOL = 1e-5


@pytest.fixture(scope="module")
def fk():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import flashlog_b200.flashlog_kernel as fk
    from flashlog_b200 import _lib
    _lib.lib()
    return fk


@pytest.fixture(scope="module")
def g1(fk):
    cfg, train, csr_np = config1_graph()
    t = torch.from_numpy(train).cuda()
    csr = fk.build_csr_structure(t[:, 0], t[:, 2], t[:, 1], cfg.entities)
    return cfg, train, csr_np, csr


def _cuda(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def _state(rng, B, L, E, per_row, zero_frac=0.05, ties=False, neg=False):
    rows, ents = [], []
    for r in range(B * L):
        k = int(rng.integers(1, per_row + 1))
        rows.append(np.full(k, r))
        ents.append(np.sort(rng.choice(E, k, replace=False)))
    row = np.concatenate(rows).astype(np.int64)
    ent = np.concatenate(ents).astype(np.int64)
    val = ((rng.integers(0, 5, row.size) / 4.0) if ties else rng.random(row.size)).astype(np.float32)
    if neg:
        val = np.where(rng.random(row.size) < 0.3, -val, val).astype(np.float32)
    val[rng.random(row.size) < zero_frac] = 0
    return row, ent, val


def _w(rng, B, L, n, ties):
    if ties:
        return (rng.integers(0, 4, size=(B, L, n)) / 4.0).astype(np.float32)
    x = rng.standard_normal((B, L, n)).astype(np.float32)
    e = np.exp(x - x.max(-1, keepdims=True))
    return (e / e.sum(-1, keepdims=True)).astype(np.float32)


def _grad_w_exact(ref, g, row, val, w):
    """grad_w of a recorded oracle forward, accumulated in float64: the
    library's grad_w is the exactly rounded sum, while the fp32 sequential
    sum of the reference CPU (and the oracle) drifts with the term count."""
    f = ref["fact_out"] >= 0
    c = ref["fact_rel"][f].astype(np.int64)
    i = ref["fact_entry"][f]
    terms = g[ref["fact_out"][f]].astype(np.float64) * val[i].astype(np.float64) * ref["fact_m"][f].astype(np.float64)
    out = np.zeros(w.shape, np.float64).reshape(-1, w.shape[-1])
    np.add.at(out, (row[i], c), terms)
    return out.reshape(w.shape)


def _sp(row, ent, val, B, L, E, requires_grad=False):
    idx = _cuda(np.stack([row // L, row % L, ent]))
    v = _cuda(val).requires_grad_(requires_grad)
    return torch.sparse_coo_tensor(idx, v, (B, L, E), is_coalesced=True), v


def _keys(sp, L, E):
    i = sp.indices().cpu().numpy()
    return (i[0] * L + i[1]) * E + i[2]


# ---------------------------------------------------------------------------
def test_csr_build_matches_oracle(fk, g1):
    cfg, train, csr_np, csr = g1
    for i, (a, b) in enumerate(zip(csr, csr_np)):
        assert a.dtype == torch.from_numpy(b).dtype, i
        assert np.array_equal(a.cpu().numpy(), b), i


def test_csr_build_tiny_golden(fk, golden):
    d = golden("csr_tiny.npz")
    tri = _cuda(d["triples"])
    csr = fk.build_csr_structure(tri[:, 0], tri[:, 2], tri[:, 1], int(d["E"]))
    for i, c in enumerate(csr):
        assert np.array_equal(c.cpu().numpy(), d[f"f{i}"]), i


def test_csr_build_rejects_bad_ids(fk):
    with pytest.raises(ValueError):
        fk.build_csr_structure(_cuda(np.array([0, 7])), _cuda(np.array([1, 2])), _cuda(np.array([0, 0])), 4)


def test_topc_matches_oracle(fk):
    from flashlog_b200 import ops
    rng = np.random.default_rng(3)
    for c1, ties, neg in [(5, False, False), (5, True, False), (3, True, True), (0, False, False), (1, True, False),
                          (20, False, False)]:
        row, ent, val = _state(rng, 6, 3, 800, 40, ties=ties, neg=neg)
        rp, en, bad = ops.coo_to_rows(_cuda(row // 3), _cuda(row % 3), _cuda(ent), 6, 3, 800)
        assert int(bad.item()) == 0
        _, _, sel_val, src = ops.topc_select(rp, en, _cuda(val), c1)
        ref = O.topc(row, val, c1)
        ref = np.arange(row.size) if ref is None else ref
        assert np.array_equal(src.cpu().numpy(), ref), (c1, ties, neg)
        assert np.array_equal(sel_val.cpu().numpy(), val[ref])


def test_topc_golden(fk, golden):
    from flashlog_b200 import ops
    d = golden("topc.npz")
    for ci in range(int(d["n"])):
        row, ent, val, c1 = d[f"c{ci}_row"], d[f"c{ci}_ent"], d[f"c{ci}_val"], int(d[f"c{ci}_c1"])
        rp, en, _ = ops.coo_to_rows(_cuda(row // 3), _cuda(row % 3), _cuda(ent), 4, 3, 500)
        _, _, _, src = ops.topc_select(rp, en, _cuda(val), c1)
        ref = d[f"c{ci}_kept"]
        ref = np.arange(row.size) if (ref.size == 1 and ref[0] == -1) else ref
        assert np.array_equal(src.cpu().numpy(), ref), ci


def test_topc_sampled_scores(fk):
    """Sampled c1 keeps the c1 largest log(v) - log(noise) per row (flashlog_kernel.py:1125-1136)."""
    from flashlog_b200 import ops
    rng = np.random.default_rng(4)
    row, ent, val = _state(rng, 4, 3, 600, 50, zero_frac=0.1)
    rp, en, _ = ops.coo_to_rows(_cuda(row // 3), _cuda(row % 3), _cuda(ent), 4, 3, 600)
    c1 = 7
    ncand = ops.topc_candidates(rp, _cuda(val), c1)
    noise = rng.exponential(size=ncand)
    _, _, _, src = ops.topc_select(rp, en, _cuda(val), c1, noise=_cuda(noise))
    # numpy restatement of the exponential race
    keep = []
    k = 0
    for r in range(12):
        idx = np.flatnonzero(row == r)
        nz = idx[val[idx] != 0]
        if nz.size <= c1:
            keep.extend(idx.tolist())
            continue
        sc = np.log(val[nz].astype(np.float64)) - np.log(noise[k:k + nz.size])
        k += nz.size
        order = np.argsort(-sc, kind="stable")[:c1]
        keep.extend(sorted(nz[order].tolist()))
    assert np.array_equal(src.cpu().numpy(), np.array(sorted(keep)))


@pytest.mark.parametrize("topk,ties,wot_i", [(3, True, False), (7, False, False), (200, False, False),
                                             (1 << 60, True, False), (4, True, True)])
def test_hop_topk_forward_backward(fk, g1, topk, ties, wot_i):
    cfg, train, csr_np, csr = g1
    E, R = cfg.entities, cfg.relations
    n = 2 * R + 1
    rng = np.random.default_rng(topk % 97 + (5 if ties else 0) + (11 if wot_i else 0))
    B, L = 5, 3
    row, ent, val = _state(rng, B, L, E, 40)
    w = _w(rng, B, L, n, ties)
    mask = rng.random(train.shape[0]) > 0.15
    sp, v = _sp(row, ent, val, B, L, E, requires_grad=True)
    wt = _cuda(w).requires_grad_(True)
    out = fk.vectorized_operation_sparse3d_csr_sum(sp, wt, csr, _cuda(mask), R, wot_i=wot_i, use_topk=True,
                                                   topk_edges=topk)
    fw = O.hop_forward(row, ent, val, w, csr_np, R, E, topk_edges=topk, mode=O.MODE_TOPK, mask=mask, wot_i=wot_i)
    assert np.array_equal(_keys(out, L, E), fw["out_key"])
    assert np.array_equal(out.values().detach().cpu().numpy(), fw["out_val"])
    g = rng.standard_normal(fw["out_key"].size).astype(np.float32)
    (out.values() * _cuda(g)).sum().backward()
    gv, gw = O.hop_backward(fw, g, row, val, w, R)
    np.testing.assert_allclose(v.grad.cpu().numpy(), gv, rtol=RTOL, atol=1e-6)
    np.testing.assert_allclose(wt.grad.cpu().numpy(), gw, rtol=RTOL, atol=1e-6)


def _topk_apply(fn, sp, v, w, csr, mask, weight, R, topk, score):
    """The reference's 33-argument positional call of a top-k operator."""
    idx = sp.indices()
    B, L, E = sp.shape
    return fn.apply(idx[0], idx[1], idx[2], v, w, *csr, mask, weight, B, L, E, R, False, topk, score, None, True,
                    False)


@pytest.mark.parametrize("score", [False, True])
@pytest.mark.parametrize("op", ["sum", "max"])
def test_topk_learnable_edge_weights(fk, g1, op, score):
    """Learnable edge weights (--use_soft): the forward multiplies each fact by
    mask * sigmoid(ew) (or mask * ew for scores), and the weights' gradient
    is the reference's g * v * w * m * (1 - sigmoid(ew)) per fact that reached
    an output (flashlog_kernel.py:1306-1336; MAX: winners only, 1590-1614).
    Against the oracle: outputs, and the gradients of values, w and ew."""
    cfg, train, csr_np, csr = g1
    E, R = cfg.entities, cfg.relations
    n = 2 * R + 1
    rng = np.random.default_rng(41 + 2 * int(score) + (op == "max"))
    B, L, topk = 4, 3, 7
    row, ent, val = _state(rng, B, L, E, 30, zero_frac=0.0)
    w = _w(rng, B, L, n, False)
    mask = rng.random(train.shape[0]) > 0.15
    M = train.shape[0]
    ew = (rng.random(M) if score else rng.standard_normal(M)).astype(np.float32)
    sp, v = _sp(row, ent, val, B, L, E, requires_grad=True)
    wt = _cuda(w).requires_grad_(True)
    ewt = _cuda(ew).requires_grad_(True)
    fn = fk.FlashLogFunctionSparse3DTopKSum if op == "sum" else fk.FlashLogFunctionSparse3DTopKMax
    out = _topk_apply(fn, sp, v, wt, csr, _cuda(mask), ewt, R, topk, score)
    if op == "sum":
        fw = O.hop_forward(row, ent, val, w, csr_np, R, E, topk_edges=topk,
                           mode=O.MODE_TOPK | (O.EDGE_SCORE if score else 0), mask=mask, edge_weight=ew,
                           record_edges=True)
    else:
        fw = O.hop_forward_max(row, ent, val, w, csr_np, R, E, topk_edges=topk, mask=mask, edge_weight=ew,
                               edge_score=score)
    assert np.array_equal(_keys(out, L, E), fw["out_key"])
    np.testing.assert_allclose(out.values().detach().cpu().numpy(), fw["out_val"], rtol=RTOL, atol=0)
    g = rng.standard_normal(fw["out_key"].size).astype(np.float32)
    (out.values() * _cuda(g)).sum().backward()
    want = O.edge_weight_grad(fw, g, row, val, w, ew)
    assert np.count_nonzero(want) > 50
    got = ewt.grad.cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=1e-6 * np.abs(want).max())
    if op == "sum":
        gv, gw = O.hop_backward(fw, g, row, val, w, R)
        np.testing.assert_allclose(v.grad.cpu().numpy(), gv, rtol=RTOL, atol=1e-6)
        np.testing.assert_allclose(wt.grad.cpu().numpy(), gw, rtol=RTOL, atol=1e-6)


def test_edge_weights_without_a_mask_are_rejected(fk, g1):
    cfg, train, csr_np, csr = g1
    E, R = cfg.entities, cfg.relations
    rng = np.random.default_rng(3)
    row, ent, val = _state(rng, 2, 2, E, 10)
    sp, v = _sp(row, ent, val, 2, 2, E)
    w = _cuda(_w(rng, 2, 2, 2 * R + 1, False))
    with pytest.raises(ValueError):
        _topk_apply(fk.FlashLogFunctionSparse3DTopKSum, sp, v, w, csr, None,
                    torch.zeros(train.shape[0], device="cuda"), R, 5, False)


def test_hop_all_edges_forward_backward(fk, g1):
    cfg, train, csr_np, csr = g1
    E, R = cfg.entities, cfg.relations
    n = 2 * R + 1
    rng = np.random.default_rng(8)
    B, L = 4, 3
    row, ent, val = _state(rng, B, L, E, 30)
    w = _w(rng, B, L, n, False)
    w[0, 0, :3] = 0.0  # zero-weight groups still emit (zero-valued) facts on this path
    mask = (rng.random(train.shape[0]) > 0.2).astype(np.float32)
    sp, v = _sp(row, ent, val, B, L, E, requires_grad=True)
    wt = _cuda(w).requires_grad_(True)
    out = fk.vectorized_operation_sparse3d_csr_sum(sp, wt, csr, _cuda(mask), R, use_topk=False)
    fw = O.hop_forward(row, ent, val, w, csr_np, R, E, mode=O.MODE_ALL_EDGES, mask=mask)
    assert np.array_equal(_keys(out, L, E), fw["out_key"])
    assert np.array_equal(out.values().detach().cpu().numpy(), fw["out_val"])
    g = rng.standard_normal(fw["out_key"].size).astype(np.float32)
    (out.values() * _cuda(g)).sum().backward()
    gv, gw = O.hop_backward(fw, g, row, val, w, R)
    np.testing.assert_allclose(v.grad.cpu().numpy(), gv, rtol=RTOL, atol=1e-6)
    np.testing.assert_allclose(wt.grad.cpu().numpy(), gw, rtol=RTOL, atol=1e-6)


@pytest.mark.parametrize("name", ["topk3_ties", "topk200", "notopk", "topk5_c1", "wot_i"])
def test_sum_norm_matches_reference_golden(fk, g1, golden, name):
    """The fused sum+normalize operator against the reference CPU operator's own outputs."""
    d = golden("hop_config1.npz")
    cfg, train, csr_np, csr = g1
    E, R = cfg.entities, cfg.relations
    row, ent, val, w = d[f"{name}_row"], d[f"{name}_ent"], d[f"{name}_val"], d[f"{name}_w"]
    B, L = w.shape[0], w.shape[1]
    c1 = int(d[f"{name}_c1"])
    sp, v = _sp(row, ent, val, B, L, E, requires_grad=True)
    wt = _cuda(w).requires_grad_(True)
    y = fk.vectorized_operation_sparse3d_csr_sum_norm(
        sp, wt, csr, _cuda(d[f"{name}_mask"].astype(bool)), R, wot_i=bool(d[f"{name}_wot_i"]),
        use_topk=bool(d[f"{name}_use_topk"]), topk_edges=int(d[f"{name}_topk"]), topk_nodes=None if c1 < 0 else c1)
    keys = _keys(y, L, E)
    yv = y.values().detach().cpu().numpy()
    gkeys, gy, gg = d[f"{name}_out_key"], d[f"{name}_out_y"], d[f"{name}_g"]
    if bool(d[f"{name}_use_topk"]):
        assert np.array_equal(keys, gkeys)
        np.testing.assert_allclose(yv, gy, rtol=RTOL, atol=0)
        g = gg
    else:
        # Without budgets the CUDA all-edges path keeps hidden edges as explicit
        # zeros, the reference CPU path drops them: compare as value maps.
        nz = yv != 0
        assert np.array_equal(keys[nz], gkeys[gy != 0])
        np.testing.assert_allclose(yv[nz], gy[gy != 0], rtol=RTOL, atol=0)
        assert np.isin(gkeys, keys).all()
        g = np.zeros(keys.size, np.float32)
        g[np.searchsorted(keys, gkeys)] = gg
    (y.values() * _cuda(g)).sum().backward()
    np.testing.assert_allclose(v.grad.cpu().numpy(), d[f"{name}_grad_v"], rtol=RTOL, atol=1e-6)
    np.testing.assert_allclose(wt.grad.cpu().numpy(), d[f"{name}_grad_w"], rtol=RTOL, atol=1e-6)


def test_sum_norm_errors_and_own_outputs(fk, g1):
    """Out-of-range state indices raise ValueError and non-finite weights
    RuntimeError, before any expansion; a state the operator returned chains
    without the index check and gives the same result as a rebuilt copy."""
    cfg, train, csr_np, csr = g1
    E, R = cfg.entities, cfg.relations
    rng = np.random.default_rng(5)
    row, ent, val = _state(rng, 2, 3, E, 20)
    w = _cuda(_w(rng, 2, 3, 2 * R + 1, False))
    mask = torch.ones(train.shape[0], dtype=torch.bool, device="cuda")
    sp, _ = _sp(row, ent, val, 2, 3, E)
    kw = dict(use_topk=True, topk_edges=4, topk_nodes=10)
    idx = sp.indices().clone()
    idx[2, -1] = E + 5
    bad = torch.sparse_coo_tensor(idx, sp.values(), (2, 3, E), is_coalesced=True)
    with pytest.raises(ValueError):
        fk.vectorized_operation_sparse3d_csr_sum_norm(bad, w, csr, mask, R, **kw)
    wbad = w.clone()
    wbad[1, 2, 3] = float("nan")
    with pytest.raises(RuntimeError):
        fk.vectorized_operation_sparse3d_csr_sum_norm(sp, wbad, csr, mask, R, **kw)
    y = fk.vectorized_operation_sparse3d_csr_sum_norm(sp, w, csr, mask, R, **kw)
    y2 = fk.vectorized_operation_sparse3d_csr_sum_norm(y, w, csr, mask, R, **kw)
    copy = torch.sparse_coo_tensor(y.indices().clone(), y.values().clone(), y.shape, is_coalesced=True)
    y3 = fk.vectorized_operation_sparse3d_csr_sum_norm(copy, w, csr, mask, R, **kw)
    assert torch.equal(y2.indices(), y3.indices())
    assert torch.equal(y2.values(), y3.values())


def test_sum_norm_keeps_explicit_zeros_past_rows_times_c1(fk, g1):
    """A row with at most c1 nonzero values keeps all its entries, explicit
    zeros included (flashlog_kernel.py:1114-1117).  Here the kept total is
    far above rows * c1, so the operator's sync-free selection overflows and
    selects again at the input's size: outputs and gradients against the
    oracle."""
    cfg, train, csr_np, csr = g1
    E, R = cfg.entities, cfg.relations
    n = 2 * R + 1
    rng = np.random.default_rng(21)
    B, L, c1 = 2, 3, 6
    rows_, ents, vals = [], [], []
    for r in range(B * L):
        k = 30
        e = np.sort(rng.choice(E, k, replace=False))
        v = rng.random(k).astype(np.float32) + 0.1
        nz = 12 if r % 3 == 0 else 4  # rows 0 and 3 are over the limit; the others keep all 30 entries
        v[rng.permutation(k)[nz:]] = 0
        rows_.append(np.full(k, r))
        ents.append(e)
        vals.append(v)
    row = np.concatenate(rows_).astype(np.int64)
    ent = np.concatenate(ents).astype(np.int64)
    val = np.concatenate(vals).astype(np.float32)
    w = _w(rng, B, L, n, False)
    mask = rng.random(train.shape[0]) > 0.15
    sp, v = _sp(row, ent, val, B, L, E, requires_grad=True)
    wt = _cuda(w).requires_grad_(True)
    y = fk.vectorized_operation_sparse3d_csr_sum_norm(sp, wt, csr, _cuda(mask), R, use_topk=True, topk_edges=4,
                                                      topk_nodes=c1)
    h = oracle_hop_norm(row, ent, val, w, csr_np, R, E, 4, True, c1, mask, False, mode=O.MODE_TOPK)
    assert h["sel"].size > B * L * c1
    assert np.array_equal(_keys(y, L, E), h["fw"]["out_key"])
    np.testing.assert_allclose(y.values().detach().cpu().numpy(), h["y"], rtol=RTOL, atol=0)
    g = rng.standard_normal(h["y"].size).astype(np.float32)
    (y.values() * _cuda(g)).sum().backward()
    gv, gw = oracle_hop_norm_backward(h, g, row, val, w, R)
    np.testing.assert_allclose(v.grad.cpu().numpy(), gv, rtol=RTOL, atol=1e-6)
    np.testing.assert_allclose(wt.grad.cpu().numpy(), gw, rtol=RTOL, atol=1e-6)


def test_drum3_dropin_chain_matches_reference_golden(fk, g1, golden):
    """Three chained drop-in sum+normalize hops, as the reference model calls
    them, and the readout loss: outputs, loss and logits gradient against the
    reference's own run of the same chain.  Covers the c1 selection without a
    host sync and the gradient handed over on the output's own indices."""
    d = golden("drum3_config1.npz")
    cfg, train, csr_np, csr = g1
    E, R = cfg.entities, cfg.relations
    logits = _cuda(d["logits"]).requires_grad_(True)
    heads, tails = _cuda(d["heads"]), _cuda(d["tails"])
    B, T, L = logits.shape[0], logits.shape[1], logits.shape[2]
    sb = torch.arange(B, device="cuda").repeat_interleave(L)
    sl = torch.arange(L, device="cuda").repeat(B)
    se = heads.repeat_interleave(L)
    state = torch.sparse_coo_tensor(torch.stack([sb, sl, se]), torch.ones(B * L, device="cuda"), (B, L, E),
                                    is_coalesced=True)
    mask = _cuda(d["mask"].astype(bool))
    for t in range(T):
        state = fk.vectorized_operation_sparse3d_csr_sum_norm(
            state, torch.softmax(logits[:, t], dim=-1), csr, mask, R, use_topk=True, topk_edges=int(d["c2"]) // 2,
            topk_nodes=int(d["c1"]))
    idx, vals = state.indices(), state.values()
    hit = idx[2] == tails[idx[0]]
    score = torch.zeros(B, device="cuda").index_add(0, idx[0][hit], vals[hit])
    loss = -torch.mean(torch.log(torch.clamp(score, min=1e-7)))
    np.testing.assert_allclose(loss.item(), float(d["loss"]), rtol=RTOL)
    loss.backward()
    np.testing.assert_allclose(logits.grad.cpu().numpy(), d["grad_logits"], rtol=1e-4, atol=1e-6)
    final = torch.sparse_coo_tensor(torch.stack([idx[0], idx[2]]), vals.detach(), (B, E)).coalesce()
    fi = final.indices().cpu().numpy()
    assert np.array_equal(fi[0] * E + fi[1], d["final_key"])
    np.testing.assert_allclose(final.values().cpu().numpy(), d["final_val"], rtol=RTOL, atol=1e-7)


def test_drum3_engine_matches_reference_golden(fk, g1, golden):
    from flashlog_b200 import engine
    from flashlog_b200.ops import Graph
    d = golden("drum3_config1.npz")
    cfg, train, csr_np, csr = g1
    E, R = cfg.entities, cfg.relations
    logits = _cuda(d["logits"]).requires_grad_(True)
    heads, tails = _cuda(d["heads"]), _cuda(d["tails"])
    N = logits.shape[2]
    rp, ent, val = engine.drum_propagate(heads, logits, Graph.of(csr), R, c1=int(d["c1"]), c2=int(d["c2"]),
                                         mask_triple=_cuda(d["mask"]))
    loss = engine.readout_loss(rp, ent, val, tails, N)
    np.testing.assert_allclose(loss.item(), float(d["loss"]), rtol=RTOL)
    loss.backward()
    np.testing.assert_allclose(logits.grad.cpu().numpy(), d["grad_logits"], rtol=1e-4, atol=1e-6)
    # channel readout of the final state (buffers keep capacity; live count rp[-1])
    counts = (rp[1:] - rp[:-1]).cpu().numpy()
    live = int(rp[-1].item())
    row = np.repeat(np.arange(counts.size), counts)
    keys = (row // N) * E + ent[:live].cpu().numpy()
    fk_, fv_ = O.coalesce_sum(keys, val[:live].detach().cpu().numpy())
    assert np.array_equal(fk_, d["final_key"])
    np.testing.assert_allclose(fv_, d["final_val"], rtol=RTOL, atol=1e-9)


@pytest.mark.parametrize("nh", [2500, 500, 100])
def test_large_rows_histogram_and_dense_paths(fk, nh):
    """Rows above one shared-memory tile, a hub destination reached by nh x 6
    facts (2500: above a tile, dense windows; 500: a bin sorted by the whole
    block; 100: a bin sorted by one warp in shared memory) and a wide entity
    range."""
    from flashlog_b200 import ops
    from flashlog_b200.ops import Graph
    rng = np.random.default_rng(12 + nh)
    for E in (60_000, 5_000_000):
        R = 6
        m_rand = 120_000
        h = rng.integers(0, 30_000, m_rand)
        t = rng.integers(0, E, m_rand)
        r = rng.integers(0, R, m_rand)
        hub = E - 17
        hs = np.repeat(np.arange(nh), R)
        hr = np.tile(np.arange(R), nh)
        tri = np.unique(np.concatenate([np.stack([h, r, t], 1), np.stack([hs, hr, np.full(hs.size, hub)], 1)]), axis=0)
        csr_np = O.build_csr(tri[:, 0], tri[:, 2], tri[:, 1], E)
        tt = _cuda(tri)
        csr = fk.build_csr_structure(tt[:, 0], tt[:, 2], tt[:, 1], E)
        B, L = 2, 1
        ent = np.concatenate([np.arange(0, 2500), np.sort(rng.choice(np.arange(2500, 30_000), 1500, replace=False))])
        row = np.zeros(ent.size, np.int64)
        ent2 = np.sort(rng.choice(30_000, 300, replace=False))
        row = np.concatenate([row, np.ones(ent2.size, np.int64)])
        ent = np.concatenate([ent, ent2]).astype(np.int64)
        val = rng.random(ent.size).astype(np.float32)
        w = _w(rng, B, L, 2 * R + 1, False)
        mask = np.ones(tri.shape[0], np.uint8)
        rp, en, _ = ops.coo_to_rows(_cuda(row), _cuda(row * 0), _cuda(ent), B, L, E)
        fw = ops.hop_forward(rp, en, _cuda(val), _cuda(w), Graph.of(csr), R, 1 << 62,
                             1 | 2, mask_triple=_cuda(mask))
        ref = O.hop_forward(row, ent, val, w, csr_np, R, E, mode=O.MODE_TOPK, mask=mask)
        counts = (fw.out_row_ptr[1:] - fw.out_row_ptr[:-1]).cpu().numpy()
        keys = np.repeat(np.arange(B * L), counts) * E + fw.out_ent.cpu().numpy()
        assert ref["n_facts"] > 12288
        assert np.array_equal(keys, ref["out_key"]), E
        assert np.array_equal(fw.out_x.cpu().numpy(), ref["out_val"]), E
        # backward through the dense window as well
        g = rng.standard_normal(keys.size).astype(np.float32)
        gv, gw = ops.hop_backward(fw, rp, _cuda(val), _cuda(w), _cuda(g), normalize=False)
        rgv, _ = O.hop_backward(ref, g, row, val, w, R)
        np.testing.assert_allclose(gv.cpu().numpy(), rgv, rtol=RTOL, atol=1e-5)
        np.testing.assert_allclose(gw.cpu().numpy(), _grad_w_exact(ref, g, row, val, w), rtol=RTOL, atol=1e-5)


def test_sampled_c2_matches_oracle(fk, g1):
    from flashlog_b200 import ops, _lib as Lb
    from flashlog_b200.ops import Graph
    cfg, train, csr_np, csr = g1
    E, R = cfg.entities, cfg.relations
    rng = np.random.default_rng(21)
    B, L = 4, 3
    row, ent, val = _state(rng, B, L, E, 30, zero_frac=0.0)
    w = _w(rng, B, L, 2 * R + 1, False)
    mask = (rng.random(train.shape[0]) > 0.1).astype(np.uint8)
    seed = 987654321123
    rp, en, _ = ops.coo_to_rows(_cuda(row // L), _cuda(row % L), _cuda(ent), B, L, E)
    for topk in (2, 5, 40):
        fw = ops.hop_forward(rp, en, _cuda(val), _cuda(w), Graph.of(csr), R, topk,
                             Lb.FL_SKIP_NONPOS_W | Lb.FL_DROP_MASKED | Lb.FL_SAMPLED, mask_triple=_cuda(mask), seed=seed)
        ref = O.hop_forward(row, ent, val, w, csr_np, R, E, topk_edges=topk, mode=O.MODE_TOPK, mask=mask,
                            sampling_seed=seed)
        counts = (fw.out_row_ptr[1:] - fw.out_row_ptr[:-1]).cpu().numpy()
        keys = np.repeat(np.arange(B * L), counts) * E + fw.out_ent.cpu().numpy()
        assert np.array_equal(keys, ref["out_key"]), topk
        assert np.array_equal(fw.out_x.cpu().numpy(), ref["out_val"]), topk


def test_topk_rows_with_equal_weights(fk, g1):
    """Rows whose weights are equal bit for bit (queries of one relation, as
    in a training batch): the selections equal the oracle's."""
    from flashlog_b200 import ops, _lib as Lb
    from flashlog_b200.ops import Graph
    cfg, train, csr_np, csr = g1
    E, R = cfg.entities, cfg.relations
    rng = np.random.default_rng(23)
    B, L = 6, 3
    row, ent, val = _state(rng, B, L, E, 30, zero_frac=0.0)
    w = _w(rng, B, L, 2 * R + 1, False)
    w[2] = w[0]
    w[4] = w[0]
    w[5, 1] = w[3, 1]  # one channel row equal across queries
    mask = (rng.random(train.shape[0]) > 0.1).astype(np.uint8)
    rp, en, _ = ops.coo_to_rows(_cuda(row // L), _cuda(row % L), _cuda(ent), B, L, E)
    for topk in (2, 5, 40):
        fw = ops.hop_forward(rp, en, _cuda(val), _cuda(w), Graph.of(csr), R, topk,
                             Lb.FL_SKIP_NONPOS_W | Lb.FL_DROP_MASKED, mask_triple=_cuda(mask))
        ref = O.hop_forward(row, ent, val, w, csr_np, R, E, topk_edges=topk, mode=O.MODE_TOPK, mask=mask)
        counts = (fw.out_row_ptr[1:] - fw.out_row_ptr[:-1]).cpu().numpy()
        keys = np.repeat(np.arange(B * L), counts) * E + fw.out_ent.cpu().numpy()
        assert np.array_equal(keys, ref["out_key"]), topk
        assert np.array_equal(fw.out_x.cpu().numpy(), ref["out_val"]), topk


def test_normalize_matches_reference_golden(fk, golden):
    d = golden("normalize.npz")
    row, ent, val = d["row"], d["ent"], d["val"]
    sp, v = _sp(row, ent, val, 5, 3, 400, requires_grad=True)
    y = fk.normalize_sparse3d(sp)
    np.testing.assert_allclose(y.values().detach().cpu().numpy(), d["y"], rtol=RTOL, atol=0)
    (y.values() * _cuda(d["g"])).sum().backward()
    np.testing.assert_allclose(v.grad.cpu().numpy(), d["grad"], rtol=RTOL, atol=1e-6)


def test_fixed_relation_matches_oracle(fk, g1):
    cfg, train, csr_np, csr = g1
    E, R = cfg.entities, cfg.relations
    rng = np.random.default_rng(31)
    Bq, Lr = 5, 7
    row, ent, val = _state(rng, Bq, Lr, E, 20, zero_frac=0.0)
    val = np.round(val * 4).astype(np.float32)
    ops_ = rng.integers(0, 2 * R + 1, size=(Bq, Lr))
    ops_[0, 0] = 2 * R
    sp, _ = _sp(row, ent, val, Bq, Lr, E)
    out = fk.vectorized_operation_sparse3d_fixed_relation(sp, _cuda(ops_), csr, R)
    rk, rv = O.fixed_relation(row // Lr, row % Lr, ent, val, ops_, csr_np, R, E)
    assert np.array_equal(_keys(out, Lr, E), rk)
    assert np.array_equal(out.values().cpu().numpy(), rv)


def test_filtered_ranks_match_oracle_and_golden(fk, golden):
    d = golden("ranks.npz")
    for ci in range(int(d["n"])):
        keys, B, E = d[f"r{ci}_keys"], int(d[f"r{ci}_B"]), int(d[f"r{ci}_E"])
        targets = d[f"r{ci}_targets"]
        filt = np.unique(np.concatenate([d[f"r{ci}_fb"] * E + d[f"r{ci}_fe"], np.arange(B) * E + targets]))
        eql = bool(d[f"r{ci}_eql"])
        ranks = fk.sparse2d_filtered_ranks_cuda(_cuda(keys // E), _cuda(keys % E), _cuda(d[f"r{ci}_vals"]),
                                                _cuda(targets), _cuda(filt), B, E, eql).cpu().numpy()
        ref = O.filtered_ranks(keys // E, keys % E, d[f"r{ci}_vals"], targets, filt, B, E, eql)
        assert np.array_equal(ranks, ref)
        hits = np.zeros(10)
        for r in ranks:
            hits += (float(r) <= np.arange(1, 11))
        np.testing.assert_array_equal(hits, d[f"r{ci}_hits"])


def test_filtered_ranks_skip_queries_out_of_range(fk, golden):
    """A score entry or a filter key whose query lies outside [0, B) is
    skipped: the ranks equal those computed without it (the counters are
    never indexed by it)."""
    d = golden("ranks.npz")
    keys, B, E = d["r0_keys"], int(d["r0_B"]), int(d["r0_E"])
    targets = d["r0_targets"]
    filt = np.unique(np.concatenate([d["r0_fb"] * E + d["r0_fe"], np.arange(B) * E + targets]))
    vals = d["r0_vals"]
    want = fk.sparse2d_filtered_ranks_cuda(_cuda(keys // E), _cuda(keys % E), _cuda(vals), _cuda(targets),
                                           _cuda(filt), B, E, True).cpu().numpy()
    ib = np.concatenate([keys // E, [B, B + 5]])
    ie = np.concatenate([keys % E, [0, 1]])
    v = np.concatenate([vals, np.float32([0.5, 0.25])]).astype(np.float32)
    filt2 = np.concatenate([filt, [B * E + 3, (B + 7) * E]])
    # through the C ABI: the Python operator rejects such indices before the launch
    import ctypes
    from flashlog_b200 import _lib
    lb = _lib.lib()
    t = [_cuda(x) for x in (ib, ie, v, targets, filt2)]
    ranks = torch.empty(B, dtype=torch.float32, device="cuda")
    ws = torch.empty(lb.fl_filtered_ranks_workspace(B), dtype=torch.uint8, device="cuda")
    rc = lb.fl_filtered_ranks(t[0].data_ptr(), t[1].data_ptr(), t[2].data_ptr(), v.size, t[3].data_ptr(),
                              t[4].data_ptr(), filt2.size, B, E, 1, ranks.data_ptr(), ws.data_ptr(), ws.numel(),
                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    assert np.array_equal(ranks.cpu().numpy(), want)


def test_hop_is_deterministic(fk, g1):
    cfg, train, csr_np, csr = g1
    E, R = cfg.entities, cfg.relations
    rng = np.random.default_rng(41)
    row, ent, val = _state(rng, 6, 3, E, 200)
    w = _w(rng, 6, 3, 2 * R + 1, False)
    outs = []
    for _ in range(2):
        sp, v = _sp(row, ent, val, 6, 3, E, requires_grad=True)
        wt = _cuda(w).requires_grad_(True)
        y = fk.vectorized_operation_sparse3d_csr_sum_norm(sp, wt, csr, torch.ones(train.shape[0], dtype=torch.bool,
                                                                                  device="cuda"),
                                                          R, use_topk=True, topk_edges=6, topk_nodes=50)
        (y.values() * torch.arange(y.values().numel(), device="cuda").float().sin()).sum().backward()
        outs.append((y.indices().cpu().numpy(), y.values().detach().cpu().numpy(), v.grad.cpu().numpy(),
                     wt.grad.cpu().numpy()))
    for a, b in zip(outs[0], outs[1]):
        assert a.tobytes() == b.tobytes()


@pytest.mark.parametrize("R,ties", [(1100, True), (9000, True), (9000, False)])
@pytest.mark.parametrize("topk", [5, 40, 300])
def test_threshold_paths_and_visibility(fk, topk, R, ties):
    """Entries with <= 8, 9-32, 33-1024 and > 1024 relation groups per side
    (team, warp-register, staged and global threshold paths; rank bins of 3
    and 18 relations), tied and distinct weights, hidden triples read through
    `order` and through the CSR-ordered visibility: bit-identical to the
    oracle either way."""
    from flashlog_b200 import ops
    from flashlog_b200.ops import Graph
    rng = np.random.default_rng(77 + topk + R)
    E = 5000
    h = rng.integers(0, E, 60_000)
    r = rng.integers(0, R, 60_000)
    t = rng.integers(0, E, 60_000)
    parts = [np.stack([h, r, t], 1)]
    for hub in range(5):  # ori side: all 1100 relations (global path)
        parts.append(np.stack([np.full(R, hub), np.arange(R), rng.integers(0, E, R)], 1))
    for hub in range(5, 10):  # inv side: 600 relations (staged path), 3 edges each
        rr = np.repeat(np.arange(600), 3)
        parts.append(np.stack([rng.integers(0, E, rr.size), rr, np.full(rr.size, hub)], 1))
    for hub in range(10, 20):  # 20 relations (warp register path)
        rr = np.repeat(np.arange(20), 2)
        parts.append(np.stack([np.full(rr.size, hub), rr, rng.integers(0, E, rr.size)], 1))
    tri = np.unique(np.concatenate(parts), axis=0)
    csr_np = O.build_csr(tri[:, 0], tri[:, 2], tri[:, 1], E)
    tt = _cuda(tri)
    csr = fk.build_csr_structure(tt[:, 0], tt[:, 2], tt[:, 1], E)
    graph = Graph.of(csr)
    B, L = 2, 2
    rows_ = []
    ents_ = []
    for rrow in range(B * L):
        e = np.unique(np.concatenate([np.arange(20), rng.choice(E, 300, replace=False)]))
        rows_.append(np.full(e.size, rrow))
        ents_.append(e)
    row = np.concatenate(rows_).astype(np.int64)
    ent = np.concatenate(ents_).astype(np.int64)
    val = rng.random(ent.size).astype(np.float32)
    w = _w(rng, B, L, 2 * R + 1, ties)
    mask = (rng.random(tri.shape[0]) > 0.1).astype(np.uint8)
    ref = O.hop_forward(row, ent, val, w, csr_np, R, E, topk_edges=topk, mode=O.MODE_TOPK, mask=mask)
    rp, en, _ = ops.coo_to_rows(_cuda(row // L), _cuda(row % L), _cuda(ent), B, L, E)
    mt = _cuda(mask)
    for vis, rank_select in ((None, True), (ops.csr_visibility(graph, mt), True), (None, False)):
        fw = ops.hop_forward(rp, en, _cuda(val), _cuda(w), graph, R, topk, 1 | 2, mask_triple=mt, vis=vis,
                             rank_select=rank_select)
        counts = (fw.out_row_ptr[1:] - fw.out_row_ptr[:-1]).cpu().numpy()
        keys = np.repeat(np.arange(B * L), counts) * E + fw.out_ent.cpu().numpy()
        assert np.array_equal(keys, ref["out_key"])
        assert np.array_equal(fw.out_x.cpu().numpy(), ref["out_val"])
        g = rng.standard_normal(keys.size).astype(np.float32)
        gv, gw = ops.hop_backward(fw, rp, _cuda(val), _cuda(w), _cuda(g), normalize=False)
        rgv, rgw = O.hop_backward(ref, g, row, val, w, R)
        np.testing.assert_allclose(gv.cpu().numpy(), rgv, rtol=RTOL, atol=1e-5)
        np.testing.assert_allclose(gw.cpu().numpy(), rgw, rtol=RTOL, atol=1e-5)


@pytest.mark.parametrize("R", [7, 822, 14824])
def test_relation_rank(R):
    """fl_relation_rank: each relation's position in (w desc, id asc) order
    among the relations with w > 0, 0xffff (-1 as int16) for the others."""
    from flashlog_b200 import ops
    rng = np.random.default_rng(R)
    rows = 5
    w = (rng.integers(-2, 6, size=(rows, 2 * R + 1)) / 4.0).astype(np.float32)  # ties, zeros, negatives
    w[0] = rng.random(2 * R + 1).astype(np.float32)
    rank = ops.relation_rank(_cuda(w), R).cpu().numpy().reshape(rows, 2, R)
    for r in range(rows):
        for d in range(2):
            x = w[r, d * R:(d + 1) * R]
            want = np.full(R, -1, dtype=np.int16)
            pos = np.flatnonzero(x > 0)
            order = pos[np.lexsort((pos, -x[pos]))]
            want[order] = np.arange(order.size)
            assert np.array_equal(rank[r, d], want)


@pytest.mark.parametrize("name", ["max_ties", "max_topk200", "max_wot_i", "max_notopk"])
def test_sparse_max_matches_reference_golden(fk, g1, golden, name):
    """FlashLogFunctionSparse3DTopKMax: outputs equal the reference MAX
    coalesce (flashlog_kernel.py:399-478) fixture bit for bit; the backward
    reaches only the winning facts (flashlog.cu:2363-2406), as in the oracle."""
    cfg, train, csr_np, csr = g1
    E, R = cfg.entities, cfg.relations
    g = golden("max_config1.npz")
    p = lambda k: g[f"{name}_{k}"]
    row, ent, val, w, mask = p("row"), p("ent"), p("val"), p("w"), p("mask")
    B, L = w.shape[0], w.shape[1]
    topk, wot_i = int(p("topk")), bool(p("wot_i"))
    sp, v = _sp(row, ent, val, B, L, E, requires_grad=True)
    wt = _cuda(w).requires_grad_(True)
    out = fk.FlashLogFunctionSparse3DTopKMax.apply(
        sp.indices()[0], sp.indices()[1], sp.indices()[2], v, wt, *csr, _cuda(mask), None, B, L, E, R, wot_i, topk,
        False, None, True, False)
    assert np.array_equal(_keys(out, L, E), p("out_key"))
    assert np.array_equal(out.values().detach().cpu().numpy(), p("out_val"))
    ref = O.hop_forward_max(row, ent, val, w, csr_np, R, E, topk_edges=topk, mask=mask, wot_i=wot_i)
    gout = np.random.default_rng(3).standard_normal(ref["out_key"].size).astype(np.float32)
    (out.values() * _cuda(gout)).sum().backward()
    rgv, rgw = O.hop_backward(ref, gout, row, val, w, R)
    np.testing.assert_allclose(v.grad.cpu().numpy(), rgv, rtol=RTOL, atol=1e-6)
    np.testing.assert_allclose(wt.grad.cpu().numpy(), rgw, rtol=RTOL, atol=1e-6)


@pytest.mark.parametrize("reduce", ["sum", "max"])
def test_rows_of_many_duplicates(fk, reduce):
    """A row of ~100k facts over 2000 destinations (about 50 facts each):
    every destination bin is above the per-fact rank size, together above one
    block-wide sort, so they are sorted one warp per bin; against the oracle."""
    from flashlog_b200 import ops
    from flashlog_b200.ops import Graph
    rng = np.random.default_rng(31 if reduce == "sum" else 32)
    E, R = 2000, 4
    h = rng.integers(0, E, 110_000)
    t = rng.integers(0, E, 110_000)
    r = rng.integers(0, R, 110_000)
    tri = np.unique(np.stack([h, r, t], 1), axis=0)
    csr_np = O.build_csr(tri[:, 0], tri[:, 2], tri[:, 1], E)
    tt = _cuda(tri)
    csr = fk.build_csr_structure(tt[:, 0], tt[:, 2], tt[:, 1], E)
    ent = np.arange(E, dtype=np.int64)
    row = np.zeros(E, np.int64)
    val = ((rng.integers(1, 4, E) / 4.0) if reduce == "max" else rng.random(E)).astype(np.float32)
    w = _w(rng, 1, 1, 2 * R + 1, reduce == "max")
    mask = (rng.random(tri.shape[0]) > 0.05).astype(np.uint8)
    rp, en, _ = ops.coo_to_rows(_cuda(row), _cuda(row * 0), _cuda(ent), 1, 1, E)
    fw = ops.hop_forward(rp, en, _cuda(val), _cuda(w), Graph.of(csr), R, 1 << 62, 1, mask_triple=_cuda(mask),
                         reduce=reduce)
    if reduce == "max":
        ref = O.hop_forward_max(row, ent, val, w, csr_np, R, E, mask=mask)
        assert np.array_equal(fw.out_ent.cpu().numpy().astype(np.int64), ref["out_key"] % E)
    else:
        ref = O.hop_forward(row, ent, val, w, csr_np, R, E, mode=O.MODE_TOPK, mask=mask)
        counts = (fw.out_row_ptr[1:] - fw.out_row_ptr[:-1]).cpu().numpy()
        keys = np.repeat(np.arange(1), counts) * E + fw.out_ent.cpu().numpy()
        assert np.array_equal(keys, ref["out_key"])
    assert ref["n_facts"] > 100_000
    assert np.array_equal(fw.out_x.cpu().numpy(), ref["out_val"])
    g = rng.standard_normal(ref["out_key"].size).astype(np.float32)
    gv, gw = ops.hop_backward(fw, rp, _cuda(val), _cuda(w), _cuda(g), normalize=False)
    rgv, _ = O.hop_backward(ref, g, row, val, w, R)
    np.testing.assert_allclose(gv.cpu().numpy(), rgv, rtol=RTOL, atol=1e-5)
    np.testing.assert_allclose(gw.cpu().numpy(), _grad_w_exact(ref, g, row, val, w), rtol=RTOL, atol=1e-5)


@pytest.mark.parametrize("nh", [2500, 500, 100])
def test_sparse_max_large_rows(fk, nh):
    """MAX coalesce of rows above a tile with a hub destination of nh x 6
    facts (dense windows, a block-sorted bin, a warp-sorted bin), against the
    oracle."""
    from flashlog_b200 import ops
    from flashlog_b200.ops import Graph
    rng = np.random.default_rng(19 + nh)
    E, R = 60_000, 6
    h = rng.integers(0, 30_000, 120_000)
    t = rng.integers(0, E, 120_000)
    r = rng.integers(0, R, 120_000)
    hub = E - 17
    hs = np.repeat(np.arange(nh), R)
    hr = np.tile(np.arange(R), nh)
    tri = np.unique(np.concatenate([np.stack([h, r, t], 1), np.stack([hs, hr, np.full(hs.size, hub)], 1)]), axis=0)
    csr_np = O.build_csr(tri[:, 0], tri[:, 2], tri[:, 1], E)
    tt = _cuda(tri)
    csr = fk.build_csr_structure(tt[:, 0], tt[:, 2], tt[:, 1], E)
    ent = np.concatenate([np.arange(0, 2500), np.sort(rng.choice(np.arange(2500, 30_000), 1500, replace=False))])
    row = np.zeros(ent.size, np.int64)
    val = (rng.integers(1, 4, ent.size) / 4.0).astype(np.float32)  # ties in value
    w = _w(rng, 1, 1, 2 * R + 1, True)
    mask = (rng.random(tri.shape[0]) > 0.1).astype(np.uint8)
    rp, en, _ = ops.coo_to_rows(_cuda(row), _cuda(row * 0), _cuda(ent), 1, 1, E)
    fw = ops.hop_forward(rp, en, _cuda(val), _cuda(w), Graph.of(csr), R, 1 << 62, 1, mask_triple=_cuda(mask),
                         reduce="max")
    ref = O.hop_forward_max(row, ent, val, w, csr_np, R, E, mask=mask)
    assert np.array_equal(fw.out_ent.cpu().numpy().astype(np.int64), ref["out_key"] % E)
    assert np.array_equal(fw.out_x.cpu().numpy(), ref["out_val"])
    g = rng.standard_normal(ref["out_key"].size).astype(np.float32)
    gv, gw = ops.hop_backward(fw, rp, _cuda(val), _cuda(w), _cuda(g), normalize=False)
    rgv, _ = O.hop_backward(ref, g, row, val, w, R)
    np.testing.assert_allclose(gv.cpu().numpy(), rgv, rtol=RTOL, atol=1e-5)
    np.testing.assert_allclose(gw.cpu().numpy(), _grad_w_exact(ref, g, row, val, w), rtol=RTOL, atol=1e-5)


@pytest.mark.parametrize("name", ["dense_plain", "dense_topk", "dense_wot_i", "dense_ties"])
def test_dense_sum_matches_reference_golden(fk, g1, golden, name):
    """Dense propagation through vectorized_operation_csr and dense_csr_sum_cuda:
    outputs bit for bit equal to the reference CPU path, gradients to rel 1e-5."""
    cfg, train, csr_np, csr = g1
    R = cfg.relations
    g = golden("dense_config1.npz")
    p = lambda k: g[f"{name}_{k}"]
    use_topk, c1, c2, wot_i = bool(p("use_topk")), int(p("c1")), int(p("c2")), bool(p("wot_i"))
    for entry in (fk.vectorized_operation_csr, fk.dense_csr_sum_cuda):
        A = _cuda(p("A")).requires_grad_(True)
        w = _cuda(p("w")).requires_grad_(True)
        s_i, s_h, s_t = entry(A, w, csr, _cuda(p("mask")).bool(), R, wot_i=wot_i, use_topk=use_topk, topk_nodes=c1,
                              topk_edges=c2)
        assert np.array_equal(s_i.detach().cpu().numpy(), p("s_i"))
        assert np.array_equal(s_h.detach().cpu().numpy(), p("s_h"))
        assert np.array_equal(s_t.detach().cpu().numpy(), p("s_t"))
        ((s_i * _cuda(p("gi"))).sum() + (s_h * _cuda(p("gh"))).sum() + (s_t * _cuda(p("gt"))).sum()).backward()
        np.testing.assert_allclose(A.grad.cpu().numpy(), p("grad_A"), rtol=RTOL, atol=1e-6)
        np.testing.assert_allclose(w.grad.cpu().numpy(), p("grad_w"), rtol=RTOL, atol=1e-6)


@pytest.mark.parametrize("name", ["dense_plain", "dense_topk", "dense_ties"])
def test_dense_max_matches_oracle(fk, g1, golden, name):
    """dense_csr_max: per direction the fact with the largest fp32 bit pattern,
    ties to the lower CSR position (flashlog.cu:103-121, 523-637); gradients to
    the winning edges only (flashlog.cu:639-726)."""
    cfg, train, csr_np, csr = g1
    R = cfg.relations
    g = golden("dense_config1.npz")
    p = lambda k: g[f"{name}_{k}"]
    use_topk, c1, c2, wot_i = bool(p("use_topk")), int(p("c1")), int(p("c2")), bool(p("wot_i"))
    A_np, w_np, mask = p("A"), p("w"), p("mask")
    A = _cuda(A_np).requires_grad_(True)
    w = _cuda(w_np).requires_grad_(True)
    s_i, s_h, s_t = fk.dense_csr_max(A, w, csr, _cuda(mask).bool(), R, wot_i=wot_i, use_topk=use_topk,
                                     topk_nodes=c1, topk_edges=c2)
    from test_oracle_golden import _dense_keep
    keep = _dense_keep(A_np, c1) if use_topk else np.ones(A_np.shape, bool)
    Ap = (A_np * keep).astype(np.float32)
    topk = c2 if (use_topk and c2 > 0) else 1 << 60
    ref = O.dense_forward(Ap, w_np, csr_np, mask, R, topk_edges=topk, wot_i=wot_i, mode="max")
    assert np.array_equal(s_i.detach().cpu().numpy(), ref["out_ind"])
    assert np.array_equal(s_h.detach().cpu().numpy(), ref["out_ori"])
    assert np.array_equal(s_t.detach().cpu().numpy(), ref["out_inv"])
    gi, gh, gt = p("gi"), p("gh"), p("gt")
    ((s_i * _cuda(gi)).sum() + (s_h * _cuda(gh)).sum() + (s_t * _cuda(gt)).sum()).backward()
    rgA, rgw = O.dense_backward(ref, Ap, w_np, gi, gh, gt, R, wot_i=wot_i)
    np.testing.assert_allclose(A.grad.cpu().numpy(), np.where(keep, rgA, 0), rtol=RTOL, atol=1e-6)
    np.testing.assert_allclose(w.grad.cpu().numpy(), rgw, rtol=RTOL, atol=1e-6)


@pytest.mark.parametrize("ci", [0, 1, 2])
def test_max_product_matches_reference_golden(fk, g1, golden, ci):
    """flashlog_b200.rules.score (max-product rule bank, smDRUM sum / mmDRUM max
    over ranks) against the reference's own score(reduction='max')."""
    from flashlog_b200 import rules as RB
    from test_oracle_golden import _rule_bank
    cfg, train, csr_np, csr = g1
    g = golden("maxproduct_config1.npz")
    bodies, weights = _rule_bank(g, ci)
    rules = [{"body": b, "rank_weights": [float(x) for x in w]} for b, w in zip(bodies, weights)]
    out = RB.score(None, _cuda(g[f"r{ci}_sources"]), rules, csr, cfg.relations, cfg.entities,
                   int(g[f"r{ci}_chunk"]), final_max=bool(g[f"r{ci}_final_max"])).coalesce()
    oi = out.indices().cpu().numpy()
    assert np.array_equal(oi[0] * cfg.entities + oi[1], g[f"r{ci}_key"])
    np.testing.assert_allclose(out.values().cpu().numpy(), g[f"r{ci}_val"], rtol=RTOL, atol=1e-9)


@pytest.mark.parametrize("rows", [1, 7, 1536, 5000, 16384])
def test_row_order_is_a_stable_descending_argsort(fk, rows):
    """fl_row_order: rows by descending slot count, ties to the lower row."""
    import ctypes
    from flashlog_b200 import _lib
    rng = np.random.default_rng(rows)
    entries = rng.integers(0, 4, rows)                      # entries per row
    row_ptr = np.concatenate([[0], np.cumsum(entries)]).astype(np.int64)
    slots = rng.integers(0, 6, row_ptr[-1])                 # few distinct counts: many ties
    slot_base = np.concatenate([[0], np.cumsum(slots)]).astype(np.int64)
    order = torch.empty(rows, dtype=torch.int32, device="cuda")
    rp, sb = _cuda(row_ptr), _cuda(slot_base)
    rc = _lib.lib().fl_row_order(rp.data_ptr(), sb.data_ptr(), rows, order.data_ptr(),
                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    counts = slot_base[row_ptr[1:]] - slot_base[row_ptr[:-1]]
    want = np.argsort(-counts, kind="stable")
    assert np.array_equal(order.cpu().numpy(), want)
