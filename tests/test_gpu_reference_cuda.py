"""The CUDA-only paths against fixtures recorded from the reference's own CUDA code.

tests/golden/make_golden_cuda.py ran the reference's extension (flashlog.cu,
compiled from its sources into oracle/_ref) on a B200 and saved inputs and raw
outputs in tests/golden/ref_cuda.npz:

* the top-k fill (flashlog.cu:1368-1559), deterministic c2 thresholds and the
  sampled c2 quotas with their SplitMix64 phase (1458-1528), on the config-1
  graph and on a graph whose hubs have up to 299 relation groups per side;
* the fixed-relation rule step (1561-1741);
* the dense MAX forward and backward (523-726, 997-1255);
* the CSR-ordered masks of apply_mask_cuda (1286-1340), plain and with
  learnable edge weights.

Selections, fact coordinates, relation columns, triple ids, MAX winners and
output coordinates are compared bit for bit; values and gradients at rel
1e-5 (the reference sums with float atomics in no fixed order).
"""
import functools
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

RTOL = 1e-5
HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURE = os.path.join(HERE, "golden", "ref_cuda.npz")


@functools.lru_cache(maxsize=None)
def _fixture():
    return dict(np.load(FIXTURE, allow_pickle=False))


@functools.lru_cache(maxsize=None)
def _graph(name):
    from flashlog_b200.flashlog_kernel import build_csr_structure
    from flashlog_b200.ops import Graph
    d = _fixture()
    if name == "hub":
        tri = d["hub_triples"].astype(np.int64)
        E, R = int(d["hub_E"]), int(d["hub_R"])
    else:
        from flashlog_b200.synthetic import CONFIGS, load_or_generate
        cfg = CONFIGS[1]
        tri, _, _ = load_or_generate(cfg)
        E, R = cfg.entities, cfg.relations
    t = torch.from_numpy(tri).cuda()
    csr = build_csr_structure(t[:, 0], t[:, 2], t[:, 1], E)
    return csr, Graph.of(csr), E, R, tri.shape[0]


@pytest.fixture(scope="module")
def ready():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    if not os.path.exists(FIXTURE):
        pytest.skip(f"{FIXTURE} is not recorded yet (tests/golden/make_golden_cuda.py on a GPU)")
    return _fixture()


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _topk_ids():
    if not os.path.exists(FIXTURE):
        return []
    return [int(k) for k in _fixture()["topk_cases"]]


@pytest.mark.parametrize("k", _topk_ids())
def test_topk_fill_matches_reference_cuda(ready, k):
    """Per source entry, the kept facts in the reference's emission order
    (forward groups, inverse groups, identity), after the visibility filter of
    flashlog_kernel.py:1217-1228: destination, relation column, triple id and
    value; then the coalesced sums."""
    from flashlog_b200 import _lib as Lb
    from flashlog_b200 import ops
    d = ready
    p = lambda s: d[f"t{k}_{s}"]
    csr, graph, E, R, _ = _graph(str(p("graph")))
    B, L = int(p("B")), int(p("L"))
    topk, seed, wot_i = int(p("topk")), int(p("seed")), bool(p("wot_i"))
    row, ent, val, w, mask = p("row"), p("ent"), p("val"), p("w"), p("mask")
    flags = Lb.FL_SKIP_NONPOS_W | Lb.FL_DROP_MASKED | (Lb.FL_WOT_I if wot_i else 0) | (Lb.FL_SAMPLED if seed >= 0 else 0)
    rp, en, _ = ops.coo_to_rows(_cuda(row // L), _cuda(row % L), _cuda(ent), B, L, E)
    fw = ops.hop_forward(rp, en, _cuda(val), _cuda(w), graph, R, topk, flags, mask_triple=_cuda(mask), seed=seed,
                         keep_facts=True, record_edge=True)
    S = row.size
    base = fw.slot_base[:S].cpu().numpy()
    cnt = fw.entry_count[:S].cpu().numpy().astype(np.int64)
    slots = np.concatenate([np.arange(b, b + c) for b, c in zip(base, cnt)]) if S else np.zeros(0, np.int64)
    g_dst = fw.fact_dst.cpu().numpy()[slots].astype(np.int64)
    g_val = fw.fact_val.cpu().numpy()[slots]
    g_rel = fw.fact_rel.cpu().numpy()[slots].astype(np.int64)
    g_edge = fw.fact_edge.cpu().numpy()[slots].astype(np.int64)
    g_entry = np.repeat(np.arange(S), cnt)
    # the reference's facts, visible ones only, per entry in emission order
    parts = []
    for side, off_rel in (("ori", 0), ("inv", R)):
        vis = p(f"{side}_m") != 0
        parts.append((p(f"{side}_entry")[vis], p(f"{side}_e")[vis], p(f"{side}_v")[vis],
                      p(f"{side}_rel")[vis].astype(np.int64) + off_rel, p(f"{side}_edge")[vis], np.full(vis.sum(), 0 if side == "ori" else 1)))
    if not wot_i:
        parts.append((np.arange(S), p("ind_e"), p("ind_v"), np.full(S, 2 * R), np.full(S, -1), np.full(S, 2)))
    r_entry, r_e, r_v, r_rel, r_edge, r_side = (np.concatenate(x) for x in zip(*parts))
    order = np.lexsort((np.arange(r_entry.size), r_side, r_entry))  # entry, then side, then emission order
    r_entry, r_e, r_v, r_rel, r_edge = (x[order] for x in (r_entry, r_e, r_v, r_rel, r_edge))
    assert np.array_equal(g_entry, r_entry), "facts per entry"
    assert np.array_equal(g_dst, r_e.astype(np.int64)), "fact destinations"
    assert np.array_equal(g_rel, r_rel), "fact relation columns"
    edge_facts = g_rel != 2 * R
    assert np.array_equal(g_edge[edge_facts], r_edge[edge_facts].astype(np.int64)), "fact triple ids"
    np.testing.assert_allclose(g_val, r_v, rtol=RTOL, atol=0)
    # coalesced sums against the reference's facts summed in float64
    keys = (row[r_entry] * E + r_e).astype(np.int64)
    uk, inv = np.unique(keys, return_inverse=True)
    sums = np.zeros(uk.size, np.float64)
    np.add.at(sums, inv, r_v.astype(np.float64))
    counts = (fw.out_row_ptr[1:] - fw.out_row_ptr[:-1]).cpu().numpy()
    ours = np.repeat(np.arange(B * L), counts) * E + fw.out_ent.cpu().numpy()
    assert np.array_equal(ours, uk)
    np.testing.assert_allclose(fw.out_x.cpu().numpy(), sums, rtol=RTOL, atol=0)


def test_topk_fixture_reaches_the_rank_select(ready):
    """At least one hub case thresholds more than 32 relation groups of one side."""
    d = ready
    csr, _, E, R, _ = _graph("hub")
    gp = csr[8].cpu().numpy()
    hub_cases = [k for k in d["topk_cases"] if str(d[f"t{k}_graph"]) == "hub"]
    assert hub_cases
    ents = np.concatenate([d[f"t{k}_ent"] for k in hub_cases])
    assert (gp[ents + 1] - gp[ents]).max() > 32


@pytest.mark.parametrize("j", [0, 1, 2])
def test_fixed_relation_matches_reference_cuda(ready, j):
    import flashlog_b200.flashlog_kernel as fk
    d = ready
    p = lambda s: d[f"f{j}_{s}"]
    csr, _, E, R, _ = _graph("c1")
    Bq, Lr = int(p("B")), int(p("L"))
    row, ent, val, ops_ = p("row"), p("ent"), p("val"), p("ops")
    idx = _cuda(np.stack([row // Lr, row % Lr, ent]))
    sp = torch.sparse_coo_tensor(idx, _cuda(val), (Bq, Lr, E), is_coalesced=True)
    out = fk.vectorized_operation_sparse3d_fixed_relation(sp, _cuda(ops_), csr, R)
    keys = ((p("out_b") * Lr + p("out_l")) * E + p("out_e")).astype(np.int64)
    uk, inv = np.unique(keys, return_inverse=True)
    sums = np.zeros(uk.size, np.float64)
    np.add.at(sums, inv, p("out_v").astype(np.float64))
    oi = out.indices().cpu().numpy()
    assert np.array_equal((oi[0] * Lr + oi[1]) * E + oi[2], uk)
    # integer-valued path counts: exact
    assert np.array_equal(out.values().cpu().numpy().astype(np.float64), sums)


@pytest.mark.parametrize("name", ["dense_plain", "dense_topk", "dense_ties"])
def test_dense_max_matches_reference_cuda(ready, golden, name):
    """Outputs bit for bit (the packed CAS-max keeps the lowest CSR position
    among equal maxima); gradients to the winners only, at rel 1e-5."""
    import flashlog_b200.flashlog_kernel as fk
    from test_oracle_golden import _dense_keep
    d = ready
    g = golden("dense_config1.npz")
    q = lambda s: g[f"{name}_{s}"]
    csr, _, E, R, _ = _graph("c1")
    use_topk, c1, c2, wot_i = bool(q("use_topk")), int(q("c1")), int(q("c2")), bool(q("wot_i"))
    A_np, w_np, mask = q("A"), q("w"), q("mask")
    A = _cuda(A_np).requires_grad_(True)
    w = _cuda(w_np).requires_grad_(True)
    s_i, s_h, s_t = fk.dense_csr_max(A, w, csr, _cuda(mask).bool(), R, wot_i=wot_i, use_topk=use_topk,
                                     topk_nodes=c1, topk_edges=c2)
    r = lambda s: d[f"{name}_{s}"]
    assert np.array_equal(s_i.detach().cpu().numpy(), r("out_ind"))
    assert np.array_equal(s_h.detach().cpu().numpy(), r("out_ori"))
    assert np.array_equal(s_t.detach().cpu().numpy(), r("out_inv"))
    ((s_i * _cuda(q("gi"))).sum() + (s_h * _cuda(q("gh"))).sum() + (s_t * _cuda(q("gt"))).sum()).backward()
    keep = _dense_keep(A_np, c1) if use_topk else np.ones(A_np.shape, bool)
    np.testing.assert_allclose(A.grad.cpu().numpy(), np.where(keep, r("gA"), 0), rtol=RTOL, atol=1e-6)
    np.testing.assert_allclose(w.grad.cpu().numpy(), r("gw"), rtol=RTOL, atol=1e-6)


@pytest.mark.parametrize("label", ["plain", "soft"])
def test_csr_masks_match_reference_cuda(ready, label):
    """prepare_csr_masks (fl_csr_mask) against apply_mask_cuda: bit for bit
    without weights; with learnable weights the sigmoid 1 / (1 + exp(-x)) at
    rel 1e-6."""
    import flashlog_b200.flashlog_kernel as fk
    d = ready
    csr, _, E, R, _ = _graph("c1")
    mask = _cuda(d["mask_mask"]).bool()
    weight = _cuda(d["mask_weight"]) if label == "soft" else None
    mo, mi = fk.prepare_csr_masks(csr, mask, weight)
    for got, want in ((mo, d[f"mask_{label}_ori"]), (mi, d[f"mask_{label}_inv"])):
        if label == "plain":
            assert np.array_equal(got.cpu().numpy(), want)
        else:
            np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-6, atol=0)
    # a float mask gives the same gather
    mo2, _ = fk.prepare_csr_masks(csr, mask.float(), weight)
    assert torch.equal(mo2, mo)
    with pytest.raises(ValueError):
        fk.prepare_csr_masks(csr, mask[:-1], weight)
