"""The max-product rule-bank evaluator at scale: pruning, the sparse accumulator, routed ranks.

* The sparse accumulation (rank rows reduced by the MAX row reduction, no
  dense [ranks, B, E] buffer) gives the reference's own score()
  (rules/shared_inference.py with reduction 'max', fixtures in
  maxproduct_config1.npz) on the same rule banks as the dense path.
* First-operator pruning (rules/shared_inference.py:34-47) drops rules that
  cannot ground and changes no score.
* evaluate_rule_bank (queries routed to the rules of their relation,
  compacted per (head, body), grounded as batches of (query, rule)
  instances, scored and ranked with filtered tie-averaged ranks) against the
  oracle's restatement run query group by query group: ranks equal, on a
  seeded 4,000-rule bank over config-2 test queries, for smDRUM (sum over
  ranks) and mmDRUM (max over ranks), with steps and scores in one range and
  split into many.
Values are compared at rel 1e-5, keys and ranks exactly.
"""
import numpy as np
import pytest

from helpers import O, config1_graph

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

RTOL = 1e-5


@pytest.fixture(scope="module")
def g1():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import flashlog_b200.flashlog_kernel as fk
    cfg, train, csr_np = config1_graph()
    t = torch.from_numpy(train).cuda()
    return cfg, train, csr_np, fk.build_csr_structure(t[:, 0], t[:, 2], t[:, 1], cfg.entities)


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("ci", [0, 1, 2])
@pytest.mark.parametrize("budget", [0, 1 << 20])
def test_sparse_accumulator_matches_reference_golden(g1, golden, ci, budget):
    """budget 0: every query batch accumulates sparsely; 1 MiB: batches of a
    few queries on the dense accumulator.  Both equal the reference."""
    from flashlog_b200 import rules as RB
    from test_oracle_golden import _rule_bank
    cfg, train, csr_np, csr = g1
    g = golden("maxproduct_config1.npz")
    bodies, weights = _rule_bank(g, ci)
    rules = [{"body": b, "rank_weights": [float(x) for x in w]} for b, w in zip(bodies, weights)]
    stats = {}
    out = RB.max_product_scores(_cuda(g[f"r{ci}_sources"]), rules, csr, cfg.relations, cfg.entities,
                                int(g[f"r{ci}_chunk"]), final_max=bool(g[f"r{ci}_final_max"]),
                                accumulator_bytes=budget, query_batch=3, stats=stats).coalesce()
    assert stats["dense_accumulation"] == (budget > 0)
    oi = out.indices().cpu().numpy()
    assert np.array_equal(oi[0] * cfg.entities + oi[1], g[f"r{ci}_key"])
    np.testing.assert_allclose(out.values().cpu().numpy(), g[f"r{ci}_val"], rtol=RTOL, atol=1e-9)


def test_first_operator_pruning_changes_no_score(g1):
    from flashlog_b200 import rules as RB
    cfg, train, csr_np, csr = g1
    R, E = cfg.relations, cfg.entities
    rng = np.random.default_rng(5)
    src = rng.integers(0, E, 6)
    avail = RB.available_first_operators(_cuda(src), csr, R).cpu().numpy()
    # the oracle's view of the same sources
    want = np.zeros(2 * R + 1, bool)
    want[2 * R] = True
    for d, (gp, gr) in enumerate(((csr_np[8], csr_np[9]), (csr_np[12], csr_np[13]))):
        for s in src:
            want[gr[gp[s]:gp[s + 1]].astype(np.int64) + d * R] = True
    assert np.array_equal(avail, want)
    absent = [o for o in range(2 * R) if not avail[o]]
    assert absent, "the sample needs an operator no source has"
    bodies = [(absent[0],), (absent[0], 0), tuple(int(x) for x in rng.integers(0, 2 * R, 2)), (2 * R, 1), ()]
    weights = rng.random((len(bodies), 3)).astype(np.float32)
    rules = [{"body": b, "rank_weights": [float(x) for x in w]} for b, w in zip(bodies, weights)]
    stats = {}
    out = RB.max_product_scores(_cuda(src), rules, csr, R, E, 2, stats=stats).coalesce()
    assert stats["rules_before"] == 5 and stats["rules_after"] == 3
    keys, vals = O.max_product(src, bodies, weights, csr_np, R, E)
    oi = out.indices().cpu().numpy()
    assert np.array_equal(oi[0] * E + oi[1], keys)
    np.testing.assert_allclose(out.values().cpu().numpy(), vals, rtol=RTOL, atol=1e-9)


def oracle_routed_ranks(src, rel, dst, rules, csr_np, R, E, final_max, sparse=False):
    """Ranks of the routed evaluation computed by the oracle, relation by relation."""
    from flashlog_b200.rules import compact_routed_rules
    by_head = {}
    for r in compact_routed_rules(rules):
        by_head.setdefault(r["head"], []).append(r)
    ranks = np.zeros(src.size, np.float32)
    fn = O.max_product_sparse if sparse else O.max_product
    for h in np.unique(rel):
        q = np.flatnonzero(rel == h)
        hr = by_head.get(int(h), [])
        if hr:
            keys, vals = fn(src[q], [r["body"] for r in hr], np.array([r["rank_weights"] for r in hr], np.float32),
                            csr_np, R, E, final_max)
        else:
            keys, vals = np.zeros(0, np.int64), np.zeros(0, np.float32)
        fk = np.arange(q.size) * E + dst[q]
        ranks[q] = O.filtered_ranks(keys // E, keys % E, vals, dst[q], fk, q.size, E, True)
    return ranks


@pytest.mark.parametrize("final_max", [False, True])
@pytest.mark.parametrize("mode", ["sorted", "split", "dense", "auto", "parts"])
def test_routed_evaluation_matches_oracle(final_max, mode):
    """mode: "sorted" reduces every step by the row reduction and every
    query's maxima by rank facts; "split" does the same in budgets of 4000
    facts (many ranges of instances and of queries); "dense" takes every
    step through entity bitmaps and every query through the dense
    accumulator; "auto" chooses per instance and per query; "parts" caps a
    batch at 64 instances, so every query with more rules is grounded in
    parts that meet in its dense accumulator."""
    budget = 4000 if mode == "split" else 1 << 29
    big = {"sorted": 1 << 62, "split": 1 << 62, "dense": 0, "auto": None, "parts": None}[mode]
    instances = 64 if mode == "parts" else 1 << 20
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import flashlog_b200.flashlog_kernel as fk
    from flashlog_b200 import rules as RB
    from flashlog_b200.synthetic import CONFIGS, evaluation_queries, load_or_generate, rule_bank
    cfg = CONFIGS[2]
    train, valid, test = load_or_generate(cfg)
    R, E = cfg.relations, cfg.entities
    t = torch.from_numpy(train).cuda()
    csr = fk.build_csr_structure(t[:, 0], t[:, 2], t[:, 1], E)
    csr_np = O.build_csr(train[:, 0], train[:, 2], train[:, 1], E)
    src, rel, dst = evaluation_queries(test, R, 150)
    rules = rule_bank(train, rel, R, 4000)
    stats = {}
    got = RB.evaluate_rule_bank(_cuda(src), _cuda(rel), _cuda(dst), rules, csr, R, E, final_max=final_max,
                                query_batch=32, fact_budget=budget, stats=stats, bitmap_min_facts=big,
                                dense_min_entries=big, instance_budget=instances).cpu().numpy()
    want = oracle_routed_ranks(src, rel, dst, rules, csr_np, R, E, final_max)
    assert np.array_equal(got, want)
    assert stats["batches"] >= src.size // 32
    if mode == "split":
        assert stats["step_ranges"] > stats["batches"] * 3 and stats["score_ranges"] > stats["batches"]
    if mode in ("sorted", "split"):
        assert stats.get("bitmap_rows", 0) == 0 and stats["dense_queries"] == 0
    if mode == "dense":
        assert stats["bitmap_rows"] > 0 and stats["dense_queries"] > 0
    if mode == "parts":
        assert stats["split_queries"] > 0
    assert (want < 0.5 * E).sum() > 10  # some targets are reached by rules
