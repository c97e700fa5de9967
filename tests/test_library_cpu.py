"""Host-side checks that need no GPU: the C ABI library and the drop-in's host logic."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(REPO, "include", "flashlog_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fl_[a-z0-9_]+)\s*\(", text)))


def test_library_builds_and_exports_every_declared_symbol():
    from flashlog_b200 import _lib
    _lib.build()
    handle = ctypes.CDLL(_lib.LIB_PATH)
    syms = declared_symbols()
    assert len(syms) >= 20
    for s in syms:
        assert hasattr(handle, s), s
    # every declared symbol has a ctypes signature in the binding
    assert set(syms) <= set(_lib.SIGNATURES), set(syms) - set(_lib.SIGNATURES)
    assert _lib.lib().fl_version() == 1


def test_library_is_built_for_sm100a():
    from flashlog_b200 import _lib
    assert "arch=compute_100a,code=sm_100a" in " ".join(_lib.NVCC_FLAGS)
    assert "-fmad=false" in _lib.NVCC_FLAGS  # products are rounded separately, as in the reference


def test_error_message_roundtrip():
    from flashlog_b200 import _lib
    lib = _lib.lib()
    rc = lib.fl_coo_to_rows(None, None, None, 0, 0, 0, 0, None, None, None, None)
    assert rc == 1
    assert b"invalid" in lib.fl_last_error()
    with pytest.raises(ValueError):
        _lib.check(rc, "coo_to_rows")


def test_cpu_tensors_are_rejected():
    import flashlog_b200.flashlog_kernel as fk
    idx = torch.tensor([[0], [0], [1]])
    sp = torch.sparse_coo_tensor(idx, torch.ones(1), (1, 1, 4)).coalesce()
    w = torch.softmax(torch.randn(1, 1, 3), -1)
    csr = tuple(torch.zeros(2, dtype=torch.int32) for _ in range(16))
    with pytest.raises(ValueError):
        fk.vectorized_operation_sparse3d_csr_sum(sp, w, csr, torch.ones(1, dtype=torch.bool), 1, use_topk=True,
                                                 topk_edges=2)
    with pytest.raises(ValueError):
        fk.vectorized_operation_sparse3d_csr_sum_norm(sp, w, csr, torch.ones(1, dtype=torch.bool), 1)
    with pytest.raises(ValueError):
        fk.vectorized_operation_sparse3d_fixed_relation(sp, torch.zeros(1, 1, dtype=torch.long), csr, 1)
    from flashlog_b200 import dropout, ops
    with pytest.raises(ValueError):
        ops.value_dropout(torch.ones(8), 0.1, 0)
    with pytest.raises(ValueError):
        dropout.sparse_dropout(sp, 0.1, seed=1)


def test_exports_match_reference_names():
    import flashlog_b200
    for name in ("FlashLogFunction", "_compute_active_nodes", "build_csr_structure", "prepare_csr_masks",
                 "vectorized_operation_csr", "vectorized_operation_sparse3d_csr_sum",
                 "vectorized_operation_sparse3d_csr_sum_norm", "vectorized_operation_sparse3d_fixed_relation",
                 "FlashLogFunctionSparse3DTopKSum", "FlashLogFunctionSparse3DAllEdgesSum",
                 "FlashLogFunctionSparse3DTopKMax", "sampled_sparse_propagation", "normalize_sparse3d",
                 "configure_flashlog_cpu_threads", "_group_starts_and_counts", "sparse2d_filtered_ranks_cuda"):
        assert hasattr(flashlog_b200, name), name


def test_configure_cpu_threads_env(monkeypatch):
    import flashlog_b200.flashlog_kernel as fk
    before = torch.get_num_threads()
    try:
        monkeypatch.setenv("FLASHLOG_CPU_THREADS", "off")
        assert fk.configure_flashlog_cpu_threads(force=True) == before
        monkeypatch.setenv("FLASHLOG_CPU_THREADS", "2")
        assert fk.configure_flashlog_cpu_threads(force=True) == min(2, os.cpu_count())
    finally:
        torch.set_num_threads(before)


def test_group_starts_and_counts():
    import flashlog_b200.flashlog_kernel as fk
    v = torch.tensor([0, 0, 1, 1, 1, 3])
    r = torch.tensor([2, 2, 0, 1, 1, 0])
    s, c = fk._group_starts_and_counts(v, r)
    assert s.tolist() == [0, 2, 3, 5] and c.tolist() == [2, 1, 2, 1]
    s, c = fk._group_starts_and_counts(v)
    assert s.tolist() == [0, 2, 5] and c.tolist() == [2, 3, 1]


def test_synthetic_graph_is_seeded_and_shaped():
    from flashlog_b200.synthetic import CONFIGS, generate_triples, training_queries
    cfg = CONFIGS[1]
    a = generate_triples(cfg)
    b = generate_triples(cfg)
    assert all(np.array_equal(x, y) for x, y in zip(a, b))
    train, valid, test = a
    assert train.shape == (22_400, 3) and valid.shape[0] == 2_800 and test.shape[0] == 2_800
    assert np.unique(np.concatenate([train, valid, test]), axis=0).shape[0] == 28_000
    ids, h, r, t = training_queries(train, cfg)
    assert h.size == 2 * cfg.batch_size
    assert np.array_equal(r[1::2], r[0::2] + cfg.relations)


def test_python_constants_match_header():
    """Every FL_* constant the Python side uses has the header's value."""
    import re
    from flashlog_b200 import _lib as L
    src = open(os.path.join(REPO, "include", "flashlog_b200.h")).read()
    header = {m.group(1): m.group(2) for m in re.finditer(r"\b(FL_[A-Z0-9_]+)\s*=\s*([^,}\n/]+)", src)}
    checked = 0
    for name in dir(L):
        if name.startswith("FL_") and name in header:
            assert getattr(L, name) == eval(header[name].strip()), name
            checked += 1
    assert checked >= 12


def test_step_capacity_bounds():
    """The graph step's static buffer bounds (host arithmetic): each hop's
    input is the previous hop's output bound; c1 caps the selection at
    rows * c1 (times zero_slack when dropout keeps explicit zeros); facts
    are capped by k_max per entry and by the per-row entity capacities K;
    outputs by one per entity and row."""
    from flashlog_b200.step import capacities
    rows, k_max, K, E = 1536, 401, 46_000_000, 4_600_000
    C, S, F, U = capacities(rows, 3, 1000, k_max, K, E)
    assert C[0] == rows and S[0] == rows and F[0] == rows * k_max
    assert all(C[t + 1] == U[t] for t in range(2))
    assert S[2] == rows * 1000 and F[2] == rows * 1000 * k_max
    C2, S2, F2, U2 = capacities(rows, 3, 1000, k_max, K, E, zero_slack=2.0)
    assert S2[2] == 2 * S[2] and F2[2] == 2 * F[2] and S2[:2] == S[:2]
    Cn, Sn, Fn, Un = capacities(4, 2, None, 3, 10, 5)
    assert Sn == Cn == [4, 12] and Fn == [12, 36] and Un == [12, 20]


def test_default_zero_slack_covers_rows_kept_whole():
    """With dropout p a row of n entries keeps all of them (zeros included)
    while at most c1 values survive, so the rows kept whole hold about
    c1 / (1 - p) entries: the default slack covers the largest such row in a
    simulation of 1536 rows per p, including p = 0.5 and beyond; p = 1
    leaves the selection unbounded."""
    import math

    import numpy as np

    from flashlog_b200.step import capacities, default_zero_slack
    assert default_zero_slack(0.0) == 1.0
    assert math.isinf(default_zero_slack(1.0))
    rng = np.random.default_rng(5)
    c1, rows = 1000, 1536
    for p in (0.1, 0.3, 0.5, 0.7):
        slack = default_zero_slack(p)
        assert slack >= 1.0 / (1.0 - p)
        n = rng.integers(0, 4 * int(c1 / (1 - p)), rows)
        survivors = rng.binomial(n, 1.0 - p)
        kept = np.where(survivors <= c1, n, c1)
        assert kept.max() <= c1 * slack, p
        assert kept.sum() <= rows * c1 * slack, p
    C, S, F, U = capacities(8, 2, 10, 3, 100, 50, zero_slack=math.inf)
    assert S == C


def test_routed_instances_cover_every_query_with_its_relations_rules():
    """Host side of evaluate_rule_bank: batches in relation order, within
    both budgets, every query once, with exactly the rules of its relation."""
    from flashlog_b200.rules import route_instances
    rng = np.random.default_rng(3)
    heads = np.sort(rng.integers(0, 12, 200))
    rel = rng.integers(0, 14, 500)  # relations 12, 13 have no rules
    seen = []
    for budget, qb in ((1 << 20, 4096), (50, 7), (1, 3)):
        seen = []
        last_rel = -1
        for bq, q_inst, inst_rule in route_instances(rel, heads, qb, budget):
            assert 1 <= bq.size <= qb
            assert q_inst[0] == 0 and q_inst[-1] == inst_rule.size
            assert bq.size == 1 or q_inst[-1] <= budget
            assert rel[bq[0]] >= last_rel and np.all(np.diff(rel[bq]) >= 0)
            last_rel = rel[bq[-1]]
            for k, q in enumerate(bq):
                mine = inst_rule[q_inst[k]:q_inst[k + 1]]
                assert np.array_equal(mine, np.flatnonzero(heads == rel[q]))
            seen.extend(bq.tolist())
        assert sorted(seen) == list(range(rel.size))

