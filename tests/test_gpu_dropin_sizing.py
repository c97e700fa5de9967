"""Buffer sizing of the drop-in hop (vectorized_operation_sparse3d_csr_sum_norm).

The first call of a hop reads its exact fact count before the expansion.
A later call with the same key (graph, rows, input size class, c2, c1,
flags) sizes its fact buffers from the count it saw and reads the output
count, the overflow status and the weights' finiteness once, after the
reduction.  When that capacity falls short, the hop runs again with exact
sizing.  Every path must give the same outputs and gradients, bit for bit,
and the state's own row layout must be reused on the next hop.
"""
import numpy as np
import pytest

from helpers import config1_graph

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _hop(fk, state, logits, csr, mask, R, c1, c2):
    w = torch.softmax(logits, dim=-1)
    out = fk.vectorized_operation_sparse3d_csr_sum_norm(state, w, csr, mask, R, use_topk=True,
                                                       topk_edges=c2 // 2, topk_nodes=c1)
    return out


def _run(fk, csr, heads, logits_np, mask, R, E, c1, c2, hops=3):
    dev = torch.device("cuda")
    Q, N = heads.size, logits_np.shape[2]
    logits = torch.from_numpy(logits_np).to(dev).requires_grad_(True)
    b = torch.arange(Q, device=dev).repeat_interleave(N)
    lv = torch.arange(N, device=dev).repeat(Q)
    e = torch.from_numpy(heads).to(dev).repeat_interleave(N)
    state = torch.sparse_coo_tensor(torch.stack([b, lv, e]), torch.ones(Q * N, device=dev), (Q, N, E),
                                    is_coalesced=True)
    outs = []
    for t in range(hops):
        state = _hop(fk, state, logits[:, t], csr, mask, R, c1, c2)
        outs.append((state.indices().cpu().numpy(), state.values().detach().cpu().numpy()))
    state.values().sum().backward()
    return outs, logits.grad.cpu().numpy()


def test_speculative_sizing_matches_exact_sizing():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import flashlog_b200.flashlog_kernel as fk
    cfg, train, _ = config1_graph()
    E, R = cfg.entities, cfg.relations
    dev = torch.device("cuda")
    t = torch.from_numpy(train).to(dev)
    csr = fk.build_csr_structure(t[:, 0], t[:, 2], t[:, 1], E)
    rng = np.random.default_rng(7)
    heads = rng.integers(0, E, 24)
    logits = rng.standard_normal((24, 3, 3, 2 * R + 1)).astype(np.float32)
    mask = torch.ones(train.shape[0], dtype=torch.bool, device=dev)
    mask[torch.from_numpy(rng.choice(train.shape[0], 500, replace=False)).to(dev)] = False
    c1, c2 = 50, 40
    fk._FACTS_SEEN.clear()
    exact, g_exact = _run(fk, csr, heads, logits, mask, R, E, c1, c2)  # every hop sized exactly
    assert len(fk._FACTS_SEEN) == 3
    spec, g_spec = _run(fk, csr, heads, logits, mask, R, E, c1, c2)  # every hop from the counts seen
    for k in list(fk._FACTS_SEEN):
        fk._FACTS_SEEN[k] = 1  # capacities of 1,025 facts: the larger hops run out and size again
    short, g_short = _run(fk, csr, heads, logits, mask, R, E, c1, c2)
    for run, g in ((spec, g_spec), (short, g_short)):
        for (ia, va), (ib, vb) in zip(exact, run):
            assert np.array_equal(ia, ib)
            assert np.array_equal(va, vb)
        assert np.array_equal(g_exact, g)
    assert exact[-1][1].size > 1025  # the last hop is larger than the short capacity


def test_nonfinite_weights_raise_on_the_speculative_path():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import flashlog_b200.flashlog_kernel as fk
    cfg, train, _ = config1_graph()
    E, R = cfg.entities, cfg.relations
    dev = torch.device("cuda")
    t = torch.from_numpy(train).to(dev)
    csr = fk.build_csr_structure(t[:, 0], t[:, 2], t[:, 1], E)
    rng = np.random.default_rng(8)
    heads = rng.integers(0, E, 8)
    logits = rng.standard_normal((8, 3, 3, 2 * R + 1)).astype(np.float32)
    mask = torch.ones(train.shape[0], dtype=torch.bool, device=dev)
    fk._FACTS_SEEN.clear()
    _run(fk, csr, heads, logits, mask, R, E, 20, 40, hops=1)
    bad = logits.copy()
    bad[0, 0, 0, 3] = np.nan
    with pytest.raises(RuntimeError, match="non-finite"):
        _run(fk, csr, heads, bad, mask, R, E, 20, 40, hops=1)
