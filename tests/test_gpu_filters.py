"""Filter keys for filtered ranking on the GPU, against the reference's own
build_filter_indices_csr outputs (training-CSR and per-split lookup paths)
and the oracle."""
import numpy as np
import pytest
import torch

from helpers import O, config1_graph

pytestmark = pytest.mark.gpu


def _keys(b, e, E):
    return np.sort(b.cpu().numpy().astype(np.int64) * E + e.cpu().numpy().astype(np.int64))


@pytest.fixture(scope="module")
def data():
    import flashlog_b200 as fk
    from flashlog_b200.synthetic import CONFIGS, load_or_generate
    cfg = CONFIGS[1]
    train, valid, test = load_or_generate(cfg)
    t = torch.from_numpy(train).cuda()
    csr = fk.build_csr_structure(t[:, 0], t[:, 2], t[:, 1], cfg.entities)
    return cfg, train, valid, test, csr


def test_filter_indices_from_training_csr(golden, data):
    from flashlog_b200 import filters
    cfg, train, valid, test, csr = data
    d = golden("filter_config1.npz")
    E = cfg.entities
    b, e = filters.build_filter_indices_csr(torch.from_numpy(d["qx"]).cuda(), torch.from_numpy(d["qr"]).cuda(),
                                            cfg.relations, csr)
    assert b.dtype == torch.long and e.dtype == torch.long and b.is_cuda
    assert np.array_equal(_keys(b, e, E), np.sort(d["csr_batch"] * E + d["csr_entity"]))


def test_filter_indices_from_split_lookups(golden, data):
    """create_eval_filter_csr (train, then valid + test) on the device, and
    lookups in the reference's own sorted-key format: both equal the
    reference's per-split lookup path."""
    from flashlog_b200 import filters
    cfg, train, valid, test, csr = data
    d = golden("filter_config1.npz")
    E, R = cfg.entities, cfg.relations
    held = np.concatenate([valid, test])
    splits = [(train[:, 0], train[:, 1], train[:, 2]), (held[:, 0], held[:, 1], held[:, 2])]
    lk, _, _ = filters.create_eval_filter_csr(splits, R, E, torch.device("cuda"))
    qx, qr = torch.from_numpy(d["qx"]).cuda(), torch.from_numpy(d["qr"]).cuda()
    want = np.sort(d["lookup_batch"] * E + d["lookup_entity"])
    b, e = filters.build_filter_indices_csr(qx, qr, R, lk)
    assert np.array_equal(_keys(b, e, E), want)

    def ref_format(h, r, t):  # (group_keys, starts, counts, columns) sorted by key, as src/main.py:154-169
        keys = h.astype(np.int64) * R + r
        order = np.argsort(keys, kind="stable")
        sk = keys[order]
        starts = np.flatnonzero(np.r_[True, sk[1:] != sk[:-1]])
        counts = np.diff(np.r_[starts, sk.size])
        return (torch.from_numpy(sk[starts]), torch.from_numpy(starts), torch.from_numpy(counts),
                torch.from_numpy(t[order].astype(np.int32)))
    ref_lk = {"filter_lookups": [(ref_format(h, r, t), ref_format(t, r, h)) for h, r, t in splits]}
    b2, e2 = filters.build_filter_indices_csr(qx, qr, R, ref_lk)
    assert np.array_equal(_keys(b2, e2, E), want)


def test_filter_indices_edge_cases(data):
    from flashlog_b200 import filters
    cfg, train, valid, test, csr = data
    R = cfg.relations
    e = torch.empty(0, dtype=torch.long, device="cuda")
    b0, e0 = filters.build_filter_indices_csr(e, e, R, csr)
    assert b0.numel() == 0 and e0.numel() == 0
    with pytest.raises(ValueError):
        filters.build_filter_indices_csr(torch.tensor([0], device="cuda"), torch.tensor([2 * R], device="cuda"), R,
                                         csr)


def test_filter_keys_for_batch(data):
    """filter_keys_for_batch_flashlog: the CSR's answers of every (source,
    relation), the split's known answers and the targets, sorted unique."""
    from flashlog_b200 import filters
    cfg, train, valid, test, csr = data
    E, R = cfg.entities, cfg.relations
    _, _, csr_np = config1_graph()
    rng = np.random.default_rng(3)
    pick = test[rng.choice(test.shape[0], 64, replace=False)]
    batch = [(int(h), int(r) + (R if k % 2 else 0), int(t)) for k, (h, r, t) in enumerate(pick)]
    known = {(batch[0][0], batch[0][1]): {5, 7}, (batch[3][0], batch[3][1]): {11}}
    sources = torch.tensor([s for s, _, _ in batch], dtype=torch.long, device="cuda")
    got = filters.filter_keys_for_batch_flashlog(csr, batch, sources, known, R, E).cpu().numpy()
    ob, oe = O.filter_indices(np.array([s for s, _, _ in batch]), np.array([r for _, r, _ in batch]), R, csr_np)
    extra = [bi * E + a for bi, (s, r, t) in enumerate(batch) for a in known.get((s, r), set()) | {t}]
    want = np.unique(np.concatenate([ob * E + oe, np.array(extra, np.int64)]))
    assert np.array_equal(got, want)


@pytest.mark.parametrize("case", [0, 1, 2])
@pytest.mark.parametrize("name", ["sum", "max"])
def test_channel_readouts_match_reference_golden(golden, case, name):
    """sum_sp_3d / max_sp_3d against the model files' own functions: output
    coordinates exact, values (sums in channel order; maxima exact) and the
    values' gradient, ties in max split evenly."""
    from flashlog_b200 import readout
    d = golden("readout.npz")
    B, L, E = (int(x) for x in d[f"c{case}_shape"])
    row, ent, val = d[f"c{case}_row"], d[f"c{case}_ent"], d[f"c{case}_val"]
    idx = torch.from_numpy(np.stack([row // L, row % L, ent])).cuda()
    v = torch.from_numpy(val.copy()).cuda().requires_grad_(True)
    y = getattr(readout, f"{name}_sp_3d")(torch.sparse_coo_tensor(idx, v, (B, L, E), is_coalesced=True))
    yi = y.indices().cpu().numpy()
    assert np.array_equal(yi[0] * E + yi[1], d[f"c{case}_{name}_key"])
    if name == "max":
        assert np.array_equal(y.values().detach().cpu().numpy(), d[f"c{case}_{name}_val"])
    else:
        np.testing.assert_allclose(y.values().detach().cpu().numpy(), d[f"c{case}_{name}_val"], rtol=1e-6, atol=0)
    (y.values() * torch.from_numpy(d[f"c{case}_{name}_g"]).cuda()).sum().backward()
    np.testing.assert_allclose(v.grad.cpu().numpy(), d[f"c{case}_{name}_grad"], rtol=1e-6, atol=1e-7)
