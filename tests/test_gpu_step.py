"""The static-buffer DRUM step (flashlog_b200.step) against the autograd engine.

Both run the same kernels; the static step sizes every buffer by a bound and
never reads counts back to the host.  One step on the config-1 graph must give
the same loss, the same final state and the same attention-table gradient
(up to the order of the float atomics of the table's index_add)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

RTOL = 1e-5


@pytest.fixture(scope="module")
def setup():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from flashlog_b200.flashlog_kernel import build_csr_structure
    from flashlog_b200.ops import Graph
    from flashlog_b200.synthetic import CONFIGS, generate_triples
    cfg = CONFIGS[1]
    train, _, _ = generate_triples(cfg)
    tt = torch.from_numpy(train).cuda()
    csr = build_csr_structure(tt[:, 0], tt[:, 2], tt[:, 1], cfg.entities)
    return cfg, train, Graph.of(csr)


@pytest.mark.parametrize("c1,c2,dropout", [(40, 16, 0.0), (None, 0, 0.0), (5, 6, 0.0), (40, 16, 0.1)])
def test_static_step_matches_autograd_engine(setup, c1, c2, dropout):
    """With dropout, the step's first replay (counter 1) and the engine with
    dropout_counter=1 draw the same keep bits per hop."""
    from flashlog_b200 import engine
    from flashlog_b200.step import DrumTrainStep
    from flashlog_b200.synthetic import training_queries
    cfg, train, graph = setup
    R, T, N = cfg.relations, 3, 3
    n = 2 * R + 1
    ids, h, r, t = training_queries(train, cfg, step=3)
    ids, h, r, t = ids[:6], h[:12], r[:12], t[:12]
    Q = h.size
    gen = torch.Generator(device="cpu").manual_seed(7)
    table = torch.randn(2 * R, T, N, n, generator=gen).cuda()
    dev = torch.device("cuda")
    d = lambda a: torch.from_numpy(a).to(dev)
    # autograd engine
    tab = table.clone().requires_grad_(True)
    mask = torch.ones(train.shape[0], dtype=torch.uint8, device=dev)
    mask[d(ids)] = 0
    rp, ent, val = engine.drum_propagate(d(h), tab[d(r)], graph, R, c1=c1, c2=c2, mask_triple=mask,
                                         dropout=dropout, dropout_seed=5, dropout_counter=1)
    loss = engine.readout_loss(rp, ent, val, d(t), N)
    loss.backward()
    # static step
    step = DrumTrainStep(graph, R, Q, T, N, c1, c2, table.clone(), n_hide=ids.size, apply_update=False,
                         dropout=dropout, dropout_seed=5)
    step.load(d(h), d(t), d(r), d(ids))
    sloss = step.run()
    torch.cuda.synchronize()
    step.check()
    assert float(sloss) == pytest.approx(float(loss), rel=1e-6)
    live = int(rp[-1])
    srp = step.out_rp[T - 1]
    assert torch.equal(srp, rp)
    assert torch.equal(step.out_ent[T - 1][:live], ent[:live])
    assert torch.equal(step.out_y[T - 1][:live], val[:live].detach())
    np.testing.assert_allclose(step.grad.cpu().numpy(), tab.grad.cpu().numpy(), rtol=RTOL, atol=1e-7)
    # the step restores the visibility it changed
    assert int(step.vis[0].min()) == 1 and int(step.vis[1].min()) == 1


@pytest.mark.parametrize("dropout", [0.0, 0.1])
def test_static_step_replays_as_cuda_graph(setup, dropout):
    """Replays equal eager runs; with dropout, replay k draws the masks of
    eager run k (the device counter advances inside the graph)."""
    from flashlog_b200.step import DrumTrainStep
    from flashlog_b200.synthetic import training_queries
    cfg, train, graph = setup
    R, T, N = cfg.relations, 3, 3
    n = 2 * R + 1
    dev = torch.device("cuda")
    d = lambda a: torch.from_numpy(a).to(dev)
    gen = torch.Generator(device="cpu").manual_seed(9)
    table = torch.randn(2 * R, T, N, n, generator=gen).cuda()
    batches = []
    for s in range(3):
        ids, h, r, t = training_queries(train, cfg, step=10 + s)
        batches.append((d(ids[:8]), d(h[:16]), d(r[:16]), d(t[:16])))
    eager = DrumTrainStep(graph, R, 16, T, N, 40, 16, table.clone(), n_hide=8, apply_update=False, dropout=dropout)
    ref = []
    for ids, h, r, t in batches:
        eager.load(h, t, r, ids)
        ref.append((float(eager.run()), eager.grad.clone()))
    step = DrumTrainStep(graph, R, 16, T, N, 40, 16, table.clone(), n_hide=8, apply_update=False, dropout=dropout)
    ids, h, r, t = batches[0]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step.load(h, t, r, ids)
        step.run()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step.run()
    step.drop_counter.zero_()  # the warm-up run counted once
    for (ids, h, r, t), (l_ref, g_ref) in zip(batches, ref):
        step.load(h, t, r, ids)
        g.replay()
        torch.cuda.synchronize()
        assert float(step.loss) == pytest.approx(l_ref, rel=1e-6)
        np.testing.assert_allclose(step.grad.cpu().numpy(), g_ref.cpu().numpy(), rtol=RTOL, atol=1e-7)
    step.check()


def test_step_update_touches_only_the_batch_rows(setup):
    """apply_update: table[rels] -= lr * gradient, equal to the dense update
    from the gradient of a step run without it; other rows unchanged."""
    from flashlog_b200.step import DrumTrainStep
    from flashlog_b200.synthetic import training_queries
    cfg, train, graph = setup
    R, T, N = cfg.relations, 3, 3
    n = 2 * R + 1
    dev = torch.device("cuda")
    d = lambda a: torch.from_numpy(a).to(dev)
    gen = torch.Generator(device="cpu").manual_seed(11)
    table = torch.randn(2 * R, T, N, n, generator=gen).cuda()
    ids, h, r, t = training_queries(train, cfg, step=21)
    args = (d(h[:16]), d(t[:16]), d(r[:16]), d(ids[:8]))
    plain = DrumTrainStep(graph, R, 16, T, N, 40, 16, table.clone(), n_hide=8, apply_update=False, lr=0.05)
    plain.load(*args)
    plain.run()
    upd = DrumTrainStep(graph, R, 16, T, N, 40, 16, table.clone(), n_hide=8, apply_update=True, lr=0.05)
    upd.load(*args)
    upd.run()
    torch.cuda.synchronize()
    want = table - 0.05 * plain.grad
    np.testing.assert_allclose(upd.table.cpu().numpy(), want.cpu().numpy(), rtol=1e-6, atol=1e-6)
    untouched = torch.ones(2 * R, dtype=torch.bool, device=dev)
    untouched[d(r[:16])] = False
    assert torch.equal(upd.table[untouched], table[untouched])
