"""Dropout of hop values (nn.Dropout on s.values(), src/model_DRUM_kernel_sp.py:189-192)
on the GPU: fl_value_dropout bit-exact against the oracle's keep bits, the
live-count and in-place forms, the autograd op and the sparse-state helper."""
import numpy as np
import pytest
import torch

from helpers import O

pytestmark = pytest.mark.gpu


def _x(n, seed=0):
    return np.random.default_rng(seed).standard_normal(n).astype(np.float32)


@pytest.mark.parametrize("p", [0.0, 0.1, 0.5, 0.9, 1.0])
def test_value_dropout_matches_oracle(p):
    from flashlog_b200 import ops
    x = _x(100_003)
    seed, counter, subseq = (1 << 63) + 5, 7, 2
    y = ops.value_dropout(torch.from_numpy(x).cuda(), p, seed, torch.tensor([counter], device="cuda"), subseq)
    want, _ = O.value_dropout(x, p, seed, counter, subseq)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_value_dropout_live_count_in_place_and_errors():
    from flashlog_b200 import ops
    x = _x(10_000, 1)
    xd = torch.from_numpy(x).cuda()
    live = torch.tensor([6_001], device="cuda")
    ops.value_dropout(xd, 0.3, 11, None, 4, live=live, out=xd)
    want, _ = O.value_dropout(x, 0.3, 11, 0, 4)
    got = xd.cpu().numpy()
    assert np.array_equal(got[:6_001], want[:6_001]) and np.array_equal(got[6_001:], x[6_001:])
    with pytest.raises(ValueError):
        ops.value_dropout(xd, 1.5, 0)
    with pytest.raises(ValueError):
        ops.value_dropout(xd, 0.1, 0, None, 1 << 16)
    with pytest.raises(ValueError):
        ops.value_dropout(xd.double(), 0.1, 0)


def test_sparse_dropout_autograd():
    """Values and the gradient (the upstream gradient through the same keep
    bits and scale) against the oracle; indices unchanged; identity outside
    training."""
    from flashlog_b200.dropout import sparse_dropout
    rng = np.random.default_rng(2)
    B, L, E, nnz = 4, 3, 500, 900
    key = np.unique(rng.integers(0, B * L * E, nnz))
    idx = torch.from_numpy(np.stack([key // (L * E), (key // E) % L, key % E])).cuda()
    v = torch.from_numpy(_x(key.size, 3)).cuda().requires_grad_(True)
    s = torch.sparse_coo_tensor(idx, v, (B, L, E), is_coalesced=True)
    assert sparse_dropout(s, 0.2, training=False) is s
    y = sparse_dropout(s, 0.2, seed=17, counter=3, subseq=1)
    assert torch.equal(y.indices(), s.indices())
    want, keep = O.value_dropout(v.detach().cpu().numpy(), 0.2, 17, 3, 1)
    assert np.array_equal(y.values().detach().cpu().numpy(), want)
    g = _x(key.size, 4)
    (y.values() * torch.from_numpy(g).cuda()).sum().backward()
    assert np.array_equal(v.grad.cpu().numpy(), O.value_dropout(g, 0.2, 17, 3, 1)[0])


def test_fused_dropout_equals_the_separate_pass():
    """fl_scatter_grad with an fl_dropout descriptor writes exactly what the
    plain scatter followed by fl_value_dropout over the full vector leaves
    (the graph step fuses the gradients' dropout this way); a bad descriptor
    is rejected."""
    import ctypes
    from flashlog_b200 import _lib as L
    from flashlog_b200.ops import _p, _stream
    lib = L.lib()
    rng = np.random.default_rng(8)
    n_full, n_sel = 50_000, 12_000
    src = torch.from_numpy(np.sort(rng.choice(n_full, n_sel, replace=False))).cuda()
    g = torch.from_numpy(_x(n_sel, 9)).cuda()
    counter = torch.tensor([5], device="cuda")
    drop = L.fl_dropout(0.25, 77, counter.data_ptr(), 3)
    fused = torch.empty(n_full, device="cuda")
    plain = torch.empty(n_full, device="cuda")
    assert lib.fl_scatter_grad(_p(g), _p(src), n_sel, None, _p(fused), n_full, None, ctypes.byref(drop), _stream()) == 0
    assert lib.fl_scatter_grad(_p(g), _p(src), n_sel, None, _p(plain), n_full, None, None, _stream()) == 0
    assert lib.fl_value_dropout(_p(plain), _p(plain), n_full, None, ctypes.c_double(0.25), 77, _p(counter), 3,
                                _stream()) == 0
    assert torch.equal(fused.view(torch.int32), plain.view(torch.int32))
    full = np.zeros(n_full, np.float32)
    full[src.cpu().numpy()] = g.cpu().numpy()
    assert np.array_equal(fused.cpu().numpy(), O.value_dropout(full, 0.25, 77, 5, 3)[0])
    bad = L.fl_dropout(1.5, 0, None, 0)
    assert lib.fl_scatter_grad(_p(g), _p(src), n_sel, None, _p(fused), n_full, None, ctypes.byref(bad),
                               _stream()) == 1
