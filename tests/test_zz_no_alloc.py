"""fl_filtered_ranks_noalloc: filtered ranks for callers that cannot allocate.

Some callers have no device allocator at hand (a plain C host program, or an
evaluation loop that must not call cudaMalloc because it synchronizes the
device).  fl_filtered_ranks_noalloc keeps its counters in a fixed array inside
the library instead of a caller workspace.  These tests call both entry points
through the C ABI and require identical ranks, on two calls in a row with
different inputs (the second call must not see the first call's counts).
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _case(seed, B, E, n_scores, n_filter, ties):
    rng = np.random.default_rng(seed)
    keys = np.unique(rng.integers(0, B * E, n_scores))
    vals = (rng.integers(0, 6, keys.size) / 5.0) if ties else rng.random(keys.size)
    targets = rng.integers(0, E, B)
    filt = np.unique(np.concatenate([rng.integers(0, B * E, n_filter), np.arange(B) * E + targets]))
    dev = torch.device("cuda")
    t = lambda a, d=torch.int64: torch.from_numpy(np.ascontiguousarray(a)).to(dev, d)
    return (t(keys // E), t(keys % E), t(vals, torch.float32), t(targets), t(filt))


def _ranks_with_workspace(lib, case, B, E, use_eql):
    ib, ie, v, tg, fk = case
    out = torch.empty(B, dtype=torch.float32, device="cuda")
    ws = torch.empty(lib.fl_filtered_ranks_workspace(B), dtype=torch.uint8, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.fl_filtered_ranks(_ptr(ib), _ptr(ie), _ptr(v), v.numel(), _ptr(tg), _ptr(fk), fk.numel(), B, E,
                               int(use_eql), _ptr(out), _ptr(ws), ws.numel(), stream)
    assert rc == 0, lib.fl_last_error()
    return out


def _ranks_no_alloc(lib, case, B, E, use_eql):
    ib, ie, v, tg, fk = case
    out = torch.empty(B, dtype=torch.float32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.fl_filtered_ranks_noalloc(_ptr(ib), _ptr(ie), _ptr(v), v.numel(), _ptr(tg), _ptr(fk), fk.numel(), B,
                                       E, int(use_eql), _ptr(out), stream)
    assert rc == 0, lib.fl_last_error()
    return out


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from flashlog_b200 import _lib
    return _lib.lib()


def test_no_alloc_ranks_match_workspace_ranks_twice(lib):
    # Two calls in a row with different sizes and contents: the fixed counters
    # must be cleared by each call.
    for seed, B, E, use_eql, ties in ((1, 4096, 900, True, True), (2, 700, 2500, False, False),
                                      (3, 65536, 64, True, True)):
        case = _case(seed, B, E, 6 * B, 2 * B, ties)
        a = _ranks_no_alloc(lib, case, B, E, use_eql)
        b = _ranks_with_workspace(lib, case, B, E, use_eql)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy())


def test_no_alloc_rejects_too_many_queries(lib):
    B, E = 65537, 8
    dummy = torch.zeros(1, dtype=torch.int64, device="cuda")
    out = torch.empty(1, dtype=torch.float32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.fl_filtered_ranks_noalloc(_ptr(dummy), _ptr(dummy), _ptr(out), 0, _ptr(dummy), _ptr(dummy), 0, B, E, 1,
                                       _ptr(out), stream)
    assert rc == 1
    assert b"65536" in lib.fl_last_error()
