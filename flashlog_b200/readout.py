"""Channel readouts of a [B, N, E] sparse state (the model files' sum_sp_3d
and max_sp_3d).

* sum_sp_3d (src/model_DRUM_kernel_sp.py:22-28): [B, E] sum over channels.
* max_sp_3d (src/model_mmDRUM_kernel_sp.py:17-32): [B, E] max over channels;
  the gradient of tied channels is split evenly, as torch's
  scatter_reduce(amax) gives it in the reference.

The merge of the channel rows -- each query's sorted union of entities and
every entry's output position -- runs in the library's row reduction
(ops.channel_merge); sums are taken in channel order.
"""
from __future__ import annotations

import torch
from torch import autograd

from . import ops


class _GatherGrad(autograd.Function):
    """Forward: precomputed sums; backward: each entry gets its output's gradient."""

    @staticmethod
    def forward(ctx, values, position, sums):
        ctx.save_for_backward(position)
        return sums

    @staticmethod
    def backward(ctx, g):
        (position,) = ctx.saved_tensors
        g = g.to_dense() if g.is_sparse else g
        return g[position], None, None


def _merge(s):
    s = s.coalesce()
    if not s.is_cuda:
        raise ValueError("channel readouts run on CUDA tensors")
    idx, val = s.indices(), s.values()
    B, N, E = s.shape
    row_ptr, ent, bad = ops.coo_to_rows(idx[0], idx[1], idx[2], B, N, E)
    if int(bad.item()):
        raise ValueError("sparse state indices are out of range or not coalesced")
    out_row_ptr, out_ent, out_x, position = ops.channel_merge(row_ptr, ent, val.detach(), B, N, E)
    out_idx = ops.rows_to_coo(out_row_ptr, out_ent, 1)
    return s, val, (B, E), torch.stack([out_idx[0], out_idx[2]]), out_x, position


def sum_sp_3d(s):
    """[B, N, E] -> [B, E], summed over channels (src/model_DRUM_kernel_sp.py:22-28)."""
    s, val, shape, out_idx, out_x, position = _merge(s)
    out_val = _GatherGrad.apply(val, position, out_x.to(val.dtype))
    return torch.sparse_coo_tensor(out_idx, out_val, shape, is_coalesced=True)


def max_sp_3d(s):
    """[B, N, E] -> [B, E], max over channels (src/model_mmDRUM_kernel_sp.py:17-32)."""
    s, val, shape, out_idx, out_x, position = _merge(s)
    out_val = torch.zeros(out_x.numel(), device=val.device, dtype=val.dtype)
    out_val = out_val.scatter_reduce(0, position, val, reduce="amax", include_self=False)
    return torch.sparse_coo_tensor(out_idx, out_val, shape, is_coalesced=True)
