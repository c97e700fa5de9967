"""Dropout of the hop values during training.

The sparse models drop values of every hop's normalized state in training
(src/model_DRUM_kernel_sp.py:189-192, src/model_mmDRUM_kernel_sp.py:144,
src/model_NeuralLP_kernel_sp.py:195):

    s = torch.sparse_coo_tensor(s.indices(), nn.Dropout(p)(s.values()), s.shape, is_coalesced=True)

Here the keep bits come from a counter-based hash of (seed, counter, subseq,
position) in fl_value_dropout, so the backward re-derives the mask instead of
storing it, and a captured step draws a new mask per replay from a device
counter.  Kept values are scaled by 1 / (1 - p), dropped ones are 0; the
indices are untouched (dropped entries stay in the state with value 0, as in
the reference).
"""
from __future__ import annotations

import torch

from . import flashlog_kernel as _fk
from . import ops


def draw_seed() -> int:
    """A 62-bit seed from torch's default CPU generator (follows torch.manual_seed)."""
    return int(torch.randint(0, 1 << 62, (1,)).item())


class ValueDropout(torch.autograd.Function):
    """y = dropout(val); the backward applies the same keep bits and scale to the gradient."""

    @staticmethod
    def forward(ctx, val, p, seed, counter, subseq, live):
        ctx.args = (float(p), int(seed), counter, int(subseq), live)
        return ops.value_dropout(val.detach(), p, seed, counter, subseq, live)

    @staticmethod
    def backward(ctx, g):
        p, seed, counter, subseq, live = ctx.args
        return ops.value_dropout(g.contiguous(), p, seed, counter, subseq, live), None, None, None, None, None


def device_counter(value: int, device) -> torch.Tensor:
    # a fill kernel, not a copy from host memory: the host does not wait for the stream
    return torch.full((1,), int(value), dtype=torch.int64, device=device)


class SparseValueDropout(torch.autograd.Function):
    """Dropout of a coalesced sparse state's values as one node: the output
    shares the input's index tensor, and the backward hands back a sparse
    gradient on that same index tensor.  A gradient that arrives on the
    output's own indices (as the next hop's gives it) aligns without a sort,
    and torch's generic sparse-constructor backward (a coalesce and a
    masked projection of the gradient) never runs."""

    @staticmethod
    def forward(ctx, s, p, seed, counter, subseq):
        idx = s._indices()
        ctx.args = (float(p), int(seed), counter, int(subseq))
        ctx.idx, ctx.shape = idx, s.shape
        val = ops.value_dropout(s._values().detach(), p, seed, counter, subseq)
        return torch.sparse_coo_tensor(idx, val, s.shape, is_coalesced=True)

    @staticmethod
    def backward(ctx, g):
        p, seed, counter, subseq = ctx.args
        B, Lch, E = ctx.shape
        gv = _fk._align_sparse_grad_to_output(g, ctx.idx, Lch, E).to(torch.float32)
        gx = ops.value_dropout(gv, p, seed, counter, subseq)
        return torch.sparse_coo_tensor(ctx.idx, gx, ctx.shape, is_coalesced=True), None, None, None, None


def sparse_dropout(s: torch.Tensor, p: float, training: bool = True, seed: int | None = None, counter: int = 0,
                   subseq: int = 0) -> torch.Tensor:
    """The models' value dropout of a coalesced sparse [B, L, E] state
    (identity outside training or for p = 0)."""
    if not training or p == 0.0:
        return s
    s = s if s.is_coalesced() else s.coalesce()
    if s.dim() != 3:
        raise ValueError("sparse_dropout takes a [B, L, E] state")
    seed = draw_seed() if seed is None else seed
    # the output shares the input's index tensor, so a hop that returned the
    # input also recognizes the output as its own (flashlog_kernel._own_rows)
    return SparseValueDropout.apply(s, p, seed, device_counter(counter, s.device), subseq)
