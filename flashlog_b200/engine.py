"""Multi-hop DRUM propagation that keeps the state in the row layout between hops.

This is the hot path of one sparse DRUM training step
(src/model_DRUM_kernel_sp.py:92-204 with the deterministic c1/c2 budgets):
for t in range(T): w_t = softmax(w_all[:, t] / tau_1); state = normalize(hop(state, w_t));
then the channel readout and log loss of src/utils.py:36-47.  Each hop is one
autograd node whose forward and backward run in the library's kernels; the
state never goes through the COO round trip of the operator API.

Host synchronization: one per hop (the planned fact count sizes the fact
buffers).  Selected entries and outputs keep capacity-sized buffers whose live
counts stay on the device (row_ptr[-1]); work that would not fit those
capacities is skipped and flagged in a sticky device status word, which
`check_status` reads once after the step (or after many steps).
"""
from __future__ import annotations

import torch

from . import _lib as L
from . import ops
from .ops import Graph


class HopNorm(torch.autograd.Function):
    """c1 selection + expansion + coalesce-sum + normalization of one hop.

    `stats` (optional) collects per-hop counts and gets a `timer` with
    record_start / record_end around the hop's expansion and reduction.
    """

    @staticmethod
    def forward(ctx, val, w, row_ptr, ent, graph, r_size, topk_edges, c1, flags, mask_triple, eps, stats, status,
                vis=None, keep_zeros=False):
        v = val.detach().contiguous()
        rows = row_ptr.numel() - 1
        ctx.pruned = None
        ctx.n_in = v.numel()
        ctx.sel_live = None
        ctx.in_live = row_ptr[rows:]  # live entries of the (capacity-sized) input
        if c1 is not None and c1 >= 0:
            # a row with at most c1 nonzero values keeps its explicit zeros too
            # (flashlog_kernel.py:1114-1117): with zeros in the state (dropout)
            # only the input's size bounds the selection; otherwise an
            # underflow to zero past rows * c1 is flagged in `status`
            cap = v.numel() if keep_zeros else min(v.numel(), rows * int(c1))
            rp, en, vv, src = ops.topc_select(row_ptr, ent, v, int(c1), sync=False, out_capacity=cap, status=status)
            row_ptr, ent, v, ctx.pruned = rp, en, vv, src
            ctx.sel_live = rp[rows:]
        wf = w.detach().contiguous()
        fw = ops.hop_forward(row_ptr, ent, v, wf, graph, r_size, topk_edges, flags, mask_triple=mask_triple, eps=eps,
                             timing=None if stats is None else stats.timer, status=status, out_sync=False, vis=vis)
        if stats is not None:
            stats.append((ent, row_ptr[rows:], fw.entry_count, fw.out_row_ptr[rows:]))
        ctx.fw = fw
        ctx.save_for_backward(row_ptr, v, wf)
        ctx.mark_non_differentiable(fw.out_row_ptr, fw.out_ent)
        return fw.out_y, fw.out_row_ptr, fw.out_ent

    @staticmethod
    def backward(ctx, g_y, _g_rp, _g_ent):
        row_ptr, v, wf = ctx.saved_tensors
        grad_v, grad_w = ops.hop_backward(ctx.fw, row_ptr, v, wf, g_y, normalize=True)
        if ctx.pruned is not None:
            grad_v = ops.scatter_grad(grad_v, ctx.pruned, ctx.n_in, n_live=ctx.sel_live, full_live=ctx.in_live)
        return grad_v, grad_w, None, None, None, None, None, None, None, None, None, None, None, None, None


class Readout(torch.autograd.Function):
    """Channel-summed score of each query's target entity."""

    @staticmethod
    def forward(ctx, val, row_ptr, ent, targets, N):
        ctx.save_for_backward(row_ptr, ent, targets)
        ctx.N = N
        ctx.n_val = val.numel()
        return ops.readout(row_ptr, ent, val.detach(), N, targets)

    @staticmethod
    def backward(ctx, g):
        row_ptr, ent, targets = ctx.saved_tensors
        return (ops.readout_backward(row_ptr, ent, ctx.N, targets, g, ctx.n_val, val_live=row_ptr[-1:]),
                None, None, None, None)


def initial_state(heads: torch.Tensor, N: int):
    """One entry (h, value 1) per (query, channel) row."""
    Q = heads.numel()
    dev = heads.device
    row_ptr = torch.arange(Q * N + 1, dtype=torch.int64, device=dev)
    ent = heads.to(torch.int32).repeat_interleave(N)
    val = torch.ones(Q * N, dtype=torch.float32, device=dev)
    return row_ptr, ent, val


def readout_loss(row_ptr, ent, val, tails, N: int, tau_2: float = 1.0, thr: float = 1e-7):
    """log_loss_common_sp of the channel-summed scores (src/utils.py:36-47)."""
    score = Readout.apply(val, row_ptr, ent, tails, N)
    return -torch.mean(torch.log(torch.maximum(score / tau_2, torch.full_like(score, thr))))


def new_status(device):
    """Sticky device status word for the hop kernels (FL_STATUS_* bits)."""
    return torch.zeros(1, dtype=torch.int32, device=device)


def check_status(status):
    """Raise if any hop ran out of its buffers (one host sync)."""
    v = int(status.item())
    if v & L.FL_STATUS_SLOT_OVERFLOW:
        raise RuntimeError("a hop exceeded its entry or fact capacity; results of this step are invalid")


def drum_propagate(heads, w_all, graph: Graph, r_size: int, *, c1=None, c2=0, mask_triple=None, tau_1=1.0,
                   eps=1e-7, stats=None, status=None, dropout=0.0, dropout_seed=None, dropout_counter=0):
    """T hops of the sparse DRUM operator; w_all is [Q, T, N, n] logits.

    dropout > 0: the training dropout of each hop's values
    (src/model_DRUM_kernel_sp.py:189-192), hop t drawing its keep bits from
    (dropout_seed, dropout_counter, t) -- the masks DrumTrainStep draws on its
    replay number dropout_counter.

    Returns the final state (row_ptr, ent, val) with capacity-sized ent/val
    (live count row_ptr[-1]).
    """
    Q, T, N, n = w_all.shape
    row_ptr, ent, val = initial_state(heads, N)
    topk = c2 // 2 if c2 and c2 > 0 else L.NO_BUDGET
    flags = L.FL_SKIP_NONPOS_W | L.FL_DROP_MASKED
    own_status = status is None
    if own_status:
        status = new_status(heads.device)
    # hidden triples in CSR order, shared by the T hops
    vis = ops.csr_visibility(graph, mask_triple) if mask_triple is not None else None
    drop = None
    if dropout:
        from .dropout import device_counter, draw_seed, ValueDropout
        drop = (float(dropout), draw_seed() if dropout_seed is None else int(dropout_seed),
                device_counter(dropout_counter, heads.device))
    for t in range(T):
        w_t = torch.softmax(w_all[:, t] / tau_1, dim=-1)
        val, row_ptr, ent = HopNorm.apply(val, w_t, row_ptr, ent, graph, r_size, topk, c1, flags, mask_triple, eps,
                                          stats, status, vis, drop is not None)
        if drop is not None:
            val = ValueDropout.apply(val, drop[0], drop[1], drop[2], t, row_ptr[-1:])
    if own_status:
        check_status(status)
    return row_ptr, ent, val
