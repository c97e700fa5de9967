"""Drop-in replacement of the reference operator module flashlog_kernel.flashlog_kernel.

Same public names, argument orders, return types and error behaviour as the
reference's flashlog_kernel/flashlog_kernel.py; the work runs in the sm_100a
kernels of libflashlog_b200.so.  There is no CPU path: CPU tensors raise
ValueError (the reference's OpenMP path is this build's timed CPU baseline,
not a fallback).
"""
from __future__ import annotations

import dataclasses
import os
import time

import weakref

import torch
from torch import autograd

from . import _lib as L
from . import ops
from .ops import Graph

_FLASHLOG_CPU_THREADS_CONFIGURED = False


# ---------------------------------------------------------------------------
# Host configuration (flashlog_kernel.py:13-102)
# ---------------------------------------------------------------------------
def _flashlog_available_logical_cpus():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def configure_flashlog_cpu_threads(force=False):
    """Apply FLASHLOG_CPU_THREADS / FLASHLOG_CPU_INTEROP_THREADS to torch's host threads.

    Semantics of flashlog_kernel.py:60-102: unset/off/none/false/0 leaves torch
    alone, "auto" picks a bandwidth-friendly count, an integer forces it.
    """
    global _FLASHLOG_CPU_THREADS_CONFIGURED
    if _FLASHLOG_CPU_THREADS_CONFIGURED and not force:
        return torch.get_num_threads()
    setting = os.environ.get("FLASHLOG_CPU_THREADS", "off").strip().lower()
    logical = max(1, _flashlog_available_logical_cpus())
    if setting in ("off", "none", "false", "0"):
        _FLASHLOG_CPU_THREADS_CONFIGURED = True
        return torch.get_num_threads()
    if setting in ("", "auto"):
        target = logical if logical < 24 else min(16, max(8, logical // 2))
    else:
        try:
            target = int(setting)
        except ValueError:
            target = logical
    target = max(1, min(target, logical))
    if torch.get_num_threads() != target:
        torch.set_num_threads(target)
    interop = os.environ.get("FLASHLOG_CPU_INTEROP_THREADS")
    if interop is not None:
        try:
            n = max(1, int(interop))
            if torch.get_num_interop_threads() != n:
                torch.set_num_interop_threads(n)
        except (ValueError, RuntimeError):
            pass
    _FLASHLOG_CPU_THREADS_CONFIGURED = True
    return torch.get_num_threads()


def _kernel_stage_timing_enabled():
    return os.environ.get("FLASHLOG_STAGE_TIMING", "") == "1"


def _kernel_log(stage, start_time):
    """StageTiming lines of flashlog_kernel.py:158-165 (FLASHLOG_STAGE_TIMING=1)."""
    if not _kernel_stage_timing_enabled():
        return
    if torch.cuda.is_available():
        torch.cuda.synchronize()
    print("StageTiming flashlog_kernel stage:{} seconds:{:.4f}".format(stage, time.perf_counter() - float(start_time)))


def get_module():
    """The native library (the reference JIT-builds a torch extension here)."""
    return L.lib()


def score_function(x):
    return torch.sigmoid(x)


def _cuda_or_raise(t, what="operator"):
    if not t.is_cuda:
        raise ValueError(f"flashlog_b200 {what} requires CUDA tensors (no CPU path)")


# ---------------------------------------------------------------------------
# CSR construction (flashlog_kernel.py:626-697)
# ---------------------------------------------------------------------------
def _group_starts_and_counts(sorted_values, sorted_relations=None):
    """Group boundaries of sorted keys (flashlog_kernel.py:637-660); returns int32 (starts, counts)."""
    n = sorted_values.numel()
    if not n:
        return torch.empty(0, dtype=torch.int32), torch.empty(0, dtype=torch.int32)
    flags = torch.ones(n, dtype=torch.bool, device=sorted_values.device)
    flags[1:] = sorted_values[1:] != sorted_values[:-1]
    if sorted_relations is not None:
        flags[1:] |= sorted_relations[1:] != sorted_relations[:-1]
    starts = flags.nonzero().flatten().to(torch.int32)
    counts = torch.empty_like(starts)
    counts[:-1] = starts[1:] - starts[:-1]
    counts[-1] = n - starts[-1]
    return starts, counts


def build_csr_structure(row_indices, col_indices, r_indices, num_nodes):
    """16-tuple CSR of both directions, built on the GPU (replaces csr.cpp:12-69).

    Output layout and ordering are those of the reference (edges by source,
    relation, triple id); tensors are returned on the input's device.
    """
    device = row_indices.device
    cdev = device if device.type == "cuda" else torch.device("cuda", torch.cuda.current_device())
    row, col, rel = (x.detach().to(device=cdev, dtype=torch.int64).contiguous()
                     for x in (row_indices, col_indices, r_indices))
    relations = int(rel.max().item()) + 1 if rel.numel() else 0
    if rel.numel() and (int(rel.min().item()) < 0 or relations - 1 > 32767):
        raise ValueError("CSR entity or relation ID outside supported range")
    nodes = int(num_nodes)
    ori = ops.build_csr_side(row, col, rel, nodes, relations)
    inv = ops.build_csr_side(col, row, rel, nodes, relations)
    out = (*ori[:4], *inv[:4], *ori[4:], *inv[4:])
    if device != cdev:
        out = tuple(t.to(device) for t in out)
    return out


def _apply_mask_order(mask_values, order, weight=None):
    """CSR-ordered float mask of one side through fl_csr_mask (flashlog.cu:1286-1340)."""
    mask_f = (mask_values if mask_values.dtype == torch.bool else mask_values.float()).contiguous().view(-1)
    _cuda_or_raise(mask_f, "mask preparation")
    order_i = order.to(device=mask_f.device, dtype=torch.int32).contiguous()
    wt = None
    if weight is not None:
        wt = weight.to(device=mask_f.device, dtype=torch.float32).squeeze(-1).contiguous().view(-1)
    return ops.csr_mask(mask_f, order_i, wt)


def _prepared_mask_pair(mask_values):
    if (isinstance(mask_values, (tuple, list)) and len(mask_values) == 2 and
            torch.is_tensor(mask_values[0]) and torch.is_tensor(mask_values[1])):
        return mask_values[0].contiguous().float(), mask_values[1].contiguous().float()
    return None


def prepare_csr_masks(csr_struct, mask_values, weight=None):
    """CSR-ordered ORI/INV masks for one model forward (flashlog_kernel.py:250-255)."""
    return (_apply_mask_order(mask_values, csr_struct[3], weight),
            _apply_mask_order(mask_values, csr_struct[7], weight))


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------
def _coo(row_ptr, ent, values, B, Lch, E):
    idx = ops.rows_to_coo(row_ptr, ent, Lch)
    return torch.sparse_coo_tensor(idx, values, [B, Lch, E], is_coalesced=True)


def _align_sparse_grad_to_output(grad, out_indices, Lch, E):
    """Upstream gradient at the forward's output coordinates (the role of
    flashlog_kernel.py:360-376), looked up on the row layout by fl_align_rows.

    A dense gradient is indexed directly.  A sparse gradient that sits on the
    output's own index tensor aligns one to one.  Any other sparse gradient is
    coalesced, put in the row layout, and every output coordinate is searched
    in its own row (missing coordinates get 0)."""
    if not grad.is_sparse:
        return grad[tuple(out_indices)].contiguous()
    raw = grad._indices()
    if raw.shape == out_indices.shape and raw.data_ptr() == out_indices.data_ptr():
        return grad._values().contiguous()
    grad = grad.coalesce()
    B = int(grad.shape[0])
    gi = grad.indices()
    g_row_ptr, g_ent, _ = ops.coo_to_rows(gi[0], gi[1], gi[2], B, Lch, E)
    return ops.align_rows(out_indices, Lch, B * Lch, g_row_ptr, g_ent, grad.values().to(torch.float32).contiguous())


def _rows(sp_batch, sp_level, sp_entity, B, Lch, E, graph=None):
    if graph is not None and graph.E < E:
        raise ValueError(f"the CSR covers {graph.E} entities but the state has {E}")
    row_ptr, ent, bad = ops.coo_to_rows(sp_batch, sp_level, sp_entity, B, Lch, E)
    return row_ptr, ent, bad


def _check_bad(bad):
    if int(bad.item()):
        raise ValueError("sparse state indices are out of range or not coalesced")


def _select_sources(ctx, row_ptr, ent, val, topk_nodes, sampling):
    """c1 selection; records the kept indices for the backward (flashlog_kernel.py:1140-1155)."""
    ctx.pruned = None
    ctx.original_input_size = val.numel()
    if topk_nodes is None:
        return row_ptr, ent, val
    if topk_nodes < 0:
        raise ValueError("topk_nodes/c must be nonnegative")
    if val.numel() <= topk_nodes:
        return row_ptr, ent, val
    noise = None
    if sampling:
        ncand = ops.topc_candidates(row_ptr, val, int(topk_nodes))
        if ncand:
            nz = val[val != 0]
            if not bool(torch.isfinite(nz).all()) or bool((nz <= 0).any()):
                raise ValueError("Entity sampling requires finite nonnegative state scores")
            # Exponential race noise from torch's generator, one draw per candidate in state order.
            noise = torch.empty(ncand, device=val.device, dtype=torch.float64).exponential_()
    sel_row_ptr, sel_ent, sel_val, src = ops.topc_select(row_ptr, ent, val, int(topk_nodes), noise)
    if src.numel() == val.numel():
        return row_ptr, ent, val
    ctx.pruned = src
    return sel_row_ptr, sel_ent, sel_val


def _select_sources_async(ctx, row_ptr, ent, val, topk_nodes, rows, status=None, full=False):
    """Deterministic c1 without a host sync: outputs keep min(S, 2 * rows * c1)
    entries (S with full=True), their live count stays on the device
    (row_ptr[rows]).  A row with at most c1 nonzero values keeps its explicit
    zeros too (flashlog_kernel.py:1114-1117), so rows * c1 is no bound once
    the state holds zeros (training dropout puts a few percent past it; the
    factor 2 absorbs that).  When even that falls short,
    FL_STATUS_SLOT_OVERFLOW is set in `status` and the caller selects again
    with full=True."""
    ctx.pruned = None
    ctx.n_live = None
    ctx.original_input_size = val.numel()
    if topk_nodes is None:
        return row_ptr, ent, val
    if topk_nodes < 0:
        raise ValueError("topk_nodes/c must be nonnegative")
    if val.numel() <= topk_nodes:
        return row_ptr, ent, val
    cap = val.numel() if full else min(val.numel(), 2 * rows * int(topk_nodes))
    sel_row_ptr, sel_ent, sel_val, src = ops.topc_select(row_ptr, ent, val, int(topk_nodes), sync=False,
                                                         out_capacity=cap, status=status)
    ctx.pruned = src
    ctx.n_live = sel_row_ptr[rows:]
    return sel_row_ptr, sel_ent, sel_val


def _restore(ctx, grad):
    if ctx.pruned is None:
        return grad
    return ops.scatter_grad(grad, ctx.pruned, ctx.original_input_size, n_live=getattr(ctx, "n_live", None))


def _graph_topk(csr_args):
    (ori_row_ptr, ori_col_ind, ori_r_ind, ori_order, inv_row_ptr, inv_col_ind, inv_r_ind, inv_order,
     ori_gp, ori_gr, ori_gs, ori_gc, inv_gp, inv_gr, inv_gs, inv_gc) = csr_args
    return Graph.of((ori_row_ptr, ori_col_ind, ori_r_ind, ori_order, inv_row_ptr, inv_col_ind, inv_r_ind,
                     inv_order, ori_gp, ori_gr, ori_gs, ori_gc, inv_gp, inv_gr, inv_gs, inv_gc))


_VISIBILITY = {}  # the last (graph, mask, mask version) -> CSR-ordered visibility bytes
_VISIBILITY_MAX_EDGES = 1 << 26


def _visibility(graph, mask_values):
    """CSR-ordered visibility bytes (ops.csr_visibility) of a triple mask, for
    the top-k hops without edge weights: a hop then reads one byte beside the
    edge instead of mask[order[p]].  The model calls every hop of a step with
    the same mask tensor, so the bytes are kept for the last (graph, mask) and
    rebuilt when torch's version counter of the mask changes (an in-place
    write such as mask[hide] = False).  Returns None for a mask that is not a
    CUDA tensor with one entry per triple, and for graphs of more than 2^26
    edges per side: the bytes are rebuilt for every mask version (every
    training step), and on such graphs the rebuild costs more than the per-fact
    mask reads it saves (the hop then reads the mask)."""
    if (mask_values is None or not isinstance(mask_values, torch.Tensor) or not mask_values.is_cuda
            or mask_values.numel() < graph.csr[1].numel() or graph.csr[1].numel() > _VISIBILITY_MAX_EDGES):
        return None
    hit = _VISIBILITY.get("last")
    if (hit is not None and hit[0]() is graph and hit[1]() is mask_values and hit[2] == mask_values._version):
        return hit[3]
    vis = ops.csr_visibility(graph, mask_values)
    _VISIBILITY["last"] = (weakref.ref(graph), weakref.ref(mask_values), mask_values._version, vis)
    return vis


def _graph_groups(ori_col, ori_gp, ori_gr, ori_gs, ori_gc, inv_col, inv_gp, inv_gr, inv_gs, inv_gc):
    """Graph view from group arrays only (the all-edges operator passes no row_ptr/order)."""
    dev = ori_col.device
    z = torch.empty(0, dtype=torch.int32, device=dev)
    return Graph.of((ori_gp, ori_col, z.to(torch.int16), z, inv_gp, inv_col, z.to(torch.int16), z,
                     ori_gp, ori_gr, ori_gs, ori_gc, inv_gp, inv_gr, inv_gs, inv_gc))


def _topk_flags(weight, edge_weight_is_score, sampling, wot_i):
    flags = L.FL_SKIP_NONPOS_W | L.FL_DROP_MASKED
    if weight is not None:
        flags |= L.FL_EDGE_WEIGHT
        if edge_weight_is_score:
            flags |= L.FL_EDGE_SCORE
    if sampling:
        flags |= L.FL_SAMPLED
    if wot_i:
        flags |= L.FL_WOT_I
    return flags


def _check_w(w):
    if not bool(torch.isfinite(w).all()):
        raise RuntimeError("FlashLog sparse top-k received non-finite attention weights; "
                           "aborting before edge count/fill to prevent uninitialized indices")


# The row layouts of the last states the fused operator returned, keyed by
# their index tensor: a state on one of these index tensors (the output
# itself, or a state built on its indices, as the models' value dropout
# does) skips the host read of the index check (its indices were written by
# the library, in range and coalesced) and the COO -> row conversion.  Each
# entry holds its index tensor, so the storage cannot be reused while it is
# listed; torch's version counter catches an in-place write to the indices.
_OWN_ROWS = []  # (indices, version, row_ptr, ent), newest last
_OWN_ROWS_KEEP = 2


def _mark_own_output(t, row_ptr, ent):
    idx = t._indices()
    _OWN_ROWS.append((idx, idx._version, row_ptr, ent))
    del _OWN_ROWS[:-_OWN_ROWS_KEEP]


def _own_rows(t):
    """(row_ptr, ent) of a state on the indices of a recent output, else None."""
    idx = t._indices()
    for i, v, rp, e in reversed(_OWN_ROWS):
        if (i.data_ptr() == idx.data_ptr() and i.shape == idx.shape and i.stride() == idx.stride()
                and i._version == v):
            return rp, e
    return None


def _check_bad_and_w(bad, w):
    """_check_bad then _check_w with one host read of both device flags."""
    flags = torch.stack([bad.reshape(-1)[0].to(torch.int32),
                         (~torch.isfinite(w)).any().to(torch.int32)]).cpu()
    if int(flags[0]):
        raise ValueError("sparse state indices are out of range or not coalesced")
    if int(flags[1]):
        raise RuntimeError("FlashLog sparse top-k received non-finite attention weights; "
                           "aborting before edge count/fill to prevent uninitialized indices")


# ---------------------------------------------------------------------------
# Sparse SUM operators
# ---------------------------------------------------------------------------
class FlashLogFunctionSparse3DTopKSum(autograd.Function):
    """Sparse sum with c1/c2 budgets (flashlog_kernel.py:1158-1348), 33 positional arguments."""

    @staticmethod
    def forward(ctx, sp_batch, sp_level, sp_entity, sp_value, w,
                ori_row_ptr, ori_col_ind, ori_r_ind, ori_order,
                inv_row_ptr, inv_col_ind, inv_r_ind, inv_order,
                ori_row_group_ptr, ori_group_rel, ori_group_edge_start, ori_group_edge_count,
                inv_row_group_ptr, inv_group_rel, inv_group_edge_start, inv_group_edge_count,
                mask_values, weight, B, L_, E, r_size, wot_i, topk_edges,
                edge_weight_is_score=False, topk_nodes=None, cache_backward=True, sampling=False):
        _cuda_or_raise(sp_value)
        t0 = time.perf_counter()
        graph = _graph_topk((ori_row_ptr, ori_col_ind, ori_r_ind, ori_order, inv_row_ptr, inv_col_ind, inv_r_ind,
                             inv_order, ori_row_group_ptr, ori_group_rel, ori_group_edge_start,
                             ori_group_edge_count, inv_row_group_ptr, inv_group_rel, inv_group_edge_start,
                             inv_group_edge_count))
        val = sp_value.detach().to(torch.float32).contiguous()
        row_ptr, ent, bad = _rows(sp_batch, sp_level, sp_entity, B, L_, E, graph)
        _check_bad(bad)
        row_ptr, ent, val = _select_sources(ctx, row_ptr, ent, val, topk_nodes, sampling)
        _kernel_log("sparse3d_topk_sum.select", t0)
        t0 = time.perf_counter()
        wf = w.detach().to(torch.float32).contiguous()
        _check_w(wf)
        seed = int(torch.randint(0, 2 ** 63 - 1, ()).item()) if sampling else -1
        learn_ew = weight is not None and bool(getattr(weight, "requires_grad", False))
        vis = _visibility(graph, mask_values) if weight is None else None
        fw = ops.hop_forward(row_ptr, ent, val, wf, graph, r_size, int(topk_edges),
                             _topk_flags(weight, edge_weight_is_score, sampling, wot_i),
                             mask_triple=None if vis is not None else mask_values, vis=vis,
                             edge_weight=None if weight is None else weight.detach(),
                             seed=seed, record_edge=learn_ew)
        _kernel_log("sparse3d_topk_sum.cuda_forward", t0)
        ctx.fw = fw
        ctx.save_for_backward(row_ptr, val, wf)
        ctx.B, ctx.L, ctx.E = B, L_, E
        ctx.edge_weight = weight.detach() if learn_ew else None
        out = _coo(fw.out_row_ptr, fw.out_ent, fw.out_x, B, L_, E)
        ctx.out_indices = out.indices()
        return out

    @staticmethod
    def backward(ctx, grad_out):
        row_ptr, val, wf = ctx.saved_tensors
        g = _align_sparse_grad_to_output(grad_out, ctx.out_indices, ctx.L, ctx.E).to(torch.float32)
        grad_val, grad_w = ops.hop_backward(ctx.fw, row_ptr, val, wf, g, normalize=False)
        grad_ew = _edge_weight_grad(ctx, row_ptr, val, wf, g)
        grad_val = _restore(ctx, grad_val)
        grads = (None, None, None, grad_val, grad_w) + (None,) * 17 + (grad_ew,) + (None,) * 10
        return grads[:len(ctx.needs_input_grad)]


def _edge_weight_grad(ctx, row_ptr, val, wf, g):
    """Gradient of the learnable edge weights (argument 22 of the top-k
    operators), or None when they take none (flashlog_kernel.py:1306-1336,
    1590-1614)."""
    if ctx.edge_weight is None:
        return None
    return ops.edge_weight_grad(ctx.fw, row_ptr, val, wf, g, ctx.edge_weight)


class FlashLogFunctionSparse3DAllEdgesSum(autograd.Function):
    """Sparse sum over every edge (flashlog_kernel.py:1351-1447), 22 positional arguments."""

    @staticmethod
    def forward(ctx, sp_batch, sp_level, sp_entity, sp_value, w,
                ori_col_ind, ori_mask,
                ori_row_group_ptr, ori_group_rel, ori_group_edge_start, ori_group_edge_count,
                inv_col_ind, inv_mask,
                inv_row_group_ptr, inv_group_rel, inv_group_edge_start, inv_group_edge_count,
                B, L_, E, r_size, wot_i, cache_backward=True):
        _cuda_or_raise(sp_value)
        graph = _graph_groups(ori_col_ind, ori_row_group_ptr, ori_group_rel, ori_group_edge_start,
                              ori_group_edge_count, inv_col_ind, inv_row_group_ptr, inv_group_rel,
                              inv_group_edge_start, inv_group_edge_count)
        val = sp_value.detach().to(torch.float32).contiguous()
        row_ptr, ent, bad = _rows(sp_batch, sp_level, sp_entity, B, L_, E, graph)
        _check_bad(bad)
        ctx.pruned = None
        wf = w.detach().to(torch.float32).contiguous()
        flags = L.FL_WOT_I if wot_i else 0
        fw = ops.hop_forward(row_ptr, ent, val, wf, graph, r_size, L.NO_BUDGET, flags,
                             mask_csr=(ori_mask, inv_mask))
        ctx.fw = fw
        ctx.save_for_backward(row_ptr, val, wf)
        ctx.B, ctx.L, ctx.E = B, L_, E
        out = _coo(fw.out_row_ptr, fw.out_ent, fw.out_x, B, L_, E)
        ctx.out_indices = out.indices()
        return out

    @staticmethod
    def backward(ctx, grad_out):
        row_ptr, val, wf = ctx.saved_tensors
        g = _align_sparse_grad_to_output(grad_out, ctx.out_indices, ctx.L, ctx.E).to(torch.float32)
        grad_val, grad_w = ops.hop_backward(ctx.fw, row_ptr, val, wf, g, normalize=False)
        grads = (None, None, None, grad_val, grad_w) + (None,) * 18
        return grads[:len(ctx.needs_input_grad)]


# Fact counts of recent hops, by (graph, rows, input size class, c2, c1,
# flags): a hop like one seen before sizes its fact buffers from that count
# (with headroom) and skips the host read of the exact count.
_FACTS_SEEN = {}


def _remember_facts(key, n):
    if len(_FACTS_SEEN) > 256:
        _FACTS_SEEN.clear()
    _FACTS_SEEN[key] = max(int(n), 1)


def _speculative_hop(ctx, key, state, wf, graph, r_size, topk_edges, flags, topk_nodes, rows, hop_args):
    """The hop with fact buffers of 1.5x the count of the last hop with the
    same key and no host read before the launches: the output count, the
    buffers' overflow status, the c1 selection's status and the weights'
    finiteness come back in one read after the reduction.  Returns
    (fw, selected state), or None when there is no count to go by or a
    buffer ran short (the caller then sizes the buffers exactly).  Non-finite
    weights raise the top-k operators' RuntimeError."""
    seen = _FACTS_SEEN.get(key)
    if seen is None:
        return None
    dev = wf.device
    sel_status = torch.zeros(1, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    sel = _select_sources_async(ctx, *state, topk_nodes, rows, sel_status, False)
    finite = torch.isfinite(wf)
    nonfinite = (~finite).any()
    # the kernels run before the finiteness is read, so they get the weights
    # with non-finite entries zeroed; such a call raises below and its outputs are dropped
    fw = ops.hop_forward(*sel, torch.where(finite, wf, torch.zeros_like(wf)), graph, r_size, topk_edges, flags,
                         slot_capacity=seen * 3 // 2 + 1024, status=status, out_sync=False, **hop_args)
    got = torch.stack([fw.out_row_ptr[rows], fw.slot_base[sel[1].numel()], status[0].to(torch.int64),
                       sel_status[0].to(torch.int64), nonfinite.to(torch.int64)]).cpu().tolist()
    if got[4]:
        raise RuntimeError("FlashLog sparse top-k received non-finite attention weights; "
                           "aborting before edge count/fill to prevent uninitialized indices")
    if (got[2] | got[3]) & L.FL_STATUS_SLOT_OVERFLOW:
        return None
    _remember_facts(key, got[1])
    u = got[0]
    fw = dataclasses.replace(fw, out_ent=fw.out_ent[:u], out_x=fw.out_x[:u], out_y=fw.out_y[:u],
                             n_facts_slots=got[1])
    return fw, sel


class _Sparse3DSumNormFused(autograd.Function):
    """c1 + expansion + coalesce-sum + row normalization as one node.

    Equal to normalize_sparse3d(FlashLogFunctionSparse3DTopKSum(...)) of the
    reference's CUDA path (flashlog_kernel.py:1908-1916); the normalization is
    computed in the same kernel that reduces the rows.
    """

    @staticmethod
    def forward(ctx, sp_value, w, sp_batch, sp_level, sp_entity, csr, mask_values, weight, B, L_, E, r_size, wot_i,
                topk_edges, topk_nodes, sampling, all_edges, masks_csr, eps, own_rows=None):
        _cuda_or_raise(sp_value)
        val = sp_value.detach().to(torch.float32).contiguous()
        graph = Graph.of(csr)
        trusted = own_rows is not None
        if trusted:
            if graph.E < E:
                raise ValueError(f"the CSR covers {graph.E} entities but the state has {E}")
            (row_ptr, ent), bad = own_rows, None
        else:
            row_ptr, ent, bad = _rows(sp_batch, sp_level, sp_entity, B, L_, E, graph)
        wf = w.detach().to(torch.float32).contiguous()
        if all_edges:
            if not trusted:
                _check_bad(bad)
            ctx.pruned = None
            fw = ops.hop_forward(row_ptr, ent, val, wf, graph, r_size, L.NO_BUDGET, L.FL_WOT_I if wot_i else 0,
                                 mask_csr=masks_csr, eps=eps)
        elif not sampling:
            if topk_nodes is not None and topk_nodes < 0:
                raise ValueError("topk_nodes/c must be nonnegative")
            if not trusted:
                _check_bad(bad)
            state = (row_ptr, ent, val)
            sel_status = torch.zeros(1, dtype=torch.int32, device=val.device)
            vis = _visibility(graph, mask_values) if weight is None else None
            hop_args = dict(mask_triple=None if vis is not None else mask_values, vis=vis,
                            edge_weight=None if weight is None else weight.detach(), seed=-1, eps=eps)
            flags = _topk_flags(weight, False, sampling, wot_i)
            key = (id(graph), B * L_, int(ent.numel()).bit_length(), int(topk_edges), topk_nodes, flags)
            fw = _speculative_hop(ctx, key, state, wf, graph, r_size, int(topk_edges), flags, topk_nodes, B * L_,
                                  hop_args)
            if fw is not None:
                fw, (row_ptr, ent, val) = fw
            else:
                for full in (False, True):
                    row_ptr, ent, val = _select_sources_async(ctx, *state, topk_nodes, B * L_, sel_status, full)
                    try:
                        fw = ops.hop_forward(row_ptr, ent, val, wf, graph, r_size, int(topk_edges), flags,
                                             check_w=True, sel_status=None if full else sel_status, **hop_args)
                        break
                    except ops.SelectionOverflow:
                        continue  # explicit zeros past rows * c1: select again at the input's size
                _remember_facts(key, fw.n_facts_slots)
        else:
            if not trusted:
                _check_bad(bad)
            row_ptr, ent, val = _select_sources(ctx, row_ptr, ent, val, topk_nodes, sampling)
            _check_w(wf)
            seed = int(torch.randint(0, 2 ** 63 - 1, ()).item()) if sampling else -1
            fw = ops.hop_forward(row_ptr, ent, val, wf, graph, r_size, int(topk_edges),
                                 _topk_flags(weight, False, sampling, wot_i), mask_triple=mask_values,
                                 edge_weight=None if weight is None else weight.detach(), seed=seed, eps=eps)
        ctx.fw = fw
        ctx.save_for_backward(row_ptr, val, wf)
        ctx.B, ctx.L, ctx.E = B, L_, E
        out = _coo(fw.out_row_ptr, fw.out_ent, fw.out_y, B, L_, E)
        ctx.out_indices = out.indices()
        _mark_own_output(out, fw.out_row_ptr, fw.out_ent)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        row_ptr, val, wf = ctx.saved_tensors
        g = _align_sparse_grad_to_output(grad_out, ctx.out_indices, ctx.L, ctx.E).to(torch.float32)
        grad_val, grad_w = ops.hop_backward(ctx.fw, row_ptr, val, wf, g, normalize=True)
        grad_val = _restore(ctx, grad_val)
        return (grad_val, grad_w) + (None,) * 18


class Sparse3DNormalizeFunction(autograd.Function):
    """Row normalization of a coalesced sparse state (flashlog_kernel.py:536-607)."""

    @staticmethod
    def forward(ctx, sp_batch, sp_level, sp_entity, sp_value, B, L_, E, eps):
        _cuda_or_raise(sp_value)
        x = sp_value.detach().to(torch.float32).contiguous()
        row_ptr, ent, bad = _rows(sp_batch, sp_level, sp_entity, B, L_, E)
        _check_bad(bad)
        y, denom = ops.normalize_forward(row_ptr, x, float(eps))
        ctx.save_for_backward(row_ptr, x, denom)
        ctx.eps = float(eps)
        idx = torch.stack([sp_batch.long(), sp_level.long(), sp_entity.long()], dim=0)
        ctx.idx = idx
        ctx.L, ctx.E = L_, E
        return torch.sparse_coo_tensor(idx, y, [B, L_, E], is_coalesced=True)

    @staticmethod
    def backward(ctx, grad_out):
        row_ptr, x, denom = ctx.saved_tensors
        g = _align_sparse_grad_to_output(grad_out, ctx.idx, ctx.L, ctx.E).to(torch.float32)
        gx = ops.normalize_backward(row_ptr, x, denom, g, ctx.eps)
        return None, None, None, gx, None, None, None, None


def normalize_sparse3d(s, eps=1e-7):
    s = s if s.is_coalesced() else s.coalesce()
    idx = s.indices()
    B, L_, E = s.shape
    return Sparse3DNormalizeFunction.apply(idx[0], idx[1], idx[2], s.values(), B, L_, E, eps)


def _csr_parts(csr_struct):
    return tuple(csr_struct)


def vectorized_operation_sparse3d_csr_sum(sp_state, w, csr_struct, mask_values, r_size, weight=None, wot_i=False,
                                          use_topk=False, topk_edges=0, prepared_masks=None, topk_nodes=None,
                                          sampling=False):
    """One hop, coalesced sum (flashlog_kernel.py:1814-1888, CUDA dispatch)."""
    if sampling and use_topk:
        return sampled_sparse_propagation(sp_state, w, csr_struct, mask_values, r_size, weight, wot_i, topk_nodes,
                                          topk_edges, "sum")
    sp_state = sp_state.coalesce()
    _cuda_or_raise(sp_state)
    idx = sp_state.indices()
    val = sp_state.values()
    B, L_, E = sp_state.shape
    c = _csr_parts(csr_struct)
    effective_topk = topk_edges if (use_topk and topk_edges > 0) else (1 << 60)
    can_use_all_edges = not (use_topk and (topk_edges > 0 or topk_nodes is not None))
    can_use_all_edges = can_use_all_edges and not (weight is not None and bool(getattr(weight, "requires_grad", False)))
    if can_use_all_edges:
        prepared = _prepared_mask_pair(prepared_masks) if prepared_masks is not None else _prepared_mask_pair(mask_values)
        if prepared is not None:
            ori_mask, inv_mask = prepared
        else:
            ori_mask, inv_mask = prepare_csr_masks(csr_struct, mask_values, weight)
        return FlashLogFunctionSparse3DAllEdgesSum.apply(
            idx[0], idx[1], idx[2], val, w, c[1], ori_mask, c[8], c[9], c[10], c[11], c[5], inv_mask,
            c[12], c[13], c[14], c[15], B, L_, E, r_size, wot_i, torch.is_grad_enabled())
    return FlashLogFunctionSparse3DTopKSum.apply(
        idx[0], idx[1], idx[2], val, w, c[0], c[1], c[2], c[3], c[4], c[5], c[6], c[7],
        c[8], c[9], c[10], c[11], c[12], c[13], c[14], c[15],
        mask_values, weight, B, L_, E, r_size, wot_i, effective_topk,
        False, topk_nodes if use_topk else None, torch.is_grad_enabled())


def vectorized_operation_sparse3d_csr_sum_norm(sp_state, w, csr_struct, mask_values, r_size, weight=None,
                                               wot_i=False, use_topk=False, topk_edges=0, prepared_masks=None,
                                               eps=1e-7, topk_nodes=None, sampling=False):
    """One hop followed by row normalization (flashlog_kernel.py:1901-1954), fused in one kernel pass."""
    sp_state = sp_state.coalesce()
    _cuda_or_raise(sp_state)
    if weight is not None and bool(getattr(weight, "requires_grad", False)):
        return normalize_sparse3d(vectorized_operation_sparse3d_csr_sum(
            sp_state, w, csr_struct, mask_values, r_size, weight=weight, wot_i=wot_i, use_topk=use_topk,
            topk_edges=topk_edges, prepared_masks=prepared_masks, topk_nodes=topk_nodes, sampling=sampling), eps=eps)
    idx = sp_state.indices()
    B, L_, E = sp_state.shape
    sampled = bool(sampling and use_topk)
    if sampled:
        all_edges = False
        eff = topk_edges if topk_edges > 0 else (1 << 60)
        nodes = topk_nodes
    else:
        eff = topk_edges if (use_topk and topk_edges > 0) else (1 << 60)
        all_edges = not (use_topk and (topk_edges > 0 or topk_nodes is not None))
        nodes = topk_nodes if use_topk else None
    masks_csr = None
    if all_edges:
        prepared = _prepared_mask_pair(prepared_masks) if prepared_masks is not None else _prepared_mask_pair(mask_values)
        masks_csr = prepared if prepared is not None else prepare_csr_masks(csr_struct, mask_values, weight)
    # a state on the indices this operator returned: valid, coalesced, and in the row layout already
    own = _own_rows(sp_state)
    out = _Sparse3DSumNormFused.apply(sp_state.values(), w, idx[0], idx[1], idx[2], _csr_parts(csr_struct),
                                      mask_values, weight, B, L_, E, r_size, wot_i, eff, nodes, sampled,
                                      all_edges, masks_csr, eps, own)
    return out


def sampled_sparse_propagation(state, w, csr_struct, mask_values, r_size, weight=None, wot_i=False,
                               topk_nodes=None, topk_edges=0, mode="sum"):
    """Training-only c1/c2 sampling (flashlog_kernel.py:1957-1971)."""
    state = state.coalesce()
    _cuda_or_raise(state)
    idx, val = state.indices(), state.values()
    B, L_, E = state.shape
    function = FlashLogFunctionSparse3DTopKMax if mode == "max" else FlashLogFunctionSparse3DTopKSum
    return function.apply(idx[0], idx[1], idx[2], val, w, *csr_struct, mask_values, weight, B, L_, E, r_size, wot_i,
                          topk_edges if topk_edges > 0 else (1 << 60), False, topk_nodes, torch.is_grad_enabled(),
                          True)


class FlashLogFunctionSparse3DTopKMax(autograd.Function):
    """Sparse MAX propagation of smDRUM / mmDRUM (flashlog_kernel.py:1450-1626), 33 positional arguments.

    The top-k fill keeps hidden edges (value 0: the reference has no
    visibility filter on this path); every destination keeps its largest fact,
    ties going to the smaller source (ori, inv, identity) and then to the
    smaller triple id (flashlog_kernel.py:399-478).  The backward sends each
    output's gradient to its winning fact only (flashlog.cu:2363-2406).
    """

    @staticmethod
    def forward(ctx, sp_batch, sp_level, sp_entity, sp_value, w,
                ori_row_ptr, ori_col_ind, ori_r_ind, ori_order,
                inv_row_ptr, inv_col_ind, inv_r_ind, inv_order,
                ori_row_group_ptr, ori_group_rel, ori_group_edge_start, ori_group_edge_count,
                inv_row_group_ptr, inv_group_rel, inv_group_edge_start, inv_group_edge_count,
                mask_values, weight, B, L_, E, r_size, wot_i, topk_edges,
                edge_weight_is_score=False, topk_nodes=None, cache_backward=True, sampling=False):
        _cuda_or_raise(sp_value)
        t0 = time.perf_counter()
        graph = _graph_topk((ori_row_ptr, ori_col_ind, ori_r_ind, ori_order, inv_row_ptr, inv_col_ind, inv_r_ind,
                             inv_order, ori_row_group_ptr, ori_group_rel, ori_group_edge_start,
                             ori_group_edge_count, inv_row_group_ptr, inv_group_rel, inv_group_edge_start,
                             inv_group_edge_count))
        val = sp_value.detach().to(torch.float32).contiguous()
        row_ptr, ent, bad = _rows(sp_batch, sp_level, sp_entity, B, L_, E, graph)
        _check_bad(bad)
        row_ptr, ent, val = _select_sources(ctx, row_ptr, ent, val, topk_nodes, sampling)
        _kernel_log("sparse3d_topk_max.select", t0)
        t0 = time.perf_counter()
        wf = w.detach().to(torch.float32).contiguous()
        _check_w(wf)
        seed = int(torch.randint(0, 2 ** 63 - 1, ()).item()) if sampling else -1
        flags = _topk_flags(weight, edge_weight_is_score, sampling, wot_i) & ~L.FL_DROP_MASKED
        learn_ew = weight is not None and bool(getattr(weight, "requires_grad", False))
        fw = ops.hop_forward(row_ptr, ent, val, wf, graph, r_size, int(topk_edges), flags,
                             mask_triple=mask_values, edge_weight=None if weight is None else weight.detach(),
                             seed=seed, reduce="max", record_edge=learn_ew)
        _kernel_log("sparse3d_topk_max.cuda_forward", t0)
        ctx.fw = fw
        ctx.save_for_backward(row_ptr, val, wf)
        ctx.B, ctx.L, ctx.E = B, L_, E
        ctx.edge_weight = weight.detach() if learn_ew else None
        out = _coo(fw.out_row_ptr, fw.out_ent, fw.out_x, B, L_, E)
        ctx.out_indices = out.indices()
        return out

    @staticmethod
    def backward(ctx, grad_out):
        row_ptr, val, wf = ctx.saved_tensors
        g = _align_sparse_grad_to_output(grad_out, ctx.out_indices, ctx.L, ctx.E).to(torch.float32)
        grad_val, grad_w = ops.hop_backward(ctx.fw, row_ptr, val, wf, g, normalize=False)
        grad_ew = _edge_weight_grad(ctx, row_ptr, val, wf, g)  # winning facts only (fact_pos -1 elsewhere)
        grad_val = _restore(ctx, grad_val)
        grads = (None, None, None, grad_val, grad_w) + (None,) * 17 + (grad_ew,) + (None,) * 10
        return grads[:len(ctx.needs_input_grad)]


# ---------------------------------------------------------------------------
# Rule evaluator (flashlog_kernel.py:168-210)
# ---------------------------------------------------------------------------
def sparse2d_filtered_ranks_cuda(idx_b, idx_e, values, targets, filter_keys, B, E, use_eql=False):
    """Filtered tie-averaged ranks (flashlog.cu:2839-2910); filter_keys sorted ascending."""
    return ops.filtered_ranks(idx_b, idx_e, values, targets, filter_keys, int(B), int(E), bool(use_eql))


def vectorized_operation_sparse3d_fixed_relation(sp_state, operators, csr_struct, r_size):
    """Advance rule states through one fixed operator per (query, rule) (flashlog_kernel.py:182-210)."""
    if not sp_state.is_cuda:
        raise ValueError("fixed-relation rule inference currently requires CUDA")
    sp_state = sp_state.coalesce()
    indices = sp_state.indices()
    values = sp_state.values()
    B, L_, E = sp_state.shape
    if tuple(operators.shape) != (B, L_):
        raise ValueError("operators must have shape [{}, {}], got {}".format(B, L_, tuple(operators.shape)))
    c = tuple(csr_struct)
    graph = _graph_groups(c[1], c[8], c[9], c[10], c[11], c[5], c[12], c[13], c[14], c[15])
    row_ptr, ent, val = ops.fixed_relation(indices[0], indices[1], indices[2], values, operators, graph, int(r_size),
                                           B, L_)
    return _coo(row_ptr, ent, val.to(values.dtype), B, L_, E)


# ---------------------------------------------------------------------------
# Dense path (flashlog_kernel.py:700-1089)
# ---------------------------------------------------------------------------
def _compute_active_nodes(A):
    """Sorted unique active node indices of A [batch, L, E] (flashlog_kernel.py:617-623)."""
    non_zero = torch.nonzero(A.sum(1))
    if non_zero.numel() == 0:
        return torch.empty(0, dtype=torch.long, device=A.device)
    return torch.unique(non_zero[:, 1])


# ---------------------------------------------------------------------------
# Dense [B, L, E] propagation (config-1 models: src/model_DRUM_kernel.py,
# src/model_NeuralLP_kernel.py, src/model_{sm,mm}DRUM_kernel.py)
# ---------------------------------------------------------------------------
def _dense_state(A, active_nodes=None):
    """Nonzero entries of A [B, L, E] (entities in active_nodes only, when given)
    as a row layout in entity order; also their flat indices into A."""
    B, L_, E = A.shape
    BL = B * L_
    Af = A.detach().reshape(BL, E)
    nz = Af != 0
    if active_nodes is not None:
        act = torch.zeros(E, dtype=torch.bool, device=A.device)
        if active_nodes.numel():
            act[active_nodes.long()] = True
        nz &= act.unsqueeze(0)
    idx = nz.nonzero()
    rows, ent = idx[:, 0], idx[:, 1]
    counts = torch.bincount(rows, minlength=BL)
    row_ptr = torch.zeros(BL + 1, dtype=torch.int64, device=A.device)
    row_ptr[1:] = torch.cumsum(counts, 0)
    val = Af[rows, ent].to(torch.float32).contiguous()
    return row_ptr, ent.to(torch.int32).contiguous(), val, rows * E + ent


@torch.no_grad()
def _dense_topc_keep(A, topk_nodes):
    """Boolean keep mask of the dense c1 selection (flashlog_kernel.py:814-842)."""
    B, L_, E = A.shape
    row_ptr, ent, val, flat = _dense_state(A)
    _, _, _, src = ops.topc_select(row_ptr, ent, val, int(topk_nodes))
    counts = row_ptr[1:] - row_ptr[:-1]
    keep = torch.ones(B * L_ * E, dtype=torch.bool, device=A.device)
    over = (counts > topk_nodes).repeat_interleave(E)  # rows over the budget keep their chosen entries only
    keep[over] = False
    keep[flat[src]] = True
    return keep.view(B, L_, E)


def _dense_topc_state(A, topk_nodes):
    """Prune all propagation sources, identity included, per (item, rule)
    (flashlog_kernel.py:814-842): the topk_nodes largest nonzero entries, ties
    to the lower entity; rows with at most topk_nodes nonzeros stay whole."""
    if topk_nodes is None:
        return A
    if topk_nodes < 0:
        raise ValueError("topk_nodes/c must be nonnegative")
    if topk_nodes >= A.shape[-1]:
        return A
    _cuda_or_raise(A)
    keep = _dense_topc_keep(A, topk_nodes)
    return A * keep


def _dense_hops(A, w, graph, masks, r_size, wot_i, topk_edges, active_nodes, mode):
    """Forward and inverse expansions of the nonzero entries of A, reduced per
    (row, destination) by SUM or by MAX, as dense [B, L, E] outputs."""
    B, L_, E = A.shape
    BL = B * L_
    n = w.shape[-1]
    row_ptr, ent, val, flat = _dense_state(A, active_nodes)
    wf = w.detach().reshape(B, L_, n).to(torch.float32).contiguous()
    _check_w(wf)
    topk = int(min(topk_edges, L.NO_BUDGET)) if topk_edges and topk_edges > 0 else L.NO_BUDGET
    flags = L.FL_SKIP_NONPOS_W | L.FL_DROP_MASKED | L.FL_WOT_I
    if mode == "max":
        flags |= L.FL_EDGE_POS  # ties go to the lower CSR position (flashlog.cu:103-121)
    outs, fws = [], []
    for side_flag in (L.FL_NO_INV, L.FL_NO_ORI):
        fw = ops.hop_forward(row_ptr, ent, val, wf, graph, r_size, topk, flags | side_flag, mask_csr=masks,
                             reduce=mode, max_bits=(mode == "max"))
        counts = fw.out_row_ptr[1:] - fw.out_row_ptr[:-1]
        orow = torch.repeat_interleave(torch.arange(BL, device=A.device), counts)
        oflat = orow * E + fw.out_ent.to(torch.int64)
        dense = torch.zeros(BL * E, dtype=torch.float32, device=A.device)
        dense[oflat] = fw.out_x
        outs.append(dense.view(B, L_, E))
        fws.append((fw, oflat))
    out_ind = (A.detach().to(torch.float32) * wf[..., n - 1:n]) if not wot_i else torch.zeros_like(outs[0])
    return out_ind, outs[0], outs[1], (row_ptr, val, flat, wf, fws)


def _dense_backward(A, w, rec, grad_ind, grad_ori, grad_inv, wot_i):
    row_ptr, val, flat, wf, fws = rec
    B, L_, E = A.shape
    n = wf.shape[-1]
    gA = torch.zeros(B * L_ * E, dtype=torch.float32, device=A.device)
    gw = torch.zeros_like(wf)
    gv_total = torch.zeros_like(val)
    for (fw, oflat), g in zip(fws, (grad_ori, grad_inv)):
        if g is None:
            continue
        gy = g.reshape(-1).to(torch.float32)[oflat].contiguous()
        gv, gws = ops.hop_backward(fw, row_ptr, val, wf, gy, normalize=False)
        gv_total += gv
        gw += gws
    gA[flat] = gv_total
    gA = gA.view(B, L_, E)
    if grad_ind is not None and not wot_i:
        gi = grad_ind.to(torch.float32)
        gA = gA + gi * wf[..., n - 1:n]
        gw[..., n - 1] += (gi * A.detach().to(torch.float32)).sum(-1)
    return gA.to(A.dtype), gw.to(w.dtype)


class FlashLogFunction(autograd.Function):
    """Dense propagation with CSR-ordered masks (flashlog_kernel.py:700-811): returns
    (out_ind, out_ori, out_inv), each [B, L, E]; the caller sums them."""

    @staticmethod
    def forward(ctx, A, w, active_nodes,
                ori_col_ind, ori_mask,
                ori_row_group_ptr, ori_group_rel, ori_group_edge_start, ori_group_edge_count,
                inv_col_ind, inv_mask,
                inv_row_group_ptr, inv_group_rel, inv_group_edge_start, inv_group_edge_count,
                r_size, wot_i, topk_edges):
        _cuda_or_raise(A)
        graph = _graph_groups(ori_col_ind, ori_row_group_ptr, ori_group_rel, ori_group_edge_start,
                              ori_group_edge_count, inv_col_ind, inv_row_group_ptr, inv_group_rel,
                              inv_group_edge_start, inv_group_edge_count)
        masks = (ori_mask.reshape(-1).to(torch.float32).contiguous(),
                 inv_mask.reshape(-1).to(torch.float32).contiguous())
        out_ind, out_ori, out_inv, rec = _dense_hops(A, w, graph, masks, r_size, wot_i, topk_edges, active_nodes,
                                                     "sum")
        ctx.rec, ctx.wot_i = rec, wot_i
        ctx.save_for_backward(A, w)
        return out_ind.to(A.dtype), out_ori.to(A.dtype), out_inv.to(A.dtype)

    @staticmethod
    def backward(ctx, grad_ind, grad_ori, grad_inv):
        A, w = ctx.saved_tensors
        gA, gw = _dense_backward(A, w, ctx.rec, grad_ind, grad_ori, grad_inv, ctx.wot_i)
        return (gA, gw) + (None,) * 16


def vectorized_operation_csr(A, w, csr_struct, mask_values, r_size, weight=None, wot_i=False,
                             use_topk=False, topk_nodes=100000, topk_edges=0, prepared_masks=None):
    """Dense entry point (flashlog_kernel.py:845-882): returns (s_i, s_h, s_t)."""
    (ori_row_ptr, ori_col_ind, ori_r_ind, order_ori,
     inv_row_ptr, inv_col_ind, inv_r_ind, order_inv,
     ori_gp, ori_gr, ori_gs, ori_gc, inv_gp, inv_gr, inv_gs, inv_gc) = csr_struct
    prepared = _prepared_mask_pair(prepared_masks) if prepared_masks is not None else _prepared_mask_pair(mask_values)
    if prepared is not None:
        ori_mask, inv_mask = prepared
    else:
        ori_mask, inv_mask = prepare_csr_masks(csr_struct, mask_values, weight)
    A = _dense_topc_state(A, topk_nodes if use_topk else None)
    active_nodes = _compute_active_nodes(A)
    effective_topk = topk_edges if (use_topk and topk_edges > 0) else (1 << 60)
    return FlashLogFunction.apply(A, w, active_nodes, ori_col_ind, ori_mask, ori_gp, ori_gr, ori_gs, ori_gc,
                                  inv_col_ind, inv_mask, inv_gp, inv_gr, inv_gs, inv_gc, r_size, wot_i,
                                  effective_topk)


def _dense_masks(csr_parts, mask_values, weight):
    prepared = _prepared_mask_pair(mask_values)
    if prepared is not None:
        return prepared
    return prepare_csr_masks(csr_parts, mask_values, weight)


class FlashLogDenseSumFunction(autograd.Function):
    """Dense SUM propagation from raw masks (flashlog_kernel.py:885-989), 26 positional arguments."""

    @staticmethod
    def forward(ctx, A, w, ori_row_ptr, ori_col_ind, ori_r_ind, ori_order,
                inv_row_ptr, inv_col_ind, inv_r_ind, inv_order,
                ori_row_group_ptr, ori_group_rel, ori_group_edge_start, ori_group_edge_count,
                inv_row_group_ptr, inv_group_rel, inv_group_edge_start, inv_group_edge_count,
                mask_values, weight, r_size, wot_i, use_topk, topk_nodes, topk_edges, agg_mode):
        _cuda_or_raise(A)
        if agg_mode not in (0, "sum"):
            raise NotImplementedError("dense aggregation 'max' through the sum operator is not supported; "
                                      "use dense_csr_max")
        csr_parts = (ori_row_ptr, ori_col_ind, ori_r_ind, ori_order, inv_row_ptr, inv_col_ind, inv_r_ind, inv_order,
                     ori_row_group_ptr, ori_group_rel, ori_group_edge_start, ori_group_edge_count,
                     inv_row_group_ptr, inv_group_rel, inv_group_edge_start, inv_group_edge_count)
        graph = _graph_topk(csr_parts)
        masks = _dense_masks(csr_parts, mask_values, weight)
        topk = topk_edges if (use_topk and topk_edges > 0) else (1 << 60)
        out_ind, out_ori, out_inv, rec = _dense_hops(A, w, graph, masks, r_size, wot_i, topk,
                                                     _compute_active_nodes(A), "sum")
        ctx.rec, ctx.wot_i = rec, wot_i
        ctx.save_for_backward(A, w)
        return out_ind.to(A.dtype), out_ori.to(A.dtype), out_inv.to(A.dtype)

    @staticmethod
    def backward(ctx, grad_ind, grad_ori, grad_inv):
        A, w = ctx.saved_tensors
        gA, gw = _dense_backward(A, w, ctx.rec, grad_ind, grad_ori, grad_inv, ctx.wot_i)
        return (gA, gw) + (None,) * 24


class FlashLogDenseMaxFunction(autograd.Function):
    """Dense MAX propagation (flashlog_kernel.py:992-1089), 25 positional arguments.

    Every (row, destination) keeps its largest fact of each direction, compared
    as in the reference's packed (value bits, ~CSR position) CAS-max, ties to the
    lower CSR position; the gradient reaches the winning edge only
    (flashlog.cu:523-726, 997-1255).  Hidden edges (mask 0) take no part."""

    @staticmethod
    def forward(ctx, A, w, ori_row_ptr, ori_col_ind, ori_r_ind, ori_order,
                inv_row_ptr, inv_col_ind, inv_r_ind, inv_order,
                ori_row_group_ptr, ori_group_rel, ori_group_edge_start, ori_group_edge_count,
                inv_row_group_ptr, inv_group_rel, inv_group_edge_start, inv_group_edge_count,
                mask_values, weight, r_size, wot_i, use_topk, topk_nodes, topk_edges):
        _cuda_or_raise(A)
        csr_parts = (ori_row_ptr, ori_col_ind, ori_r_ind, ori_order, inv_row_ptr, inv_col_ind, inv_r_ind, inv_order,
                     ori_row_group_ptr, ori_group_rel, ori_group_edge_start, ori_group_edge_count,
                     inv_row_group_ptr, inv_group_rel, inv_group_edge_start, inv_group_edge_count)
        graph = _graph_topk(csr_parts)
        masks = _dense_masks(csr_parts, mask_values, weight)
        topk = topk_edges if (use_topk and topk_edges > 0) else (1 << 60)
        out_ind, out_ori, out_inv, rec = _dense_hops(A, w, graph, masks, r_size, wot_i, topk,
                                                     _compute_active_nodes(A), "max")
        ctx.rec, ctx.wot_i = rec, wot_i
        ctx.save_for_backward(A, w)
        return out_ind.to(A.dtype), out_ori.to(A.dtype), out_inv.to(A.dtype)

    @staticmethod
    def backward(ctx, grad_ind, grad_ori, grad_inv):
        A, w = ctx.saved_tensors
        gA, gw = _dense_backward(A, w, ctx.rec, grad_ind, grad_ori, grad_inv, ctx.wot_i)
        return (gA, gw) + (None,) * 23


def dense_csr_sum_cuda(A, w, csr_struct, mask_values, r_size, weight=None, wot_i=False, use_topk=False,
                       topk_nodes=100000, topk_edges=0, agg_mode="sum", prepared_masks=None):
    """Dense SUM entry point (flashlog_kernel.py:1629-1663): returns (s_i, s_h, s_t)."""
    agg_id = 1 if agg_mode == "max" else 0
    A = _dense_topc_state(A, topk_nodes if use_topk else None)
    mask_input = prepared_masks if prepared_masks is not None else mask_values
    weight_input = None if prepared_masks is not None else weight
    return FlashLogDenseSumFunction.apply(A, w, *csr_struct, mask_input, weight_input, r_size, wot_i, use_topk,
                                          topk_nodes, topk_edges, agg_id)


def dense_csr_max(A, w, csr_struct, mask_values, r_size, weight=None, wot_i=False, use_topk=False,
                  topk_nodes=100000, topk_edges=0, prepared_masks=None):
    """Dense MAX entry point (flashlog_kernel.py:1666-1688): returns (s_i, s_h, s_t)."""
    A = _dense_topc_state(A, topk_nodes if use_topk else None)
    mask_input = prepared_masks if prepared_masks is not None else mask_values
    weight_input = None if prepared_masks is not None else weight
    return FlashLogDenseMaxFunction.apply(A, w, *csr_struct, mask_input, weight_input, r_size, wot_i, use_topk,
                                          topk_nodes, topk_edges)
