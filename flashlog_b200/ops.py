"""Tensor-level wrappers over the C ABI (one function per stage of the hot path).

Every function takes CUDA tensors, allocates its outputs and workspace with
torch on the tensors' device and runs the library's kernels on the current
stream.  CPU tensors are rejected: there is no CPU path.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib as L
from ._lib import check, lib

EPS = 1e-7


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ws(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("flashlog_b200 runs on CUDA tensors only (no CPU fallback)")


_CSR_DTYPES = (torch.int32, torch.int32, torch.int16, torch.int32) * 2 + \
              (torch.int32, torch.int16, torch.int32, torch.int32) * 2


class Graph:
    """Device CSR of both directions in the reference's 16-tuple layout.

    csr[0:4]  ori row_ptr, col, edge_rel, order
    csr[4:8]  inv row_ptr, col, edge_rel, order
    csr[8:12] ori group_ptr, group_rel, group_start, group_count
    csr[12:16] inv group_ptr, group_rel, group_start, group_count
    """

    _cache: dict = {}

    def __init__(self, csr):
        csr = tuple(csr)
        if len(csr) != 16:
            raise ValueError("csr_struct must be the 16-tuple of build_csr_structure")
        _require_cuda(*[c for c in csr if c.numel()])
        self.csr = tuple(c if c.dtype == d else c.to(d) for c, d in zip(csr, _CSR_DTYPES))
        self.csr = tuple(c.contiguous() for c in self.csr)
        self.E = self.csr[0].numel() - 1
        c = self.csr
        self.ori = L.fl_csr_side(_p(c[0]), _p(c[1]), _p(c[3]), _p(c[8]), _p(c[10]), _p(c[11]), _p(c[9]))
        self.inv = L.fl_csr_side(_p(c[4]), _p(c[5]), _p(c[7]), _p(c[12]), _p(c[14]), _p(c[15]), _p(c[13]))
        self.device = c[0].device
        self._max_degree = None

    def max_degree(self):
        """(max out-degree, max in-degree) over entities (one host sync, cached)."""
        if self._max_degree is None:
            def side_max(gp, gs, gc):
                if gs.numel() == 0:
                    return 0
                g0, g1 = gp[:-1].long(), gp[1:].long()
                has = g1 > g0
                last = (g1 - 1).clamp(min=0)
                deg = torch.where(has, gs[last].long() + gc[last].long() - gs[g0.clamp(max=gs.numel() - 1)].long(),
                                  torch.zeros_like(g0))
                return int(deg.max().item())
            c = self.csr
            self._max_degree = (side_max(c[8], c[10], c[11]), side_max(c[12], c[14], c[15]))
        return self._max_degree

    @classmethod
    def of(cls, csr):
        """Cached view of a csr tuple (keyed by its tensors' storage)."""
        key = tuple((t.data_ptr(), t.numel(), t.dtype) for t in csr)
        g = cls._cache.get(key)
        if g is None:
            if len(cls._cache) > 8:
                cls._cache.clear()
            g = cls(csr)
            cls._cache[key] = g
        return g


# --------------------------------------------------------------------------
# CSR build
# --------------------------------------------------------------------------
def build_csr_side(src, dst, rel, nodes: int, relations: int):
    _require_cuda(src, dst, rel)
    src, dst, rel = (x.to(torch.int64).contiguous() for x in (src, dst, rel))
    m = src.numel()
    dev = src.device
    row_ptr = torch.empty(nodes + 1, dtype=torch.int32, device=dev)
    col = torch.empty(m, dtype=torch.int32, device=dev)
    erel = torch.empty(m, dtype=torch.int16, device=dev)
    order = torch.empty(m, dtype=torch.int32, device=dev)
    gptr = torch.empty(nodes + 1, dtype=torch.int32, device=dev)
    grel = torch.empty(max(m, 1), dtype=torch.int16, device=dev)
    gstart = torch.empty(max(m, 1), dtype=torch.int32, device=dev)
    gcount = torch.empty(max(m, 1), dtype=torch.int32, device=dev)
    ws = _ws(lib().fl_csr_build_workspace(m, nodes), dev)
    ng = ctypes.c_int64(0)
    check(lib().fl_csr_build_side(_p(src), _p(dst), _p(rel), m, nodes, relations, _p(row_ptr), _p(col), _p(erel),
                                  _p(order), _p(gptr), _p(grel), _p(gstart), _p(gcount), ctypes.byref(ng), _p(ws),
                                  ws.numel(), _stream()), "build_csr_side")
    g = ng.value
    return row_ptr, col, erel, order, gptr, grel[:g].clone(), gstart[:g].clone(), gcount[:g].clone()


# --------------------------------------------------------------------------
# layouts
# --------------------------------------------------------------------------
def coo_to_rows(b, l, e, B: int, Lch: int, E: int):
    """Coalesced COO -> (row_ptr i64[B*L+1], ent i32); raises on invalid input."""
    _require_cuda(b, l, e)
    b, l, e = (x.to(torch.int64).contiguous() for x in (b, l, e))
    rows = B * Lch
    row_ptr = torch.empty(rows + 1, dtype=torch.int64, device=b.device)
    ent = torch.empty(e.numel(), dtype=torch.int32, device=b.device)
    bad = torch.zeros(1, dtype=torch.int32, device=b.device)
    check(lib().fl_coo_to_rows(_p(b), _p(l), _p(e), e.numel(), Lch, rows, E, _p(row_ptr), _p(ent), _p(bad),
                               _stream()), "coo_to_rows")
    return row_ptr, ent, bad


def rows_to_coo(row_ptr, ent, Lch: int):
    U = ent.numel()
    rows = row_ptr.numel() - 1
    idx = torch.empty((3, U), dtype=torch.int64, device=ent.device)
    check(lib().fl_rows_to_coo(_p(row_ptr), _p(ent), rows, Lch, U, _p(idx), _stream()), "rows_to_coo")
    return idx


# --------------------------------------------------------------------------
# c1
# --------------------------------------------------------------------------
def topc_candidates(row_ptr, val, c1: int) -> int:
    rows = row_ptr.numel() - 1
    S = val.numel()
    ws = _ws(lib().fl_topc_workspace(rows, S), val.device)
    n = ctypes.c_int64(0)
    check(lib().fl_topc_candidates(_p(row_ptr), _p(val), rows, S, c1, ctypes.byref(n), _p(ws), ws.numel(), _stream()),
          "topc_candidates")
    return n.value


def topc_select(row_ptr, ent, val, c1: int, noise=None, sync: bool = True, out_capacity: int = 0, status=None):
    """c1 selection; returns (row_ptr, ent, val, src_index) of the kept entries.

    With sync=False the outputs keep the input's capacity and the live count
    is only on the device (row_ptr[-1]); no host synchronization happens.
    """
    _require_cuda(row_ptr, ent, val)
    rows = row_ptr.numel() - 1
    S = val.numel()
    dev = val.device
    cap = int(out_capacity) if out_capacity else S
    out_row_ptr = torch.empty(rows + 1, dtype=torch.int64, device=dev)
    out_ent = torch.empty(max(cap, 1), dtype=torch.int32, device=dev)
    out_val = torch.empty(max(cap, 1), dtype=torch.float32, device=dev)
    out_src = torch.empty(max(cap, 1), dtype=torch.int64, device=dev)
    ws = _ws(lib().fl_topc_workspace(rows, S), dev)
    if noise is not None:
        noise = noise.to(torch.float64).contiguous()
    check(lib().fl_topc_select(_p(row_ptr), _p(ent), _p(val), rows, S, int(c1), _p(noise), _p(out_row_ptr),
                               _p(out_ent), _p(out_val), _p(out_src), cap, _p(status), _p(ws), ws.numel(),
                               _stream()), "topc_select")
    if not sync:
        return out_row_ptr, out_ent[:cap], out_val[:cap], out_src[:cap]
    k = int(out_row_ptr[-1].item())
    return out_row_ptr, out_ent[:k], out_val[:k], out_src[:k]


# --------------------------------------------------------------------------
# one hop
# --------------------------------------------------------------------------
class SelectionOverflow(RuntimeError):
    """The c1 selection that fed a hop ran out of its output capacity."""


@dataclass
class HopForward:
    params: L.fl_hop_params
    slot_base: torch.Tensor
    entry_count: torch.Tensor
    fact_rel: torch.Tensor
    fact_m: torch.Tensor | None
    fact_pos: torch.Tensor | None
    out_row_ptr: torch.Tensor
    out_ent: torch.Tensor
    out_x: torch.Tensor
    out_y: torch.Tensor
    out_denom: torch.Tensor
    n_facts_slots: int
    fact_dst: torch.Tensor | None = None
    fact_val: torch.Tensor | None = None
    fact_edge: torch.Tensor | None = None  # triple id per fact (record_edge)


def hop_params(rows, Lch, n, r_size, E, topk_edges, flags, seed=-1, eps=EPS, slot_capacity=0, status=None,
               entry_info=None, vis=None, work=None, rel_rank=None):
    return L.fl_hop_params(rows, Lch, n, r_size, E, int(min(topk_edges, L.NO_BUDGET)), int(flags), int(seed),
                           float(eps), int(slot_capacity), None if status is None else status.data_ptr(),
                           None if entry_info is None else entry_info.data_ptr(),
                           None if vis is None else vis[0].data_ptr(), None if vis is None else vis[1].data_ptr(),
                           None if work is None else work.data_ptr(),
                           None if rel_rank is None else rel_rank.data_ptr(), None)


def relation_rank(w, r_size: int):
    """Per (row, direction, relation) the relation's position in the order
    (w desc, id asc) of the relations with w > 0 (0xffff, i.e. -1 as int16,
    for w <= 0); None when r_size is outside the supported range (the
    expansion then selects thresholds over the weights)."""
    if not (0 < r_size <= 16384):
        return None
    rows = w.numel() // (2 * r_size + 1)
    rank = torch.empty(max(rows * 2 * r_size, 1), dtype=torch.int16, device=w.device)
    check(lib().fl_relation_rank(_p(w), rows, r_size, None, _p(rank), _stream()), "relation_rank")
    return rank


def csr_mask(mask, order, weight=None):
    """CSR-ordered float mask: mask[order[p]] (* sigmoid(weight[order[p]])), fl_csr_mask."""
    _require_cuda(mask, order)
    m = order.numel()
    out = torch.empty(m, dtype=torch.float32, device=mask.device)
    if mask.dtype == torch.bool:
        mk, kind = mask.view(torch.uint8), L.FL_MASK_U8
    else:
        mk, kind = mask.to(torch.float32).contiguous(), L.FL_MASK_F32
    # order is a permutation of the M triple ids (one CSR position per triple):
    # the mask and the weights need one entry per triple
    if mk.numel() < m:
        raise ValueError(f"edge visibility mask must have one entry per triple ({mk.numel()} < {m})")
    if weight is not None:
        _require_cuda(weight)
        if weight.numel() < m:
            raise ValueError(f"edge weights must have one entry per triple ({weight.numel()} < {m})")
    check(lib().fl_csr_mask(_p(mk), kind, _p(order), m, _p(weight), _p(out), _stream()), "csr_mask")
    return out


def align_rows(out_indices, Lch: int, rows: int, g_row_ptr, g_ent, g_val):
    """Gradient values at out_indices (3 x n, int64) from a row-layout gradient (fl_align_rows)."""
    n = out_indices.shape[1]
    out = torch.empty(n, dtype=torch.float32, device=g_val.device)
    oi = out_indices.to(torch.int64).contiguous()
    check(lib().fl_align_rows(_p(oi[0]), _p(oi[1]), _p(oi[2]), n, Lch, rows, _p(g_row_ptr), _p(g_ent), _p(g_val),
                              _p(out), _stream()), "align_rows")
    return out


def csr_visibility(graph: Graph, mask_triple):
    """CSR-ordered visibility (u8 per edge, both sides) of a per-triple mask.

    The gather of prepare_csr_masks (flashlog_kernel.py:225-255) in one byte
    per edge; a hop given it reads visibility next to the edge instead of
    through `order`."""
    _require_cuda(mask_triple)
    m = mask_triple.reshape(-1)
    m = (m if m.dtype == torch.uint8 else (m != 0).to(torch.uint8)).contiguous()
    M = graph.csr[1].numel()
    if m.numel() < M:
        raise ValueError("edge visibility mask must have one entry per triple")
    out = []
    for order in (graph.csr[3], graph.csr[7]):
        v = torch.empty(M, dtype=torch.uint8, device=m.device)
        check(lib().fl_csr_visibility(_p(order), M, _p(m), _p(v), _stream()), "csr_visibility")
        out.append(v)
    return tuple(out)


def hop_forward(row_ptr, ent, val, w, graph: Graph, r_size: int, topk_edges: int, flags: int, *,
                mask_triple=None, mask_csr=None, edge_weight=None, seed: int = -1, eps: float = EPS,
                keep_facts: bool = False, record: bool = True, timing=None, slot_capacity=None,
                status=None, out_sync: bool = True, vis=None, reduce: str = "sum",
                max_bits: bool = False, rank_select: bool = True, check_w: bool = False,
                sel_status=None, record_edge: bool = False) -> HopForward:
    """Expansion + per-row coalesce-sum + normalization of one hop.

    slot_capacity=None sizes the fact buffers exactly (one host sync for the
    fact count, one for the output count).  With an upper bound instead, no
    host synchronization happens: outputs keep that capacity, their live
    count is out_row_ptr[-1] on the device, and work that would not fit sets
    FL_STATUS_SLOT_OVERFLOW in `status` (an int32 device tensor).  With
    out_sync=False the fact count is still read (one sync) but the outputs keep
    that capacity and their live count stays on the device.  `vis` (from
    csr_visibility of the same mask) replaces the per-fact mask_triple read.
    reduce="max" coalesces by MAX with exact winners instead
    (FlashLogFunctionSparse3DTopKMax); its out_x holds the maxima, out_y is
    None and fact_pos is -1 for the facts that did not win.  max_bits compares
    fact values by their fp32 bit patterns (the dense MAX order).
    rank_select=False makes the expansion select c2 thresholds by a radix
    select over the groups' weights instead of over relation ranks (same
    result; the path used when r_size exceeds 16384).  check_w raises the
    non-finite-weights RuntimeError of the top-k operators before the
    expansion, read in the same host sync as the fact count.  sel_status (with
    check_w): the status word of the c1 selection that produced the state,
    read in that sync too; SelectionOverflow is raised when it is set.
    record_edge keeps the triple id of every fact (fact_edge) for
    edge_weight_grad.
    """
    if reduce not in ("sum", "max"):
        raise ValueError("reduce must be 'sum' or 'max'")
    _require_cuda(row_ptr, ent, val, w)
    B, Lch, n = w.shape
    rows = B * Lch
    S = ent.numel()
    dev = val.device
    if row_ptr.numel() != rows + 1:
        raise ValueError(f"w has {rows} (item, channel) rows but the state has {row_ptr.numel() - 1}")
    if n != 2 * r_size + 1:
        raise ValueError(f"w must have 2 * r_size + 1 = {2 * r_size + 1} columns, got {n}")
    w = w.contiguous()
    sync = slot_capacity is None
    slot_base = torch.empty(S + 1, dtype=torch.int64, device=dev)
    ws = _ws(lib().fl_hop_workspace(rows, S), dev)
    total = ctypes.c_int64(0)
    entry_info = torch.empty(L.FL_ENTRY_INFO_INTS * max(S, 1), dtype=torch.int32, device=dev)
    if vis is not None and (len(vis) != 2 or any(v.numel() < graph.csr[1].numel() or v.dtype != torch.uint8
                                                 for v in vis)):
        raise ValueError("vis must be the two u8 CSR-ordered visibility arrays of csr_visibility")
    work = torch.empty(2, dtype=torch.int32, device=dev)  # the expansion's two work queues
    rel_rank = (relation_rank(w, r_size) if rank_select and (flags & L.FL_SKIP_NONPOS_W)
                and topk_edges < L.NO_BUDGET and not (flags & L.FL_SAMPLED) else None)
    params = hop_params(rows, Lch, n, r_size, graph.E, topk_edges, flags, seed, eps, slot_capacity or 0, status,
                        entry_info, vis, work, rel_rank)
    nonfinite = (~torch.isfinite(w)).any() if check_w else None
    check(lib().fl_hop_plan(ctypes.byref(params), _p(row_ptr), _p(ent), S, graph.ori, graph.inv, _p(slot_base),
                            ctypes.byref(total) if (sync and not check_w) else None, _p(ws), ws.numel(), _stream()),
          "hop_plan")
    if check_w:
        # one host read: the fact count, the weights' finiteness and the selection's status
        parts = [slot_base[S], nonfinite.to(torch.int64)]
        if sel_status is not None:
            parts.append(sel_status[0].to(torch.int64))
        got = torch.stack(parts).cpu()
        if sel_status is not None and int(got[2]) & L.FL_STATUS_SLOT_OVERFLOW:
            raise SelectionOverflow("the c1 selection exceeded its capacity")
        if int(got[1]):
            raise RuntimeError("FlashLog sparse top-k received non-finite attention weights; "
                               "aborting before edge count/fill to prevent uninitialized indices")
        total.value = int(got[0])
    T = max(total.value, 1) if sync else max(int(slot_capacity), 1)
    if not sync:
        params.slot_capacity = T
    fact_dst = torch.empty(T, dtype=torch.int32, device=dev)
    fact_val = torch.empty(T, dtype=torch.float32, device=dev)
    fact_rel = torch.empty(T, dtype=torch.int16, device=dev)
    # The mask value of each fact is needed by the backward whenever it can be
    # anything but 1: soft edge weights, CSR-ordered float masks, or hidden
    # edges kept as zero-valued facts.
    need_m = bool(flags & L.FL_EDGE_WEIGHT) or mask_csr is not None or (
        (mask_triple is not None or vis is not None) and not (flags & L.FL_DROP_MASKED))
    fact_m = torch.empty(T, dtype=torch.float32, device=dev) if need_m else None
    entry_count = torch.empty(max(S, 1), dtype=torch.int32, device=dev)
    mo = mi = None
    M = graph.csr[1].numel()
    if mask_csr is not None:
        mo, mi = (m.reshape(-1).to(torch.float32).contiguous() for m in mask_csr)
        if mo.numel() != M or mi.numel() != graph.csr[5].numel():
            raise ValueError("CSR-ordered masks must have one value per edge")
    if mask_triple is not None:
        mask_triple = mask_triple.reshape(-1)
        if mask_triple.dtype == torch.bool:
            mask_triple = mask_triple.contiguous().view(torch.uint8)  # one byte, 0 or 1: the same visibility
        elif mask_triple.dtype != torch.uint8:
            mask_triple = (mask_triple != 0).to(torch.uint8)
        mask_triple = mask_triple.contiguous()
        if mask_triple.numel() < M:
            raise ValueError("edge visibility mask must have one entry per triple")
    if edge_weight is not None:
        if mask_triple is None:
            # the multiplier is mask[triple] * sigmoid(edge_weight[triple]): the
            # weights are read through the triple-indexed mask
            raise ValueError("edge weights need the triple-indexed mask (mask_values)")
        edge_weight = edge_weight.reshape(-1).to(torch.float32).contiguous()
        if edge_weight.numel() < M:
            raise ValueError("edge weights must have one entry per triple")
    fact_pos = torch.empty(T, dtype=torch.int32, device=dev) if (record or reduce == "max") else None
    fact_edge = None
    if reduce == "max" or record_edge:
        fact_edge = torch.empty(T, dtype=torch.int32, device=dev)
        params.fact_edge = fact_edge.data_ptr()
    out_row_ptr = torch.empty(rows + 1, dtype=torch.int64, device=dev)
    out_ent = torch.empty(T, dtype=torch.int32, device=dev)
    out_x = torch.empty(T, dtype=torch.float32, device=dev)
    out_y = torch.empty(T, dtype=torch.float32, device=dev)
    out_denom = torch.empty(max(rows, 1), dtype=torch.float32, device=dev)
    ws2 = _ws(lib().fl_reduce_workspace(rows, T), dev)
    # every buffer exists before the launches: nothing on the host between them
    if timing is not None:
        timing.record_start()
    check(lib().fl_hop_expand(ctypes.byref(params), _p(row_ptr), _p(ent), _p(val), S, _p(w), graph.ori, graph.inv,
                              _p(mo), _p(mi), _p(mask_triple), _p(edge_weight), _p(slot_base), _p(fact_dst),
                              _p(fact_val), _p(fact_rel), _p(fact_m), _p(entry_count), _stream()), "hop_expand")
    if reduce == "max":
        check(lib().fl_row_reduce_max(_p(row_ptr), rows, graph.E, r_size, _p(slot_base), _p(fact_dst), _p(fact_val),
                                      _p(fact_rel), _p(fact_edge), T, _p(fact_pos), _p(out_row_ptr), _p(out_ent),
                                      _p(out_x), L.FL_MAX_BITS if max_bits else 0, _p(status), _p(ws2), ws2.numel(),
                                      _stream()), "row_reduce_max")
    else:
        check(lib().fl_row_reduce(_p(row_ptr), rows, graph.E, _p(slot_base), _p(entry_count), _p(fact_dst),
                                  _p(fact_val), T, _p(fact_pos), ctypes.c_float(eps), _p(out_row_ptr), _p(out_ent),
                                  _p(out_x), _p(out_y), _p(out_denom), _p(status), None, _p(ws2), ws2.numel(),
                                  None, _stream()),
              "row_reduce")
    if timing is not None:
        timing.record_end()
    u = int(out_row_ptr[rows].item()) if (sync and out_sync) else T
    params.fact_edge = None  # the buffer is not kept with the record
    return HopForward(params, slot_base, entry_count, fact_rel, fact_m, fact_pos, out_row_ptr, out_ent[:u],
                      out_x[:u], None if reduce == "max" else out_y[:u],
                      None if reduce == "max" else out_denom[:rows], total.value,
                      fact_dst if keep_facts else None, fact_val if keep_facts else None,
                      fact_edge if record_edge else None)


def hop_backward(fw: HopForward, row_ptr, val, w, g_y, normalize: bool = True):
    """Gradients of one hop w.r.t. the entry values and w."""
    B, Lch, n = w.shape
    rows = B * Lch
    S = val.numel()
    dev = val.device
    params = L.fl_hop_params(fw.params.rows, fw.params.L, fw.params.n, fw.params.r_size, fw.params.E,
                             fw.params.topk_edges, fw.params.flags | (0 if normalize else L.FL_NO_NORMALIZE),
                             fw.params.sampling_seed, fw.params.eps, fw.params.slot_capacity, fw.params.status)
    grad_val = torch.empty(max(S, 1), dtype=torch.float32, device=dev)
    grad_w = torch.empty((rows, n), dtype=torch.float32, device=dev)
    ws = _ws(lib().fl_hop_backward_workspace(rows, n), dev)
    g_y = g_y.to(torch.float32).contiguous()
    check(lib().fl_hop_backward(ctypes.byref(params), _p(row_ptr), _p(val), S, _p(w.contiguous()), _p(fw.slot_base),
                                _p(fw.entry_count), _p(fw.fact_pos), _p(fw.fact_rel), _p(fw.fact_m),
                                _p(fw.out_row_ptr), _p(fw.out_x), _p(fw.out_denom), _p(g_y), _p(grad_val),
                                _p(grad_w), _p(ws), ws.numel(), _stream()), "hop_backward")
    return grad_val[:S], grad_w.view(B, Lch, n)


def edge_weight_grad(fw: HopForward, row_ptr, val, w, g_x, edge_weight):
    """d loss / d edge_weight of a top-k hop with learnable edge weights
    (flashlog_kernel.py:1306-1336, 1590-1614); g_x is the gradient at the
    outputs (the MAX outputs, or the sums before normalization).  The forward
    must have run with the edge weights and record_edge=True."""
    if fw.fact_edge is None or fw.fact_m is None or fw.fact_pos is None:
        raise ValueError("edge_weight_grad needs a forward recorded with edge weights and record_edge=True")
    ew = edge_weight.detach().reshape(-1).to(torch.float32).contiguous()
    grad = torch.zeros_like(ew)
    check(lib().fl_edge_weight_grad(ctypes.byref(fw.params), _p(row_ptr), _p(val), val.numel(), _p(w.contiguous()),
                                    _p(fw.slot_base), _p(fw.entry_count), _p(fw.fact_pos), _p(fw.fact_rel),
                                    _p(fw.fact_m), _p(fw.fact_edge), _p(fw.out_row_ptr),
                                    _p(g_x.to(torch.float32).contiguous()), _p(ew), _p(grad), _stream()),
          "edge_weight_grad")
    return grad.view_as(edge_weight)


def scatter_grad(grad_sel, src_index, n_full: int, n_live=None, full_live=None):
    """grad_full[src_index[j]] = grad_sel[j]; n_live (device int64) bounds j;
    full_live (device int64) limits the zeroing to the live prefix."""
    out = torch.empty(max(n_full, 1), dtype=torch.float32, device=grad_sel.device)
    check(lib().fl_scatter_grad(_p(grad_sel.contiguous()), _p(src_index), src_index.numel(), _p(n_live), _p(out),
                                n_full, _p(full_live), None, _stream()), "scatter_grad")
    return out[:n_full]


def normalize_forward(row_ptr, x, eps=EPS):
    rows = row_ptr.numel() - 1
    y = torch.empty_like(x)
    denom = torch.empty(max(rows, 1), dtype=torch.float32, device=x.device)
    check(lib().fl_normalize_forward(_p(row_ptr), _p(x.contiguous()), rows, ctypes.c_float(eps), _p(y), _p(denom),
                                     _stream()), "normalize_forward")
    return y, denom[:rows]


def normalize_backward(row_ptr, x, denom, g, eps=EPS):
    rows = row_ptr.numel() - 1
    gx = torch.empty_like(x)
    check(lib().fl_normalize_backward(_p(row_ptr), _p(x.contiguous()), _p(denom.contiguous()),
                                      _p(g.to(torch.float32).contiguous()), rows, ctypes.c_float(eps), _p(gx),
                                      _stream()), "normalize_backward")
    return gx


# --------------------------------------------------------------------------
# rule evaluator
# --------------------------------------------------------------------------
def fixed_relation(b, l, e, v, ops_, graph: Graph, r_size: int, B: int, Lr: int):
    """One fixed-operator rule step + coalesce-sum; returns (row_ptr, ent, val)."""
    _require_cuda(b, l, e, v, ops_)
    row_ptr, ent, bad = coo_to_rows(b, l, e, B, Lr, graph.E)
    if int(bad.item()):
        raise ValueError("sparse state indices are out of range or not coalesced")
    b, l = b.to(torch.int64).contiguous(), l.to(torch.int64).contiguous()
    v = v.to(torch.float32).contiguous()
    ops_ = ops_.to(torch.int64).contiguous()
    if tuple(ops_.shape) != (B, Lr):
        raise ValueError(f"operators must have shape [{B}, {Lr}]")
    nnz = v.numel()
    dev = v.device
    slot_base = torch.empty(nnz + 1, dtype=torch.int64, device=dev)
    ws = _ws(lib().fl_fixed_relation_workspace(nnz), dev)
    total = ctypes.c_int64(0)
    check(lib().fl_fixed_relation_plan(_p(b), _p(l), _p(ent), nnz, _p(ops_), Lr, r_size, graph.ori, graph.inv,
                                       _p(slot_base), ctypes.byref(total), _p(ws), ws.numel(), _stream()),
          "fixed_relation_plan")
    T = max(total.value, 1)
    fact_dst = torch.empty(T, dtype=torch.int32, device=dev)
    fact_val = torch.empty(T, dtype=torch.float32, device=dev)
    entry_count = torch.empty(max(nnz, 1), dtype=torch.int32, device=dev)
    check(lib().fl_fixed_relation_fill(_p(b), _p(l), _p(ent), _p(v), nnz, _p(ops_), Lr, r_size, graph.ori, graph.inv,
                                       _p(slot_base), _p(fact_dst), _p(fact_val), _p(entry_count), _stream()),
          "fixed_relation_fill")
    rows = B * Lr
    out_row_ptr = torch.empty(rows + 1, dtype=torch.int64, device=dev)
    out_ent = torch.empty(T, dtype=torch.int32, device=dev)
    out_x = torch.empty(T, dtype=torch.float32, device=dev)
    out_denom = torch.empty(max(rows, 1), dtype=torch.float32, device=dev)
    ws2 = _ws(lib().fl_reduce_workspace(rows, T), dev)
    check(lib().fl_row_reduce(_p(row_ptr), rows, graph.E, _p(slot_base), _p(entry_count), _p(fact_dst), _p(fact_val),
                              T, None, ctypes.c_float(EPS), _p(out_row_ptr), _p(out_ent), _p(out_x), None,
                              _p(out_denom), None, None, _p(ws2), ws2.numel(), None, _stream()), "row_reduce")
    u = int(out_row_ptr[rows].item())
    return out_row_ptr, out_ent[:u], out_x[:u]


def row_max(slot_base, fact_dst, fact_val, rows: int, E: int):
    """Per row r, the maximum fact value of every destination among the slots
    [slot_base[r], slot_base[r + 1]) (destination -1: no fact); returns the
    row layout (row_ptr, ent, val).  One host read sizes the outputs."""
    dev = fact_val.device
    T = max(int(fact_dst.numel()), 1)
    entries = torch.arange(rows + 1, dtype=torch.int64, device=dev)
    out_row_ptr = torch.empty(rows + 1, dtype=torch.int64, device=dev)
    out_ent = torch.empty(T, dtype=torch.int32, device=dev)
    out_x = torch.empty(T, dtype=torch.float32, device=dev)
    ws = _ws(lib().fl_reduce_workspace(rows, T), dev)
    check(lib().fl_row_reduce_max(_p(entries), rows, E, 1, _p(slot_base), _p(fact_dst), _p(fact_val), None, None,
                                  fact_dst.numel(), None, _p(out_row_ptr), _p(out_ent), _p(out_x),
                                  L.FL_MAX_VALUE_ONLY, None, _p(ws), ws.numel(), _stream()), "row_max")
    u = int(out_row_ptr[rows].item())
    return out_row_ptr, out_ent[:u], out_x[:u]


def rule_rank_maxima(st_rp, st_ent, st_val, B: int, C: int, w, ranks: int, E: int, running=None):
    """Rank rows (q, r) of the largest rule weight reaching each entity: the
    grounded rows q * C + c of one rule chunk (weights w [C, ranks]) merged
    with the running maxima of earlier chunks (a rank-row layout or None)."""
    dev = st_val.device
    rows = B * ranks
    run_rp, run_ent, run_val = running if running is not None else (None, None, None)
    slot_base = torch.empty(rows + 1, dtype=torch.int64, device=dev)
    n_run = 0 if running is None else run_ent.numel()
    T = n_run + ranks * st_ent.numel()
    fact_dst = torch.empty(max(T, 1), dtype=torch.int32, device=dev)
    fact_val = torch.empty(max(T, 1), dtype=torch.float32, device=dev)
    check(lib().fl_rule_rank_facts(_p(st_rp), _p(st_ent), _p(st_val), B, C, _p(w.contiguous()), ranks, _p(run_rp),
                                   _p(run_ent), _p(run_val), _p(slot_base), _p(fact_dst), _p(fact_val), _stream()),
          "rule_rank_facts")
    return row_max(slot_base, fact_dst[:T], fact_val[:T], rows, E)


def channel_merge(row_ptr, ent, val, B: int, Lch: int, E: int):
    """Rows (b, l) of a [B, L, E] state merged into rows b: per query the
    sorted union of its channels' entities with each entity's values summed
    in channel order (the row reduction with one fact per entry).  Returns
    (out_row_ptr i64[B+1], out_ent, out_x, position i64[nnz]) where position
    is each input entry's global output index."""
    _require_cuda(row_ptr, ent, val)
    dev = val.device
    nnz = ent.numel()
    if row_ptr.numel() != B * Lch + 1:
        raise ValueError("row_ptr must have B * L + 1 entries")
    entry_row_ptr = row_ptr[::Lch].contiguous()
    slot_base = torch.arange(nnz + 1, dtype=torch.int64, device=dev)
    entry_count = torch.ones(max(nnz, 1), dtype=torch.int32, device=dev)
    fact_pos = torch.empty(max(nnz, 1), dtype=torch.int32, device=dev)
    out_row_ptr = torch.empty(B + 1, dtype=torch.int64, device=dev)
    out_ent = torch.empty(max(nnz, 1), dtype=torch.int32, device=dev)
    out_x = torch.empty(max(nnz, 1), dtype=torch.float32, device=dev)
    out_denom = torch.empty(max(B, 1), dtype=torch.float32, device=dev)
    ws = _ws(lib().fl_reduce_workspace(B, max(nnz, 1)), dev)
    check(lib().fl_row_reduce(_p(entry_row_ptr), B, int(E), _p(slot_base), _p(entry_count), _p(ent.contiguous()),
                              _p(val.to(torch.float32).contiguous()), max(nnz, 1), _p(fact_pos), ctypes.c_float(EPS),
                              _p(out_row_ptr), _p(out_ent), _p(out_x), None, _p(out_denom), None, None, _p(ws),
                              ws.numel(), None, _stream()), "channel_merge")
    u = int(out_row_ptr[B].item())
    row_of = torch.repeat_interleave(torch.arange(B, device=dev), entry_row_ptr[1:] - entry_row_ptr[:-1],
                                     output_size=nnz)
    position = out_row_ptr[row_of] + fact_pos[:nnz].to(torch.int64)
    return out_row_ptr, out_ent[:u], out_x[:u], position


def filtered_ranks(idx_b, idx_e, values, targets, filter_keys, B: int, E: int, use_eql: bool = False):
    _require_cuda(idx_b, idx_e, values, targets, filter_keys)
    idx_b, idx_e, targets, filter_keys = (x.to(torch.int64).contiguous() for x in (idx_b, idx_e, targets, filter_keys))
    values = values.to(torch.float32).contiguous()
    if idx_b.numel() and (int(idx_b.min()) < 0 or int(idx_b.max()) >= B or int(idx_e.min()) < 0 or int(idx_e.max()) >= E):
        raise ValueError("score indices out of range")
    if targets.numel() != B:
        raise ValueError("targets must have one entity per query")
    if filter_keys.numel() and (int(filter_keys.min()) < 0 or int(filter_keys.max()) >= B * E):
        raise ValueError("filter keys out of range")
    ranks = torch.empty(max(B, 1), dtype=torch.float32, device=values.device)
    ws = _ws(lib().fl_filtered_ranks_workspace(B), values.device)
    check(lib().fl_filtered_ranks(_p(idx_b), _p(idx_e), _p(values), values.numel(), _p(targets), _p(filter_keys),
                                  filter_keys.numel(), B, E, int(bool(use_eql)), _p(ranks), _p(ws), ws.numel(),
                                  _stream()), "filtered_ranks")
    return ranks[:B]


# --------------------------------------------------------------------------
# dropout of hop values
# --------------------------------------------------------------------------
def value_dropout(x, p: float, seed: int, counter=None, subseq: int = 0, live=None, out=None):
    """nn.Dropout(p) on a float32 value vector (src/model_DRUM_kernel_sp.py:189-192)
    with counter-based keep bits (fl_value_dropout): the mask is a function of
    (seed, counter[0], subseq, position), so the same call on the gradient is
    the backward.  counter: device int64 tensor or None (0); live: device
    count of the entries to write (the rest of `out` is left as it is)."""
    _require_cuda(x, counter, live)
    if x.dtype != torch.float32:
        raise ValueError("value_dropout takes float32 values")
    if not 0.0 <= float(p) <= 1.0:
        raise ValueError(f"dropout probability must lie in [0, 1], got {p}")
    x = x.contiguous()
    y = torch.empty_like(x) if out is None else out
    check(lib().fl_value_dropout(_p(x), _p(y), x.numel(), _p(live), ctypes.c_double(float(p)),
                                 int(seed) & 0xFFFFFFFFFFFFFFFF, _p(counter), int(subseq), _stream()), "value_dropout")
    return y


# --------------------------------------------------------------------------
# readout
# --------------------------------------------------------------------------
def readout(row_ptr, ent, val, N: int, targets):
    """Channel-summed scores at each query's target (sum_sp_3d + target lookup)."""
    Q = targets.numel()
    scores = torch.empty(max(Q, 1), dtype=torch.float32, device=val.device)
    check(lib().fl_readout(_p(row_ptr), _p(ent), _p(val.contiguous()), N, _p(targets.to(torch.int64).contiguous()), Q,
                           _p(scores), _stream()), "readout")
    return scores[:Q]


def readout_backward(row_ptr, ent, N: int, targets, g_scores, n_val: int, val_live=None):
    Q = targets.numel()
    grad = torch.empty(max(n_val, 1), dtype=torch.float32, device=g_scores.device)
    check(lib().fl_readout_backward(_p(row_ptr), _p(ent), N, _p(targets.to(torch.int64).contiguous()), Q,
                                    _p(g_scores.to(torch.float32).contiguous()), _p(grad), n_val, _p(val_live),
                                    None, _stream()),
          "readout_backward")
    return grad[:n_val]
