"""One sparse DRUM training step on static buffers, with no host synchronization.

This is src/model_DRUM_kernel_sp.py:92-204 (T hops of c1 selection,
expansion with the c2 budget, coalesce-sum and row normalization), the
channel readout and log loss of src/utils.py:36-47, their backward and an
SGD update of a per-query-relation attention table, written against buffers
allocated once.  Every buffer is sized by a static bound:

  selected entries of hop t   S_t = min(C_t, ceil(rows * c1 * zero_slack))
  fact slots of hop t         F_t = min(S_t * k_max, rows * K)
  outputs of hop t            C_{t+1} = min(F_t, rows * E)

where k(e) = min(deg_ori(e), c2//2) + min(deg_inv(e), c2//2) + 1 is the slot
capacity of entity e, k_max its maximum, K its sum over the entities (a row
holds every entity at most once) and C_0 = rows.  zero_slack is 1 without
dropout: a row keeps at most c1 entries unless it has at most c1 nonzero
values, and then all of them.  Such a row also keeps its explicit zeros
(flashlog_kernel.py:1114-1117).  With dropout p, a row of n entries holds
about n (1 - p) nonzero values, so the rows kept whole hold up to about
c1 / (1 - p) entries: zero_slack defaults to 1 / (1 - p) + 0.25 (see
default_zero_slack; p = 1 leaves the selection unbounded).  The kernels
read the live counts from the device (row_ptr[-1]), so nothing is read back
to the host and one step can be captured in a CUDA graph and replayed.  A
device status word flags any capacity overflow (it cannot happen under these
bounds without dropout) and `check` reads it.

The autograd path of engine.drum_propagate computes the same step with one
host synchronization per hop.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib as L
from .ops import Graph, _p, _stream, check, lib


def _buf(n, dtype, dev):
    return torch.empty(max(int(n), 1), dtype=dtype, device=dev)


def default_zero_slack(p: float) -> float:
    """Selection slack for dropout p: rows kept whole hold up to about
    c1 / (1 - p) entries (their explicit zeros included), plus a margin."""
    if p <= 0.0:
        return 1.0
    if p >= 1.0:
        return math.inf
    return 1.0 / (1.0 - p) + 0.25


def capacities(rows: int, T: int, c1, k_max: int, K: int, E: int, zero_slack: float = 1.0):
    """Static bounds of the step's buffers per hop, as lists (C, S, F, U):
    C_t inputs, S_t selected entries, F_t fact slots, U_t = C_{t+1} outputs,
    with C_0 = rows, S_t = min(C_t, ceil(rows * c1 * zero_slack)) (C_t
    without c1, or with an infinite slack), F_t = min(S_t * k_max, rows * K),
    U_t = min(F_t, rows * E)."""
    Cs, Ss, Fs, Us = [], [], [], []
    C = rows
    for _ in range(T):
        S = min(C, math.ceil(rows * c1 * zero_slack)) if (c1 is not None and math.isfinite(zero_slack)) else C
        F = min(S * k_max, rows * K)
        Cs.append(C)
        Ss.append(S)
        Fs.append(F)
        C = min(F, rows * E)
        Us.append(C)
    return Cs, Ss, Fs, Us


class DrumTrainStep:
    """Static-buffer DRUM step: forward (T hops), loss, backward, SGD.

    table: [2R, T, N, n] attention logits (the parameter); a query with
    relation r uses table[r].  Inputs per step are copied into the static
    tensors heads, tails, rels (i64[Q]) and hide (i64[H], triple ids hidden
    during the step) with `load`.  With apply_update the step ends with the
    SGD update table[rels] -= lr * d loss / d logits (only the batch's rows
    are touched); without it the dense gradient of the table is left in
    `grad` (for an all-reduce across ranks before the caller's update),
    hop by hop in grad_hop[t] as the backward reaches it (see `parts`).
    dropout > 0 applies the training dropout of each hop's values
    (src/model_DRUM_kernel_sp.py:189-192) in place; replay k (from 1) draws
    hop t's keep bits from (dropout_seed, k, t), counted on the device.
    A step whose forward overflowed a buffer (status word nonzero) leaves
    the table and the gradient untouched (the gradient is scaled by 0 on the
    device); `check` then raises.
    """

    def __init__(self, graph: Graph, r_size: int, Q: int, T: int, N: int, c1, c2: int, table: torch.Tensor,
                 n_hide: int, lr: float = 0.01, eps: float = 1e-7, thr: float = 1e-7, stats: bool = True,
                 apply_update: bool = True, dropout: float = 0.0, dropout_seed: int = 0, zero_slack=None,
                 record_grad_w: bool = False):
        dev = table.device
        self.dev, self.graph, self.r_size, self.Q, self.T, self.N = dev, graph, r_size, Q, T, N
        self.n = 2 * r_size + 1
        self.c1 = None if c1 is None or c1 < 0 else int(c1)
        self.topk = c2 // 2 if c2 and c2 > 0 else L.NO_BUDGET
        self.flags = L.FL_SKIP_NONPOS_W | L.FL_DROP_MASKED
        self.eps, self.thr, self.lr = eps, thr, lr
        self.apply_update = apply_update
        if not 0.0 <= float(dropout) <= 1.0:
            raise ValueError(f"dropout probability must lie in [0, 1], got {dropout}")
        self.dropout, self.dropout_seed = float(dropout), int(dropout_seed) & 0xFFFFFFFFFFFFFFFF
        self.drop_counter = torch.zeros(1, dtype=torch.int64, device=dev)  # replays so far
        self.zero_slack = default_zero_slack(self.dropout) if zero_slack is None else float(zero_slack)
        self.table = table
        # without the update: the dense table gradient, one contiguous [2R, N, n]
        # block per hop (grad_hop[t]); grad views it as the table's [2R, T, N, n]
        self.grad_hop = None if apply_update else torch.zeros((T,) + tuple(table.shape[:1]) + tuple(table.shape[2:]),
                                                              dtype=table.dtype, device=dev)
        self.grad = None if apply_update else self.grad_hop.permute(1, 0, 2, 3)
        rows = Q * N
        self.rows = rows
        csr = graph.csr
        M = csr[1].numel()
        E = graph.E
        d_o = (csr[0][1:] - csr[0][:-1]).to(torch.int64).clamp_max(self.topk)
        d_i = (csr[4][1:] - csr[4][:-1]).to(torch.int64).clamp_max(self.topk)
        k = d_o + d_i + 1
        k_max, K = (int(k.max().item()), int(k.sum().item())) if E > 0 else (1, 1)
        self.C, self.S, self.F, self.U = capacities(rows, T, self.c1, k_max, K, E, self.zero_slack)
        i64, i32, f32, u8, i16 = torch.int64, torch.int32, torch.float32, torch.uint8, torch.int16
        # inputs
        self.heads = _buf(Q, i64, dev)
        self.tails = _buf(Q, i64, dev)
        self.rels = _buf(Q, i64, dev)
        self.hide = _buf(n_hide, i64, dev)
        self.n_hide = n_hide
        # visibility in CSR order, with the position of every triple on each side
        self.vis = (torch.ones(M, dtype=u8, device=dev), torch.ones(M, dtype=u8, device=dev))
        self.pos = []
        for order in (csr[3], csr[7]):
            p = torch.empty(M, dtype=i64, device=dev)
            p[order.to(i64)] = torch.arange(M, dtype=i64, device=dev)
            self.pos.append(p)
        # hop-1 state
        self.rp0 = torch.arange(rows + 1, dtype=i64, device=dev)
        self.ent0 = _buf(rows, i32, dev)
        self.val0 = torch.ones(rows, dtype=f32, device=dev)
        # per hop: what the backward needs
        self.w = [_buf(rows * self.n, f32, dev) for _ in range(T)]
        self.rp_sel = [_buf(rows + 1, i64, dev) for _ in range(T)]
        self.val_sel = [_buf(self.S[t], f32, dev) for t in range(T)]
        self.src_sel = [_buf(self.S[t], i64, dev) for t in range(T)]
        self.slot_base = [_buf(self.S[t] + 1, i64, dev) for t in range(T)]
        self.entry_count = [_buf(self.S[t], i32, dev) for t in range(T)]
        self.fact_rel = [_buf(self.F[t], i16, dev) for t in range(T)]
        self.fact_pos = [_buf(self.F[t], i32, dev) for t in range(T)]
        self.out_rp = [_buf(rows + 1, i64, dev) for _ in range(T)]
        self.out_ent = [_buf(self.U[t], i32, dev) for t in range(T)]
        self.out_x = [_buf(self.U[t], f32, dev) for t in range(T)]
        self.out_y = [_buf(self.U[t], f32, dev) for t in range(T)]
        self.out_denom = [_buf(rows, f32, dev) for _ in range(T)]
        self.g_y = [_buf(self.U[t], f32, dev) for t in range(T)]
        # transient, shared by the hops
        Smax, Fmax = max(self.S), max(self.F)
        self.ent_sel = _buf(Smax, i32, dev)
        self.entry_info = _buf(L.FL_ENTRY_INFO_INTS * Smax, i32, dev)
        self.use_rank = 0 < r_size <= 16384 and self.topk < L.NO_BUDGET
        self.rel_rank = _buf(rows * 2 * r_size, i16, dev) if self.use_rank else None
        # rows of queries with one relation have one w: they share the first such row's ranks
        self.rank_row = _buf(rows, i32, dev) if self.use_rank else None
        self.chan = torch.arange(N, dtype=torch.int64, device=dev)
        # per hop: rows by descending slot count, the reduction's and the backward's block order
        self.row_order = [_buf(rows, i32, dev) for _ in range(T)]
        self.fact_dst = _buf(Fmax, i32, dev)
        self.fact_val = _buf(Fmax, f32, dev)
        self.grad_sel = _buf(Smax, f32, dev)
        # d loss / d w of the hop being differentiated; with record_grad_w one slice per hop is kept
        self.record_grad_w = bool(record_grad_w)
        self.grad_w = _buf((T if self.record_grad_w else 1) * rows * self.n, f32, dev)
        self.work = _buf(2, i32, dev)  # the expansion's two work queues
        self.status = torch.zeros(1, dtype=i32, device=dev)
        self.ok = torch.ones(1, dtype=f32, device=dev)  # 1 while the status word is clear
        self.scores = _buf(Q, f32, dev)
        self.loss = torch.zeros((), dtype=f32, device=dev)
        self.grad_logits = torch.empty((Q, T, N, self.n), dtype=f32, device=dev)
        ws = 0
        for t in range(T):
            ws = max(ws, lib().fl_topc_workspace(rows, self.C[t]), lib().fl_hop_workspace(rows, self.S[t]),
                     lib().fl_reduce_workspace(rows, self.F[t]))
        ws = max(ws, lib().fl_hop_backward_workspace(rows, self.n))
        self.ws = _buf(ws, u8, dev)
        self.stats = torch.zeros(4, dtype=i64, device=dev) if stats else None
        self.timer = None  # optional: per hop (start, after expand, after reduce) external events

    # ------------------------------------------------------------------
    def memory_bytes(self) -> int:
        seen, total = set(), 0
        for v in vars(self).values():
            for t in (v if isinstance(v, (list, tuple)) else [v]):
                if isinstance(t, torch.Tensor) and t.is_cuda and t.data_ptr() not in seen:
                    seen.add(t.data_ptr())
                    total += t.numel() * t.element_size()
        return total

    def load(self, heads, tails, rels, hide):
        """Copy one step's inputs (device tensors) into the static buffers."""
        if hide.numel() != self.n_hide or heads.numel() != self.Q:
            raise ValueError("inputs must have the static sizes given at construction")
        self.heads.copy_(heads)
        self.tails.copy_(tails)
        self.rels.copy_(rels)
        self.hide.copy_(hide)

    def grad_w_of(self, t):
        """d loss / d w of hop t as [Q, N, n] (kept for every hop only with record_grad_w)."""
        k = t if self.record_grad_w else 0
        m = self.rows * self.n
        return self.grad_w[k * m:(k + 1) * m].view(self.Q, self.N, self.n)

    def _params(self, t, flags):
        return L.fl_hop_params(self.rows, self.N, self.n, self.r_size, self.graph.E, int(self.topk), int(flags), -1,
                               float(self.eps), int(self.F[t]), self.status.data_ptr(), self.entry_info.data_ptr(),
                               self.vis[0].data_ptr(), self.vis[1].data_ptr(), self.work.data_ptr(),
                               self.rel_rank.data_ptr() if self.use_rank else None,
                               self.rank_row.data_ptr() if self.use_rank else None,
                               self.row_order[t].data_ptr())

    # ------------------------------------------------------------------
    def run(self):
        """Forward, loss, backward and (optionally) the SGD update; returns the loss tensor."""
        for part in self.parts():
            part()
        return self.loss

    def parts(self):
        """The step as T + 1 stream-ordered callables, run in order: the
        forward, the loss and the backward of hop T-1; then the backward of
        hops T-2, ..., 0, one per part; last the update.  After part k < T the
        gradient of hop T-1-k is complete (in grad_hop[T-1-k] when the step
        does not apply the update itself), so a caller can start that hop's
        collective while the later parts run; each part can be captured in a
        CUDA graph of its own."""
        T = self.T
        return [self._part_forward] + [lambda t=t: self._backward_hop(t) for t in reversed(range(T - 1))] + \
            [self._finish]

    def _part_forward(self):
        lb, st, g = lib(), _stream(), self.graph
        rows, N, Q, T = self.rows, self.N, self.Q, self.T
        ws, wsn = _p(self.ws), self.ws.numel()
        if self.dropout > 0:
            self.drop_counter.add_(1)
        # hide the batch's own triples (src/main.py:888), remembering what was there
        hid = [self.pos[k][self.hide] for k in range(2)]
        old = [self.vis[k][hid[k]] for k in range(2)]
        for k in range(2):
            self.vis[k].index_fill_(0, hid[k], 0)
        if self.use_rank:
            # first query with the same relation (argmax returns the first maximum)
            first = (self.rels[:, None] == self.rels[None, :]).to(torch.int32).argmax(dim=1)
            self.rank_row.view(Q, N).copy_(first[:, None] * N + self.chan[None, :])
        self.ent0[:rows].view(Q, N).copy_(self.heads.view(Q, 1).expand(Q, N))
        rp_in, ent_in, val_in = self.rp0, self.ent0, self.val0
        for t in range(T):
            # this hop's attention rows [Q, N, n], gathered contiguous, then softmax
            self.w[t][:rows * self.n].view(Q, N, self.n).copy_(
                torch.softmax(self.table[:, t].index_select(0, self.rels), dim=-1))
            # c1
            if self.c1 is not None:
                check(lb.fl_topc_select(_p(rp_in), _p(ent_in), _p(val_in), rows, self.C[t], self.c1, None,
                                        _p(self.rp_sel[t]), _p(self.ent_sel), _p(self.val_sel[t]),
                                        _p(self.src_sel[t]), self.S[t], _p(self.status), ws, wsn, st), "topc_select")
                rp_s, ent_s, val_s = self.rp_sel[t], self.ent_sel, self.val_sel[t]
            else:
                rp_s, ent_s, val_s = rp_in, ent_in, val_in
                self.rp_sel[t].copy_(rp_in)
                self.val_sel[t][:self.S[t]].copy_(val_in[:self.S[t]])
            if self.use_rank:
                check(lb.fl_relation_rank(_p(self.w[t]), rows, self.r_size, _p(self.rank_row), _p(self.rel_rank), st),
                      "relation_rank")
            params = self._params(t, self.flags)
            check(lb.fl_hop_plan(ctypes.byref(params), _p(rp_s), _p(ent_s), self.S[t], g.ori, g.inv,
                                 _p(self.slot_base[t]), None, ws, wsn, st), "hop_plan")
            # rows by descending slot count: the reduction and the backward take the heaviest first
            if rows <= 16384:
                check(lb.fl_row_order(_p(rp_s), _p(self.slot_base[t]), rows, _p(self.row_order[t]), st), "row_order")
            else:
                rows_facts = self.slot_base[t][rp_s[1:]] - self.slot_base[t][rp_s[:-1]]
                self.row_order[t].copy_(torch.argsort(rows_facts, descending=True, stable=True))
            if self.timer is not None:
                self.timer[t][0].record()
            check(lb.fl_hop_expand(ctypes.byref(params), _p(rp_s), _p(ent_s), _p(val_s), self.S[t], _p(self.w[t]),
                                   g.ori, g.inv, None, None, None, None, _p(self.slot_base[t]), _p(self.fact_dst),
                                   _p(self.fact_val), _p(self.fact_rel[t]), None, _p(self.entry_count[t]), st),
                  "hop_expand")
            if self.timer is not None and len(self.timer[t]) > 2:
                self.timer[t][1].record()
            check(lb.fl_row_reduce(_p(rp_s), rows, g.E, _p(self.slot_base[t]), _p(self.entry_count[t]),
                                   _p(self.fact_dst), _p(self.fact_val), self.F[t], _p(self.fact_pos[t]),
                                   ctypes.c_float(self.eps), _p(self.out_rp[t]), _p(self.out_ent[t]),
                                   _p(self.out_x[t]), _p(self.out_y[t]), _p(self.out_denom[t]), _p(self.status),
                                   _p(self.row_order[t]), ws, wsn, self._drop(t), st), "row_reduce")
            if self.timer is not None:
                self.timer[t][-1].record()
            if self.stats is not None:
                check(lb.fl_hop_stats(_p(rp_s), rows, _p(ent_s), self.S[t], g.ori, g.inv, _p(self.entry_count[t]),
                                      _p(self.out_rp[t]), 0, _p(self.stats), st), "hop_stats")
            rp_in, ent_in, val_in = self.out_rp[t], self.out_ent[t], self.out_y[t]
        # the backward reads no visibility: restore what the batch hid
        for k in range(2):
            self.vis[k].index_put_((hid[k],), old[k])
        # readout + loss (src/utils.py:36-47)
        check(lb.fl_readout(_p(rp_in), _p(ent_in), _p(val_in), N, _p(self.tails), Q, _p(self.scores), st), "readout")
        score = self.scores[:Q]
        self.loss.copy_(-torch.mean(torch.log(torch.clamp_min(score, self.thr))))
        g_score = torch.where(score > self.thr, -1.0 / (Q * torch.clamp_min(score, self.thr)),
                              torch.zeros_like(score))
        check(lb.fl_readout_backward(_p(rp_in), _p(ent_in), N, _p(self.tails), Q, _p(g_score), _p(self.g_y[T - 1]),
                                     self.U[T - 1], _p(self.out_rp[T - 1][rows:]), self._drop(T - 1), st),
              "readout_backward")
        # a forward that overflowed a buffer updates nothing: its gradient is scaled by 0
        self.ok.copy_(self.status == 0)
        self._backward_hop(T - 1)

    def _backward_hop(self, t):
        """Backward of hop t; g_y[t] arrived through hop t's dropout (the same
        keep bits and scale), applied where it is written."""
        lb, st = lib(), _stream()
        rows, N, Q = self.rows, self.N, self.Q
        ws, wsn = _p(self.ws), self.ws.numel()
        params = self._params(t, self.flags)
        check(lb.fl_hop_backward(ctypes.byref(params), _p(self.rp_sel[t]), _p(self.val_sel[t]), self.S[t],
                                 _p(self.w[t]), _p(self.slot_base[t]), _p(self.entry_count[t]),
                                 _p(self.fact_pos[t]), _p(self.fact_rel[t]), None, _p(self.out_rp[t]),
                                 _p(self.out_x[t]), _p(self.out_denom[t]), _p(self.g_y[t]), _p(self.grad_sel),
                                 _p(self.grad_w_of(t)), ws, wsn, st), "hop_backward")
        if t > 0:
            src = self.src_sel[t] if self.c1 is not None else None
            if src is not None:
                check(lb.fl_scatter_grad(_p(self.grad_sel), _p(src), self.S[t], _p(self.rp_sel[t][rows:]),
                                         _p(self.g_y[t - 1]), self.U[t - 1], _p(self.out_rp[t - 1][rows:]),
                                         self._drop(t - 1), st),
                      "scatter_grad")
            else:
                self.g_y[t - 1][:self.S[t]].copy_(self.grad_sel[:self.S[t]])
                if self.dropout > 0:
                    self._dropout(self.g_y[t - 1], t - 1, st)
        # softmax backward, d logits = w * (g - sum(g * w)): torch's own kernel
        wt = self.w[t][:rows * self.n].view(Q, N, self.n)
        gw = self.grad_w_of(t)
        torch.mul(torch._softmax_backward_data(gw, wt, -1, torch.float32), self.ok, out=self.grad_logits[:, t])
        if not self.apply_update:
            # hop t's dense table gradient, complete once this part has run
            self.grad_hop[t].zero_()
            self.grad_hop[t].index_add_(0, self.rels, self.grad_logits[:, t])

    def _finish(self):
        if self.apply_update:
            # SGD on the rows of the batch's relations only: no dense gradient
            self.table.index_add_(0, self.rels, self.grad_logits, alpha=-self.lr)

    def _drop(self, t):
        """fl_dropout of hop t for the kernels that write its values or their gradient (None: no dropout)."""
        if self.dropout <= 0:
            return None
        return ctypes.byref(L.fl_dropout(self.dropout, self.dropout_seed, self.drop_counter.data_ptr(), t))

    def _dropout(self, x, t, st):
        check(lib().fl_value_dropout(_p(x), _p(x), self.U[t], _p(self.out_rp[t][self.rows:]),
                                     ctypes.c_double(self.dropout), self.dropout_seed, _p(self.drop_counter), t, st),
              "value_dropout")

    def check(self):
        """Raise if any hop ran out of its buffers (one host read)."""
        if int(self.status.item()) & L.FL_STATUS_SLOT_OVERFLOW:
            raise RuntimeError("a hop exceeded its static capacity")
