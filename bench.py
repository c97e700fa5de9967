"""Benchmark: propagated facts/s of one L=3 sparse DRUM fwd+bwd step.

Workload (default): config 4 of the benchmark configs -- 4.6M entities, 822
base relations (+ inverses), 20.6M training triples; DRUM with T=3 hops,
N=3 channels, batch 256 (512 queries: every sampled triple gives (h, r, t) and
(t, r + R, h)), c1 = 1000 entity budget, c2 = 400 fact budget, deterministic
top-k.  Seeded synthetic data (the reference's datasets are unavailable).

A fact is one emitted (query, channel, src -> dst) contribution through a
kept, visible graph edge in a hop's forward; identity terms are not counted.
value = sum of facts over the timed steps / device time of those steps (hop
forward + backward, readout, loss, gradient all-reduce and the parameter
update), inputs resident in HBM.  e2e = the same metric through the
reference-facing operator API (COO states,
vectorized_operation_sparse3d_csr_sum_norm per hop) with the step's query
batch copied from pinned host memory and the loss read back every step.

The per-query attention w_t = softmax(table[r_q, t] / tau_1) is a learnable
table indexed by the query relation; it stands in for the reference's LSTM
over the relation embedding (outside the propagation hot path).

Multi-GPU (torchrun): every rank runs its own 512 queries on a replica of the
CSR (weak scaling); per step one NCCL all_gather of the batch triple ids (so
every replica hides the union, src/main.py:888) and one all_reduce of the
attention gradients.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

from flashlog_b200.synthetic import CONFIGS, load_graph, load_or_generate, training_queries  # noqa: E402

PROFILE_TRAFFIC = os.path.join(REPO, "profiles", "hop_forward_traffic.json")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", type=int, default=4)
    ap.add_argument("--batch-size", type=int, default=0, help="override --batch_size (queries = 2x)")
    ap.add_argument("--e2e-steps", type=int, default=0, help="timed e2e steps (default: --steps)")
    ap.add_argument("--cpu-queries", type=int, default=16)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--dropout", type=float, default=0.1,
                    help="training dropout of each hop's values (src/main.py:1008 default 0.1)")
    ap.add_argument("--engine", default="graph", choices=["graph", "autograd"],
                    help="graph: static-buffer step replayed as CUDA graphs; autograd: engine.drum_propagate")
    ap.add_argument("--rules", type=int, default=0,
                    help="instead of the training step: max-product rule-bank evaluation of this many test "
                         "queries (sharded over the ranks), --rule-bank rules, queries/s")
    ap.add_argument("--rule-bank", type=int, default=50_000)
    ap.add_argument("--union-rows", action="store_true",
                    help="N > 1: all-reduce only the table rows of the ranks' batch relations (one host read "
                         "per step to find them) instead of the whole hop gradient")
    ap.add_argument("--rule-timing", action="store_true",
                    help="synchronize between the evaluator's phases and report their host times")
    ap.add_argument("--rule-ops", choices=("edge", "uniform"), default="edge",
                    help="body operators drawn by edge frequency (default) or uniformly over the 2R operators")
    ap.add_argument("--rule-max", action="store_true", help="mmDRUM (max over ranks); default smDRUM (sum)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi samples (clocks, throttle reasons) during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (FileNotFoundError, OSError):
            self.proc = None

    def wait_first(self, timeout=10.0):
        """Block until nvidia-smi has printed one sample, so its start-up is not timed."""
        t_end = time.time() + timeout
        while self.proc is not None and not self.lines and time.time() < t_end and self.proc.poll() is None:
            time.sleep(0.02)
        self.skip = len(self.lines)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lines = self.lines[getattr(self, "skip", 0):] or self.lines[-1:]
        for ln in lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, flag in zip(names, parts[5:9]):
                if flag.lower() in ("active", "1", "yes"):
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


class HopTimer:
    """CUDA events around each hop forward (expand + row reduction) on the launching stream."""

    def __init__(self):
        self.pairs = []
        self.enabled = False

    def record_start(self):
        if self.enabled:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.pairs.append([e, None])

    def record_end(self):
        if self.enabled:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.pairs[-1][1] = e

    def total_ms(self):
        return sum(a.elapsed_time(b) for a, b in self.pairs)


class Stats:
    """Per-hop counts (device tensors, reduced after the timed region)."""

    def __init__(self, graph):
        self.graph = graph
        self.records = []
        self.timer = HopTimer()

    def append(self, rec):
        self.records.append(rec)

    def reduce(self):
        g = self.graph.csr
        S = G = F = U = 0
        for ent, s_live, entry_count, u_live in self.records:
            n = int(s_live.item())
            e = ent[:n].to(torch.int64)
            S += n
            G += int(((g[8][e + 1] - g[8][e]).sum() + (g[12][e + 1] - g[12][e]).sum()).item())
            F += int(entry_count[:n].to(torch.int64).sum().item()) - n  # identity terms excluded
            U += int(u_live.item())
        return S, G, F, U


# ---------------------------------------------------------------------------
def setup(args, rank, world, device):
    cfg = CONFIGS[args.config]
    if args.batch_size:
        import dataclasses
        cfg = dataclasses.replace(cfg, batch_size=args.batch_size)
    train, tt = load_graph(cfg, device)
    from flashlog_b200.flashlog_kernel import build_csr_structure
    csr = build_csr_structure(tt[:, 0], tt[:, 2], tt[:, 1], cfg.entities)
    del tt
    torch.cuda.empty_cache()
    return cfg, train, csr


def batches_for(cfg, train, n, rank, seed_base=1234):
    out = []
    for s in range(n):
        ids, h, r, t = training_queries(train, cfg, step=s, seed=seed_base + 7919 * rank)
        out.append((ids, h, r, t))
    return out


TABLE_MAX_BYTES = 4 << 30


def attention_table(cfg, data, device):
    """The learnable attention logits [rows, T, N, n] and the batches with
    their query relations mapped to table rows.

    Up to TABLE_MAX_BYTES the table has one row per query relation (2R rows,
    drawn on the host from seed 1234).  Beyond (config 5: 29,648 x 9 x
    29,649 fp32 would take 31.6 GB) it has one row per distinct query
    relation of the run's batches, drawn on the device; only the row index
    changes, the softmax, propagation and update are the same."""
    R, T, N = cfg.relations, cfg.T, cfg.N
    n = 2 * R + 1
    if 2 * R * T * N * n * 4 <= TABLE_MAX_BYTES:
        gen = torch.Generator(device="cpu").manual_seed(1234)
        return torch.randn(2 * R, T, N, n, generator=gen).to(device), data
    rels = np.unique(np.concatenate([b[2] for b in data]))
    mapped = [(ids, h, np.searchsorted(rels, r).astype(np.int64), t) for ids, h, r, t in data]
    gen = torch.Generator(device=device).manual_seed(1234)
    return torch.randn(rels.size, T, N, n, generator=gen, device=device), mapped


def run_value_arm(args, cfg, train, csr, rank, world, device):
    from flashlog_b200 import _lib, engine
    from flashlog_b200.ops import Graph
    import torch.distributed as dist

    graph = Graph.of(csr)
    R, T, N = cfg.relations, cfg.T, cfg.N
    n = 2 * R + 1
    mask = torch.ones(train.shape[0], dtype=torch.uint8, device=device)
    nb = args.warmup + args.steps
    table, data = attention_table(cfg, batches_for(cfg, train, nb, rank), device)
    table.requires_grad_(True)
    dev_data = [tuple(torch.from_numpy(x).to(device) for x in b) for b in data]
    stats = Stats(graph)
    status = engine.new_status(device)
    lr = 0.01
    k = 0  # steps so far: the dropout counter

    def step(ids, h, r, t, collect):
        from flashlog_b200 import multigpu as MG
        hide = MG.gather_hidden_triples(ids) if world > 1 else ids
        mask[hide] = 0
        w_all = table[r]
        nonlocal k
        k += 1
        rp, ent, val = engine.drum_propagate(h, w_all, graph, R, c1=cfg.c1 or None, c2=cfg.c2, mask_triple=mask,
                                             stats=stats if collect else None, status=status, dropout=args.dropout,
                                             dropout_seed=1234 + rank, dropout_counter=k)
        loss = engine.readout_loss(rp, ent, val, t, N)
        table.grad = None
        loss.backward()
        if world > 1:
            MG.allreduce_mean_(table.grad)
        with torch.no_grad():
            table.sub_(lr * table.grad)
        mask[hide] = 1
        return loss

    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()  # before the warm-up: nvidia-smi's start-up must not fall in the timed region
    for b in dev_data[:args.warmup]:
        step(*b, collect=False)
    torch.cuda.synchronize()
    clocks.wait_first()
    if world > 1:
        dist.barrier()
    launches0 = _lib.lib().fl_launch_count()
    stats.timer.enabled = True
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for b in dev_data[args.warmup:]:
        step(*b, collect=True)
    t1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = t0.elapsed_time(t1)
    engine.check_status(status)  # no hop ran out of its buffers
    launches = _lib.lib().fl_launch_count() - launches0
    clk = clocks.stop()
    S, G, F, U = stats.reduce()
    hop_ms = stats.timer.total_ms()
    n_hops = len(stats.timer.pairs)
    return dict(ms=ms, facts=F, S=S, G=G, U=U, hop_ms=hop_ms, n_hops=n_hops, launches=launches, clocks=clk,
                data=data, table=table)


def run_graph_arm(args, cfg, train, csr, rank, world, device):
    """The training step of flashlog_b200.step.DrumTrainStep, one CUDA graph per timed step.

    Each graph holds its own external CUDA events around every hop's
    expansion + row reduction, so the hop-forward kernel time is read from the
    timed replays themselves; the work counts (S, G, F, U) are accumulated on
    the device by the step.  Kernel launches per step are counted while the
    step is captured.
    """
    from flashlog_b200 import _lib
    from flashlog_b200.ops import Graph
    from flashlog_b200.step import DrumTrainStep
    import torch.distributed as dist

    graph = Graph.of(csr)
    R, T, N = cfg.relations, cfg.T, cfg.N
    n = 2 * R + 1
    nb = args.warmup + args.steps
    table, data = attention_table(cfg, batches_for(cfg, train, nb, rank), device)
    dev_data = [tuple(torch.from_numpy(x).to(device) for x in b) for b in data]
    n_ids = dev_data[0][0].numel()
    step = DrumTrainStep(graph, R, cfg.queries, T, N, cfg.c1 or None, cfg.c2, table, n_hide=n_ids * world,
                         apply_update=(world == 1), dropout=args.dropout, dropout_seed=1234 + rank)
    lr = step.lr

    from flashlog_b200 import multigpu as MG

    def hide_of(ids):
        return MG.gather_hidden_triples(ids) if world > 1 else ids

    # N > 1: the step runs as T + 1 parts; as soon as the part that completes
    # hop t's table gradient has been issued, that gradient's all-reduce is
    # issued on a communication stream, so it overlaps the remaining backward
    # parts; the update waits for all of them.
    comm = torch.cuda.Stream() if world > 1 else None

    # N > 1 with --union-rows: only the union of the ranks' batch relations
    # (rows of the table) can hold gradient, so those rows alone are
    # all-reduced and updated; finding the union costs a host read per step
    def run_parts(parts, rels):
        if world > 1:
            rows = MG.union_rows(rels, table.shape[0]) if args.union_rows else None
            MG.run_parts_with_overlapped_allreduce(parts, step.grad_hop, step.grad, table, lr, comm, rows=rows)
        else:
            for part in parts:
                part()

    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()  # before the warm-up: nvidia-smi's start-up must not fall in the timed region
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # warm-up (also sets kernel attributes before any capture)
        for b in dev_data[:args.warmup]:
            ids, h, r, t = b
            step.load(h, t, r, hide_of(ids))
            run_parts(step.parts(), r)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    step.check()
    # graphs per timed step (one for the whole step at N = 1, one per part at
    # N > 1, the collectives between them), each step with its own hop events
    graphs, timers = [], []
    pool = None
    launches_per_step = 0
    for k in range(args.steps):
        timer = [tuple(torch.cuda.Event(enable_timing=True, external=True) for _ in range(3)) for _ in range(T)]
        step.timer = timer
        l0 = _lib.lib().fl_launch_count()
        chunks = [step.run] if world == 1 else step.parts()[:T]  # the last part is empty without the update
        gs = []
        for fn in chunks:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=pool):
                fn()
            pool = g.pool()
            gs.append(g)
        launches_per_step = _lib.lib().fl_launch_count() - l0
        graphs.append(gs)
        timers.append(timer)
    step.timer = None
    torch.cuda.synchronize()
    step.stats.zero_()
    clocks.wait_first()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for k, b in enumerate(dev_data[args.warmup:]):
        ids, h, r, t = b
        step.load(h, t, r, hide_of(ids))
        if world == 1:
            graphs[k][0].replay()
        else:
            run_parts([g.replay for g in graphs[k]], r)
    t1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = t0.elapsed_time(t1)
    clk = clocks.stop()
    step.check()  # no hop ran out of its buffers
    S, G, F, U = (int(x) for x in step.stats.tolist())
    hop_ms = sum(a.elapsed_time(c) for timer in timers for a, b, c in timer)
    expand_ms = sum(a.elapsed_time(b) for timer in timers for a, b, c in timer)
    reduce_ms = sum(b.elapsed_time(c) for timer in timers for a, b, c in timer)
    del graphs
    return dict(ms=ms, facts=F, S=S, G=G, U=U, hop_ms=hop_ms, expand_ms=expand_ms, reduce_ms=reduce_ms,
                n_hops=args.steps * T,
                launches=launches_per_step * args.steps, clocks=clk, data=data, table=table,
                memory_gb=step.memory_bytes() / 1e9)


def run_e2e_arm(args, cfg, train, csr, data, table, rank, world, device, steps):
    """Same metric through the reference-facing operator API with host buffers."""
    import flashlog_b200.flashlog_kernel as fk
    from flashlog_b200 import engine, ops
    import torch.distributed as dist

    from flashlog_b200.dropout import sparse_dropout
    R, T, N, E = cfg.relations, cfg.T, cfg.N, cfg.entities
    mask = torch.ones(train.shape[0], dtype=torch.bool, device=device)
    pinned = [tuple(torch.from_numpy(x).pin_memory() for x in b) for b in data]
    k = 0  # steps so far: the dropout counter
    h2d = sum(x.numel() * x.element_size() for x in pinned[0])
    tab = table.detach().clone().requires_grad_(True)

    def step(ids_h, h_h, r_h, t_h):
        nonlocal k
        k += 1
        ids = ids_h.to(device, non_blocking=True)
        h = h_h.to(device, non_blocking=True)
        r = r_h.to(device, non_blocking=True)
        t = t_h.to(device, non_blocking=True)
        from flashlog_b200 import multigpu as MG
        hide = MG.gather_hidden_triples(ids) if world > 1 else ids
        mask[hide] = False
        Q = h.numel()
        w_all = tab[r]
        sb = torch.arange(Q, device=device).repeat_interleave(N)
        sl = torch.arange(N, device=device).repeat(Q)
        se = h.repeat_interleave(N)
        state = torch.sparse_coo_tensor(torch.stack([sb, sl, se]), torch.ones(Q * N, device=device),
                                        (Q, N, E), is_coalesced=True)
        for hop in range(T):
            w_t = torch.softmax(w_all[:, hop], dim=-1)
            state = fk.vectorized_operation_sparse3d_csr_sum_norm(state, w_t, csr, mask, R, use_topk=True,
                                                                 topk_edges=cfg.c2 // 2, topk_nodes=cfg.c1)
            # the models' training dropout of the values (src/model_DRUM_kernel_sp.py:189-192)
            state = sparse_dropout(state, args.dropout, seed=1234 + rank, counter=k, subseq=hop)
        # readout + log loss (src/utils.py:36-47) through the library's readout
        idx = state.indices()
        rp, ent, _ = ops.coo_to_rows(idx[0], idx[1], idx[2], Q, N, E)
        loss = engine.readout_loss(rp, ent, state.values(), t, N)
        tab.grad = None
        loss.backward()
        if world > 1:
            MG.allreduce_mean_(tab.grad)
        with torch.no_grad():
            tab.sub_(0.01 * tab.grad)
        mask[hide] = True
        return loss.item()  # device -> host read of the step's result

    for b in pinned[:args.warmup]:
        step(*b)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for b in pinned[args.warmup:args.warmup + steps]:
        step(*b)
    e1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    return e0.elapsed_time(e1), h2d, 4


def cpu_baseline(args, cfg, train, csr):
    """The reference's OpenMP path on a bounded sample of the same workload."""
    from oracle import cpu_baseline as CB
    torch.set_num_threads(os.cpu_count() or 1)
    csr_np = tuple(c.cpu().numpy() for c in csr)
    R, T, N = cfg.relations, cfg.T, cfg.N
    n = 2 * R + 1
    rng = np.random.default_rng(99)
    batches = []
    for s in range(4):
        ids, h, r, t = training_queries(train, cfg, step=1000 + s)
        q = args.cpu_queries
        h, r, t, ids = h[:q], r[:q], t[:q], ids[:q // 2]
        w_all = rng.standard_normal((q, T, N, n)).astype(np.float32)
        mask = np.ones(train.shape[0], np.uint8)
        mask[ids] = 0
        batches.append((h, t, w_all, mask))
    rate, facts, secs, steps, kind = CB.time_sample(csr_np, batches, R, cfg.entities, cfg.c1, cfg.c2,
                                                    min_seconds=args.cpu_seconds, max_seconds=3 * args.cpu_seconds,
                                                    dropout=args.dropout)
    return dict(value=rate, unit="facts/s", cores=torch.get_num_threads(), kind=kind,
                sample=f"{steps} steps x {args.cpu_queries} queries of config {cfg.index} "
                       f"({facts} facts in {secs:.1f} s); c1 via the oracle port, expansion/reduction/"
                       f"normalization fwd+bwd in the reference's compiled OpenMP extension; "
                       f"dropout {args.dropout} on every hop's values")


def run_rules(args, rank, world, device):
    """Max-product rule-bank evaluation (rules/evaluate.py routed_normalized,
    reduction 'max'): the config's test split gives args.rules queries
    (both directions of each triple), a seeded bank of args.rule_bank rules
    (heads by query-relation frequency, bodies of 1-3 operators by edge
    frequency, weights U(0, 1), three groups) routes to them, and every rank
    ranks its contiguous share of the queries (filtered by the targets).
    value = queries / device time (max over ranks)."""
    from flashlog_b200 import multigpu as MG
    from flashlog_b200 import rules as RB
    from flashlog_b200.flashlog_kernel import build_csr_structure
    from flashlog_b200.synthetic import (evaluation_queries, generate_triples_device, host_generation_fits,
                                         rule_bank)
    import torch.distributed as dist
    cfg = CONFIGS[args.config]
    if host_generation_fits(cfg):
        train, _, test = load_or_generate(cfg)
        tt = torch.from_numpy(train).to(device)
    else:
        tt, _, test_dev = generate_triples_device(cfg, device=device)
        train, test = tt.cpu().numpy(), test_dev.cpu().numpy()
        del test_dev
    csr = build_csr_structure(tt[:, 0], tt[:, 2], tt[:, 1], cfg.entities)
    del tt
    torch.cuda.empty_cache()
    src, rel, dst = evaluation_queries(test, cfg.relations, (args.rules + 1) // 2)
    src, rel, dst = src[:args.rules], rel[:args.rules], dst[:args.rules]
    rules = rule_bank(train, rel, cfg.relations, args.rule_bank, uniform_ops=args.rule_ops == "uniform")
    lo, hi = MG.shard_bounds(src.size, rank, world)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a[lo:hi])).to(device)
    s_d, r_d, t_d = d(src), d(rel), d(dst)
    stats = {"timing": bool(args.rule_timing)}
    # warm-up: the first relation group (kernel attributes, allocator)
    w_n = min(64, hi - lo)
    RB.evaluate_rule_bank(s_d[:w_n], r_d[:w_n], t_d[:w_n], rules, csr, cfg.relations, cfg.entities,
                          final_max=args.rule_max)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    from flashlog_b200 import _lib
    l0 = _lib.lib().fl_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall = time.perf_counter()
    e0.record()
    ranks = RB.evaluate_rule_bank(s_d, r_d, t_d, rules, csr, cfg.relations, cfg.entities, final_max=args.rule_max,
                                  stats=stats)
    e1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t_wall
    ms = e0.elapsed_time(e1)
    launches = _lib.lib().fl_launch_count() - l0
    all_ranks = MG.gather_varlen(ranks) if world > 1 else ranks
    n_q = hi - lo
    if world > 1:
        ms, n_q = MG.max_time_sum_work(ms, n_q, device)
    if rank == 0:
        r = all_ranks.cpu().numpy()
        line = {"metric": "rule-bank queries/sec (max-product, routed_normalized)", "value": n_q / (ms / 1000.0),
                "unit": "queries/s", "n_gpus": world, "ms_total": ms, "wall_s_rank0": wall,
                "higher_is_better": True, "scaling": "strong", "dtype": "f32", "data": "synthetic",
                "config": {"workload": f"config {cfg.index}: {cfg.entities} entities, {cfg.train_triples} triples; "
                                       f"{args.rules} test queries, {args.rule_bank} rules "
                                       f"(body operators by {'edge frequency' if args.rule_ops == 'edge' else 'uniform draw'}), "
                                       f"{'mmDRUM (max)' if args.rule_max else 'smDRUM (sum)'} over 3 ranks",
                           "parallelism": f"query-sharded dp{world}"},
                "metrics": {"mrr": float((1.0 / r).mean()), "hits@10": float((r <= 10).mean())},
                "rule_instances_rank0": stats.get("instances"), "batches_rank0": stats.get("batches"),
                "entries_rank0": stats.get("entries"), "bitmap_rows_rank0": stats.get("bitmap_rows"),
                "dense_queries_rank0": stats.get("dense_queries"),
                "phase_s_rank0": {k: stats[k] for k in ("ground_s", "score_s") if k in stats},
                "compacted_rules": stats.get("rules_after"),
                "gpu_launches": launches}
        print(json.dumps(line))


def workload_desc(cfg, world):
    return (f"config {cfg.index}: {cfg.entities} entities, {cfg.relations} relations (+inverses), "
            f"{cfg.train_triples} triples; DRUM T={cfg.T} N={cfg.N}, batch {cfg.batch_size} "
            f"({cfg.queries} queries) per GPU, c1={cfg.c1} c2={cfg.c2}, deterministic top-k")


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cfg0 = CONFIGS[args.config]
    metric = "propagated facts/sec (L=3 DRUM fwd+bwd)"

    if args.impl == "reference":
        if rank != 0:
            return
        import dataclasses
        cfg = dataclasses.replace(cfg0, batch_size=args.batch_size) if args.batch_size else cfg0
        from oracle import oracle as O
        from oracle import reference as Rf
        from flashlog_b200.synthetic import host_generation_fits
        if host_generation_fits(cfg):
            train, _, _ = load_or_generate(cfg)
        else:  # config 5: drawn on the device (the host generator cannot key 68-bit triples)
            train, tt = load_graph(cfg, torch.device("cuda", local))
            del tt
            torch.cuda.empty_cache()
        # the reference's own CSR builder (csr.cpp) when built, else the oracle's restatement
        build = Rf.build_csr if Rf.available() else O.build_csr
        csr_np = build(train[:, 0], train[:, 2], train[:, 1], cfg.entities)
        from oracle import cpu_baseline as CB
        torch.set_num_threads(os.cpu_count() or 1)
        rng = np.random.default_rng(99)
        R, T, N = cfg.relations, cfg.T, cfg.N
        vals = []
        steps_done = 0
        t_all = time.perf_counter()
        for s in range(args.warmup + args.steps):
            ids, h, r, t = training_queries(train, cfg, step=2000 + s)
            q = args.cpu_queries
            w_all = rng.standard_normal((q, T, N, 2 * R + 1)).astype(np.float32)
            mask = np.ones(train.shape[0], np.uint8)
            mask[ids[:q // 2]] = 0
            t0 = time.perf_counter()
            f, _, kind = CB.drum_step(csr_np, h[:q], t[:q], w_all, mask, R, cfg.entities, cfg.c1, cfg.c2,
                                      dropout=args.dropout, seed=2000 + s)
            el = time.perf_counter() - t0
            if s >= args.warmup:
                vals.append((f, el))
                steps_done += 1
        facts = sum(f for f, _ in vals)
        secs = sum(e for _, e in vals)
        value = facts / secs if secs > 0 else 0.0
        line = {"impl": "reference", "metric": metric, "value": value, "unit": "facts/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * secs / max(steps_done, 1),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic",
                "config": {"workload": workload_desc(cfg, 1) + f"; CPU sample of {args.cpu_queries} queries per step",
                           "global_batch": args.cpu_queries, "parallelism": "OpenMP host threads"},
                "cpu_baseline": {"value": value, "unit": "facts/s", "cores": torch.get_num_threads(), "kind": kind,
                                 "sample": f"{steps_done} steps x {args.cpu_queries} queries"},
                "e2e": {"value": value, "unit": "facts/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    import torch.distributed as dist
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))
    if args.rules:
        run_rules(args, rank, world, device)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    cfg, train, csr = setup(args, rank, world, device)
    if args.engine == "graph":
        res = run_graph_arm(args, cfg, train, csr, rank, world, device)
    else:
        res = run_value_arm(args, cfg, train, csr, rank, world, device)
    ms = res["ms"]
    facts = res["facts"]
    hop_ms = res["hop_ms"]
    if world > 1:
        from flashlog_b200 import multigpu as MG
        ms, facts = MG.max_time_sum_work(ms, facts, device)
        facts = int(facts)
    value = facts / (ms / 1000.0)
    e2e = None
    if not args.no_e2e:
        steps_e2e = args.e2e_steps or args.steps
        e2e_ms, h2d, d2h = run_e2e_arm(args, cfg, train, csr, res["data"], res["table"], rank, world, device,
                                       steps_e2e)
        local_facts = res["facts"] * steps_e2e / args.steps
        if world > 1:
            from flashlog_b200 import multigpu as MG
            e2e_ms, local_facts = MG.max_time_sum_work(e2e_ms, local_facts, device)
        e2e = {"value": local_facts / (e2e_ms / 1000.0), "unit": "facts/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms / steps_e2e,
               "api": "vectorized_operation_sparse3d_csr_sum_norm per hop (COO in/out)"}
    peaks_path = os.path.join(REPO, "MEASURED_PEAKS.json")
    peak, peak_src = 6650.0, "fallback"
    if os.path.exists(peaks_path):
        try:
            peak = float(json.load(open(peaks_path))["hbm_gbs"])
            peak_src = "measured"
        except Exception:
            pass
    S, G, U = res["S"], res["G"], res["U"]
    alg_bytes = 24 * S + 14 * G + 5 * res["facts"] + 8 * U
    # per kernel, the kernel's own compulsory I/O over the timed hops
    # (expansion: its inputs 24 S + 14 G + 5 F and the facts it writes, 10 F
    # with S identity facts; reduction + compaction: the facts it reads 8 F,
    # fact positions 4 F, per-row outputs 8 U written and re-read, 12 U
    # packed), each over its own CUDA-event time
    per_kernel = None
    if res.get("expand_ms") is not None and res["expand_ms"] > 0 and res["reduce_ms"] > 0:
        Fi = res["facts"] + S
        kb = {"hop_expand": 24 * S + 14 * G + 5 * res["facts"] + 10 * Fi, "row_reduce+compact": 12 * Fi + 28 * U}
        kt = {"hop_expand": res["expand_ms"], "row_reduce+compact": res["reduce_ms"]}
        per_kernel = {k: {"bytes": kb[k], "ms": kt[k], "achieved_gbs": kb[k] / (kt[k] / 1000.0) / 1e9,
                          "frac": kb[k] / (kt[k] / 1000.0) / 1e9 / peak}
                      for k in kb}
    achieved = alg_bytes / (hop_ms / 1000.0) / 1e9 if hop_ms > 0 else 0.0
    # DRAM bytes per hop forward: ncu's count on a small case of the same
    # configuration (profiles/hop_forward_traffic.json), scaled to this run's
    # hops by their algorithmic bytes
    traffic = None
    if os.path.exists(PROFILE_TRAFFIC) and res["n_hops"] > 0:
        try:
            prof = json.load(open(PROFILE_TRAFFIC))
            if prof.get("config") == cfg.index:
                traffic = float(prof["dram_bytes_per_algorithmic_byte"]) * alg_bytes / res["n_hops"]
        except Exception:
            traffic = None
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_baseline(args, cfg, train, csr)
        except Exception as exc:  # the baseline never decides the GPU result
            cpu = {"value": None, "unit": "facts/s", "cores": os.cpu_count(), "kind": "reference",
                   "sample": f"failed: {exc}"}
    if rank == 0:
        line = {"metric": metric, "value": value, "unit": "facts/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": workload_desc(cfg, world), "global_batch": cfg.queries * world,
                           "per_gpu_queries": cfg.queries, "parallelism": f"query-sharded dp{world}",
                           "l2": "inputs larger than L2 (CSR ~0.7 GB; fresh query batch every step)",
                           "engine": ("static buffers, one CUDA graph per step (flashlog_b200.step)"
                                      if args.engine == "graph" else "autograd, one host sync per hop"),
                           "facts_per_step": facts / args.steps, "dropout": args.dropout},
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "traffic": traffic, "peak_source": peak_src,
                             "kernel": "hop forward (expand + row reduction), rank 0",
                             "algorithmic_bytes": "24*S + 14*G + 5*F + 8*U per hop",
                             "algorithmic_bytes_per_hop": alg_bytes / max(res["n_hops"], 1),
                             "units": {"S": S, "G": G, "F": res["facts"], "U": U, "hops": res["n_hops"],
                                       "hop_forward_ms": hop_ms},
                             "per_kernel": per_kernel},
                "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": res["launches"], "clocks": res["clocks"]}
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
