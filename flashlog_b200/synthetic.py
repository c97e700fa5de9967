"""Seeded synthetic knowledge graphs with the shapes of the benchmark configs.

The reference's datasets (FB15k-237, YAGO3-10, Wikidata5M, Freebase, ...) are not
available, so every workload here is a seeded synthetic stand-in with the entity,
relation and triple counts of the five benchmark configurations:

* relation ids follow a finite Zipf law over a seeded permutation of the base
  relations;
* heads are uniform (or Zipf for config 2), tails follow a Zipf law over a seeded
  entity permutation, which produces the hub entities that drive the c2 budget;
* duplicate (h, r, t) triples are dropped and resampled until the stated count
  is reached.

Queries follow the reference's ``batch_iter`` (src/dataloader.py:99-123): every
sampled training triple yields the two queries (h, r, t) and (t, r + R, h), so a
``--batch_size b`` step has ``2 b`` queries, and the batch's own triples are
hidden through the edge-visibility mask (src/main.py:888).
"""
from __future__ import annotations

import dataclasses
import os

import numpy as np

SEED = 1234


@dataclasses.dataclass(frozen=True)
class KGConfig:
    """One benchmark configuration (entities, relations, triples, model sizes)."""

    index: int
    entities: int
    relations: int          # base relations R; the model sees n = 2R + 1 operators
    train_triples: int      # triples in the training graph (the CSR)
    s_rel: float            # Zipf exponent of relation frequency
    s_tail: float           # Zipf exponent of tail frequency
    head_zipf: float        # 0.0 means uniform heads
    emb: int
    batch_size: int         # --batch_size; a training step has 2 * batch_size queries
    c1: int                 # entity budget per (query, channel); 0 disables top-k
    c2: int                 # fact budget per source (c2 // 2 per direction)
    T: int = 3              # hops (--L in the reference CLI)
    N: int = 3              # channels (--N; the operator's L)
    split_all: int = 0      # config 1 states the total triple count and splits 80/10/10

    @property
    def n(self) -> int:
        return 2 * self.relations + 1

    @property
    def queries(self) -> int:
        return 2 * self.batch_size

    @property
    def use_topk(self) -> bool:
        return self.c1 > 0 or self.c2 > 0


CONFIGS = {
    1: KGConfig(1, 3_000, 12, 22_400, 1.2, 1.0, 0.0, 128, 32, 0, 0, split_all=28_000),
    2: KGConfig(2, 14_500, 237, 272_000, 1.1, 1.0, 1.0, 128, 64, 1000, 400),
    3: KGConfig(3, 123_000, 37, 1_080_000, 1.3, 1.2, 0.0, 256, 128, 1000, 400),
    4: KGConfig(4, 4_600_000, 822, 20_600_000, 1.1, 1.0, 0.0, 1024, 256, 1000, 400),
    5: KGConfig(5, 86_000_000, 14_824, 338_000_000, 1.2, 1.0, 0.0, 1024, 256, 1000, 400),
}


def scaled_config(base: KGConfig, entities: int, relations: int, train_triples: int,
                  batch_size: int | None = None) -> KGConfig:
    """A smaller graph with the same distributions, for tests and CPU baselines."""
    return dataclasses.replace(base, entities=entities, relations=relations,
                               train_triples=train_triples, split_all=0,
                               batch_size=batch_size or base.batch_size)


class _ZipfSampler:
    """Finite Zipf law P(k) ∝ k^-s over k = 1..K, by inverse CDF (float64)."""

    def __init__(self, K: int, s: float):
        ranks = np.arange(1, K + 1, dtype=np.float64)
        cdf = np.cumsum(ranks ** (-s))
        self.cdf = cdf / cdf[-1]

    def __call__(self, u: np.ndarray) -> np.ndarray:
        idx = np.searchsorted(self.cdf, u, side="right")
        return np.minimum(idx, self.cdf.size - 1)


def generate_triples(cfg: KGConfig, seed: int = SEED):
    """Return (train, valid, test) int64 arrays of shape [m, 3] (head, rel, tail)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    E, R = cfg.entities, cfg.relations
    rel_perm = rng.permutation(R)
    tail_perm = rng.permutation(E)
    head_perm = rng.permutation(E)
    rel_zipf = _ZipfSampler(R, cfg.s_rel)
    tail_zipf = _ZipfSampler(E, cfg.s_tail)
    head_zipf = _ZipfSampler(E, cfg.head_zipf) if cfg.head_zipf > 0 else None

    if cfg.split_all:
        total = cfg.split_all
    else:
        total = cfg.train_triples + 2 * (cfg.train_triples // 10)
    # Pack (h, r, t) into one int64 key for duplicate removal when it fits.
    packable = float(E) * R * E < 2.0 ** 62
    keys_seen = np.empty(0, dtype=np.int64)
    chunks = []
    have = 0
    while have < total:
        need = total - have
        draw = int(need * 1.05) + 1024
        r = rel_perm[rel_zipf(rng.random(draw))]
        t = tail_perm[tail_zipf(rng.random(draw))]
        if head_zipf is None:
            h = rng.integers(0, E, size=draw)
        else:
            h = head_perm[head_zipf(rng.random(draw))]
        tri = np.stack([h, r, t], axis=1).astype(np.int64)
        if packable:
            key = (tri[:, 0] * R + tri[:, 1]) * E + tri[:, 2]
            _, first = np.unique(key, return_index=True)
            first.sort()
            tri, key = tri[first], key[first]
            fresh = ~np.isin(key, keys_seen, assume_unique=True)
            tri, key = tri[fresh], key[fresh]
            tri, key = tri[:need], key[:need]
            keys_seen = np.concatenate([keys_seen, key])
        else:
            raise NotImplementedError("graphs whose (h, r, t) key exceeds 62 bits")
        chunks.append(tri)
        have += tri.shape[0]
    triples = np.concatenate(chunks, axis=0)
    if cfg.split_all:
        n_train = int(round(total * 0.8))
        n_valid = int(round(total * 0.1))
    else:
        n_train = cfg.train_triples
        n_valid = cfg.train_triples // 10
    train = triples[:n_train]
    valid = triples[n_train:n_train + n_valid]
    test = triples[n_train + n_valid:]
    return train, valid, test


def generate_triples_device(cfg: KGConfig, seed: int = SEED, device="cuda"):
    """(train, valid, test) int64 [m, 3] tensors on `device`, drawn there.

    For graphs too large for the host generator (config 5: 86M entities,
    14,824 relations, 405.6M triples before the split, whose (h, r, t) key
    needs 68 bits): the same distributions -- relation Zipf(s_rel) over a
    seeded permutation, uniform (or Zipf) heads, tail Zipf(s_tail) over a
    seeded entity permutation, duplicates dropped and redrawn, draw order
    kept -- with torch's device generator seeded by `seed` (a different
    stream from the host generator's, so the graph is its own seeded
    instance).  Duplicates are found by two stable sorts, tail then
    (head, relation)."""
    import torch
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(int(seed))
    E, R = cfg.entities, cfg.relations
    rel_perm = torch.randperm(R, generator=g, device=dev)
    tail_perm = torch.randperm(E, generator=g, device=dev)
    head_perm = torch.randperm(E, generator=g, device=dev)

    def zipf_cdf(K, s):
        c = torch.cumsum(torch.arange(1, K + 1, dtype=torch.float64, device=dev).pow_(-s), 0)
        return c / c[-1]

    rel_cdf = zipf_cdf(R, cfg.s_rel)
    tail_cdf = zipf_cdf(E, cfg.s_tail)
    head_cdf = zipf_cdf(E, cfg.head_zipf) if cfg.head_zipf > 0 else None

    def draw_zipf(cdf, n):
        u = torch.rand(n, generator=g, dtype=torch.float64, device=dev)
        return torch.searchsorted(cdf, u, right=True).clamp_max_(cdf.numel() - 1)

    total = cfg.split_all or cfg.train_triples + 2 * (cfg.train_triples // 10)
    kept = torch.empty((0, 3), dtype=torch.int64, device=dev)
    while kept.shape[0] < total:
        need = total - kept.shape[0]
        draw = int(need * 1.05) + 1024
        r = rel_perm[draw_zipf(rel_cdf, draw)]
        t = tail_perm[draw_zipf(tail_cdf, draw)]
        h = (torch.randint(0, E, (draw,), generator=g, device=dev) if head_cdf is None
             else head_perm[draw_zipf(head_cdf, draw)])
        cand = torch.cat([kept, torch.stack([h, r, t], 1)])
        del h, r, t
        # lexicographic order of (h * R + r, t), draw order among equals
        o = torch.sort(cand[:, 2], stable=True)[1]
        hr = cand[:, 0] * R + cand[:, 1]
        o = o[torch.sort(hr[o], stable=True)[1]]
        hr_s, t_s = hr[o], cand[o, 2]
        first = torch.ones(o.numel(), dtype=torch.bool, device=dev)
        first[1:] = (hr_s[1:] != hr_s[:-1]) | (t_s[1:] != t_s[:-1])
        keep_idx = torch.sort(o[first])[0]  # first occurrences, in draw order
        del o, hr, hr_s, t_s, first
        kept = cand[keep_idx[:total]]
        del cand, keep_idx
    n_train = cfg.train_triples if not cfg.split_all else int(round(total * 0.8))
    n_valid = cfg.train_triples // 10 if not cfg.split_all else int(round(total * 0.1))
    return kept[:n_train], kept[n_train:n_train + n_valid], kept[n_train + n_valid:]


def host_generation_fits(cfg: KGConfig) -> bool:
    """Whether generate_triples handles cfg (its duplicate key needs E * R * E < 2^62)."""
    return float(cfg.entities) * cfg.relations * cfg.entities < 2.0 ** 62


def load_or_generate(cfg: KGConfig, seed: int = SEED, cache_dir: str | None = None):
    """Generate the graph once and cache it as .npy under ``cache_dir``."""
    cache_dir = cache_dir or os.environ.get(
        "FLASHLOG_B200_CACHE", os.path.join(os.path.dirname(os.path.dirname(__file__)), ".cache"))
    tag = f"kg_e{cfg.entities}_r{cfg.relations}_m{cfg.train_triples}_s{seed}_{cfg.s_rel}_{cfg.s_tail}_{cfg.head_zipf}_{cfg.split_all}"
    path = os.path.join(cache_dir, tag + ".npz")
    if os.path.exists(path):
        data = np.load(path)
        return data["train"], data["valid"], data["test"]
    train, valid, test = generate_triples(cfg, seed)
    os.makedirs(cache_dir, exist_ok=True)
    tmp = path + f".tmp{os.getpid()}.npz"
    np.savez(tmp, train=train, valid=valid, test=test)
    os.replace(tmp, path)
    return train, valid, test


def load_graph(cfg: KGConfig, device, seed: int = SEED):
    """The training triples as (host int64 [m, 3] array, device tensor).

    Configs the host generator handles come from load_or_generate (cached);
    larger ones (config 5) are drawn on the device by generate_triples_device
    and copied to the host once."""
    import torch
    if host_generation_fits(cfg):
        train, _, _ = load_or_generate(cfg, seed)
        return train, torch.from_numpy(train).to(device)
    train_dev, valid, test = generate_triples_device(cfg, seed, device)
    del valid, test
    return train_dev.cpu().numpy(), train_dev


def training_queries(train: np.ndarray, cfg: KGConfig, step: int = 0, seed: int = SEED):
    """One training batch as in ``batch_iter``: B/2 triples give 2 queries each.

    Returns (triple_ids, heads, relations, tails) with 2 * batch_size queries
    ordered (h, r, t), (t, r + R, h) per sampled triple.
    """
    rng = np.random.Generator(np.random.PCG64([seed, step]))
    ids = rng.choice(train.shape[0], size=cfg.batch_size, replace=False)
    h, r, t = train[ids, 0], train[ids, 1], train[ids, 2]
    heads = np.stack([h, t], axis=1).reshape(-1)
    rels = np.stack([r, r + cfg.relations], axis=1).reshape(-1)
    tails = np.stack([t, h], axis=1).reshape(-1)
    return ids.astype(np.int64), heads.astype(np.int64), rels.astype(np.int64), tails.astype(np.int64)


def random_attention(queries: int, T: int, N: int, n: int, seed: int = SEED, std: float = 1.0):
    """Kernel-level stand-in for the LSTM attention: w_t = softmax(N(0, std^2))."""
    rng = np.random.Generator(np.random.PCG64([seed, 7]))
    logits = rng.standard_normal((queries, T, N, n)).astype(np.float32) * np.float32(std)
    logits -= logits.max(axis=-1, keepdims=True)
    e = np.exp(logits)
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


def evaluation_queries(test: np.ndarray, relations: int, max_triples: int | None = None):
    """Test queries as in rules/evaluate.py:122-128: every triple (h, r, t)
    gives (h, r, t) and (t, r + R, h).  Returns (sources, relations, targets)."""
    test = test if max_triples is None else test[:max_triples]
    h, r, t = test[:, 0], test[:, 1], test[:, 2]
    src = np.stack([h, t], 1).reshape(-1).astype(np.int64)
    rel = np.stack([r, r + relations], 1).reshape(-1).astype(np.int64)
    dst = np.stack([t, h], 1).reshape(-1).astype(np.int64)
    return src, rel, dst


def rule_bank(train: np.ndarray, query_relations: np.ndarray, relations: int, n_rules: int = 50_000,
              seed: int = SEED, uniform_ops: bool = False, groups: int = 3):
    """A seeded Horn-rule bank in the reference's rule format (rules/evaluate.py:63-92).

    Heads are drawn in proportion to the frequency of the query relations;
    body lengths are uniform on {1, 2, 3}; body operators are directed
    relations (r forward, r + R inverse) drawn in proportion to their edge
    counts in the training graph, so bodies ground (uniform over the 2R
    operators with uniform_ops); weights ~ U(0, 1); group_id ~ U{0, 1, 2}.
    Each rule is a dict with rule_id, head, body (tuple), weight, group_id
    and rank_weights None, as load_rules returns."""
    rng = np.random.Generator(np.random.PCG64([seed, 11]))
    R = relations
    head_freq = np.bincount(np.asarray(query_relations, np.int64), minlength=2 * R).astype(np.float64)
    heads = rng.choice(2 * R, size=n_rules, p=head_freq / head_freq.sum())
    lengths = rng.integers(1, 4, size=n_rules)
    if uniform_ops:
        op_p = np.full(2 * R, 1.0 / (2 * R))
    else:
        edge = np.bincount(np.asarray(train[:, 1], np.int64), minlength=R).astype(np.float64)
        op_p = np.concatenate([edge, edge])
        op_p /= op_p.sum()
    ops_ = rng.choice(2 * R, size=(n_rules, 3), p=op_p)
    weights = rng.random(n_rules)
    group = rng.integers(0, groups, size=n_rules)
    # a (head, body, group) instance appears once (rules/evaluate.py:110-111
    # rejects duplicates); later draws of the same instance are dropped
    seen, out = set(), []
    for k in range(n_rules):
        body = tuple(int(o) for o in ops_[k, :lengths[k]])
        key = (int(heads[k]), body, int(group[k]))
        if key in seen:
            continue
        seen.add(key)
        out.append({"rule_id": len(out), "head": key[0], "body": body, "weight": float(weights[k]),
                    "rank_weights": None, "group_id": key[2]})
    return out


def write_rules_tsv(path: str, rules) -> None:
    """The rule TSV read by rules/evaluate.py:63-92 (head_id, body_ids, weight, group_id)."""
    with open(path, "w") as f:
        f.write("head_id\tbody_ids\tweight\tgroup_id\n")
        for r in rules:
            f.write(f"{r['head']}\t{' '.join(str(o) for o in r['body'])}\t{r['weight']!r}\t{r['group_id']}\n")
