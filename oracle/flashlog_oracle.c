/*
 * flashlog_oracle.c -- CPU restatement of FlashLog's soft-grounding hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library in flashlog_b200/csrc.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py may load it; the product never
 * calls it and has no CPU fallback.
 *
 * Every routine restates the reference algorithm (paths relative to the
 * reference project root) in plain single-threaded C with a fixed summation
 * order, so the results are deterministic:
 *
 *   flo_build_side        flashlog_kernel/source/csr.cpp:12-69
 *   flo_group_threshold   flashlog_kernel/source/flashlog.cpp:13-35
 *                         (GPU twin flashlog.cu:26-63, 1342-1366)
 *   flo_topc              flashlog_kernel/flashlog_kernel.py:1092-1137
 *   flo_hop_forward       flashlog_kernel/source/flashlog.cpp:506-578, 706-989,
 *                         1231-1610 (CPU) and flashlog.cu:1402-1559,
 *                         1743-1854 (CUDA fill semantics), coalesce
 *                         flashlog_kernel.py:258-357
 *   flo_hop_backward      flashlog_kernel/source/flashlog.cpp:991-1134
 *   flo_normalize_*       flashlog_kernel/flashlog_kernel.py:536-607,
 *                         flashlog.cu:2480-2691, flashlog.cpp:1136-1230
 *   flo_fixed_relation    flashlog.cu:1561-1741 + flashlog_kernel.py:182-210
 *   flo_filtered_ranks    flashlog.cu:2754-2910
 *   flo_sample_quota      flashlog.cu:1458-1528
 *
 * Parity is pinned against the reference's own CPU extension compiled from
 * its sources (oracle/build_ref.py) and against committed golden vectors
 * (tests/golden).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>

#define FLO_EXPORT __attribute__((visibility("default")))

/* ---------------------------------------------------------------------- */
/* CSR build: two stable counting passes, relation first then source.      */
/* csr.cpp:12-69.  Returns the number of groups, or -1 on invalid input.   */
/* group arrays must have room for `edges` entries.                        */
/* ---------------------------------------------------------------------- */
FLO_EXPORT int64_t flo_build_side(int64_t edges, const int64_t *s, const int64_t *t,
                                  const int64_t *r, int64_t nodes,
                                  int32_t *row_ptr, int32_t *columns, int16_t *edge_rel,
                                  int32_t *order, int32_t *group_ptr, int16_t *group_rel,
                                  int32_t *group_start, int32_t *group_count) {
    if (nodes < 0 || nodes > INT32_MAX || edges > INT32_MAX) return -1;
    int64_t relations = 0;
    for (int64_t i = 0; i < edges; ++i) {
        if (s[i] < 0 || s[i] >= nodes || t[i] < 0 || t[i] >= nodes || r[i] < 0 || r[i] > INT16_MAX)
            return -1;
        if (r[i] + 1 > relations) relations = r[i] + 1;
    }
    int64_t ncur = nodes > relations ? nodes : relations;
    int64_t *cursor = (int64_t *)calloc((size_t)(ncur > 0 ? ncur : 1), sizeof(int64_t));
    int32_t *tmp = (int32_t *)malloc((size_t)(edges > 0 ? edges : 1) * sizeof(int32_t));
    for (int64_t i = 0; i < edges; ++i) ++cursor[r[i]];
    int64_t off = 0;
    for (int64_t i = 0; i < relations; ++i) { int64_t c = cursor[i]; cursor[i] = off; off += c; }
    for (int64_t i = 0; i < edges; ++i) tmp[cursor[r[i]]++] = (int32_t)i;
    memset(cursor, 0, (size_t)ncur * sizeof(int64_t));
    for (int64_t i = 0; i < edges; ++i) ++cursor[s[i]];
    off = 0;
    for (int64_t i = 0; i < nodes; ++i) { int64_t c = cursor[i]; row_ptr[i] = (int32_t)off; cursor[i] = off; off += c; }
    row_ptr[nodes] = (int32_t)edges;
    for (int64_t k = 0; k < edges; ++k) { int32_t i = tmp[k]; order[cursor[s[i]]++] = i; }
    memset(group_ptr, 0, (size_t)(nodes + 1) * sizeof(int32_t));
    int64_t g = -1;
    for (int64_t j = 0; j < edges; ++j) {
        int64_t i = order[j];
        columns[j] = (int32_t)t[i];
        edge_rel[j] = (int16_t)r[i];
        if (j == 0 || s[i] != s[order[j - 1]] || r[i] != r[order[j - 1]]) {
            if (g >= 0) group_count[g] = (int32_t)(j - group_start[g]);
            ++g;
            group_start[g] = (int32_t)j;
            group_rel[g] = (int16_t)r[i];
            ++group_ptr[s[i] + 1];
        }
    }
    if (g >= 0) group_count[g] = (int32_t)(edges - group_start[g]);
    for (int64_t i = 0; i < nodes; ++i) group_ptr[i + 1] += group_ptr[i];
    free(cursor);
    free(tmp);
    return g + 1;
}

/* ---------------------------------------------------------------------- */
/* c2: weighted order statistic over relation groups (flashlog.cpp:13-35). */
/* Returns the threshold weight, or -1 when everything fits the budget;    */
/* *remaining is the number of edges kept at the threshold weight.         */
/* ---------------------------------------------------------------------- */
typedef struct { float w; int32_t c; } flo_wc;

static int flo_wc_desc(const void *a, const void *b) {
    float x = ((const flo_wc *)a)->w, y = ((const flo_wc *)b)->w;
    return (x < y) - (x > y);
}

FLO_EXPORT float flo_group_threshold(const float *w_dir, const int16_t *grel, const int32_t *gcount,
                                     int64_t g0, int64_t g1, int64_t budget, int64_t *remaining) {
    int64_t total = 0, m = 0;
    flo_wc *buf = (flo_wc *)malloc((size_t)((g1 - g0) > 0 ? (g1 - g0) : 1) * sizeof(flo_wc));
    for (int64_t g = g0; g < g1; ++g) {
        float sc = w_dir[grel[g]];
        if (sc > 0.0f) { buf[m].w = sc; buf[m].c = gcount[g]; ++m; total += gcount[g]; }
    }
    *remaining = 0;
    if (total <= budget) { free(buf); return -1.0f; }
    /* Only the order of distinct weights matters for the result. */
    qsort(buf, (size_t)m, sizeof(flo_wc), flo_wc_desc);
    int64_t consumed = 0, higher = 0;
    float prev = -1.0f;
    for (int64_t i = 0; i < m; ++i) {
        if (buf[i].w != prev) { higher = consumed; prev = buf[i].w; }
        if (consumed + buf[i].c >= budget) { *remaining = budget - higher; float res = buf[i].w; free(buf); return res; }
        consumed += buf[i].c;
    }
    free(buf);
    return -1.0f;
}

/* Per-group take under a threshold (flashlog.cpp:62-79, flashlog.cu:1342-1366). */
static int32_t flo_take(float w, int32_t count, float thr, int64_t keep_thr, int64_t *seen, int skip_nonpos) {
    int32_t take = (!skip_nonpos || w > 0.0f) ? count : 0;
    if (take > 0 && thr >= 0.0f) {
        if (w < thr) take = 0;
        else if (w == thr) {
            int64_t left = keep_thr - *seen;
            take = left > 0 ? (int32_t)(left < count ? left : count) : 0;
            *seen += take;
        }
    }
    return take;
}

/* ---------------------------------------------------------------------- */
/* SplitMix64 rounding phase and weighted quotas of the sampled c2 path.   */
/* flashlog.cu:1458-1528.  take[g - g0] receives each group's quota.       */
/* ---------------------------------------------------------------------- */
FLO_EXPORT double flo_sampling_phase(int64_t seed, int64_t b, int64_t l, int64_t src, int is_inv) {
    uint64_t z = (uint64_t)seed ^ ((uint64_t)b * 0x9e3779b97f4a7c15ULL)
               ^ ((uint64_t)l * 0xbf58476d1ce4e5b9ULL) ^ ((uint64_t)src * 0x94d049bb133111ebULL)
               ^ (is_inv ? 0xd1b54a32d192ed03ULL : 0x8cb92baa3f3d8dd7ULL);
    z += 0x9e3779b97f4a7c15ULL;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    z ^= z >> 31;
    return (double)(z >> 11) * 0x1.0p-53;
}

FLO_EXPORT void flo_sample_quota(const float *w_dir, const int16_t *grel, const int32_t *gcount,
                                 int64_t g0, int64_t g1, int64_t budget, double phase, int32_t *take) {
    int64_t capacity = 0;
    double wsum = 0.0;
    for (int64_t g = g0; g < g1; ++g) {
        double wt = w_dir[grel[g]];
        if (wt > 0 && gcount[g] > 0) { capacity += gcount[g]; wsum += wt; }
    }
    int64_t target = budget < capacity ? budget : capacity;
    int64_t allocated = capacity;
    if (target < capacity) {
        allocated = 0;
        for (int64_t g = g0; g < g1; ++g) {
            double wt = w_dir[grel[g]];
            int64_t c = gcount[g];
            if (wt > 0 && c > 0) allocated += (int64_t)fmin((double)c, floor((double)target * wt / wsum));
        }
    }
    int64_t residual = target - allocated, spare_total = capacity - allocated;
    int64_t left = residual, cap_left = spare_total, prefix = 0;
    for (int64_t g = g0; g < g1; ++g) {
        float sc = w_dir[grel[g]];
        int32_t c = gcount[g];
        int64_t cur = sc > 0.0f ? c : 0;
        if (cur > 0 && spare_total > 0) {
            int64_t base = (int64_t)fmin((double)c, floor((double)target * (double)sc / wsum));
            int64_t spare = (int64_t)c - base;
            prefix += spare;
            cap_left -= spare;
            int64_t cumulative = prefix == spare_total ? residual
                : (int64_t)floor((double)residual * (double)prefix / (double)spare_total + phase);
            int64_t extra = cumulative - (residual - left);
            int64_t lim = spare < left ? spare : left;
            if (extra > lim) extra = lim;
            if (extra < 0) extra = 0;
            if (extra < left - cap_left) extra = left - cap_left;
            left -= extra;
            cur = base + extra;
        }
        take[g - g0] = (int32_t)cur;
    }
}

/* ---------------------------------------------------------------------- */
/* c1: keep the c1 largest nonzero values per (item, channel) row of a     */
/* coalesced state; ties keep the lower entity (stable descending sort).   */
/* Rows with <= c1 nonzeros are untouched (zeros included); rows above     */
/* keep only the selected nonzeros.  flashlog_kernel.py:1092-1137.         */
/* Returns the number of kept entries, or -1 when nothing is pruned.       */
/* ---------------------------------------------------------------------- */
typedef struct { float v; int64_t i; } flo_vi;

static int flo_vi_desc(const void *a, const void *b) {
    const flo_vi *x = (const flo_vi *)a, *y = (const flo_vi *)b;
    if (x->v > y->v) return -1;
    if (x->v < y->v) return 1;
    return (x->i > y->i) - (x->i < y->i);
}

FLO_EXPORT int64_t flo_topc(int64_t nnz, const int64_t *row, const float *val, int64_t c1,
                            uint8_t *keep) {
    if (nnz <= c1) return -1;
    int any_over = 0;
    int64_t kept = 0;
    flo_vi *buf = (flo_vi *)malloc((size_t)(nnz > 0 ? nnz : 1) * sizeof(flo_vi));
    for (int64_t s = 0; s < nnz;) {
        int64_t e = s;
        int64_t nz = 0;
        while (e < nnz && row[e] == row[s]) { if (val[e] != 0.0f) ++nz; ++e; }
        if (nz <= c1) {
            for (int64_t i = s; i < e; ++i) keep[i] = 1;
        } else {
            any_over = 1;
            int64_t m = 0;
            for (int64_t i = s; i < e; ++i) {
                keep[i] = 0;
                if (val[i] != 0.0f) { buf[m].v = val[i]; buf[m].i = i; ++m; }
            }
            qsort(buf, (size_t)m, sizeof(flo_vi), flo_vi_desc);
            for (int64_t k = 0; k < c1 && k < m; ++k) keep[buf[k].i] = 1;
        }
        s = e;
    }
    free(buf);
    if (!any_over) return -1;
    for (int64_t i = 0; i < nnz; ++i) kept += keep[i];
    return kept;
}

/* ---------------------------------------------------------------------- */
/* One propagation hop: expansion + coalesce-sum (+ optional normalize).   */
/* ---------------------------------------------------------------------- */
typedef struct {
    const int32_t *col, *order, *gptr, *gstart, *gcount;
    const int16_t *grel;
} flo_side;

enum {
    FLO_SKIP_NONPOS_W = 1,   /* groups with w <= 0 take nothing (top-k / CPU paths)     */
    FLO_DROP_MASKED = 2,     /* facts with m == 0 are not emitted (top-k / CPU paths)   */
    FLO_MASK_BY_TRIPLE = 4,  /* mask indexed by triple id via order[p] (top-k CUDA path) */
    FLO_WOT_I = 8,           /* no identity term                                        */
    FLO_SAMPLED = 16,        /* c2 by weighted quotas with a SplitMix64 phase            */
    FLO_EDGE_SCORE = 32,     /* edge_weight already holds scores (no sigmoid)            */
    FLO_EDGE_POS = 1024      /* fact_edge records the CSR position p, not order[p]       */
};

typedef struct { float *acc; int64_t *mark; int64_t *touched; int64_t ntouched; int64_t *pos; } flo_row_acc;

static int flo_i64_cmp(const void *a, const void *b) {
    int64_t x = *(const int64_t *)a, y = *(const int64_t *)b;
    return (x > y) - (x < y);
}

/*
 * sp_row[i] = b * L + l of entry i (entries sorted by (row, entity)),
 * sp_ent[i], sp_val[i]; w is [rows, n].
 * mask: CSR-ordered float per side (mask_ori / mask_inv) unless
 * FLO_MASK_BY_TRIPLE, in which case mask_triple[order[p]] (nonzero = visible)
 * and optional edge_weight[order[p]] (sigmoid unless FLO_EDGE_SCORE).
 * Outputs (capacity checked by the caller): out_key[u] = row * E + e sorted,
 * out_val[u] (pre-normalization sums), and per-fact provenance in emission
 * order: fact_entry, fact_rel (relation column in w, i.e. rel + offset),
 * fact_m, fact_out (output position).  Identity facts use rel = n - 1, m = 1.
 * Returns the number of outputs; *n_facts receives the number of facts.
 */
/* fact_edge (with fact_entry, may be NULL): triple id of each graph fact
 * (order[p]) and 0 for identity facts: the tie key of the MAX coalesce
 * (flashlog_kernel.py:399-478, meta_edge of flashlog.cu:1539-1557). */
FLO_EXPORT int64_t flo_hop_forward_edges(
    int64_t nnz, const int64_t *sp_row, const int64_t *sp_ent, const float *sp_val,
    const float *w, int64_t L, int64_t n, int64_t E, int64_t r_size,
    const int32_t *ori_col, const int32_t *ori_order, const int32_t *ori_gptr,
    const int16_t *ori_grel, const int32_t *ori_gstart, const int32_t *ori_gcount,
    const int32_t *inv_col, const int32_t *inv_order, const int32_t *inv_gptr,
    const int16_t *inv_grel, const int32_t *inv_gstart, const int32_t *inv_gcount,
    const float *mask_ori, const float *mask_inv, const uint8_t *mask_triple,
    const float *edge_weight, int64_t topk_edges, int64_t flags, int64_t sampling_seed,
    int64_t *out_key, float *out_val, int64_t *fact_entry, int32_t *fact_rel,
    float *fact_m, int64_t *fact_out, int64_t *fact_edge, int64_t *n_facts) {
    flo_side sides[2] = {
        {ori_col, ori_order, ori_gptr, ori_gstart, ori_gcount, ori_grel},
        {inv_col, inv_order, inv_gptr, inv_gstart, inv_gcount, inv_grel}};
    const float *csr_mask[2] = {mask_ori, mask_inv};
    float *acc = (float *)calloc((size_t)E, sizeof(float));
    int64_t *mark = (int64_t *)malloc((size_t)E * sizeof(int64_t));
    int64_t *slot = (int64_t *)malloc((size_t)E * sizeof(int64_t));
    for (int64_t e = 0; e < E; ++e) mark[e] = -1;
    int64_t cap_touched = 1024, ntouch = 0;
    int64_t *touched = (int64_t *)malloc((size_t)cap_touched * sizeof(int64_t));
    int32_t *take_buf = NULL;
    int64_t take_cap = 0;
    int64_t nf = 0, nu = 0;
    int64_t row_fact_begin = 0;
    const int skip_nonpos = (flags & FLO_SKIP_NONPOS_W) != 0;
    for (int64_t s = 0; s < nnz;) {
        int64_t row = sp_row[s];
        int64_t e_end = s;
        while (e_end < nnz && sp_row[e_end] == row) ++e_end;
        ntouch = 0;
        row_fact_begin = nf;
        const float *w_row = w + row * n;
#define FLO_ADD(dst, value, ent_i, relc, mval, edge_id)                          \
        do {                                                                      \
            int64_t d_ = (dst);                                                   \
            if (mark[d_] != row) {                                                \
                mark[d_] = row; acc[d_] = 0.0f;                                   \
                if (ntouch == cap_touched) {                                      \
                    cap_touched *= 2;                                             \
                    touched = (int64_t *)realloc(touched, (size_t)cap_touched * sizeof(int64_t)); \
                }                                                                 \
                touched[ntouch++] = d_;                                           \
            }                                                                     \
            acc[d_] += (value);                                                   \
            if (fact_entry) { fact_entry[nf] = (ent_i); fact_rel[nf] = (int32_t)(relc); \
                              fact_m[nf] = (mval); fact_out[nf] = d_;             \
                              if (fact_edge) fact_edge[nf] = (edge_id); }         \
            ++nf;                                                                 \
        } while (0)
        for (int64_t i = s; i < e_end; ++i) {
            int64_t src = sp_ent[i];
            float sv = sp_val[i];
            for (int dir = 0; dir < 2; ++dir) {
                const flo_side *sd = &sides[dir];
                int64_t off = dir ? r_size : 0;
                int64_t g0 = sd->gptr[src], g1 = sd->gptr[src + 1];
                if (g0 == g1) continue;
                const float *w_dir = w_row + off;
                int64_t keep_thr = 0, seen = 0;
                float thr = -1.0f;
                if (flags & FLO_SAMPLED) {
                    if (take_cap < g1 - g0) { take_cap = g1 - g0; take_buf = (int32_t *)realloc(take_buf, (size_t)take_cap * sizeof(int32_t)); }
                    flo_sample_quota(w_dir, sd->grel, sd->gcount, g0, g1, topk_edges,
                                     flo_sampling_phase(sampling_seed, row / L, row % L, src, dir),
                                     take_buf);
                } else if (skip_nonpos) {
                    thr = flo_group_threshold(w_dir, sd->grel, sd->gcount, g0, g1, topk_edges, &keep_thr);
                }
                for (int64_t g = g0; g < g1; ++g) {
                    int64_t rel = sd->grel[g];
                    float wv = w_dir[rel];
                    int32_t take;
                    if (flags & FLO_SAMPLED) take = take_buf[g - g0];
                    else take = flo_take(wv, sd->gcount[g], thr, keep_thr, &seen, skip_nonpos);
                    if (take <= 0) continue;
                    int64_t p0 = sd->gstart[g];
                    float prod = sv * wv;
                    for (int64_t p = p0; p < p0 + take; ++p) {
                        float m;
                        if (flags & FLO_MASK_BY_TRIPLE) {
                            int64_t edge = sd->order[p];
                            m = mask_triple[edge] ? 1.0f : 0.0f;
                            if (edge_weight) {
                                float ew = edge_weight[edge];
                                m *= (flags & FLO_EDGE_SCORE) ? ew : 1.0f / (1.0f + expf(-ew));
                            }
                            if ((flags & FLO_DROP_MASKED) && !mask_triple[edge]) continue;
                        } else {
                            m = csr_mask[dir][p];
                            if ((flags & FLO_DROP_MASKED) && m == 0.0f) continue;
                        }
                        FLO_ADD(sd->col[p], prod * m, i, rel + off, m,
                                (flags & FLO_EDGE_POS) ? p : (int64_t)sd->order[p]);
                    }
                }
            }
            if (!(flags & FLO_WOT_I)) FLO_ADD(src, sv * w_row[n - 1], i, n - 1, 1.0f, (int64_t)0);
        }
#undef FLO_ADD
        qsort(touched, (size_t)ntouch, sizeof(int64_t), flo_i64_cmp);
        for (int64_t k = 0; k < ntouch; ++k) {
            int64_t d = touched[k];
            slot[d] = nu + k;
            out_key[nu + k] = row * E + d;
            out_val[nu + k] = acc[d];
        }
        if (fact_entry)
            for (int64_t f = row_fact_begin; f < nf; ++f) fact_out[f] = slot[fact_out[f]];
        nu += ntouch;
        s = e_end;
    }
    free(acc); free(mark); free(slot); free(touched); free(take_buf);
    *n_facts = nf;
    return nu;
}

FLO_EXPORT int64_t flo_hop_forward(
    int64_t nnz, const int64_t *sp_row, const int64_t *sp_ent, const float *sp_val,
    const float *w, int64_t L, int64_t n, int64_t E, int64_t r_size,
    const int32_t *ori_col, const int32_t *ori_order, const int32_t *ori_gptr,
    const int16_t *ori_grel, const int32_t *ori_gstart, const int32_t *ori_gcount,
    const int32_t *inv_col, const int32_t *inv_order, const int32_t *inv_gptr,
    const int16_t *inv_grel, const int32_t *inv_gstart, const int32_t *inv_gcount,
    const float *mask_ori, const float *mask_inv, const uint8_t *mask_triple,
    const float *edge_weight, int64_t topk_edges, int64_t flags, int64_t sampling_seed,
    int64_t *out_key, float *out_val, int64_t *fact_entry, int32_t *fact_rel,
    float *fact_m, int64_t *fact_out, int64_t *n_facts) {
    return flo_hop_forward_edges(nnz, sp_row, sp_ent, sp_val, w, L, n, E, r_size, ori_col, ori_order, ori_gptr,
                                 ori_grel, ori_gstart, ori_gcount, inv_col, inv_order, inv_gptr, inv_grel, inv_gstart,
                                 inv_gcount, mask_ori, mask_inv, mask_triple, edge_weight, topk_edges, flags,
                                 sampling_seed, out_key, out_val, fact_entry, fact_rel, fact_m, fact_out, NULL,
                                 n_facts);
}

/* Upper bound on facts for flo_hop_forward (degree sum + identity). */
FLO_EXPORT int64_t flo_fact_bound(int64_t nnz, const int64_t *sp_ent, const int32_t *ori_rowptr,
                                  const int32_t *inv_rowptr) {
    int64_t f = nnz;
    for (int64_t i = 0; i < nnz; ++i) {
        int64_t e = sp_ent[i];
        f += (int64_t)(ori_rowptr[e + 1] - ori_rowptr[e]) + (int64_t)(inv_rowptr[e + 1] - inv_rowptr[e]);
    }
    return f;
}

/* Sampled variant needs (b, l) for the SplitMix64 phase; rows = b * L + l. */
FLO_EXPORT void flo_sampled_takes(const float *w_dir, const int16_t *grel, const int32_t *gcount,
                                  int64_t g0, int64_t g1, int64_t budget, int64_t seed,
                                  int64_t b, int64_t l, int64_t src, int is_inv, int32_t *take) {
    flo_sample_quota(w_dir, grel, gcount, g0, g1, budget,
                     flo_sampling_phase(seed, b, l, src, is_inv), take);
}

/* ---------------------------------------------------------------------- */
/* Backward of one hop from the recorded facts (flashlog.cpp:991-1134).    */
/* g_out[u] is the gradient of output u; the loops follow the reference's  */
/* single-thread order: all graph facts in emission order, identity facts  */
/* included where they were emitted.                                       */
/* ---------------------------------------------------------------------- */
FLO_EXPORT void flo_hop_backward(int64_t n_facts, const int64_t *fact_entry, const int32_t *fact_rel,
                                 const float *fact_m, const int64_t *fact_out, const float *g_out,
                                 int64_t nnz, const int64_t *sp_row, const float *sp_val,
                                 const float *w, int64_t n, int64_t r_size, float *grad_v, float *grad_w) {
    memset(grad_v, 0, (size_t)nnz * sizeof(float));
    /* Three passes as in the reference: ori facts, inv facts, identity. */
    for (int pass = 0; pass < 3; ++pass) {
        int64_t lo = pass == 0 ? 0 : (pass == 1 ? r_size : n - 1);
        int64_t hi = pass == 0 ? r_size : (pass == 1 ? 2 * r_size : n);
        for (int64_t f = 0; f < n_facts; ++f) {
            int64_t c = fact_rel[f];
            if (c < lo || c >= hi) continue;
            if (fact_out[f] < 0) continue;  /* a losing fact of a MAX coalesce */
            float g = g_out[fact_out[f]];
            if (g == 0.0f) continue;
            int64_t i = fact_entry[f];
            int64_t row = sp_row[i];
            float m = fact_m[f];
            grad_v[i] += g * w[row * n + c] * m;
            grad_w[row * n + c] += g * sp_val[i] * m;
        }
    }
}

/* ---------------------------------------------------------------------- */
/* Row normalization (flashlog_kernel.py:550-559 forward, flashlog.cpp:     */
/* 1136-1230 backward).  rows of key / E give the (b, l) row of each value. */
/* ---------------------------------------------------------------------- */
FLO_EXPORT void flo_normalize_forward(int64_t u, const int64_t *out_row, const float *x, int64_t rows,
                                      float eps, float *denom, float *y) {
    memset(denom, 0, (size_t)rows * sizeof(float));
    for (int64_t k = 0; k < u; ++k) denom[out_row[k]] += x[k];
    for (int64_t k = 0; k < u; ++k) {
        float d = denom[out_row[k]];
        y[k] = x[k] / (d > eps ? d : eps);
    }
}

FLO_EXPORT void flo_normalize_backward(int64_t u, const int64_t *out_row, const float *x,
                                       const float *denom, const float *g, int64_t rows, float eps,
                                       float *gx) {
    float *sgx = (float *)calloc((size_t)(rows > 0 ? rows : 1), sizeof(float));
    for (int64_t k = 0; k < u; ++k) sgx[out_row[k]] += g[k] * x[k];
    for (int64_t k = 0; k < u; ++k) {
        float d0 = denom[out_row[k]];
        float d = d0 > eps ? d0 : eps;
        float v = g[k] / d;
        if (d0 >= eps) v -= sgx[out_row[k]] / (d * d);
        gx[k] = v;
    }
    free(sgx);
}

/* ---------------------------------------------------------------------- */
/* Rule step: one fixed operator per (query, rule) row, identity at 2R.    */
/* flashlog.cu:1561-1675; the caller coalesces (sum) the emitted facts.    */
/* Returns the number of emitted facts (capacity `cap`).                   */
/* ---------------------------------------------------------------------- */
static int64_t flo_find_group(const int32_t *gptr, const int16_t *grel, int64_t src, int relation) {
    int64_t lo = gptr[src], hi = gptr[src + 1];
    while (lo < hi) {
        int64_t mid = lo + (hi - lo) / 2;
        if ((int)grel[mid] < relation) lo = mid + 1; else hi = mid;
    }
    if (lo < gptr[src + 1] && (int)grel[lo] == relation) return lo;
    return -1;
}

FLO_EXPORT int64_t flo_fixed_relation(int64_t nnz, const int64_t *sp_b, const int64_t *sp_l,
                                      const int64_t *sp_e, const float *sp_v, const int64_t *ops,
                                      int64_t L, int64_t r_size,
                                      const int32_t *ori_col, const int32_t *ori_gptr,
                                      const int16_t *ori_grel, const int32_t *ori_gstart,
                                      const int32_t *ori_gcount,
                                      const int32_t *inv_col, const int32_t *inv_gptr,
                                      const int16_t *inv_grel, const int32_t *inv_gstart,
                                      const int32_t *inv_gcount,
                                      int64_t cap, int64_t *ob, int64_t *ol, int64_t *oe, float *ov) {
    int64_t nf = 0;
    for (int64_t i = 0; i < nnz; ++i) {
        int64_t op = ops[sp_b[i] * L + sp_l[i]];
        if (op == 2 * r_size) {
            if (nf < cap) { ob[nf] = sp_b[i]; ol[nf] = sp_l[i]; oe[nf] = sp_e[i]; ov[nf] = sp_v[i]; }
            ++nf;
            continue;
        }
        int inv = op >= r_size;
        int rel = (int)(inv ? op - r_size : op);
        int64_t g = inv ? flo_find_group(inv_gptr, inv_grel, sp_e[i], rel)
                        : flo_find_group(ori_gptr, ori_grel, sp_e[i], rel);
        if (g < 0) continue;
        int64_t p0 = inv ? inv_gstart[g] : ori_gstart[g];
        int64_t c = inv ? inv_gcount[g] : ori_gcount[g];
        const int32_t *col = inv ? inv_col : ori_col;
        for (int64_t p = p0; p < p0 + c; ++p) {
            if (nf < cap) { ob[nf] = sp_b[i]; ol[nf] = sp_l[i]; oe[nf] = col[p]; ov[nf] = sp_v[i]; }
            ++nf;
        }
    }
    return nf;
}

/* Coalesce (sum) raw COO facts in emission order per key (flashlog.cpp:408-494). */
typedef struct { int64_t k; int64_t i; } flo_ki;
static int flo_ki_cmp(const void *a, const void *b) {
    const flo_ki *x = (const flo_ki *)a, *y = (const flo_ki *)b;
    if (x->k != y->k) return (x->k > y->k) - (x->k < y->k);
    return (x->i > y->i) - (x->i < y->i);
}

FLO_EXPORT int64_t flo_coalesce_sum(int64_t m, const int64_t *keys, const float *vals,
                                    int64_t *out_keys, float *out_vals) {
    flo_ki *buf = (flo_ki *)malloc((size_t)(m > 0 ? m : 1) * sizeof(flo_ki));
    for (int64_t i = 0; i < m; ++i) { buf[i].k = keys[i]; buf[i].i = i; }
    qsort(buf, (size_t)m, sizeof(flo_ki), flo_ki_cmp);
    int64_t u = 0;
    for (int64_t j = 0; j < m; ++j) {
        if (u > 0 && out_keys[u - 1] == buf[j].k) out_vals[u - 1] += vals[buf[j].i];
        else { out_keys[u] = buf[j].k; out_vals[u] = vals[buf[j].i]; ++u; }
    }
    free(buf);
    return u;
}

/* ---------------------------------------------------------------------- */
/* Filtered, tie-averaged ranks (flashlog.cu:2754-2910).                   */
/* filter_keys (b * E + e) must be sorted ascending.                       */
/* ---------------------------------------------------------------------- */
static int flo_bsearch64(const int64_t *keys, int64_t n, int64_t key) {
    int64_t lo = 0, hi = n;
    while (lo < hi) { int64_t mid = lo + ((hi - lo) >> 1); if (keys[mid] < key) lo = mid + 1; else hi = mid; }
    return lo < n && keys[lo] == key;
}

FLO_EXPORT void flo_filtered_ranks(int64_t nnz, const int64_t *idx_b, const int64_t *idx_e,
                                   const float *values, const int64_t *targets, int64_t n_filter,
                                   const int64_t *filter_keys, int64_t B, int64_t E, int use_eql,
                                   float *ranks) {
    float *truth = (float *)calloc((size_t)(B > 0 ? B : 1), sizeof(float));
    int64_t *greater = (int64_t *)calloc((size_t)(B > 0 ? B : 1), sizeof(int64_t));
    int64_t *equal = (int64_t *)calloc((size_t)(B > 0 ? B : 1), sizeof(int64_t));
    int64_t *expl = (int64_t *)calloc((size_t)(B > 0 ? B : 1), sizeof(int64_t));
    int64_t *fcount = (int64_t *)calloc((size_t)(B > 0 ? B : 1), sizeof(int64_t));
    /* The reference writes truth[b] from every matching entry; with a
     * coalesced input there is at most one. */
    for (int64_t i = 0; i < nnz; ++i) if (idx_e[i] == targets[idx_b[i]]) truth[idx_b[i]] = values[i];
    for (int64_t i = 0; i < n_filter; ++i) fcount[filter_keys[i] / E] += 1;
    for (int64_t i = 0; i < nnz; ++i) {
        int64_t b = idx_b[i];
        if (flo_bsearch64(filter_keys, n_filter, b * E + idx_e[i])) continue;
        expl[b] += 1;
        if (values[i] > truth[b]) greater[b] += 1;
        else if (values[i] == truth[b]) equal[b] += 1;
    }
    for (int64_t b = 0; b < B; ++b) {
        if (use_eql) {
            /* fp32 count arithmetic as in flashlog.cu:2829-2834 */
            float missing = (float)E - (float)fcount[b] - (float)expl[b];
            float eq = (float)equal[b] + (truth[b] == 0.0f ? missing : 0.0f);
            eq += 1.0f;
            ranks[b] = (float)greater[b] + (eq + 1.0f) * 0.5f;
        } else {
            ranks[b] = (float)greater[b] + 1.0f;
        }
    }
    free(truth); free(greater); free(equal); free(expl); free(fcount);
}
