/*
 * flashlog_b200.h -- C ABI of the B200 (sm_100a) FlashLog propagation library
 * (libflashlog_b200.so).
 *
 * Plain device pointers, sizes, a CUDA stream and an int status; no torch
 * types.  Every call is ordered on the stream it is given and never allocates
 * device memory: callers pass a workspace sized by the matching *_workspace
 * query.  Calls documented as "syncs" copy a size to a host pointer and
 * synchronize the stream.
 *
 * Status codes: FL_OK, FL_EINVAL (bad argument), FL_ECUDA (a CUDA call or
 * launch failed).  fl_last_error() returns a thread-local message for the last
 * failure.
 *
 * Layouts (the reference's formats, flashlog_kernel/flashlog_kernel.py:678-697
 * and flashlog_kernel/source/csr.cpp:12-69):
 *   CSR side  row_ptr i32[E+1], col i32[M], order i32[M] (CSR position ->
 *             triple id), group_ptr i32[E+1], group_rel i16[G],
 *             group_start i32[G], group_count i32[G]; edges sorted by
 *             (source, relation, triple id).
 *   state     a coalesced [B, L, E] COO held as rows r = b * L + l:
 *             row_ptr i64[rows+1], ent i32[S] ascending per row, val f32[S].
 *   weights   w f32[B, L, n], n = 2R + 1: columns [0, R) forward relations,
 *             [R, 2R) inverse relations, n - 1 identity.
 *   facts     per source entry i a slot range [slot_base[i], slot_base[i] +
 *             entry_count[i]) holding (dst i32, value f32, relation column
 *             i16 [, m f32]) in the reference's canonical order: forward
 *             groups, inverse groups, identity.
 */
#ifndef FLASHLOG_B200_H
#define FLASHLOG_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *fl_stream_t;

enum { FL_OK = 0, FL_EINVAL = 1, FL_ECUDA = 2 };

/* Expansion flags: which reference path a hop follows. */
enum {
    FL_SKIP_NONPOS_W = 1,  /* groups with w <= 0 take no edge (top-k fill, flashlog.cu:1511) */
    FL_DROP_MASKED = 2,    /* hidden edges emit no fact (flashlog_kernel.py:1217-1228)      */
    FL_WOT_I = 8,          /* no identity term                                             */
    FL_SAMPLED = 16,       /* c2 by weighted quotas, SplitMix64 phase (flashlog.cu:1458-1528) */
    FL_EDGE_SCORE = 32,    /* edge_weight holds scores, not logits                         */
    FL_EDGE_WEIGHT = 64,   /* multiply facts by sigmoid(edge_weight[triple])               */
    FL_NO_ORI = 256,       /* expand the inverse side only (dense outputs by source)       */
    FL_NO_INV = 512,       /* expand the forward side only                                 */
    FL_EDGE_POS = 1024,    /* fact_edge holds the CSR position p instead of order[p]        */
    FL_NO_NORMALIZE = 1 << 20  /* backward: g_y is the gradient of the sums, not of the normalized rows */
};

typedef struct {
    const int32_t *row_ptr, *col, *order, *group_ptr, *group_start, *group_count;
    const int16_t *group_rel;
} fl_csr_side;

typedef struct {
    int64_t rows, L, n, r_size, E; /* rows = B * L                              */
    int64_t topk_edges;             /* c2 // 2 per direction; >= 2^62: no budget */
    int64_t flags;                  /* FL_* flags                                */
    int64_t sampling_seed;          /* FL_SAMPLED only                           */
    float eps;                      /* row normalization epsilon                 */
    int64_t slot_capacity;          /* > 0: length of the fact / output buffers;
                                       work beyond it is skipped and flagged      */
    int32_t *status;                /* device int (or NULL): FL_STATUS_* bits     */
    int32_t *entry_info;            /* i32[FL_ENTRY_INFO_INTS * S] or NULL: per entry
                                       its row and the group ranges of both sides,
                                       written by
                                       fl_hop_plan and read by fl_hop_expand (NULL:
                                       the expansion looks them up)               */
    const uint8_t *vis_ori, *vis_inv; /* u8[M] or NULL: CSR-ordered visibility from
                                       fl_csr_visibility; replaces the mask_triple
                                       read through `order` (same result)         */
    uint32_t *work;                 /* device u32[2] or NULL: the two work queues of
                                       fl_hop_expand (it zeroes them); NULL:
                                       static assignment                          */
    const uint16_t *rel_rank;       /* u16[rows * 2 * r_size] or NULL: from
                                       fl_relation_rank of the same w             */
    const int32_t *rank_row;        /* i32[rows] or NULL: the row whose ranks a
                                       row uses (rows with equal w share one)     */
    const int32_t *row_order;       /* i32[rows] or NULL: the order in which
                                       fl_hop_backward takes the rows (a
                                       permutation; heaviest first balances the
                                       tail), NULL: row order                     */
    int32_t *fact_edge;             /* i32[slots] or NULL: fl_hop_expand writes each
                                       fact's triple id (order[p]; 0 for identity),
                                       the tie key of fl_row_reduce_max          */
} fl_hop_params;

/* Dropout of hop values fused into the kernels that write them (the models'
 * training dropout, src/model_DRUM_kernel_sp.py:189-192), with the keep bits
 * of fl_value_dropout: the same (seed, *counter, subseq, position) gives the
 * same mask.  Passed as an optional pointer; NULL means no dropout. */
typedef struct fl_dropout {
    double p;                /* drop probability, 0 <= p <= 1                   */
    uint64_t seed;
    const int64_t *counter;  /* device int64 or NULL (counts as 0)              */
    uint64_t subseq;         /* < 65536, e.g. the hop index                     */
} fl_dropout;

/* int32 values per entry in fl_hop_params.entry_info. */
enum { FL_ENTRY_INFO_INTS = 5 };

/* Device status bits set by the hop kernels. */
enum { FL_STATUS_SLOT_OVERFLOW = 1 };

const char *fl_last_error(void);
int fl_version(void);
int fl_device_sm_count(void);
/* Number of kernels this library has launched in the process so far. */
unsigned long long fl_launch_count(void);

/* CSR build on the device.  Replaces build_side (csr.cpp:12-69).  src, dst,
 * rel are i64[m]; ids outside [0, nodes) / [0, relations) are rejected before
 * any write.  Group arrays need room for m entries; *n_groups (host) receives
 * the number of groups (syncs). */
size_t fl_csr_build_workspace(int64_t m, int64_t nodes);
int fl_csr_build_side(const int64_t *src, const int64_t *dst, const int64_t *rel, int64_t m, int64_t nodes,
                      int64_t relations, int32_t *row_ptr, int32_t *col, int16_t *edge_rel, int32_t *order,
                      int32_t *group_ptr, int16_t *group_rel, int32_t *group_start, int32_t *group_count,
                      int64_t *n_groups, void *ws, size_t ws_bytes, fl_stream_t stream);

/* COO (b, l, e i64, coalesced order) -> row layout; *bad (device int, caller
 * zeroed) is set when ids are out of range or unsorted.  Replaces the index
 * handling of flashlog_kernel.py:1821-1824 / 1167-1178. */
int fl_coo_to_rows(const int64_t *b, const int64_t *l, const int64_t *e, int64_t nnz, int64_t L, int64_t rows,
                   int64_t E, int64_t *row_ptr, int32_t *ent, int *bad, fl_stream_t stream);
/* Row layout -> COO indices i64[3, U] (b, l, e). */
int fl_rows_to_coo(const int64_t *row_ptr, const int32_t *ent, int64_t rows, int64_t L, int64_t U, int64_t *indices,
                   fl_stream_t stream);

/* c1 entity budget.  Replaces _sparse_topc_entries (flashlog_kernel.py:1092-1137).
 * Rows with at most c1 nonzeros are kept whole; larger rows keep their c1
 * largest nonzero values, ties to the lower entity.  noise (f64, or NULL)
 * selects the sampled mode: candidate k (nonzero entries of over-budget rows
 * in state order) scores log(v) - log(noise[k]).  out_src[j] is the input
 * index of kept entry j.  Outputs have out_capacity entries (0: S); rows that
 * do not fit are truncated in out_row_ptr and set FL_STATUS_SLOT_OVERFLOW in
 * *status (device int, may be NULL). */
size_t fl_topc_workspace(int64_t rows, int64_t S);
int fl_topc_select(const int64_t *row_ptr, const int32_t *ent, const float *val, int64_t rows, int64_t S, int64_t c1,
                   const double *noise, int64_t *out_row_ptr, int32_t *out_ent, float *out_val, int64_t *out_src,
                   int64_t out_capacity, int32_t *status, void *ws, size_t ws_bytes, fl_stream_t stream);
/* Number of sampled-mode candidates (syncs). */
int fl_topc_candidates(const int64_t *row_ptr, const float *val, int64_t rows, int64_t S, int64_t c1,
                       int64_t *n_candidates, void *ws, size_t ws_bytes, fl_stream_t stream);

/* Hop planning: per-entry fact capacity (degree capped by topk_edges per
 * direction, + identity) and its scan into slot_base i64[S+1]; *total_slots
 * (host) receives slot_base[S] (syncs), unless total_slots is NULL (no host
 * synchronization).  S may exceed the live entry count row_ptr[rows]: entries
 * beyond it get no slots, so callers can run on upper-bound buffers.  Replaces the count kernels and the
 * two .item() calls of flashlog.cu:2040-2062 / 2160-2182. */
size_t fl_hop_workspace(int64_t rows, int64_t S);
int fl_hop_plan(const fl_hop_params *p, const int64_t *row_ptr, const int32_t *ent, int64_t S, fl_csr_side ori,
                fl_csr_side inv, int64_t *slot_base, int64_t *total_slots, void *ws, size_t ws_bytes,
                fl_stream_t stream);

/* Per (row, direction): rank u16[rows * 2 * r_size], the position of each
 * relation in the order (w descending, relation ascending) of the relations
 * with w > 0, and 0xffff for w <= 0.  fl_hop_expand uses it (through
 * fl_hop_params.rel_rank) for the c2 threshold of sides with more than 32
 * relation groups: taking a side's groups in rank order until the budget is
 * spent is the reference's selection (flashlog.cu:26-63), found by a scan
 * over rank bins instead of a radix select over the groups' weights.
 * rank_row (i32[rows] or NULL): rows with rank_row[r] != r are skipped (they
 * read the ranks of row rank_row[r], whose w must equal theirs).
 * r_size <= 16384. */
int fl_relation_rank(const float *w, int64_t rows, int64_t r_size, const int32_t *rank_row, uint16_t *rank,
                     fl_stream_t stream);

/* CSR-ordered visibility of one side: vis[p] = mask_triple[order[p]] != 0.
 * The gather of prepare_csr_masks / apply_mask_cuda (flashlog_kernel.py:225-255,
 * flashlog.cu:1291-1340) in one byte per edge; built once per step and shared
 * by the hops. */
int fl_csr_visibility(const int32_t *order, int64_t m, const uint8_t *mask_triple, uint8_t *vis, fl_stream_t stream);

/* The order in which the row reduction and the backward take the rows
 * (fl_hop_params.row_order): rows by descending slot count
 * slot_base[row_ptr[r + 1]] - slot_base[row_ptr[r]], ties to the lower row.
 * One block; at most 16384 rows (FL_EINVAL above). */
int fl_row_order(const int64_t *row_ptr, const int64_t *slot_base, int64_t rows, int32_t *order, fl_stream_t stream);

/* Kinds of the triple-indexed mask of fl_csr_mask. */
enum { FL_MASK_U8 = 0, FL_MASK_F32 = 1 };

/* CSR-ordered float mask of one side: out[p] = mask[order[p]], times
 * 1 / (1 + exp(-weight[order[p]])) when weight is not NULL (learnable edge
 * weights, --use_soft).  Replaces prepare_csr_masks / _apply_mask_order /
 * apply_mask_cuda (flashlog_kernel.py:225-255, flashlog.cu:1286-1340).
 * mask is u8 (0 / 1, a bool tensor's bytes) or f32 per triple. */
int fl_csr_mask(const void *mask, int mask_kind, const int32_t *order, int64_t m, const float *weight, float *out,
                fl_stream_t stream);

/* Upstream gradient of a hop's output at the output's coordinates: out[i] =
 * the value of the gradient state at (out_b[i], out_l[i], out_e[i]), or 0
 * where the gradient has no entry.  The gradient is a row layout (g_row_ptr
 * i64[rows+1], g_ent i32 ascending per row, g_val f32); every lookup is a
 * binary search in its own row.  Replaces _align_sparse_grad_to_output
 * (flashlog_kernel.py:360-376). */
int fl_align_rows(const int64_t *out_b, const int64_t *out_l, const int64_t *out_e, int64_t n, int64_t L,
                  int64_t rows, const int64_t *g_row_ptr, const int32_t *g_ent, const float *g_val, float *out,
                  fl_stream_t stream);

/* Hop expansion (8-lane teams for entries with at most 8 relation groups per
 * side, one warp otherwise).  Replaces
 * fill_sparse3d_topk_kernel / fill_sparse3d_all_edges_kernel /
 * fill_sparse3d_identity_kernel (flashlog.cu:1402-1559, 1759-1854).  The edge
 * visibility comes from mask_triple (u8 per triple, read through order, the
 * top-k path) or mask_csr_ori / mask_csr_inv (f32 per CSR position, the
 * all-edges path), or is 1 when all are NULL.  fact_m may be NULL unless
 * FL_EDGE_WEIGHT is set. */
int fl_hop_expand(const fl_hop_params *p, const int64_t *row_ptr, const int32_t *ent, const float *val, int64_t S,
                  const float *w, fl_csr_side ori, fl_csr_side inv, const float *mask_csr_ori,
                  const float *mask_csr_inv, const uint8_t *mask_triple, const float *edge_weight,
                  const int64_t *slot_base, int32_t *fact_dst, float *fact_val, int16_t *fact_rel, float *fact_m,
                  int32_t *entry_count, fl_stream_t stream);

/* Per-row coalesce-sum (+ normalization) of expanded facts.  Replaces the
 * coalesce of flashlog_kernel.py:258-357 (argsort + unique + scatter_add) and
 * sparse3d_normalize_forward_cuda (flashlog.cu:2593-2649).  Sums follow the
 * canonical fact order.  fact_pos (i32 per slot, may be NULL) receives each
 * fact's output index within its row.  Outputs out_ent / out_x / out_y have
 * capacity total_slots, out_row_ptr i64[rows+1] (its last entry is the
 * output count), out_denom f32[rows] (raw row sums).  Stream-ordered; no
 * host synchronization.  total_slots is the length of the fact and output
 * buffers; rows whose slots lie beyond it are skipped and set
 * FL_STATUS_SLOT_OVERFLOW in *status (device int, may be NULL).  row_order
 * (i32[rows], a permutation, or NULL) is the order in which the rows are
 * taken: heaviest first shortens the tail; results do not depend on it.
 * drop (or NULL): out_y[i] is written as fl_value_dropout would leave it
 * (out_x and out_denom are not affected). */
size_t fl_reduce_workspace(int64_t rows, int64_t total_slots);
int fl_row_reduce(const int64_t *row_ptr, int64_t rows, int64_t E, const int64_t *slot_base, const int32_t *entry_count,
                  const int32_t *fact_dst, const float *fact_val, int64_t total_slots, int32_t *fact_pos, float eps,
                  int64_t *out_row_ptr, int32_t *out_ent, float *out_x, float *out_y, float *out_denom,
                  int32_t *status, const int32_t *row_order, void *ws, size_t ws_bytes, const fl_dropout *drop,
                  fl_stream_t stream);

/* MAX coalesce of expanded facts (FlashLogFunctionSparse3DTopKMax,
 * flashlog_kernel.py:386-478): per (row, destination) the largest fact value;
 * equal values go to the smaller source (ori < inv < identity, read from the
 * fact's relation column: < r_size, < 2 r_size, 2 r_size) and then to the
 * smaller triple id (fact_edge).  fact_pos gets the output index of every
 * winning fact and -1 for the others, so fl_hop_backward (with
 * FL_NO_NORMALIZE) sends gradients to the winners only
 * (flashlog.cu:2363-2406).  Outputs are the unnormalized maxima. */
int fl_row_reduce_max(const int64_t *row_ptr, int64_t rows, int64_t E, int64_t r_size, const int64_t *slot_base,
                      const int32_t *fact_dst, const float *fact_val, const int16_t *fact_rel,
                      const int32_t *fact_edge, int64_t total_slots, int32_t *fact_pos, int64_t *out_row_ptr,
                      int32_t *out_ent, float *out_x, int max_flags, int32_t *status, void *ws, size_t ws_bytes,
                      fl_stream_t stream);
/* max_flags of fl_row_reduce_max: compare values by their fp32 bit patterns as
 * unsigned integers, the order of the packed (value, ~position) CAS-max of the
 * dense MAX path (flashlog.cu:103-121, 523-581). */
enum { FL_MAX_BITS = 1,
       FL_MAX_VALUE_ONLY = 2 /* only the maxima are wanted: fact_rel and fact_edge may be NULL,
                                equal values tie at no key (any of them gives the same value) */ };

/* Hop backward (+ normalization backward unless FL_NO_NORMALIZE).  Replaces
 * flashlog_backward_sparse3d_cached_cuda (flashlog.cu:2317-2361) and
 * sparse3d_normalize_backward_cuda (flashlog.cu:2651-2691).  g_y f32[U]
 * (gradient of out_y, or of out_x with FL_NO_NORMALIZE) -> grad_val f32[S]
 * and grad_w f32[rows, n] (every column written). */
size_t fl_hop_backward_workspace(int64_t rows, int64_t n);
int fl_hop_backward(const fl_hop_params *p, const int64_t *row_ptr, const float *val, int64_t S, const float *w,
                    const int64_t *slot_base, const int32_t *entry_count, const int32_t *fact_pos,
                    const int16_t *fact_rel, const float *fact_m, const int64_t *out_row_ptr, const float *out_x,
                    const float *out_denom, const float *g_y, float *grad_val, float *grad_w, void *ws,
                    size_t ws_bytes, fl_stream_t stream);

/* Row normalization alone.  Replaces sparse3d_normalize_{forward,backward}_cuda
 * (flashlog.cu:2593-2691). */
int fl_normalize_forward(const int64_t *row_ptr, const float *x, int64_t rows, float eps, float *y, float *denom,
                         fl_stream_t stream);
int fl_normalize_backward(const int64_t *row_ptr, const float *x, const float *denom, const float *g, int64_t rows,
                          float eps, float *gx, fl_stream_t stream);

/* Work counts of one hop, added to acc (device i64[4]): live entries S,
 * relation groups of both sides G, facts through graph edges F, live
 * outputs U.  No synchronization; the measurement of bench.py reads them
 * after its timed region. */
int fl_hop_stats(const int64_t *row_ptr, int64_t rows, const int32_t *ent, int64_t S, fl_csr_side ori,
                 fl_csr_side inv, const int32_t *entry_count, const int64_t *out_row_ptr, int wot_i, int64_t *acc,
                 fl_stream_t stream);

/* Gradient of learnable edge weights (the --use_soft path): replaces the
 * chunk loops of flashlog_kernel.py:1306-1336 (SUM) and 1590-1614 (MAX).
 * Every edge fact f of the first min(S, row_ptr[rows]) entries with
 * fact_pos[f] >= 0 (its position within its row's outputs) adds
 *   g[out_row_ptr[r] + fact_pos[f]] * val[i] * w[r, fact_rel[f]] * fact_m[f] * (1 - sigmoid(edge_weight[e]))
 * to grad_edge[e], r = row(i), e = fact_edge[f] (the triple id).  The facts
 * are those fl_hop_expand recorded with fact_m and fact_edge and the row
 * reduction placed (fact_pos, out_row_ptr); g is the gradient at the outputs
 * (before any normalization); the identity fact has no edge.  grad_edge is
 * accumulated (zero it first) with float atomics. */
int fl_edge_weight_grad(const fl_hop_params *p, const int64_t *row_ptr, const float *val, int64_t S, const float *w,
                        const int64_t *slot_base, const int32_t *entry_count, const int32_t *fact_pos,
                        const int16_t *fact_rel, const float *fact_m, const int32_t *fact_edge,
                        const int64_t *out_row_ptr, const float *g, const float *edge_weight, float *grad_edge,
                        fl_stream_t stream);

/* grad_full[src_index[j]] = grad_sel[j] for j < n_sel (and j < *n_live when
 * n_live, a device count, is given), zeros elsewhere: all of grad_full[0,
 * n_full), or only its first *full_live entries when full_live (a device
 * count) is given.  Replaces _restore_pruned_gradient
 * (flashlog_kernel.py:1150-1155).  drop (or NULL): each written value is
 * multiplied by the dropout factor of its position in grad_full (the backward
 * of a dropout of the full vector), as fl_value_dropout on grad_full would. */
int fl_scatter_grad(const float *grad_sel, const int64_t *src_index, int64_t n_sel, const int64_t *n_live,
                    float *grad_full, int64_t n_full, const int64_t *full_live, const fl_dropout *drop,
                    fl_stream_t stream);

/* Channel readout at the targets: scores[q] = sum over channels l (in order)
 * of the state's value at (q, l, targets[q]) (0 when absent).  Rows are
 * r = q * N + l.  Replaces sum_sp_3d + the target lookup of
 * log_loss_common_sp (src/model_DRUM_kernel_sp.py:22-28, src/utils.py:36-47).
 * The backward writes g_scores[q] at every entry read and zeros the rest of
 * grad_val (n_val entries, or the first *val_live when that device count is
 * given).  drop (or NULL): the written gradients get the dropout factor of
 * their position, as fl_value_dropout on grad_val would. */
int fl_readout(const int64_t *row_ptr, const int32_t *ent, const float *val, int64_t N, const int64_t *targets,
               int64_t Q, float *scores, fl_stream_t stream);
int fl_readout_backward(const int64_t *row_ptr, const int32_t *ent, int64_t N, const int64_t *targets, int64_t Q,
                        const float *g_scores, float *grad_val, int64_t n_val, const int64_t *val_live,
                        const fl_dropout *drop, fl_stream_t stream);

/* Dropout of hop values (nn.Dropout on s.values() in training,
 * src/model_DRUM_kernel_sp.py:189-192; the other sparse models do the same).
 * y[i] = x[i] * (keep(i) ? scale : 0) for i < n (or the first
 * *live, a device count, when live is given); y may be x.  keep(i) is a pure
 * function of (seed, *counter, subseq, i): with
 *   key = splitmix64(seed ^ splitmix64((*counter << 16) | subseq)),
 * i is kept iff (splitmix64(key + i) >> 32) >= floor(p * 2^32)
 * (splitmix64: the SplitMix64 output function; *counter is 0 when counter is
 * NULL) and scale = (float)(1 / (double)(float)(1 - p)), torch's rounding.  A device counter lets a captured step draw a new mask per replay;
 * the backward is the same call on the gradient.  Needs 0 <= p <= 1 and
 * subseq < 65536 (FL_EINVAL otherwise). */
int fl_value_dropout(const float *x, float *y, int64_t n, const int64_t *live, double p, uint64_t seed,
                     const int64_t *counter, uint64_t subseq, fl_stream_t stream);

/* Rule step with one fixed operator per (query, rule) row: ops i64[B, Lr]
 * holds a forward relation, inverse relation + R, or identity 2R.  Replaces
 * flashlog_forward_sparse3d_fixed_relation_cuda (flashlog.cu:1677-1741); the
 * facts are then reduced by fl_row_reduce.  plan: *total (host) receives the
 * number of facts (syncs).  l may be NULL (every entry in column 0, as for a
 * state whose rows are rule instances with ops i64[B, 1]); val may be NULL
 * (every value 1, a Boolean state). */
size_t fl_fixed_relation_workspace(int64_t nnz);
int fl_fixed_relation_plan(const int64_t *b, const int64_t *l, const int32_t *ent, int64_t nnz, const int64_t *ops,
                           int64_t Lr, int64_t r_size, fl_csr_side ori, fl_csr_side inv, int64_t *slot_base,
                           int64_t *total, void *ws, size_t ws_bytes, fl_stream_t stream);
int fl_fixed_relation_fill(const int64_t *b, const int64_t *l, const int32_t *ent, const float *val, int64_t nnz,
                           const int64_t *ops, int64_t Lr, int64_t r_size, fl_csr_side ori, fl_csr_side inv,
                           const int64_t *slot_base, int32_t *fact_dst, float *fact_val, int32_t *entry_count,
                           fl_stream_t stream);

/* Filtered tie-averaged ranks; filter_keys (b * E + e) sorted ascending.
 * Replaces sparse2d_filtered_ranks_cuda (flashlog.cu:2839-2910). */
/* Max-product rule scores of one chunk of C rules (rules/shared_inference.py
 * :123-206 with reduction 'max', the dense accumulator of 200-206): the state
 * has rows q * C + c (query q, rule c) with Boolean values; every entry with a
 * positive value raises acc[rank * B * E + q * E + entity] to the fp32 bit
 * pattern of weights[c * ranks + rank].  acc (u32, caller zeroed) then holds,
 * as fp32, the largest rank weight of the rules reaching each entity.
 * weights must be finite and nonnegative.  Order-independent and exact.
 * val may be NULL (a Boolean state: every entry counts). */
int fl_rule_max_reduce(const int64_t *row_ptr, int64_t rows, const int32_t *ent, const float *val, int64_t C,
                       const float *weights, int64_t ranks, int64_t B, int64_t E, uint32_t *acc, fl_stream_t stream);

/* Sparse max-product accumulation (rules/shared_inference.py:176-206 when
 * the dense [ranks, B, E] accumulator does not fit, as with 86M entities): the
 * facts of the rank rows (q, r), r < ranks, laid out for fl_row_reduce_max.
 * The grounded state has rows q * C + c (row_ptr st_rp[B*C+1], entities
 * st_ent, values st_val); the running maxima of earlier chunks are rank rows
 * (run_rp[B*ranks+1], run_ent, run_val), or NULL for the first chunk.  Row
 * (q, r) holds its running maxima, then every entry of the rows (q, c) with
 * its rule's weight w[c * ranks + r] as value (destination -1, no fact, where
 * the weight or the state value is 0).  slot_base i64[B*ranks+1] gets the row
 * starts (run_rp[row] + ranks * st_rp[q*C] + r * (entries of query q)),
 * fact_dst / fact_val i32 / f32[slot_base[B*ranks]] the facts. */
int fl_rule_rank_facts(const int64_t *st_rp, const int32_t *st_ent, const float *st_val, int64_t B, int64_t C,
                       const float *w, int64_t ranks, const int64_t *run_rp, const int32_t *run_ent,
                       const float *run_val, int64_t *slot_base, int32_t *fact_dst, float *fact_val,
                       fl_stream_t stream);

/* The rank-row facts of a state whose rows are rule instances (one query's
 * instances contiguous: query q owns rows [q_inst[q], q_inst[q + 1]),
 * q_inst i64[B + 1]; rows st_rp[rows + 1], entities st_ent): row (q, r)
 * holds every entry of the query's instance rows in instance order with the
 * instance's weight w[instance * ranks + r] as value (destination -1 where
 * the weight is 0).  slot_base i64[B*ranks+1] gets ranks * (st_rp[q_inst[q]]
 * - st_rp[q_inst[0]]) + r * (entries of query q), so a range of queries
 * (q_inst offset to its first query) has facts from slot 0; fact_dst /
 * fact_val the facts, for
 * fl_row_reduce_max (FL_MAX_VALUE_ONLY).  The routed evaluation of
 * rules/evaluate.py:1015-1095, where every query has the rules of its own
 * relation, as one state over many queries. */
int fl_rule_instance_facts(const int64_t *st_rp, const int32_t *st_ent, const int64_t *q_inst, int64_t B,
                           const float *w, int64_t ranks, int64_t *slot_base, int32_t *fact_dst, float *fact_val,
                           fl_stream_t stream);

/* The same rank maxima as fl_rule_instance_facts + fl_row_reduce_max, into a
 * dense accumulator for queries that reach a large share of the entities:
 * acc u32[nq * ranks * E] (caller zeroed) gets at (q * ranks + r) * E + e
 * the largest fp32 bit pattern of w[instance * ranks + r] over the instances
 * of query q (rows q_inst[q] .. q_inst[q + 1] - 1, q < nq) whose row holds e.
 * Weights must be finite and nonnegative; order-independent and exact. */
int fl_rule_instance_max(const int64_t *st_rp, const int32_t *st_ent, const int64_t *q_inst, int64_t nq,
                         const float *w, int64_t ranks, int64_t E, uint32_t *acc, fl_stream_t stream);

/* Boolean fixed-operator step into per-row bitmaps, for the rows of a rule
 * state with more facts than their bitmap has words: every listed entry
 * entries[k] (k < n) of row entry_row[entries[k]] sets, in the bitmap of slot
 * row_slot[row] (words u32 words each, caller zeroed), the bit of every
 * destination of the row's operator ops[row] (identity 2R: the entity
 * itself).  The rows' next states are then read out in entity order by
 * fl_bitmap_rows_count (row_ptr i64[nb+1]; chunk_off i64[nb*words/256+1]
 * kept for the emit) and fl_bitmap_rows_emit (ent i32[row_ptr[nb]]).  words
 * must be a multiple of 256.  The set semantics are the Boolean projection
 * after every rule step of rules/shared_inference.py:123-126. */
int fl_fixed_relation_bitmap(const int64_t *entries, int64_t n, const int64_t *entry_row, const int32_t *row_slot,
                             const int32_t *ent, const int64_t *ops, int64_t r_size, fl_csr_side ori,
                             fl_csr_side inv, uint32_t *bitmap, int64_t words, fl_stream_t stream);
size_t fl_bitmap_rows_workspace(int64_t nb, int64_t words);
/* Copies every row of a row layout (src_rp i64[rows+1], src_ent) to the
 * start of the same row in another layout (dst_rp i64[rows], dst_ent), for
 * merging the results of disjoint row sets. */
int fl_rows_copy(const int64_t *src_rp, const int32_t *src_ent, int64_t rows, const int64_t *dst_rp, int32_t *dst_ent,
                 fl_stream_t stream);
int fl_bitmap_rows_count(const uint32_t *bitmap, int64_t nb, int64_t words, int64_t *chunk_off, int64_t *row_ptr,
                         void *ws, size_t ws_bytes, fl_stream_t stream);
int fl_bitmap_rows_emit(const uint32_t *bitmap, int64_t nb, int64_t words, const int64_t *chunk_off, int32_t *ent,
                        fl_stream_t stream);

size_t fl_filtered_ranks_workspace(int64_t B);
int fl_filtered_ranks(const int64_t *idx_b, const int64_t *idx_e, const float *values, int64_t nnz,
                      const int64_t *targets, const int64_t *filter_keys, int64_t n_filter, int64_t B, int64_t E,
                      int use_eql, float *ranks, void *ws, size_t ws_bytes, fl_stream_t stream);

/* fl_filtered_ranks for callers that cannot allocate device memory (no
 * reference counterpart: the reference allocates its counters with torch on
 * every call).  Same inputs, outputs and results as fl_filtered_ranks, but the
 * per-query counters live in a fixed 1.25 MiB array inside this library's
 * device memory, which every GPU that loads the library keeps until the
 * process exits; the call itself allocates nothing.  At most 65536 queries
 * (B) per call -- larger B returns FL_EINVAL.  The first call on each device
 * looks up that array's device address (cudaGetSymbolAddress) with the device
 * current; make that first call before any stream capture, and do not reset
 * the device (cudaDeviceReset) between calls, since the looked-up address
 * belongs to the context that was current then.  All calls share
 * the one array and each call clears it before counting, so calls that
 * overlap on the GPU (concurrent streams, or host threads sharing a device)
 * race and must be serialized by the caller. */
int fl_filtered_ranks_noalloc(const int64_t *idx_b, const int64_t *idx_e, const float *values, int64_t nnz,
                              const int64_t *targets, const int64_t *filter_keys, int64_t n_filter, int64_t B,
                              int64_t E, int use_eql, float *ranks, fl_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* FLASHLOG_B200_H */
