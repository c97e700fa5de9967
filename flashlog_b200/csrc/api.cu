// api.cu -- the extern "C" boundary of libflashlog_b200.so.
//
// Each entry point validates its arguments, runs stream-ordered kernels on the
// caller's stream and returns an int status; fl_last_error() holds a
// thread-local message for the last failure.
#include <stdarg.h>
#include <string.h>

#include <atomic>

#include "common.cuh"
#include "hop.cuh"

namespace fl {

static thread_local char g_err[512] = "";
static std::atomic<unsigned long long> g_launches{0};

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

int check_launch(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error("%s: %s", what, cudaGetErrorString(e));
        return FL_ECUDA;
    }
    return FL_OK;
}

// Declarations of the kernels' host wrappers defined in other units.
size_t csr_build_workspace(int64_t m, int64_t nodes);
int csr_build_side(const int64_t *src, const int64_t *dst, const int64_t *rel, int64_t m, int64_t nodes,
                   int64_t relations, int32_t *row_ptr, int32_t *col, int16_t *edge_rel, int32_t *order,
                   int32_t *group_ptr, int16_t *group_rel, int32_t *group_start, int32_t *group_count,
                   int64_t *n_groups, void *ws, size_t ws_bytes, cudaStream_t st);
size_t fixed_relation_workspace(int64_t nnz);
int fixed_relation_plan(const int64_t *b, const int64_t *l, const int32_t *ent, int64_t nnz, const int64_t *ops,
                        int64_t Lr, int64_t R, const fl_csr_side &ori, const fl_csr_side &inv, int64_t *slot_base,
                        int64_t *total, void *ws, size_t ws_bytes, cudaStream_t st);
int fixed_relation_fill(const int64_t *b, const int64_t *l, const int32_t *ent, const float *val, int64_t nnz,
                        const int64_t *ops, int64_t Lr, int64_t R, const fl_csr_side &ori, const fl_csr_side &inv,
                        const int64_t *slot_base, int32_t *fact_dst, float *fact_val, int32_t *entry_count,
                        cudaStream_t st);
size_t filtered_ranks_workspace(int64_t B);
int rule_rank_facts(const int64_t *st_rp, const int32_t *st_ent, const float *st_val, int64_t B, int64_t C,
                    const float *w, int64_t ranks, const int64_t *run_rp, const int32_t *run_ent, const float *run_val,
                    int64_t *slot_base, int32_t *fact_dst, float *fact_val, cudaStream_t st);
int rule_instance_facts(const int64_t *st_rp, const int32_t *st_ent, const int64_t *q_inst, int64_t B,
                        const float *w, int64_t ranks, int64_t *slot_base, int32_t *fact_dst, float *fact_val,
                        cudaStream_t st);
int rule_instance_max(const int64_t *st_rp, const int32_t *st_ent, const int64_t *q_inst, int64_t nq, const float *w,
                      int64_t ranks, int64_t E, unsigned int *acc, cudaStream_t st);
int rows_copy(const int64_t *src_rp, const int32_t *src_ent, int64_t rows, const int64_t *dst_rp, int32_t *dst_ent,
              cudaStream_t st);
size_t bitmap_rows_workspace(int64_t nb, int64_t words);
int fixed_relation_bitmap(const int64_t *entries, int64_t n, const int64_t *entry_row, const int32_t *row_slot,
                          const int32_t *ent, const int64_t *ops, int64_t R, const fl_csr_side &ori,
                          const fl_csr_side &inv, uint32_t *bitmap, int64_t words, cudaStream_t st);
int bitmap_rows_count(const uint32_t *bitmap, int64_t nb, int64_t words, int64_t *chunk_off, int64_t *row_ptr,
                      void *ws, size_t ws_bytes, cudaStream_t st);
int bitmap_rows_emit(const uint32_t *bitmap, int64_t nb, int64_t words, const int64_t *chunk_off, int32_t *ent,
                     cudaStream_t st);
int rule_max_reduce(const int64_t *row_ptr, int64_t rows, const int32_t *ent, const float *val, int64_t C,
                    const float *weights, int64_t ranks, int64_t B, int64_t E, unsigned int *acc, cudaStream_t st);
int filtered_ranks(const int64_t *ib, const int64_t *ie, const float *v, int64_t nnz, const int64_t *targets,
                   const int64_t *fk, int64_t nf, int64_t B, int64_t E, int use_eql, float *ranks, void *ws,
                   size_t ws_bytes, cudaStream_t st);
int filtered_ranks_noalloc(const int64_t *ib, const int64_t *ie, const float *v, int64_t nnz, const int64_t *targets,
                           const int64_t *fk, int64_t nf, int64_t B, int64_t E, int use_eql, float *ranks,
                           cudaStream_t st);

int csr_mask(const void *mask, int mask_kind, const int32_t *order, int64_t m, const float *weight, float *out,
             cudaStream_t st);
int align_rows(const int64_t *out_b, const int64_t *out_l, const int64_t *out_e, int64_t n, int64_t L, int64_t rows,
               const int64_t *g_row_ptr, const int32_t *g_ent, const float *g_val, float *out, cudaStream_t st);

int readout(const int64_t *row_ptr, const int32_t *ent, const float *val, int64_t N, const int64_t *targets, int64_t Q,
            float *scores, cudaStream_t st);
int value_dropout(const float *x, float *y, int64_t n, const int64_t *live, double p, uint64_t seed,
                  const int64_t *counter, uint64_t subseq, cudaStream_t st);
int readout_backward(const int64_t *row_ptr, const int32_t *ent, int64_t N, const int64_t *targets, int64_t Q,
                     const float *g, float *grad_val, int64_t n_val, const int64_t *val_live, const fl_dropout *drop,
                     cudaStream_t st);

namespace {

// COO (b, l, e) sorted by key -> row_ptr by binary search per row; entity ids
// narrowed to int32.  Out-of-range or unsorted input sets *bad.
__global__ void coo_rows_kernel(const int64_t *b, const int64_t *l, int64_t nnz, int64_t L, int64_t rows,
                                int64_t *row_ptr) {
    int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (r > rows) return;
    int64_t lo = 0, hi = nnz;  // first i with key(i) >= r
    while (lo < hi) {
        int64_t mid = lo + ((hi - lo) >> 1);
        if (b[mid] * L + l[mid] < r) lo = mid + 1; else hi = mid;
    }
    row_ptr[r] = lo;
}

__global__ void coo_ent_kernel(const int64_t *b, const int64_t *l, const int64_t *e, int64_t nnz, int64_t L,
                               int64_t rows, int64_t E, int32_t *ent, int *bad) {
    int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= nnz) return;
    const int64_t key = b[i] * L + l[i];
    bool ok = e[i] >= 0 && e[i] < E && l[i] >= 0 && l[i] < L && key >= 0 && key < rows;
    if (ok && i > 0) {
        const int64_t pk = b[i - 1] * L + l[i - 1];
        ok = pk < key || (pk == key && e[i - 1] < e[i]);
    }
    if (!ok) atomicExch(bad, 1);
    ent[i] = static_cast<int32_t>(e[i]);
}

__global__ void rows_coo_kernel(const int64_t *row_ptr, const int32_t *ent, int64_t rows, int64_t L, int64_t U,
                                int64_t *idx) {
    const int64_t r = blockIdx.x;
    if (r >= rows) return;
    const int64_t a = row_ptr[r], z = row_ptr[r + 1];
    for (int64_t k = a + threadIdx.x; k < z; k += blockDim.x) {
        idx[k] = r / L;
        idx[U + k] = r % L;
        idx[2 * U + k] = ent[k];
    }
}

}  // namespace
}  // namespace fl

using namespace fl;

extern "C" {

const char *fl_last_error(void) { return g_err; }

int fl_version(void) { return 1; }

unsigned long long fl_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int fl_device_sm_count(void) {
    // cached per device: launches made while a stream is being captured must
    // not query the device
    static std::atomic<int> cache[64];
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (dev >= 0 && dev < 64 && (n = cache[dev].load(std::memory_order_relaxed)) > 0) return n;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    if (dev >= 0 && dev < 64) cache[dev].store(n, std::memory_order_relaxed);
    return n;
}

size_t fl_csr_build_workspace(int64_t m, int64_t nodes) { return csr_build_workspace(m, nodes); }

int fl_csr_build_side(const int64_t *src, const int64_t *dst, const int64_t *rel, int64_t m, int64_t nodes,
                      int64_t relations, int32_t *row_ptr, int32_t *col, int16_t *edge_rel, int32_t *order,
                      int32_t *group_ptr, int16_t *group_rel, int32_t *group_start, int32_t *group_count,
                      int64_t *n_groups, void *ws, size_t ws_bytes, fl_stream_t stream) {
    return csr_build_side(src, dst, rel, m, nodes, relations, row_ptr, col, edge_rel, order, group_ptr, group_rel,
                          group_start, group_count, n_groups, ws, ws_bytes, as_stream(stream));
}

int fl_coo_to_rows(const int64_t *b, const int64_t *l, const int64_t *e, int64_t nnz, int64_t L, int64_t rows,
                   int64_t E, int64_t *row_ptr, int32_t *ent, int *bad, fl_stream_t stream) {
    FL_REQUIRE(L > 0 && rows >= 0 && nnz >= 0, "invalid state shape");
    cudaStream_t st = as_stream(stream);
    launch(coo_rows_kernel, static_cast<unsigned>((rows + 1 + 255) / 256), 256, 0, st, b, l, nnz, L, rows, row_ptr);
    if (nnz > 0)
        launch(coo_ent_kernel, static_cast<unsigned>((nnz + 255) / 256), 256, 0, st, b, l, e, nnz, L, rows, E, ent, bad);
    return check_launch("coo_to_rows");
}

int fl_rows_to_coo(const int64_t *row_ptr, const int32_t *ent, int64_t rows, int64_t L, int64_t U, int64_t *indices,
                   fl_stream_t stream) {
    FL_REQUIRE(L > 0, "invalid L");
    if (rows > 0 && U > 0)
        launch(rows_coo_kernel, static_cast<unsigned>(rows), 256, 0, as_stream(stream), row_ptr, ent, rows, L, U, indices);
    return check_launch("rows_to_coo");
}

size_t fl_topc_workspace(int64_t rows, int64_t S) { return topc_workspace(rows, S); }

int fl_topc_select(const int64_t *row_ptr, const int32_t *ent, const float *val, int64_t rows, int64_t S, int64_t c1,
                   const double *noise, int64_t *out_row_ptr, int32_t *out_ent, float *out_val, int64_t *out_src,
                   int64_t out_capacity, int32_t *status, void *ws, size_t ws_bytes, fl_stream_t stream) {
    return topc_select(row_ptr, ent, val, rows, S, c1, noise, out_row_ptr, out_ent, out_val, out_src, out_capacity,
                       status, ws, ws_bytes, as_stream(stream));
}

int fl_topc_candidates(const int64_t *row_ptr, const float *val, int64_t rows, int64_t S, int64_t c1,
                       int64_t *n_candidates, void *ws, size_t ws_bytes, fl_stream_t stream) {
    return topc_candidates(row_ptr, val, rows, S, c1, n_candidates, ws, ws_bytes, as_stream(stream));
}

size_t fl_hop_workspace(int64_t rows, int64_t S) { return hop_workspace(rows, S); }

int fl_hop_plan(const fl_hop_params *p, const int64_t *row_ptr, const int32_t *ent, int64_t S, fl_csr_side ori,
                fl_csr_side inv, int64_t *slot_base, int64_t *total_slots, void *ws, size_t ws_bytes,
                fl_stream_t stream) {
    FL_REQUIRE(p != nullptr && p->n == 2 * p->r_size + 1, "w must have n = 2 * r_size + 1 columns");
    return hop_plan(p, row_ptr, ent, S, ori, inv, slot_base, total_slots, ws, ws_bytes, as_stream(stream));
}

int fl_relation_rank(const float *w, int64_t rows, int64_t r_size, const int32_t *rank_row, uint16_t *rank,
                     fl_stream_t stream) {
    FL_REQUIRE(rows >= 0 && (rows == 0 || (w && rank)), "fl_relation_rank: bad arguments");
    return relation_rank(w, rows, r_size, rank_row, rank, as_stream(stream));
}

int fl_row_order(const int64_t *row_ptr, const int64_t *slot_base, int64_t rows, int32_t *order, fl_stream_t stream) {
    FL_REQUIRE(rows == 0 || (row_ptr && slot_base && order), "fl_row_order: null pointer");
    return row_order(row_ptr, slot_base, rows, order, as_stream(stream));
}

int fl_csr_visibility(const int32_t *order, int64_t m, const uint8_t *mask_triple, uint8_t *vis, fl_stream_t stream) {
    FL_REQUIRE(m >= 0 && (m == 0 || (order && mask_triple && vis)), "fl_csr_visibility: bad arguments");
    return csr_visibility(order, m, mask_triple, vis, as_stream(stream));
}

int fl_csr_mask(const void *mask, int mask_kind, const int32_t *order, int64_t m, const float *weight, float *out,
                fl_stream_t stream) {
    return csr_mask(mask, mask_kind, order, m, weight, out, as_stream(stream));
}

int fl_align_rows(const int64_t *out_b, const int64_t *out_l, const int64_t *out_e, int64_t n, int64_t L,
                  int64_t rows, const int64_t *g_row_ptr, const int32_t *g_ent, const float *g_val, float *out,
                  fl_stream_t stream) {
    return align_rows(out_b, out_l, out_e, n, L, rows, g_row_ptr, g_ent, g_val, out, as_stream(stream));
}

int fl_hop_expand(const fl_hop_params *p, const int64_t *row_ptr, const int32_t *ent, const float *val, int64_t S,
                  const float *w, fl_csr_side ori, fl_csr_side inv, const float *mask_csr_ori,
                  const float *mask_csr_inv, const uint8_t *mask_triple, const float *edge_weight,
                  const int64_t *slot_base, int32_t *fact_dst, float *fact_val, int16_t *fact_rel, float *fact_m,
                  int32_t *entry_count, fl_stream_t stream) {
    FL_REQUIRE(p != nullptr && p->n == 2 * p->r_size + 1, "w must have n = 2 * r_size + 1 columns");
    FL_REQUIRE(p->n - 1 <= 32767, "relation columns exceed int16");
    FL_REQUIRE(!((p->flags & FL_SAMPLED) && p->sampling_seed < 0), "sampled mode needs a seed");
    return hop_expand(p, row_ptr, ent, val, S, w, ori, inv, mask_csr_ori, mask_csr_inv, mask_triple, edge_weight,
                      slot_base, fact_dst, fact_val, fact_rel, fact_m, entry_count, as_stream(stream));
}

size_t fl_reduce_workspace(int64_t rows, int64_t total_slots) { return row_reduce_workspace(rows, total_slots); }

int fl_row_reduce_max(const int64_t *row_ptr, int64_t rows, int64_t E, int64_t r_size, const int64_t *slot_base,
                      const int32_t *fact_dst, const float *fact_val, const int16_t *fact_rel,
                      const int32_t *fact_edge, int64_t total_slots, int32_t *fact_pos, int64_t *out_row_ptr,
                      int32_t *out_ent, float *out_x, int max_flags, int32_t *status, void *ws, size_t ws_bytes,
                      fl_stream_t stream) {
    return row_reduce_max(row_ptr, rows, E, r_size, slot_base, fact_dst, fact_val, fact_rel, fact_edge, total_slots,
                          fact_pos, out_row_ptr, out_ent, out_x, (max_flags & FL_MAX_BITS) ? 2 : 1,
                          (max_flags & FL_MAX_VALUE_ONLY) != 0, status, ws, ws_bytes, as_stream(stream));
}

int fl_row_reduce(const int64_t *row_ptr, int64_t rows, int64_t E, const int64_t *slot_base, const int32_t *entry_count,
                  const int32_t *fact_dst, const float *fact_val, int64_t total_slots, int32_t *fact_pos, float eps,
                  int64_t *out_row_ptr, int32_t *out_ent, float *out_x, float *out_y, float *out_denom,
                  int32_t *status, const int32_t *row_order, void *ws, size_t ws_bytes, const fl_dropout *drop,
                  fl_stream_t stream) {
    return row_reduce(row_ptr, rows, E, slot_base, entry_count, fact_dst, fact_val, total_slots, fact_pos, eps,
                      out_row_ptr, out_ent, out_x, out_y, out_denom, status, row_order, ws, ws_bytes, drop,
                      as_stream(stream));
}

size_t fl_hop_backward_workspace(int64_t rows, int64_t n) { return hop_backward_workspace(rows, n); }

int fl_hop_backward(const fl_hop_params *p, const int64_t *row_ptr, const float *val, int64_t S, const float *w,
                    const int64_t *slot_base, const int32_t *entry_count, const int32_t *fact_pos,
                    const int16_t *fact_rel, const float *fact_m, const int64_t *out_row_ptr, const float *out_x,
                    const float *out_denom, const float *g_y, float *grad_val, float *grad_w, void *ws,
                    size_t ws_bytes, fl_stream_t stream) {
    FL_REQUIRE(p != nullptr, "null params");
    return hop_backward(p, row_ptr, val, S, w, slot_base, entry_count, fact_pos, fact_rel, fact_m, out_row_ptr, out_x,
                        out_denom, g_y, grad_val, grad_w, ws, ws_bytes, as_stream(stream));
}

int fl_normalize_forward(const int64_t *row_ptr, const float *x, int64_t rows, float eps, float *y, float *denom,
                         fl_stream_t stream) {
    return normalize_forward(row_ptr, x, rows, eps, y, denom, as_stream(stream));
}

int fl_normalize_backward(const int64_t *row_ptr, const float *x, const float *denom, const float *g, int64_t rows,
                          float eps, float *gx, fl_stream_t stream) {
    return normalize_backward(row_ptr, x, denom, g, rows, eps, gx, as_stream(stream));
}

int fl_hop_stats(const int64_t *row_ptr, int64_t rows, const int32_t *ent, int64_t S, fl_csr_side ori,
                 fl_csr_side inv, const int32_t *entry_count, const int64_t *out_row_ptr, int wot_i, int64_t *acc,
                 fl_stream_t stream) {
    FL_REQUIRE(acc != nullptr && rows >= 0 && S >= 0, "fl_hop_stats: bad arguments");
    return hop_stats(row_ptr, rows, ent, S, ori, inv, entry_count, out_row_ptr, wot_i, acc, as_stream(stream));
}

int fl_edge_weight_grad(const fl_hop_params *p, const int64_t *row_ptr, const float *val, int64_t S, const float *w,
                        const int64_t *slot_base, const int32_t *entry_count, const int32_t *fact_pos,
                        const int16_t *fact_rel, const float *fact_m, const int32_t *fact_edge,
                        const int64_t *out_row_ptr, const float *g, const float *edge_weight, float *grad_edge,
                        fl_stream_t stream) {
    return edge_weight_grad(p, row_ptr, val, S, w, slot_base, entry_count, fact_pos, fact_rel, fact_m, fact_edge,
                            out_row_ptr, g, edge_weight, grad_edge, as_stream(stream));
}

int fl_scatter_grad(const float *grad_sel, const int64_t *src_index, int64_t n_sel, const int64_t *n_live,
                    float *grad_full, int64_t n_full, const int64_t *full_live, const fl_dropout *drop,
                    fl_stream_t stream) {
    return scatter_grad(grad_sel, src_index, n_sel, n_live, grad_full, n_full, full_live, drop, as_stream(stream));
}

size_t fl_fixed_relation_workspace(int64_t nnz) { return fixed_relation_workspace(nnz); }

int fl_fixed_relation_plan(const int64_t *b, const int64_t *l, const int32_t *ent, int64_t nnz, const int64_t *ops,
                           int64_t Lr, int64_t r_size, fl_csr_side ori, fl_csr_side inv, int64_t *slot_base,
                           int64_t *total, void *ws, size_t ws_bytes, fl_stream_t stream) {
    return fixed_relation_plan(b, l, ent, nnz, ops, Lr, r_size, ori, inv, slot_base, total, ws, ws_bytes,
                               as_stream(stream));
}

int fl_fixed_relation_fill(const int64_t *b, const int64_t *l, const int32_t *ent, const float *val, int64_t nnz,
                           const int64_t *ops, int64_t Lr, int64_t r_size, fl_csr_side ori, fl_csr_side inv,
                           const int64_t *slot_base, int32_t *fact_dst, float *fact_val, int32_t *entry_count,
                           fl_stream_t stream) {
    return fixed_relation_fill(b, l, ent, val, nnz, ops, Lr, r_size, ori, inv, slot_base, fact_dst, fact_val,
                               entry_count, as_stream(stream));
}

size_t fl_filtered_ranks_workspace(int64_t B) { return filtered_ranks_workspace(B); }

int fl_rule_max_reduce(const int64_t *row_ptr, int64_t rows, const int32_t *ent, const float *val, int64_t C,
                       const float *weights, int64_t ranks, int64_t B, int64_t E, uint32_t *acc, fl_stream_t stream) {
    return rule_max_reduce(row_ptr, rows, ent, val, C, weights, ranks, B, E, acc, as_stream(stream));
}

int fl_rule_rank_facts(const int64_t *st_rp, const int32_t *st_ent, const float *st_val, int64_t B, int64_t C,
                       const float *w, int64_t ranks, const int64_t *run_rp, const int32_t *run_ent,
                       const float *run_val, int64_t *slot_base, int32_t *fact_dst, float *fact_val,
                       fl_stream_t stream) {
    return rule_rank_facts(st_rp, st_ent, st_val, B, C, w, ranks, run_rp, run_ent, run_val, slot_base, fact_dst,
                           fact_val, as_stream(stream));
}

int fl_rule_instance_facts(const int64_t *st_rp, const int32_t *st_ent, const int64_t *q_inst, int64_t B,
                           const float *w, int64_t ranks, int64_t *slot_base, int32_t *fact_dst, float *fact_val,
                           fl_stream_t stream) {
    return rule_instance_facts(st_rp, st_ent, q_inst, B, w, ranks, slot_base, fact_dst, fact_val, as_stream(stream));
}

int fl_fixed_relation_bitmap(const int64_t *entries, int64_t n, const int64_t *entry_row, const int32_t *row_slot,
                             const int32_t *ent, const int64_t *ops, int64_t r_size, fl_csr_side ori,
                             fl_csr_side inv, uint32_t *bitmap, int64_t words, fl_stream_t stream) {
    return fixed_relation_bitmap(entries, n, entry_row, row_slot, ent, ops, r_size, ori, inv, bitmap, words,
                                 as_stream(stream));
}

int fl_rule_instance_max(const int64_t *st_rp, const int32_t *st_ent, const int64_t *q_inst, int64_t nq,
                         const float *w, int64_t ranks, int64_t E, uint32_t *acc, fl_stream_t stream) {
    return rule_instance_max(st_rp, st_ent, q_inst, nq, w, ranks, E, acc, as_stream(stream));
}

int fl_rows_copy(const int64_t *src_rp, const int32_t *src_ent, int64_t rows, const int64_t *dst_rp, int32_t *dst_ent,
                 fl_stream_t stream) {
    return rows_copy(src_rp, src_ent, rows, dst_rp, dst_ent, as_stream(stream));
}

size_t fl_bitmap_rows_workspace(int64_t nb, int64_t words) { return bitmap_rows_workspace(nb, words); }

int fl_bitmap_rows_count(const uint32_t *bitmap, int64_t nb, int64_t words, int64_t *chunk_off, int64_t *row_ptr,
                         void *ws, size_t ws_bytes, fl_stream_t stream) {
    return bitmap_rows_count(bitmap, nb, words, chunk_off, row_ptr, ws, ws_bytes, as_stream(stream));
}

int fl_bitmap_rows_emit(const uint32_t *bitmap, int64_t nb, int64_t words, const int64_t *chunk_off, int32_t *ent,
                        fl_stream_t stream) {
    return bitmap_rows_emit(bitmap, nb, words, chunk_off, ent, as_stream(stream));
}

int fl_filtered_ranks(const int64_t *idx_b, const int64_t *idx_e, const float *values, int64_t nnz,
                      const int64_t *targets, const int64_t *filter_keys, int64_t n_filter, int64_t B, int64_t E,
                      int use_eql, float *ranks, void *ws, size_t ws_bytes, fl_stream_t stream) {
    return filtered_ranks(idx_b, idx_e, values, nnz, targets, filter_keys, n_filter, B, E, use_eql, ranks, ws, ws_bytes,
                          as_stream(stream));
}

int fl_filtered_ranks_noalloc(const int64_t *idx_b, const int64_t *idx_e, const float *values, int64_t nnz,
                              const int64_t *targets, const int64_t *filter_keys, int64_t n_filter, int64_t B,
                              int64_t E, int use_eql, float *ranks, fl_stream_t stream) {
    return filtered_ranks_noalloc(idx_b, idx_e, values, nnz, targets, filter_keys, n_filter, B, E, use_eql, ranks,
                                  as_stream(stream));
}

int fl_readout(const int64_t *row_ptr, const int32_t *ent, const float *val, int64_t N, const int64_t *targets,
               int64_t Q, float *scores, fl_stream_t stream) {
    return readout(row_ptr, ent, val, N, targets, Q, scores, as_stream(stream));
}

int fl_readout_backward(const int64_t *row_ptr, const int32_t *ent, int64_t N, const int64_t *targets, int64_t Q,
                        const float *g_scores, float *grad_val, int64_t n_val, const int64_t *val_live,
                        const fl_dropout *drop, fl_stream_t stream) {
    return readout_backward(row_ptr, ent, N, targets, Q, g_scores, grad_val, n_val, val_live, drop,
                            as_stream(stream));
}

int fl_value_dropout(const float *x, float *y, int64_t n, const int64_t *live, double p, uint64_t seed,
                     const int64_t *counter, uint64_t subseq, fl_stream_t st) {
    return value_dropout(x, y, n, live, p, seed, counter, subseq, as_stream(st));
}

}  // extern "C"
