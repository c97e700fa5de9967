// rules.cu -- rule-bank evaluator kernels.
//
//   fixed-operator step   flashlog_kernel/source/flashlog.cu:1561-1741 (one
//                         operator per (query, rule) row: forward relation,
//                         inverse relation + R, or identity 2R; the value is
//                         copied) followed by the coalesce-sum of
//                         flashlog_kernel.py:206-210.  The facts go through
//                         the same per-row stable-sort reduction as a hop.
//   filtered ranks        flashlog.cu:2754-2910 (tie-averaged rank that also
//                         counts the implicit zeros when the truth is 0).
#include <mutex>

#include "common.cuh"
#include "scan.cuh"

namespace fl {
namespace {

struct SideR {
    const int32_t *col, *gptr, *gstart, *gcount;
    const int16_t *grel;
};

__device__ __forceinline__ int64_t find_group(const SideR &s, int64_t src, int rel) {
    int64_t lo = s.gptr[src], hi = s.gptr[src + 1];
    const int64_t end = hi;
    while (lo < hi) {
        int64_t mid = lo + (hi - lo) / 2;
        if (static_cast<int>(s.grel[mid]) < rel) lo = mid + 1; else hi = mid;
    }
    return (lo < end && static_cast<int>(s.grel[lo]) == rel) ? lo : -1;
}

__global__ void fixed_count_kernel(const int64_t *b, const int64_t *l, const int32_t *ent, int64_t nnz,
                                   const int64_t *ops, int64_t Lr, int64_t R, SideR ori, SideR inv, int64_t *cnt) {
    int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= nnz) return;
    const int64_t op = ops[b[i] * Lr + (l != nullptr ? l[i] : 0)];
    if (op == 2 * R) { cnt[i] = 1; return; }
    const bool inv_dir = op >= R;
    const int rel = static_cast<int>(inv_dir ? op - R : op);
    const SideR &s = inv_dir ? inv : ori;
    const int64_t g = find_group(s, ent[i], rel);
    cnt[i] = g < 0 ? 0 : s.gcount[g];
}

// One warp per entry: copy the group's destinations (coalesced int32 loads).
__global__ void fixed_fill_kernel(const int64_t *b, const int64_t *l, const int32_t *ent, const float *val,
                                  int64_t nnz, const int64_t *ops, int64_t Lr, int64_t R, SideR ori, SideR inv,
                                  const int64_t *slot_base, int32_t *fact_dst, float *fact_val, int32_t *entry_count) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); i < nnz; i += nw) {
        const int64_t op = ops[b[i] * Lr + (l != nullptr ? l[i] : 0)];
        const int64_t out = slot_base[i];
        const float v = val != nullptr ? val[i] : 1.0f;
        if (op == 2 * R) {
            if (lane == 0) { fact_dst[out] = ent[i]; fact_val[out] = v; entry_count[i] = 1; }
            continue;
        }
        const bool inv_dir = op >= R;
        const int rel = static_cast<int>(inv_dir ? op - R : op);
        const SideR &s = inv_dir ? inv : ori;
        const int64_t g = find_group(s, ent[i], rel);
        const int64_t c = g < 0 ? 0 : s.gcount[g];
        const int64_t p0 = g < 0 ? 0 : s.gstart[g];
        for (int64_t k = lane; k < c; k += 32) {
            fact_dst[out + k] = s.col[p0 + k];
            fact_val[out + k] = v;
        }
        if (lane == 0) entry_count[i] = static_cast<int32_t>(c);
    }
}

__device__ __forceinline__ bool bsearch64(const int64_t *keys, int64_t n, int64_t key) {
    int64_t lo = 0, hi = n;
    while (lo < hi) {
        int64_t mid = lo + ((hi - lo) >> 1);
        if (keys[mid] < key) lo = mid + 1; else hi = mid;
    }
    return lo < n && keys[lo] == key;
}

// Score entries and filter keys whose query lies outside [0, B) are skipped
// (the reference does not check them); the counters are never indexed by them.
__global__ void ranks_truth_kernel(const int64_t *ib, const int64_t *ie, const float *v, int64_t nnz,
                                   const int64_t *targets, int64_t B, float *truth) {
    int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= nnz) return;
    const int64_t b = ib[i];
    if (b >= 0 && b < B && ie[i] == targets[b]) truth[b] = v[i];
}

__global__ void ranks_filter_kernel(const int64_t *fk, int64_t nf, int64_t E, int64_t B, int32_t *fcount) {
    int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= nf || fk[i] < 0) return;
    const int64_t b = fk[i] / E;
    if (b < B) atomicAdd(&fcount[b], 1);
}

__global__ void ranks_count_kernel(const int64_t *ib, const int64_t *ie, const float *v, int64_t nnz,
                                   const float *truth, const int64_t *fk, int64_t nf, int64_t E, int64_t B,
                                   int32_t *greater, int32_t *equal, int32_t *expl) {
    int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= nnz) return;
    const int64_t b = ib[i];
    if (b < 0 || b >= B) return;
    if (bsearch64(fk, nf, b * E + ie[i])) return;
    const float t = truth[b];
    atomicAdd(&expl[b], 1);
    if (v[i] > t) atomicAdd(&greater[b], 1);
    else if (v[i] == t) atomicAdd(&equal[b], 1);
}

__global__ void ranks_finalize_kernel(const float *truth, const int32_t *greater, const int32_t *equal,
                                      const int32_t *expl, const int32_t *fcount, int64_t B, int64_t E, int use_eql,
                                      float *ranks) {
    int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (b >= B) return;
    if (use_eql) {
        // fp32 count arithmetic of flashlog.cu:2829-2834 (counts exact below 2^24)
        float missing = static_cast<float>(E) - static_cast<float>(fcount[b]) - static_cast<float>(expl[b]);
        float eq = static_cast<float>(equal[b]) + (truth[b] == 0.0f ? missing : 0.0f);
        eq += 1.0f;
        ranks[b] = static_cast<float>(greater[b]) + (eq + 1.0f) * 0.5f;
    } else {
        ranks[b] = static_cast<float>(greater[b]) + 1.0f;
    }
}

SideR make_side_r(const fl_csr_side &s) {
    SideR r;
    r.col = s.col; r.gptr = s.group_ptr; r.gstart = s.group_start; r.gcount = s.group_count; r.grel = s.group_rel;
    return r;
}

// Max-product rule scores (rules/shared_inference.py:123-206 with
// reduction 'max'): every reached (query, rule, entity) of a Boolean rule state
// raises acc[rank][query * E + entity] to the rule's rank weight.  Weights are
// finite and nonnegative, so the fp32 bit patterns order like the values and
// an unsigned atomic max is exact and order-independent.  One warp per
// (query, rule) row.
__global__ void rule_max_kernel(const int64_t *row_ptr, int64_t rows, const int32_t *ent, const float *val,
                                int64_t C, const float *weights, int64_t ranks, int64_t B, int64_t E,
                                unsigned int *acc) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
        const int64_t q = r / C, c = r % C;
        const int64_t a = row_ptr[r], b = row_ptr[r + 1];
        for (int64_t k = a + lane; k < b; k += 32) {
            if (val != nullptr && !(val[k] > 0.0f)) continue;
            const int64_t e = ent[k];
            for (int64_t rk = 0; rk < ranks; ++rk) {
                const unsigned int wbits = __float_as_uint(weights[c * ranks + rk]);
                if (wbits != 0u) atomicMax(acc + rk * B * E + q * E + e, wbits);
            }
        }
    }
}

// Row starts of the rank rows (q, r): the running maxima of the row, then r
// copies of query q's entries before it, after every earlier query's.
__global__ void rank_slots_kernel(const int64_t *st_rp, int64_t B, int64_t C, int64_t ranks, const int64_t *run_rp,
                                  int64_t *slot_base) {
    const int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (row > B * ranks) return;
    const int64_t q = row / ranks, r = row % ranks;
    const int64_t base = st_rp[q * C];
    const int64_t nq = q < B ? st_rp[(q + 1) * C] - base : 0;
    slot_base[row] = (run_rp != nullptr ? run_rp[row] : 0) + ranks * base + r * nq;
}

// One block per rank row (q, r): the running maxima, then the entries of the
// rule rows (q, c) in rule order with the weight of rule c at rank r.
__global__ void rank_facts_kernel(const int64_t *st_rp, const int32_t *st_ent, const float *st_val, int64_t C,
                                  const float *w, int64_t ranks, const int64_t *run_rp, const int32_t *run_ent,
                                  const float *run_val, const int64_t *slot_base, int32_t *fact_dst,
                                  float *fact_val) {
    const int64_t row = blockIdx.x;
    const int64_t q = row / ranks, r = row % ranks;
    int64_t s = slot_base[row];
    if (run_rp != nullptr) {
        const int64_t a = run_rp[row], n = run_rp[row + 1] - a;
        for (int64_t j = threadIdx.x; j < n; j += blockDim.x) {
            fact_dst[s + j] = run_ent[a + j];
            fact_val[s + j] = run_val[a + j];
        }
        s += n;
    }
    const int64_t base = st_rp[q * C];
    for (int64_t c = 0; c < C; ++c) {
        const int64_t a = st_rp[q * C + c], b = st_rp[q * C + c + 1];
        const float wv = w[c * ranks + r];
        for (int64_t i = a + threadIdx.x; i < b; i += blockDim.x) {
            const bool ok = wv != 0.0f && st_val[i] > 0.0f;
            fact_dst[s + (i - base)] = ok ? st_ent[i] : -1;
            fact_val[s + (i - base)] = wv;
        }
    }
}

// Rank-row starts of an instance-grouped state: query q owns the instance
// rows [q_inst[q], q_inst[q + 1]) and row (q, r) holds all their entries.
// Slots count from the first query's first entry.
__global__ void inst_slots_kernel(const int64_t *st_rp, const int64_t *q_inst, int64_t B, int64_t ranks,
                                  int64_t *slot_base) {
    const int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (row > B * ranks) return;
    const int64_t q = row / ranks, r = row % ranks;
    const int64_t base = st_rp[q_inst[q]];
    const int64_t nq = q < B ? st_rp[q_inst[q + 1]] - base : 0;
    slot_base[row] = ranks * (base - st_rp[q_inst[0]]) + r * nq;
}

// One block per rank row (q, r): the entries of the query's instance rows in
// instance order, each with its instance's weight at rank r.
__global__ void inst_facts_kernel(const int64_t *st_rp, const int32_t *st_ent, const int64_t *q_inst,
                                  const float *w, int64_t ranks, const int64_t *slot_base, int32_t *fact_dst,
                                  float *fact_val) {
    const int64_t row = blockIdx.x;
    const int64_t q = row / ranks, r = row % ranks;
    const int64_t s = slot_base[row];  // relative to the first query's first entry
    const int64_t c0 = q_inst[q], c1 = q_inst[q + 1];
    const int64_t base = st_rp[c0];
    for (int64_t c = c0; c < c1; ++c) {
        const int64_t a = st_rp[c], b = st_rp[c + 1];
        const float wv = w[c * ranks + r];
        for (int64_t i = a + threadIdx.x; i < b; i += blockDim.x) {
            fact_dst[s + (i - base)] = wv != 0.0f ? st_ent[i] : -1;
            fact_val[s + (i - base)] = wv;
        }
    }
}

// Dense rank maxima of an instance-grouped Boolean state (query q owns the
// instance rows [q_inst[q], q_inst[q + 1]), q < nq): for every entry of
// every instance, acc[(q * ranks + r) * E + entity] is raised to the fp32
// bits of the instance's weight at rank r.  The work is split by entries,
// not by instances (an instance can hold millions of entries): each warp
// takes runs of kMaxChunk consecutive entries, finds the instance of the
// first by binary search and walks forward from there.
constexpr int kMaxChunk = 256;
__global__ void inst_max_kernel(const int64_t *st_rp, const int32_t *st_ent, const int64_t *q_inst, int64_t nq,
                                const float *w, int64_t ranks, int64_t E, unsigned int *acc) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    const int64_t c_lo = q_inst[0], c_hi = q_inst[nq];
    const int64_t e0 = st_rp[c_lo], e1 = st_rp[c_hi];
    for (int64_t k0 = e0 + (blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5)) * kMaxChunk;
         k0 < e1; k0 += nw * kMaxChunk) {
        int64_t c = 0;
        if (lane == 0) {  // the instance holding entry k0: the last c with st_rp[c] <= k0
            int64_t lo = c_lo, hi = c_hi - 1;
            while (lo < hi) {
                const int64_t mid = (lo + hi + 1) >> 1;
                if (st_rp[mid] <= k0) lo = mid; else hi = mid - 1;
            }
            c = lo;
        }
        c = __shfl_sync(0xffffffffu, c, 0);
        int64_t q = 0;
        while (q_inst[q + 1] <= c) ++q;  // q < nq: q_inst[nq] = c_hi > c
        const int64_t k1 = (k0 + kMaxChunk) < e1 ? (k0 + kMaxChunk) : e1;
        for (int64_t k = k0 + lane; k < k1; k += 32) {
            while (st_rp[c + 1] <= k) ++c;  // c + 1 <= c_hi: st_rp[c_hi] = e1 > k
            while (q_inst[q + 1] <= c) ++q;
            const int64_t e = st_ent[k];
            unsigned int *aq = acc + q * ranks * E + e;
            for (int64_t r = 0; r < ranks; ++r) {
                const unsigned int wb = __float_as_uint(w[c * ranks + r]);
                if (wb != 0u) atomicMax(aq + r * E, wb);
            }
        }
    }
}

// Boolean fixed-operator step into per-row bitmaps (the rows of a rule
// state whose facts outnumber its bitmap's words): one warp per listed
// entry sets the bit of every destination of its row's operator.
__global__ void fixed_bitmap_kernel(const int64_t *entries, int64_t n, const int64_t *entry_row,
                                    const int32_t *row_slot, const int32_t *ent, const int64_t *ops, int64_t R,
                                    SideR ori, SideR inv, uint32_t *bitmap, int64_t words) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t k = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); k < n; k += nw) {
        const int64_t i = entries[k];
        const int64_t row = entry_row[i];
        uint32_t *bm = bitmap + static_cast<int64_t>(row_slot[row]) * words;
        const int64_t op = ops[row];
        const int32_t src = ent[i];
        if (op == 2 * R) {
            if (lane == 0) atomicOr(bm + (src >> 5), 1u << (src & 31));
            continue;
        }
        const bool inv_dir = op >= R;
        const int rel = static_cast<int>(inv_dir ? op - R : op);
        const SideR &sd = inv_dir ? inv : ori;
        const int64_t g = find_group(sd, src, rel);
        if (g < 0) continue;
        const int64_t c = sd.gcount[g], p0 = sd.gstart[g];
        for (int64_t t = lane; t < c; t += 32) {
            const int32_t d = sd.col[p0 + t];
            atomicOr(bm + (d >> 5), 1u << (d & 31));
        }
    }
}

// Row copy: one warp per row moves the row's entries to the row's start in
// another row layout (rows with no entries copy nothing).
__global__ void rows_copy_kernel(const int64_t *src_rp, const int32_t *src_ent, int64_t rows, const int64_t *dst_rp,
                                 int32_t *dst_ent) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += nw) {
        const int64_t a = src_rp[r], n = src_rp[r + 1] - a, d = dst_rp[r];
        for (int64_t k = lane; k < n; k += 32) dst_ent[d + k] = src_ent[a + k];
    }
}

// Set-bit counts of chunks of kBmChunk consecutive bitmap words, one block each.
constexpr int kBmChunk = 256;
__global__ void __launch_bounds__(kBmChunk) bitmap_count_kernel(const uint32_t *bm, int64_t *chunk_cnt) {
    __shared__ int64_t scratch[kBmChunk / 32 + 1];
    const int64_t c = blockIdx.x;
    const uint32_t w = bm[c * kBmChunk + threadIdx.x];
    int64_t tot;
    block_exclusive_scan<int64_t>(__popc(w), scratch, &tot);
    if (threadIdx.x == 0) chunk_cnt[c] = tot;
}

__global__ void bitmap_rowptr_kernel(const int64_t *chunk_off, int64_t nb, int64_t chunks_per_row, int64_t *row_ptr) {
    const int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (r <= nb) row_ptr[r] = chunk_off[r * chunks_per_row];
}

// The set bits of every row in ascending order: entity = word-in-row * 32 + bit.
__global__ void __launch_bounds__(kBmChunk) bitmap_emit_kernel(const uint32_t *bm, int64_t words,
                                                               const int64_t *chunk_off, int32_t *ent) {
    __shared__ int64_t scratch[kBmChunk / 32 + 1];
    const int64_t c = blockIdx.x;
    const int64_t wi = c * kBmChunk + threadIdx.x;
    uint32_t x = bm[wi];
    int64_t tot;
    int64_t o = block_exclusive_scan<int64_t>(__popc(x), scratch, &tot) + chunk_off[c];
    const int64_t base = (wi % words) * 32;
    while (x) {
        const int b = __ffs(x) - 1;
        x &= x - 1;
        ent[o++] = static_cast<int32_t>(base + b);
    }
}

}  // namespace

int rule_instance_max(const int64_t *st_rp, const int32_t *st_ent, const int64_t *q_inst, int64_t nq, const float *w,
                      int64_t ranks, int64_t E, unsigned int *acc, cudaStream_t st) {
    FL_REQUIRE(nq >= 0 && ranks > 0 && E > 0 && st_rp && q_inst && w && acc, "fl_rule_instance_max: bad arguments");
    if (nq > 0) {
        const int sms = fl_device_sm_count();
        launch(inst_max_kernel, static_cast<unsigned>((sms > 0 ? sms : 148) * 8), 256, 0, st, st_rp, st_ent, q_inst,
               nq, w, ranks, E, acc);
    }
    return check_launch("rule_instance_max");
}

int rows_copy(const int64_t *src_rp, const int32_t *src_ent, int64_t rows, const int64_t *dst_rp, int32_t *dst_ent,
              cudaStream_t st) {
    FL_REQUIRE(rows >= 0 && (rows == 0 || (src_rp && dst_rp)), "fl_rows_copy: bad arguments");
    if (rows > 0) {
        const int sms = fl_device_sm_count();
        int64_t blocks = (rows + 7) / 8;
        const int64_t cap = static_cast<int64_t>(sms > 0 ? sms : 148) * 16;
        if (blocks > cap) blocks = cap;
        launch(rows_copy_kernel, static_cast<unsigned>(blocks), 256, 0, st, src_rp, src_ent, rows, dst_rp, dst_ent);
    }
    return check_launch("rows_copy");
}

size_t bitmap_rows_workspace(int64_t nb, int64_t words) {
    const int64_t chunks = nb * (words / kBmChunk);
    return carve_bytes<int64_t>(chunks + 1) + scan_workspace(chunks) + 1024;
}

int fixed_relation_bitmap(const int64_t *entries, int64_t n, const int64_t *entry_row, const int32_t *row_slot,
                          const int32_t *ent, const int64_t *ops, int64_t R, const fl_csr_side &ori,
                          const fl_csr_side &inv, uint32_t *bitmap, int64_t words, cudaStream_t st) {
    FL_REQUIRE(n >= 0 && words > 0 && (n == 0 || (entries && entry_row && row_slot && ent && ops && bitmap)),
               "fl_fixed_relation_bitmap: bad arguments");
    if (n > 0) {
        const int sms = fl_device_sm_count();
        int64_t blocks = (n + 7) / 8;
        const int64_t cap = static_cast<int64_t>(sms > 0 ? sms : 148) * 16;
        if (blocks > cap) blocks = cap;
        launch(fixed_bitmap_kernel, static_cast<unsigned>(blocks), 256, 0, st, entries, n, entry_row, row_slot, ent,
               ops, R, make_side_r(ori), make_side_r(inv), bitmap, words);
    }
    return check_launch("fixed_relation_bitmap");
}

int bitmap_rows_count(const uint32_t *bitmap, int64_t nb, int64_t words, int64_t *chunk_off, int64_t *row_ptr,
                      void *ws, size_t ws_bytes, cudaStream_t st) {
    FL_REQUIRE(nb >= 0 && words > 0 && words % kBmChunk == 0 && chunk_off && row_ptr,
               "fl_bitmap_rows_count: words must be a positive multiple of 256");
    const int64_t chunks = nb * (words / kBmChunk);
    FL_REQUIRE(chunks < (int64_t(1) << 31), "fl_bitmap_rows_count: too many bitmap words");
    Carve c(ws, ws_bytes);
    int64_t *cnt = c.take<int64_t>(chunks + 1);
    const size_t sws = scan_workspace(chunks);
    void *scan_ws = c.take<char>(sws);
    FL_REQUIRE(cnt && scan_ws, "fl_bitmap_rows_count: workspace too small");
    if (chunks > 0) launch(bitmap_count_kernel, static_cast<unsigned>(chunks), kBmChunk, 0, st, bitmap, cnt);
    int rc = exclusive_scan<int64_t>(cnt, chunks, chunk_off, scan_ws, sws, st);
    if (rc) return rc;
    launch(bitmap_rowptr_kernel, static_cast<unsigned>((nb + 1 + 255) / 256), 256, 0, st, chunk_off, nb,
           words / kBmChunk, row_ptr);
    return check_launch("bitmap_rows_count");
}

int bitmap_rows_emit(const uint32_t *bitmap, int64_t nb, int64_t words, const int64_t *chunk_off, int32_t *ent,
                     cudaStream_t st) {
    FL_REQUIRE(nb >= 0 && words > 0 && words % kBmChunk == 0 && chunk_off, "fl_bitmap_rows_emit: bad arguments");
    const int64_t chunks = nb * (words / kBmChunk);
    if (chunks > 0) launch(bitmap_emit_kernel, static_cast<unsigned>(chunks), kBmChunk, 0, st, bitmap, words, chunk_off, ent);
    return check_launch("bitmap_rows_emit");
}

int rule_instance_facts(const int64_t *st_rp, const int32_t *st_ent, const int64_t *q_inst, int64_t B,
                        const float *w, int64_t ranks, int64_t *slot_base, int32_t *fact_dst, float *fact_val,
                        cudaStream_t st) {
    FL_REQUIRE(B >= 0 && ranks > 0 && st_rp && q_inst && slot_base && w, "fl_rule_instance_facts: bad arguments");
    const int64_t rows = B * ranks;
    launch(inst_slots_kernel, static_cast<unsigned>((rows + 1 + 255) / 256), 256, 0, st, st_rp, q_inst, B, ranks,
           slot_base);
    if (rows > 0)
        launch(inst_facts_kernel, static_cast<unsigned>(rows), 256, 0, st, st_rp, st_ent, q_inst, w, ranks, slot_base,
               fact_dst, fact_val);
    return check_launch("rule_instance_facts");
}

int rule_rank_facts(const int64_t *st_rp, const int32_t *st_ent, const float *st_val, int64_t B, int64_t C,
                    const float *w, int64_t ranks, const int64_t *run_rp, const int32_t *run_ent, const float *run_val,
                    int64_t *slot_base, int32_t *fact_dst, float *fact_val, cudaStream_t st) {
    FL_REQUIRE(B >= 0 && C > 0 && ranks > 0 && st_rp && slot_base && w, "fl_rule_rank_facts: bad arguments");
    const int64_t rows = B * ranks;
    launch(rank_slots_kernel, static_cast<unsigned>((rows + 1 + 255) / 256), 256, 0, st, st_rp, B, C, ranks, run_rp,
           slot_base);
    if (rows > 0)
        launch(rank_facts_kernel, static_cast<unsigned>(rows), 256, 0, st, st_rp, st_ent, st_val, C, w, ranks, run_rp,
               run_ent, run_val, slot_base, fact_dst, fact_val);
    return check_launch("rule_rank_facts");
}

size_t fixed_relation_workspace(int64_t nnz) { return carve_bytes<int64_t>(nnz + 1) + scan_workspace(nnz) + 1024; }

int fixed_relation_plan(const int64_t *b, const int64_t *l, const int32_t *ent, int64_t nnz, const int64_t *ops,
                        int64_t Lr, int64_t R, const fl_csr_side &ori, const fl_csr_side &inv, int64_t *slot_base,
                        int64_t *total, void *ws, size_t ws_bytes, cudaStream_t st) {
    Carve c(ws, ws_bytes);
    int64_t *cnt = c.take<int64_t>(nnz + 1);
    size_t sws = scan_workspace(nnz);
    void *scan_ws = c.take<char>(sws);
    FL_REQUIRE(cnt && scan_ws, "fixed_relation workspace too small");
    if (nnz > 0)
        launch(fixed_count_kernel, static_cast<unsigned>((nnz + 255) / 256), 256, 0, st, 
            b, l, ent, nnz, ops, Lr, R, make_side_r(ori), make_side_r(inv), cnt);
    int rc = exclusive_scan<int64_t>(cnt, nnz, slot_base, scan_ws, sws, st);
    if (rc) return rc;
    FL_CUDA(cudaMemcpyAsync(total, slot_base + nnz, sizeof(int64_t), cudaMemcpyDeviceToHost, st));
    FL_CUDA(cudaStreamSynchronize(st));
    return check_launch("fixed_relation_plan");
}

int fixed_relation_fill(const int64_t *b, const int64_t *l, const int32_t *ent, const float *val, int64_t nnz,
                        const int64_t *ops, int64_t Lr, int64_t R, const fl_csr_side &ori, const fl_csr_side &inv,
                        const int64_t *slot_base, int32_t *fact_dst, float *fact_val, int32_t *entry_count,
                        cudaStream_t st) {
    if (nnz == 0) return FL_OK;
    int64_t blocks = (nnz + 7) / 8;
    if (blocks > 148 * 32) blocks = 148 * 32;
    launch(fixed_fill_kernel, static_cast<unsigned>(blocks), 256, 0, st, b, l, ent, val, nnz, ops, Lr, R, make_side_r(ori),
                                                                    make_side_r(inv), slot_base, fact_dst, fact_val,
                                                                    entry_count);
    return check_launch("fixed_relation_fill");
}

size_t filtered_ranks_workspace(int64_t B) { return carve_bytes<float>(B) + 4 * carve_bytes<int32_t>(B) + 1024; }

int rule_max_reduce(const int64_t *row_ptr, int64_t rows, const int32_t *ent, const float *val, int64_t C,
                    const float *weights, int64_t ranks, int64_t B, int64_t E, unsigned int *acc, cudaStream_t st) {
    FL_REQUIRE(C > 0 && ranks > 0 && B >= 0 && E > 0 && rows == B * C, "rule_max_reduce: bad sizes");
    if (rows > 0) {
        const int sms = fl_device_sm_count();
        int64_t blocks = (rows + 7) / 8;
        const int64_t cap = static_cast<int64_t>(sms > 0 ? sms : 148) * 16;
        if (blocks > cap) blocks = cap;
        launch(rule_max_kernel, static_cast<unsigned>(blocks), 256, 0, st, row_ptr, rows, ent, val, C, weights, ranks,
               B, E, acc);
    }
    return check_launch("rule_max_reduce");
}

int filtered_ranks(const int64_t *ib, const int64_t *ie, const float *v, int64_t nnz, const int64_t *targets,
                   const int64_t *fk, int64_t nf, int64_t B, int64_t E, int use_eql, float *ranks, void *ws,
                   size_t ws_bytes, cudaStream_t st) {
    Carve c(ws, ws_bytes);
    float *truth = c.take<float>(B);
    int32_t *greater = c.take<int32_t>(B), *equal = c.take<int32_t>(B), *expl = c.take<int32_t>(B),
            *fcount = c.take<int32_t>(B);
    FL_REQUIRE(truth && greater && equal && expl && fcount, "filtered_ranks workspace too small");
    if (B == 0) return FL_OK;
    FL_CUDA(cudaMemsetAsync(truth, 0, B * sizeof(float), st));
    FL_CUDA(cudaMemsetAsync(greater, 0, B * sizeof(int32_t), st));
    FL_CUDA(cudaMemsetAsync(equal, 0, B * sizeof(int32_t), st));
    FL_CUDA(cudaMemsetAsync(expl, 0, B * sizeof(int32_t), st));
    FL_CUDA(cudaMemsetAsync(fcount, 0, B * sizeof(int32_t), st));
    if (nnz > 0)
        launch(ranks_truth_kernel, static_cast<unsigned>((nnz + 255) / 256), 256, 0, st, ib, ie, v, nnz, targets, B,
               truth);
    if (nf > 0) launch(ranks_filter_kernel, static_cast<unsigned>((nf + 255) / 256), 256, 0, st, fk, nf, E, B, fcount);
    if (nnz > 0)
        launch(ranks_count_kernel, static_cast<unsigned>((nnz + 255) / 256), 256, 0, st, ib, ie, v, nnz, truth, fk, nf, E,
               B, greater, equal, expl);
    launch(ranks_finalize_kernel, static_cast<unsigned>((B + 255) / 256), 256, 0, st, truth, greater, equal, expl, fcount, B,
                                                                                E, use_eql, ranks);
    return check_launch("filtered_ranks");
}

// ---------------------------------------------------------------------------
// Filtered ranks without any allocation.
//
// Some callers cannot allocate device memory at the moment they need ranks:
// a plain C host program that has no device allocator of its own, or code
// that must not call cudaMalloc because it synchronizes the whole device
// (for example a latency-sensitive evaluation loop running beside training
// on other streams).  This variant takes its per-query counters from a fixed
// array in the library's device memory instead of a caller workspace.
// ---------------------------------------------------------------------------
constexpr int64_t kNoAllocMaxQueries = 65536;  // 5 arrays x 64 Ki x 4 B = 1.25 MiB per device
static __device__ __align__(256) unsigned char g_rank_scratch[5 * kNoAllocMaxQueries * 4 + 5 * 256];

constexpr int kMaxDevices = 64;
static void *g_rank_scratch_addr[kMaxDevices];
static std::mutex g_rank_scratch_mutex;

static int rank_scratch_address(void **out) {
    int dev = 0;
    FL_CUDA(cudaGetDevice(&dev));
    FL_REQUIRE(dev >= 0 && dev < kMaxDevices, "device index %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_rank_scratch_mutex);
    if (g_rank_scratch_addr[dev] == nullptr) {
        // The symbol's host-side name is not a device address; look the
        // address up once per device, with that device current.  The address
        // stays valid while the device's primary context lives: a
        // cudaDeviceReset between calls would leave it stale, so callers of
        // fl_filtered_ranks_noalloc must not reset the device in between.
        void *p = nullptr;
        FL_CUDA(cudaGetSymbolAddress(&p, g_rank_scratch));
        g_rank_scratch_addr[dev] = p;
    }
    *out = g_rank_scratch_addr[dev];
    return FL_OK;
}

int filtered_ranks_noalloc(const int64_t *ib, const int64_t *ie, const float *v, int64_t nnz, const int64_t *targets,
                           const int64_t *fk, int64_t nf, int64_t B, int64_t E, int use_eql, float *ranks,
                           cudaStream_t st) {
    FL_REQUIRE(B >= 0 && B <= kNoAllocMaxQueries,
               "fl_filtered_ranks_noalloc handles at most %lld queries per call (got %lld); use fl_filtered_ranks",
               static_cast<long long>(kNoAllocMaxQueries), static_cast<long long>(B));
    void *scratch = nullptr;
    int rc = rank_scratch_address(&scratch);
    if (rc) return rc;
    // filtered_ranks clears every counter it uses before counting.
    return filtered_ranks(ib, ie, v, nnz, targets, fk, nf, B, E, use_eql, ranks, scratch, sizeof(g_rank_scratch), st);
}

}  // namespace fl
