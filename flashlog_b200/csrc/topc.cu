// topc.cu -- c1 entity budget per (query, channel) row.
//
// Semantics of the reference's _sparse_topc_entries
// (flashlog_kernel/flashlog_kernel.py:1092-1137): a row with at most c1
// nonzero values is kept whole (explicit zeros included); a row with more
// keeps exactly its c1 largest nonzero values, ties going to the lower entity
// (stable descending sort over the coalesced order).  In the sampled mode the
// score of a candidate is log(v) - log(noise) in fp64 (exponential race), with
// noise drawn by the caller in candidate order.
//
// B200 design: one CTA per row; an MSB-first radix select over order-
// preserving keys finds the c1-th key, and ordered block scans pick the tied
// entries by position, so the selection is exact and deterministic.
#include <math.h>

#include "common.cuh"
#include "scan.cuh"

namespace fl {
namespace {

constexpr int kSelThreads = 512;

__global__ void __launch_bounds__(256) topc_count_kernel(const int64_t *row_ptr, const float *val, int64_t rows,
                                                         int64_t c1, int64_t *kept, int64_t *cand) {
    __shared__ int64_t scratch[256 / 32 + 1];
    int64_t r = blockIdx.x;
    if (r >= rows) return;
    int64_t a = row_ptr[r], b = row_ptr[r + 1];
    int64_t nz = 0;
    for (int64_t i = a + threadIdx.x; i < b; i += blockDim.x) nz += (val[i] != 0.0f);
    nz = block_sum(nz, scratch);
    if (threadIdx.x == 0) {
        bool over = nz > c1;
        kept[r] = over ? c1 : (b - a);
        cand[r] = over ? nz : 0;
    }
}

template <bool kSampled>
struct KeyOf;

template <>
struct KeyOf<false> {
    using T = uint32_t;
    static constexpr int kBits = 32;
};
template <>
struct KeyOf<true> {
    using T = uint64_t;
    static constexpr int kBits = 64;
};

template <bool kSampled>
__global__ void __launch_bounds__(kSelThreads) topc_select_kernel(
    const int64_t *row_ptr, const int32_t *ent, const float *val, int64_t rows, int64_t c1,
    const double *noise, const int64_t *cand_off, const int64_t *out_row_ptr, const int64_t *kept_count,
    uint64_t *key_scratch, int32_t *out_ent, float *out_val, int64_t *out_src) {
    using Key = typename KeyOf<kSampled>::T;
    __shared__ unsigned int hist[256];
    __shared__ int64_t scan_scratch[kSelThreads / 32 + 1];
    __shared__ Key s_prefix;
    __shared__ int64_t s_krem;
    const int64_t r = blockIdx.x;
    if (r >= rows) return;
    const int64_t a = row_ptr[r], b = row_ptr[r + 1];
    const int64_t out0 = out_row_ptr[r];
    const int64_t out_end = out_row_ptr[r + 1];  // clamped to the output capacity
    const int64_t kept = kept_count[r];
    if (kept == b - a) {  // row kept whole (also covers empty rows)
        for (int64_t i = a + threadIdx.x; i < b && out0 + (i - a) < out_end; i += blockDim.x) {
            out_ent[out0 + (i - a)] = ent[i];
            out_val[out0 + (i - a)] = val[i];
            out_src[out0 + (i - a)] = i;
        }
        return;
    }
    // Keys of nonzero candidates.  Sampled keys need the candidate's rank in
    // state order (noise index), computed with an ordered block scan.
    if (kSampled) {
        int64_t carry = cand_off[r];
        for (int64_t base = a; base < b; base += blockDim.x) {
            int64_t i = base + threadIdx.x;
            bool nz = i < b && val[i] != 0.0f;
            int64_t tot;
            int64_t ex = block_exclusive_scan<int64_t>(nz ? 1 : 0, scan_scratch, &tot);
            if (nz) {
                double sc = log(static_cast<double>(val[i])) - log(noise[carry + ex]);
                key_scratch[i] = double_order_key(sc);
            }
            carry += tot;
        }
        __syncthreads();
    }
    auto key_at = [&](int64_t i) -> Key {
        if constexpr (kSampled) return static_cast<Key>(key_scratch[i]);
        else return static_cast<Key>(float_order_key(val[i]));
    };
    if (threadIdx.x == 0) { s_prefix = 0; s_krem = c1; }
    __syncthreads();
    Key prefix_mask = 0;
    for (int shift = KeyOf<kSampled>::kBits - 8; shift >= 0; shift -= 8) {
        for (int d = threadIdx.x; d < 256; d += blockDim.x) hist[d] = 0;
        __syncthreads();
        const Key prefix = s_prefix;
        for (int64_t i = a + threadIdx.x; i < b; i += blockDim.x) {
            if (val[i] == 0.0f) continue;
            Key k = key_at(i);
            if ((k & prefix_mask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            int64_t krem = s_krem;
            for (int d = 255; d >= 0; --d) {
                if (krem <= static_cast<int64_t>(hist[d])) { s_prefix = prefix | (static_cast<Key>(d) << shift); break; }
                krem -= hist[d];
            }
            s_krem = krem;
        }
        prefix_mask |= static_cast<Key>(255) << shift;
        __syncthreads();
    }
    const Key thr = s_prefix;
    const int64_t take_ties = s_krem;  // entries equal to thr to keep, by position
    int64_t tie_carry = 0, out_carry = 0;
    for (int64_t base = a; base < b; base += blockDim.x) {
        int64_t i = base + threadIdx.x;
        bool nz = i < b && val[i] != 0.0f;
        Key k = nz ? key_at(i) : Key(0);
        bool tie = nz && k == thr;
        int64_t ttot;
        int64_t tex = block_exclusive_scan<int64_t>(tie ? 1 : 0, scan_scratch, &ttot);
        bool keep = nz && (k > thr || (tie && tie_carry + tex < take_ties));
        int64_t ktot;
        int64_t kex = block_exclusive_scan<int64_t>(keep ? 1 : 0, scan_scratch, &ktot);
        if (keep && out0 + out_carry + kex < out_end) {
            int64_t o = out0 + out_carry + kex;
            out_ent[o] = ent[i];
            out_val[o] = val[i];
            out_src[o] = i;
        }
        tie_carry += ttot;
        out_carry += ktot;
    }
}

// Clamp the output row offsets to the buffers' capacity (rows past it become
// empty or truncated) and flag the overflow.
__global__ void clamp_rows_kernel(int64_t *row_ptr, int64_t rows, int64_t cap, int32_t *status) {
    int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (r > rows) return;
    if (row_ptr[r] > cap) {
        row_ptr[r] = cap;
        if (status && r == rows) atomicOr(status, FL_STATUS_SLOT_OVERFLOW);
    }
}

}  // namespace

size_t topc_workspace(int64_t rows, int64_t S) {
    return carve_bytes<int64_t>(rows + 1) * 4 + carve_bytes<uint64_t>(S > 0 ? S : 1) +
           scan_workspace(rows) + 1024;
}

int topc_counts(const int64_t *row_ptr, const float *val, int64_t rows, int64_t c1, int64_t *out_row_ptr,
                int64_t *cand_off, int64_t **kept_out, Carve &c, cudaStream_t st) {
    int64_t *kept = c.take<int64_t>(rows + 1);
    *kept_out = kept;
    int64_t *cand = c.take<int64_t>(rows + 1);
    size_t sws = scan_workspace(rows);
    void *scan_ws = c.take<char>(sws);
    FL_REQUIRE(kept && cand && scan_ws, "topc workspace too small");
    if (rows > 0) launch(topc_count_kernel, static_cast<unsigned>(rows), 256, 0, st, row_ptr, val, rows, c1, kept, cand);
    int rc = exclusive_scan<int64_t>(kept, rows, out_row_ptr, scan_ws, sws, st);
    if (rc) return rc;
    rc = exclusive_scan<int64_t>(cand, rows, cand_off, scan_ws, sws, st);
    if (rc) return rc;
    return check_launch("topc_count");
}

int topc_select(const int64_t *row_ptr, const int32_t *ent, const float *val, int64_t rows, int64_t S,
                int64_t c1, const double *noise, int64_t *out_row_ptr, int32_t *out_ent, float *out_val,
                int64_t *out_src, int64_t out_capacity, int32_t *status, void *ws, size_t ws_bytes, cudaStream_t st) {
    FL_REQUIRE(c1 >= 0, "topk_nodes/c must be nonnegative");
    Carve c(ws, ws_bytes);
    int64_t *cand_off = c.take<int64_t>(rows + 1);
    uint64_t *keys = c.take<uint64_t>(noise ? (S > 0 ? S : 1) : 1);
    FL_REQUIRE(cand_off && keys, "topc workspace too small");
    int64_t *kept = nullptr;
    int rc = topc_counts(row_ptr, val, rows, c1, out_row_ptr, cand_off, &kept, c, st);
    if (rc) return rc;
    if (rows == 0) return FL_OK;
    const int64_t cap = out_capacity > 0 ? out_capacity : S;
    launch(clamp_rows_kernel, static_cast<unsigned>((rows + 1 + 255) / 256), 256, 0, st, out_row_ptr, rows, cap, status);
    if (noise)
        launch(topc_select_kernel<true>, static_cast<unsigned>(rows), kSelThreads, 0, st, 
            row_ptr, ent, val, rows, c1, noise, cand_off, out_row_ptr, kept, keys, out_ent, out_val, out_src);
    else
        launch(topc_select_kernel<false>, static_cast<unsigned>(rows), kSelThreads, 0, st, 
            row_ptr, ent, val, rows, c1, nullptr, cand_off, out_row_ptr, kept, keys, out_ent, out_val, out_src);
    return check_launch("topc_select");
}

int topc_candidates(const int64_t *row_ptr, const float *val, int64_t rows, int64_t S, int64_t c1,
                    int64_t *n_candidates, void *ws, size_t ws_bytes, cudaStream_t st) {
    Carve c(ws, ws_bytes);
    int64_t *cand_off = c.take<int64_t>(rows + 1);
    int64_t *kept_ptr = c.take<int64_t>(rows + 1);
    FL_REQUIRE(cand_off && kept_ptr, "topc workspace too small");
    int64_t *kept = nullptr;
    int rc = topc_counts(row_ptr, val, rows, c1, kept_ptr, cand_off, &kept, c, st);
    if (rc) return rc;
    FL_CUDA(cudaMemcpyAsync(n_candidates, cand_off + rows, sizeof(int64_t), cudaMemcpyDeviceToHost, st));
    FL_CUDA(cudaStreamSynchronize(st));
    return FL_OK;
}

}  // namespace fl
