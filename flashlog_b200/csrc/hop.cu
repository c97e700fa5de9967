// hop.cu -- one soft-grounding propagation hop on B200 (sm_100a).
//
// Reference semantics (paths relative to the reference project):
//   expansion   flashlog_kernel/source/flashlog.cu:1368-1559 (top-k fill,
//               c2 threshold 26-63 / 1342-1366, sampled quotas 1458-1528),
//               1743-1854 (all-edges fill, identity)
//   coalesce    flashlog_kernel/flashlog_kernel.py:258-357 (sum per key)
//   normalize   flashlog.cu:2480-2691, flashlog_kernel.py:536-607
//   backward    flashlog.cu:1856-1959, flashlog.cpp:991-1134
//
// B200 design.  The state is a row layout over r = b * L + l.  A warp expands
// one source entry: it finds the c2 threshold by a weighted radix select over
// the entry's relation groups, then streams the taken CSR edges with
// coalesced int32 loads and writes facts (dst, value, relation) into slots
// reserved by a prefix sum of per-entry capacities, in the reference's
// canonical order (ori groups, inv groups, identity).  One CTA then reduces
// each row: facts of a destination range are gathered into shared memory in
// canonical order, stably radix-sorted by destination and summed
// sequentially per destination, which reproduces the CPU reference's
// summation order exactly and needs no atomics.  Rows larger than one tile
// are split by a destination histogram; a range too dense to split is
// accumulated into a dense shared-memory window tile by tile, still in
// canonical order.  The backward accumulates grad_w with exact 128-bit
// fixed-point adds, so its result does not depend on thread order.
#include <math.h>

#include "common.cuh"
#include "hop.cuh"
#include "scan.cuh"

namespace fl {
namespace {

constexpr int64_t kNoBudget = int64_t(1) << 62;

struct Side {
    const int32_t *row_ptr, *col, *order, *gptr, *gstart, *gcount;
    const int16_t *grel;
    const float *mask_csr;
};

__device__ __forceinline__ int64_t find_row(const int64_t *row_ptr, int64_t rows, int64_t i) {
    int64_t lo = 0, hi = rows;  // largest r with row_ptr[r] <= i
    while (lo < hi) {
        int64_t mid = (lo + hi + 1) >> 1;
        if (row_ptr[mid] <= i) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// ---------------------------------------------------------------------------
// Plan: per-entry fact capacity (budget-capped degree per side + identity)
// and the entry's row.
// ---------------------------------------------------------------------------
// Per-entry record handed from the plan to the expansion: the entry's row and
// the group ranges of both sides.
struct EntryInfo {
    int32_t row, g0o, g1o, g0i, g1i;
};
static_assert(sizeof(EntryInfo) == FL_ENTRY_INFO_INTS * sizeof(int32_t), "entry record size of the C ABI");

__global__ void hop_capacity_kernel(const int32_t *ent, const int64_t *row_ptr, int64_t rows, int64_t S, Side ori,
                                    Side inv, int64_t topk, int wot_i, int sides, int64_t *cap, EntryInfo *info) {
    int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= S) return;
    if (i >= row_ptr[rows]) { cap[i] = 0; return; }  // beyond the live entries
    int64_t src = ent[i];
    // sides: bit 0 forward, bit 1 inverse; a disabled side gets an empty group range
    const int64_t g0o = ori.gptr[src], g1o = (sides & 1) ? ori.gptr[src + 1] : g0o;
    const int64_t g0i = inv.gptr[src], g1i = (sides & 2) ? inv.gptr[src + 1] : g0i;
    if (info) {
        EntryInfo e;
        e.row = static_cast<int32_t>(find_row(row_ptr, rows, i));
        e.g0o = static_cast<int32_t>(g0o); e.g1o = static_cast<int32_t>(g1o);
        e.g0i = static_cast<int32_t>(g0i); e.g1i = static_cast<int32_t>(g1i);
        info[i] = e;
    }
    // Groups of a source are contiguous in CSR order, so a side's degree
    // follows from its first group's start and its last group's end.
    int64_t d0 = g0o == g1o ? 0 : static_cast<int64_t>(ori.gstart[g1o - 1]) + ori.gcount[g1o - 1] - ori.gstart[g0o];
    int64_t d1 = g0i == g1i ? 0 : static_cast<int64_t>(inv.gstart[g1i - 1]) + inv.gcount[g1i - 1] - inv.gstart[g0i];
    if (topk < kNoBudget) { d0 = d0 < topk ? d0 : topk; d1 = d1 < topk ? d1 : topk; }
    cap[i] = d0 + d1 + (wot_i ? 0 : 1);
}

// Rows by descending slot count, ties to the lower row (a stable descending
// argsort of the per-row slot counts): one block sorts the keys
// (~count << 32 | row) ascending in shared memory by a bitonic network.
constexpr int kRowOrderMax = 16384;
__global__ void __launch_bounds__(1024) row_order_kernel(const int64_t *row_ptr, const int64_t *slot_base, int64_t rows,
                                                        int32_t *order) {
    extern __shared__ unsigned long long okey[];
    int m = 1;
    while (m < rows) m <<= 1;
    for (int i = threadIdx.x; i < m; i += blockDim.x) {
        unsigned long long k = ~0ull;
        if (i < rows) {
            const int64_t cnt = slot_base[row_ptr[i + 1]] - slot_base[row_ptr[i]];
            k = (static_cast<unsigned long long>(~static_cast<uint32_t>(cnt)) << 32) | static_cast<uint32_t>(i);
        }
        okey[i] = k;
    }
    __syncthreads();
    for (int k = 2; k <= m; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < m; i += blockDim.x) {
                const int l = i ^ j;
                if (l > i) {
                    const unsigned long long a = okey[i], b = okey[l];
                    const bool up = (i & k) == 0;
                    if ((a > b) == up) { okey[i] = b; okey[l] = a; }
                }
            }
            __syncthreads();
        }
    }
    for (int i = threadIdx.x; i < rows; i += blockDim.x) order[i] = static_cast<int32_t>(okey[i] & 0xffffffffull);
}

// CSR-ordered visibility of one side: vis[p] = mask_triple[order[p]].
__global__ void csr_visibility_kernel(const int32_t *order, int64_t m, const uint8_t *mask_triple, uint8_t *vis) {
    for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; p < m;
         p += static_cast<int64_t>(gridDim.x) * blockDim.x)
        vis[p] = mask_triple[order[p]] != 0 ? 1 : 0;
}

// ---------------------------------------------------------------------------
// Expansion.  Entries whose two sides have at most kTeam relation groups each
// (most entries) are expanded by 8-lane teams, four entries per warp; the
// others by a whole warp, with the entry's group keys staged in shared memory
// for the c2 threshold.
// ---------------------------------------------------------------------------
constexpr int kExpandWarps = 8;
constexpr int kTeam = 8;
constexpr int kBigPass = 0, kSmallPass = 1, kBothPasses = 2;  // work-queue passes of the expansion
constexpr int kTeamMaxSlots = 24;  // entries with more reserved slots go to the whole-warp path
constexpr int kStage = 1024;  // relation groups of one side staged per warp
constexpr int kRankBins = 512;  // bins of the rank select (WarpScratch::hist)
constexpr uint32_t kNoRank = 0xffffu;

struct WarpScratch {
    // radix select: weighted digit counts [0, 256) and group counts per digit
    // [256, 512); rank select: the weighted counts of 512 rank bins
    unsigned int hist[512];
    uint32_t ckey[32];        // threshold candidates
    uint32_t ccnt[32];
    int32_t incl[32];
    int32_t start[32];
    float prod[32];
    int32_t rel[32];
    int32_t quota[32];
};

// Per-warp staging of one side's group keys (fp32 weight bits, 0 when w <= 0)
// and counts clamped to the budget.  Clamping leaves the threshold and the
// take of every group unchanged: a clamped group alone reaches the budget.
struct StageBuf {
    uint32_t key[kStage];
    uint16_t cnt[kStage];
};
// The rank select's staging: each group's relation rank and clamped count
// (4 KB per warp, so four expansion CTAs fit on an SM).  After the select
// the taking groups are compacted in place: rank = group offset, cnt = take.
struct StageRank {
    uint16_t rank[kStage];
    uint16_t cnt[kStage];
};

struct ExpandArgs {
    const int64_t *row_ptr;
    const int32_t *ent;
    const float *val;
    int64_t S, rows, n, r_size, topk, flags, seed, L, capacity;
    int32_t *status;
    const float *w;
    Side ori, inv;
    const uint8_t *mask_triple;
    const uint8_t *vis_ori, *vis_inv;  // CSR-ordered visibility (may be null)
    const float *edge_weight;
    const int64_t *slot_base;
    const EntryInfo *info;             // may be null: rows and group ranges looked up
    const uint16_t *rel_rank;          // per (row, direction, relation): position in (w desc, id asc) order,
                                       // kNoRank for w <= 0; or null
    int32_t rank_bin;                  // relation ranks per bin of the rank select (ceil(r_size / kRankBins))
    const int32_t *rank_row;           // per row: the row whose ranks it uses, or null (itself)
    uint32_t *work;                    // work-queue counter (zeroed before the launch) or null
    int32_t *fact_dst;
    float *fact_val;
    int16_t *fact_rel;
    float *fact_m;
    int32_t *fact_edge;                // triple id per fact (0 for identity) or null: the MAX tie key
    int32_t *entry_count;
};

// Multiplier m and visibility of the fact at CSR position p.
__device__ __forceinline__ void fact_mask(const ExpandArgs &a, const Side &sd, const uint8_t *vis, int64_t p,
                                          bool drop_masked, bool edge_w, bool edge_score, float *m, bool *visible) {
    *m = 1.0f;
    *visible = true;
    if (vis != nullptr && !edge_w) {
        const bool mv = vis[p] != 0;
        *m = mv ? 1.0f : 0.0f;
        if (drop_masked && !mv) *visible = false;
    } else if (a.mask_triple) {
        const int64_t edge = sd.order[p];
        const bool mv = a.mask_triple[edge] != 0;
        *m = mv ? 1.0f : 0.0f;
        if (edge_w) {
            const float ew = a.edge_weight[edge];
            *m *= edge_score ? ew : 1.0f / (1.0f + expf(-ew));
        }
        if (drop_masked && !mv) *visible = false;
    } else if (sd.mask_csr) {
        *m = sd.mask_csr[p];
        if (drop_masked && *m == 0.0f) *visible = false;
    }
}

// Weighted order statistic over the groups' weights (flashlog.cu:26-63).
// Groups with w > 0 count with multiplicity group_count.  When their total
// exceeds the budget, returns true with *thr = the key T such that
// sum(count | key > T) < budget <= sum(count | key >= T) and *keep = the
// number of edges still to take at T; returns false when everything fits.
// Keys are the fp32 bit patterns of the (positive) weights.
__device__ __forceinline__ void group_key(const float *wdir, const Side &sd, int64_t g, int64_t g1, uint32_t *key,
                                          uint32_t *cnt) {
    *key = 0u;
    *cnt = 0u;
    if (g < g1) {
        const float wg = wdir[sd.grel[g]];
        if (wg > 0.0f) { *key = __float_as_uint(wg); *cnt = static_cast<uint32_t>(sd.gcount[g]); }
    }
}

// MSB-first radix select over 8-bit digits of n (key, count) pairs given by
// get(j, &key, &cnt); the total of the counts must exceed the budget.  Lanes
// with equal digits are merged with a warp match before the shared-memory
// add, so equal weights (groups of one relation share it) do not serialize.
// Once at most 32 groups share the selected prefix they are gathered into
// one lane each and the threshold is finished by all-pairs comparison.
template <typename Get>
__device__ void radix_threshold(int64_t n, int64_t budget, WarpScratch &ws, Get get, uint32_t *thr, int64_t *keep) {
    const int lane = threadIdx.x & 31;
    uint32_t prefix = 0, pmask = 0;
    int64_t krem = budget;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int d = lane; d < 512; d += 32) ws.hist[d] = 0;
        __syncwarp();
        for (int64_t cb = 0; cb < n; cb += 32) {
            uint32_t key, cnt;
            get(cb + lane, &key, &cnt);
            const bool part = cnt > 0u && (key & pmask) == prefix;
            const unsigned act = __ballot_sync(kFull, part);
            if (part) {
                const uint32_t d = (key >> shift) & 255u;
                const unsigned peers = __match_any_sync(act, d);
                const unsigned sum = __reduce_add_sync(peers, cnt);
                if (lane == __ffs(peers) - 1) {
                    atomicAdd(&ws.hist[d], sum);
                    atomicAdd(&ws.hist[256 + d], static_cast<unsigned>(__popc(peers)));
                }
            }
        }
        __syncwarp();
        // lane j owns digits 255 - 8j .. 248 - 8j (descending)
        int64_t part = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) part += ws.hist[255 - (lane * 8 + k)];
        const int64_t incl = warp_inclusive_scan(part);
        const int64_t excl = incl - part;
        const unsigned ball = __ballot_sync(kFull, incl >= krem && excl < krem);
        const int src_lane = __ffs(ball) - 1;  // exactly one lane crosses krem
        int digit = 0;
        int64_t above = 0;
        if (lane == src_lane) {
            int64_t acc = excl;
            for (int k = 0; k < 8; ++k) {
                const int d = 255 - (lane * 8 + k);
                const int64_t h = ws.hist[d];
                if (acc + h >= krem) { digit = d; above = acc; break; }
                acc += h;
            }
        }
        digit = __shfl_sync(kFull, digit, src_lane);
        above = __shfl_sync(kFull, above, src_lane);
        krem -= above;
        prefix |= static_cast<uint32_t>(digit) << shift;
        pmask |= 255u << shift;
        const unsigned ncand = ws.hist[256 + digit];
        __syncwarp();
        if (shift > 0 && ncand <= 32u) {
            unsigned running = 0;
            for (int64_t cb = 0; cb < n; cb += 32) {
                uint32_t key, cnt;
                get(cb + lane, &key, &cnt);
                const bool cand = cnt > 0u && (key & pmask) == prefix;
                const unsigned b = __ballot_sync(kFull, cand);
                if (cand) {
                    const unsigned p = running + __popc(b & lanemask_lt());
                    ws.ckey[p] = key;
                    ws.ccnt[p] = cnt;
                }
                running += __popc(b);
            }
            __syncwarp();
            const uint32_t key = static_cast<unsigned>(lane) < ncand ? ws.ckey[lane] : 0u;
            const int64_t cnt = static_cast<unsigned>(lane) < ncand ? static_cast<int64_t>(ws.ccnt[lane]) : 0;
            int64_t ge = 0, gt = 0;
#pragma unroll 8
            for (int j = 0; j < 32; ++j) {
                const uint32_t kj = __shfl_sync(kFull, key, j);
                const int64_t cj = __shfl_sync(kFull, cnt, j);
                ge += kj >= key ? cj : 0;
                gt += kj > key ? cj : 0;
            }
            const unsigned q = __ballot_sync(kFull, cnt > 0 && gt < krem && ge >= krem);
            const int src = __ffs(q) - 1;
            *thr = __shfl_sync(kFull, key, src);
            *keep = krem - __shfl_sync(kFull, gt, src);
            __syncwarp();
            return;
        }
    }
    *thr = prefix;
    *keep = krem;
}

// c2 threshold in rank space.  rk[rel] is the relation's position in the
// row's (w descending, relation ascending) order; kNoRank marks w <= 0.  On
// one side of one source every relation has at most one group and groups are
// in relation order, so the reference's rule (flashlog.cu:26-63: groups above
// the weight threshold whole, groups at it in group order until the budget is
// spent) takes exactly the groups of smallest rank until the budget is
// reached.  The select therefore needs no comparison of weights: the groups'
// counts (clamped to the budget, which changes no take) are summed into
// kRankBins bins of rank_bin consecutive ranks, a warp scan over the bins
// finds the bin where the running total reaches the budget, and the at most
// rank_bin <= 32 groups of that bin, one per lane, finish it.
//
// Pass 1 (`scatter`) has filled ws.hist; `members(lo, hi, quota)` must store
// the clamped count of each group with rank in [lo, hi) at quota[rank - lo].
// Returns *thr = the rank of the group at which the budget is reached and
// *keep = the edges that group still takes.
template <typename Members>
__device__ void rank_select(int64_t budget, int rank_bin, WarpScratch &ws, Members members, uint32_t *thr,
                            int64_t *keep) {
    const int lane = threadIdx.x & 31;
    constexpr int kPer = kRankBins / 32;  // bins per lane, contiguous
    uint32_t part = 0;
#pragma unroll
    for (int k = 0; k < kPer; ++k) part += ws.hist[lane * kPer + ((k + (lane >> 1)) & (kPer - 1))];
    const uint32_t krem = static_cast<uint32_t>(budget);
    const uint32_t incl = warp_inclusive_scan(part);
    const unsigned ball = __ballot_sync(kFull, incl >= krem && incl - part < krem);
    const int src = __ffs(ball) - 1;  // the clamped total reaches the budget, so one lane crosses it
    const uint32_t base = __shfl_sync(kFull, incl - part, src);
    const uint32_t hb = lane < kPer ? ws.hist[src * kPer + lane] : 0u;
    const uint32_t hi = warp_inclusive_scan(hb);
    const unsigned bb = __ballot_sync(kFull, lane < kPer && base + hi >= krem && base + hi - hb < krem);
    const int bl = __ffs(bb) - 1;
    const int bin = src * kPer + bl;
    const uint32_t above = __shfl_sync(kFull, base + hi - hb, bl);
    __syncwarp();
    ws.quota[lane] = 0;
    __syncwarp();
    const uint32_t lo = static_cast<uint32_t>(bin) * static_cast<uint32_t>(rank_bin);
    members(lo, lo + static_cast<uint32_t>(rank_bin), ws.quota);
    __syncwarp();
    const int32_t qc = lane < rank_bin ? ws.quota[lane] : 0;
    const int32_t qi = warp_inclusive_scan(qc);
    const int32_t rem = static_cast<int32_t>(krem - above);  // >= 1
    const unsigned qb = __ballot_sync(kFull, qc > 0 && qi >= rem && qi - qc < rem);
    const int ql = __ffs(qb) - 1;
    *thr = lo + static_cast<uint32_t>(ql);
    *keep = rem - (__shfl_sync(kFull, qi, ql) - __shfl_sync(kFull, qc, ql));
    __syncwarp();
}

// Threshold of one side of one entry, computed by a whole warp.  With `stg`
// the side's keys and clamped counts are left in stg for the take pass and
// *staged is set.  kRanked compiles the rank-select paths only (rk given),
// otherwise the radix select over the weights: each expansion kernel carries
// one of the two, which keeps it within the instruction cache.
template <bool kRanked>
__device__ bool group_threshold(const float *wdir, const uint16_t *rk, int rank_bin, const Side &sd, int64_t g0,
                                int64_t g1, int64_t budget, WarpScratch &ws, void *stgv, bool *staged, bool *ranked,
                                uint32_t *thr, int64_t *keep) {
    const int lane = threadIdx.x & 31;
    *staged = false;
    *ranked = false;
    if (g1 - g0 <= 32) {
        // One group per lane: every lane counts the groups at or above its own key.
        uint32_t key, cnt;
        group_key(wdir, sd, g0 + lane, g1, &key, &cnt);
        const int64_t total = warp_sum(static_cast<int64_t>(cnt));
        if (total <= budget) return false;
        int64_t ge = 0, gt = 0;
#pragma unroll 8
        for (int j = 0; j < 32; ++j) {
            const uint32_t kj = __shfl_sync(kFull, key, j);
            const int64_t cj = __shfl_sync(kFull, cnt, j);
            ge += kj >= key ? cj : 0;
            gt += kj > key ? cj : 0;
        }
        const unsigned q = __ballot_sync(kFull, cnt > 0u && gt < budget && ge >= budget);
        const int src = __ffs(q) - 1;
        *thr = __shfl_sync(kFull, key, src);
        *keep = budget - __shfl_sync(kFull, gt, src);
        return true;
    }
    const int64_t n = g1 - g0;
    if constexpr (kRanked) {
        // rank select; staged: each group's rank and clamped count
        StageRank *stg = static_cast<StageRank *>(stgv);
        *ranked = true;
        for (int d = lane; d < kRankBins; d += 32) ws.hist[d] = 0u;
        __syncwarp();
        const uint32_t cap = static_cast<uint32_t>(budget);
        int64_t total = 0;
        if (stg != nullptr && n <= kStage) {
            for (int64_t cb = 0; cb < n; cb += 128) {  // four groups per lane: the loads are issued together
                int32_t rel[4];
                uint32_t c[4], r[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int64_t j = cb + u * 32 + lane;
                    rel[u] = j < n ? static_cast<int32_t>(sd.grel[g0 + j]) : -1;
                    c[u] = j < n ? static_cast<uint32_t>(sd.gcount[g0 + j]) : 0u;
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) r[u] = rel[u] >= 0 ? static_cast<uint32_t>(rk[rel[u]]) : kNoRank;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int64_t j = cb + u * 32 + lane;
                    const uint32_t cc = r[u] != kNoRank ? c[u] : 0u;
                    const uint32_t cl = cc < cap ? cc : cap;
                    if (j < n) {
                        stg->rank[j] = static_cast<uint16_t>(r[u]);
                        stg->cnt[j] = static_cast<uint16_t>(cl);
                        if (cl > 0u) atomicAdd(&ws.hist[r[u] / static_cast<uint32_t>(rank_bin)], cl);
                    }
                    total += cc;
                }
            }
            __syncwarp();
            *staged = true;
            if (warp_sum(total) <= budget) return false;
            rank_select(budget, rank_bin, ws, [&](uint32_t lo, uint32_t hi, int32_t *quota) {
                for (int64_t j = lane; j < n; j += 32) {
                    const uint32_t r = stg->rank[j];
                    if (r >= lo && r < hi) quota[r - lo] = stg->cnt[j];
                }
            }, thr, keep);
            return true;
        }
        for (int64_t j = lane; j < n; j += 32) {
            const uint32_t r = rk[sd.grel[g0 + j]];
            const uint32_t cc = r != kNoRank ? static_cast<uint32_t>(sd.gcount[g0 + j]) : 0u;
            const uint32_t cl = cc < cap ? cc : cap;
            if (cl > 0u) atomicAdd(&ws.hist[r / static_cast<uint32_t>(rank_bin)], cl);
            total += cc;
        }
        __syncwarp();
        if (warp_sum(total) <= budget) return false;
        rank_select(budget, rank_bin, ws, [&](uint32_t lo, uint32_t hi, int32_t *quota) {
            for (int64_t j = lane; j < n; j += 32) {
                const uint32_t r = rk[sd.grel[g0 + j]];
                if (r >= lo && r < hi) {
                    const uint32_t c = static_cast<uint32_t>(sd.gcount[g0 + j]);
                    quota[r - lo] = static_cast<int32_t>(c < cap ? c : cap);
                }
            }
        }, thr, keep);
        return true;
    } else {
    StageBuf *stg = static_cast<StageBuf *>(stgv);
    if (stg != nullptr && n <= kStage && budget < 65536) {
        int64_t total = 0;
        for (int64_t cb = 0; cb < n; cb += 128) {  // four groups per lane: the loads are issued together
            int32_t rel[4];
            uint32_t c[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int64_t j = cb + u * 32 + lane;
                rel[u] = j < n ? static_cast<int32_t>(sd.grel[g0 + j]) : -1;
                c[u] = j < n ? static_cast<uint32_t>(sd.gcount[g0 + j]) : 0u;
            }
            float wv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) wv[u] = rel[u] >= 0 ? wdir[rel[u]] : 0.0f;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int64_t j = cb + u * 32 + lane;
                const bool pos = wv[u] > 0.0f;
                const uint32_t cc = pos ? c[u] : 0u;
                if (j < n) {
                    stg->key[j] = pos ? __float_as_uint(wv[u]) : 0u;
                    stg->cnt[j] = static_cast<uint16_t>(cc < budget ? cc : budget);
                }
                total += cc;
            }
        }
        __syncwarp();
        *staged = true;
        if (warp_sum(total) <= budget) return false;
        radix_threshold(n, budget, ws, [&](int64_t j, uint32_t *key, uint32_t *cnt) {
            *key = j < n ? stg->key[j] : 0u;
            *cnt = j < n ? stg->cnt[j] : 0u;
        }, thr, keep);
        return true;
    }
    int64_t total = 0;
    for (int64_t cb = g0; cb < g1; cb += 32) {
        uint32_t key, cnt;
        group_key(wdir, sd, cb + lane, g1, &key, &cnt);
        total += cnt;
    }
    if (warp_sum(total) <= budget) return false;
    radix_threshold(n, budget, ws, [&](int64_t j, uint32_t *key, uint32_t *cnt) {
        group_key(wdir, sd, g0 + j, g1, key, cnt);
    }, thr, keep);
    return true;
    }
}

__device__ __forceinline__ double splitmix_phase(int64_t seed, int64_t b, int64_t l, int64_t src, bool inv) {
    uint64_t z = static_cast<uint64_t>(seed) ^ (static_cast<uint64_t>(b) * 0x9e3779b97f4a7c15ULL) ^
                 (static_cast<uint64_t>(l) * 0xbf58476d1ce4e5b9ULL) ^ (static_cast<uint64_t>(src) * 0x94d049bb133111ebULL) ^
                 (inv ? 0xd1b54a32d192ed03ULL : 0x8cb92baa3f3d8dd7ULL);
    z += 0x9e3779b97f4a7c15ULL;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    z ^= z >> 31;
    return static_cast<double>(z >> 11) * 0x1.0p-53;
}

// Emits, in lane order, the facts of the (at most 32) groups held one per
// lane: `take` edges from CSR position `start`, each with value prod * m and
// relation column rel_abs; facts the mask hides are dropped when drop_masked.
__device__ __forceinline__ void emit_groups(const ExpandArgs &a, WarpScratch &ws, const Side &sd, const uint8_t *vis,
                                            int32_t take, int32_t start, float prod, int32_t rel_abs, int64_t out,
                                            int64_t *written, bool drop_masked, bool edge_w, bool edge_score) {
    const int lane = threadIdx.x & 31;
    const int32_t incl = warp_inclusive_scan(take);
    const int32_t tot = __shfl_sync(kFull, incl, 31);
    ws.incl[lane] = incl;
    ws.start[lane] = start;
    ws.prod[lane] = prod;
    ws.rel[lane] = rel_abs;
    __syncwarp();
    int64_t wr = *written;
    for (int32_t f0 = 0; f0 < tot; f0 += 32) {
        const int32_t f = f0 + lane;
        const bool act = f < tot;
        bool visible = false;
        int32_t dst = 0, frel = 0, edge = 0;
        float value = 0.0f, m = 1.0f;
        if (act) {
            int lo = 0, hi = 31;  // first lane with incl > f
            while (lo < hi) { int mid = (lo + hi) >> 1; if (ws.incl[mid] > f) hi = mid; else lo = mid + 1; }
            const int32_t eoff = f - (lo ? ws.incl[lo - 1] : 0);
            const int64_t p = static_cast<int64_t>(ws.start[lo]) + eoff;
            fact_mask(a, sd, vis, p, drop_masked, edge_w, edge_score, &m, &visible);
            dst = sd.col[p];
            value = ws.prod[lo] * m;
            frel = ws.rel[lo];
            if (a.fact_edge) edge = (a.flags & FL_EDGE_POS) ? static_cast<int32_t>(p) : sd.order[p];
        }
        const unsigned ball = __ballot_sync(kFull, act && visible);
        if (act && visible) {
            const int64_t pos = out + wr + __popc(ball & lanemask_lt());
            a.fact_dst[pos] = dst;
            a.fact_val[pos] = value;
            a.fact_rel[pos] = static_cast<int16_t>(frel);
            if (a.fact_m) a.fact_m[pos] = m;
            if (a.fact_edge) a.fact_edge[pos] = edge;
        }
        wr += __popc(ball);
    }
    __syncwarp();
    *written = wr;
}

// One source entry expanded by a whole warp: ori groups, inv groups, identity.
template <bool kSampled, bool kRanked>
__device__ void expand_entry_warp(const ExpandArgs &a, WarpScratch &ws, void *stgv, int64_t i) {
    const int lane = threadIdx.x & 31;
    const bool skip_nonpos = (a.flags & FL_SKIP_NONPOS_W) != 0;
    const bool drop_masked = (a.flags & FL_DROP_MASKED) != 0;
    const bool edge_w = (a.flags & FL_EDGE_WEIGHT) != 0 && a.edge_weight != nullptr;
    const bool edge_score = (a.flags & FL_EDGE_SCORE) != 0;
    const bool wot_i = (a.flags & FL_WOT_I) != 0;
    if (a.capacity > 0 && a.slot_base[i + 1] > a.capacity) {  // would write past the fact buffers
        if (lane == 0) { a.entry_count[i] = 0; if (a.status) atomicOr(a.status, FL_STATUS_SLOT_OVERFLOW); }
        return;
    }
    const int64_t src = a.ent[i];
    EntryInfo e;
    if (a.info) {
        e = a.info[i];
    } else {
        e.row = static_cast<int32_t>(find_row(a.row_ptr, a.rows, i));
        e.g0o = a.ori.gptr[src]; e.g1o = (a.flags & FL_NO_ORI) ? e.g0o : a.ori.gptr[src + 1];
        e.g0i = a.inv.gptr[src]; e.g1i = (a.flags & FL_NO_INV) ? e.g0i : a.inv.gptr[src + 1];
    }
    const int64_t row = e.row;
    const float v = a.val[i];
    const float *wrow = a.w + row * a.n;
    const int64_t out = a.slot_base[i];
    int64_t written = 0;
    for (int dir = 0; dir < 2; ++dir) {
        const Side &sd = dir ? a.inv : a.ori;
        const uint8_t *vis = dir ? a.vis_inv : a.vis_ori;
        const int64_t off = dir ? a.r_size : 0;
        const float *wdir = wrow + off;
        const int64_t g0 = dir ? e.g0i : e.g0o, g1 = dir ? e.g1i : e.g1o;
        if (g0 == g1) continue;
        bool use_thr = false, staged = false, ranked = false;
        const uint16_t *rk = nullptr;
        uint32_t thr = 0;
        int64_t keep_thr = 0;
        // sampled-mode state (lane 0 only)
        int64_t q_target = 0, q_residual = 0, q_spare = 0, q_left = 0, q_capleft = 0, q_prefix = 0;
        double q_wsum = 0.0, q_phase = 0.0;
        if constexpr (kSampled) {
            if (lane == 0) {
                int64_t capacity = 0;
                double wsum = 0.0;
                for (int64_t g = g0; g < g1; ++g) {
                    double wt = wdir[sd.grel[g]];
                    if (wt > 0 && sd.gcount[g] > 0) { capacity += sd.gcount[g]; wsum += wt; }
                }
                q_target = a.topk < capacity ? a.topk : capacity;
                q_wsum = wsum;
                int64_t allocated = capacity;
                if (q_target < capacity) {
                    allocated = 0;
                    for (int64_t g = g0; g < g1; ++g) {
                        double wt = wdir[sd.grel[g]];
                        int64_t c = sd.gcount[g];
                        if (wt > 0 && c > 0)
                            allocated += static_cast<int64_t>(fmin(static_cast<double>(c),
                                                                   floor(static_cast<double>(q_target) * wt / wsum)));
                    }
                }
                q_residual = q_target - allocated;
                q_spare = capacity - allocated;
                q_left = q_residual;
                q_capleft = q_spare;
                q_phase = splitmix_phase(a.seed, row / a.L, row % a.L, src, dir == 1);
                q_prefix = 0;
            }
        } else if (skip_nonpos && a.topk < kNoBudget) {
            rk = a.rel_rank != nullptr
                     ? a.rel_rank + ((a.rank_row != nullptr ? a.rank_row[row] : row) * 2 + dir) * a.r_size
                     : nullptr;
            use_thr = group_threshold<kRanked>(wdir, rk, a.rank_bin, sd, g0, g1, a.topk, ws, stgv, &staged, &ranked, &thr,
                                      &keep_thr);
        }
        if (kRanked && staged && ranked) {
            // The taking groups, compacted in group order in place:
            // rank = group offset, cnt = edges taken.
            StageRank *stg = static_cast<StageRank *>(stgv);
            const uint32_t last = use_thr ? thr : 0xfffffffeu;
            const int n = static_cast<int>(g1 - g0);
            int ntk = 0;
            for (int cb = 0; cb < n; cb += 32) {
                const int j = cb + lane;
                const uint32_t r = j < n ? stg->rank[j] : kNoRank;
                const int32_t cnt = j < n ? stg->cnt[j] : 0;
                const int32_t take = r == kNoRank || r > last ? 0 : (r < last ? cnt : static_cast<int32_t>(keep_thr));
                const unsigned b = __ballot_sync(kFull, take > 0);
                if (take > 0) {  // positions below cb + 32: entries of this chunk are read already
                    const int p = ntk + __popc(b & lanemask_lt());
                    stg->rank[p] = static_cast<uint16_t>(j);
                    stg->cnt[p] = static_cast<uint16_t>(take);
                }
                ntk += __popc(b);
                __syncwarp();
            }
            for (int k0 = 0; k0 < ntk; k0 += 32) {
                const int k = k0 + lane;
                const bool has = k < ntk;
                const int64_t g = g0 + (has ? stg->rank[k] : 0);
                const int32_t take = has ? stg->cnt[k] : 0;
                const int32_t rel = has ? static_cast<int32_t>(sd.grel[g]) : 0;
                const int32_t start = has ? sd.gstart[g] : 0;
                const float wg = has ? wdir[rel] : 0.0f;
                emit_groups(a, ws, sd, vis, take, start, v * wg, rel + static_cast<int32_t>(off), out, &written,
                            drop_masked, edge_w, edge_score);
            }
            continue;
        }
        int64_t tie_seen = 0;
        for (int64_t cb = g0; cb < g1; cb += 32) {
            const int64_t g = cb + lane;
            const bool valid = g < g1;
            int32_t take;
            int32_t rel = 0;
            float wg = 0.0f;
            if (!kSampled && !kRanked && staged) {
                // keys and clamped counts from the staging buffer; global
                // group data only for groups that take edges
                const StageBuf *stg = static_cast<const StageBuf *>(stgv);
                const uint32_t key = valid ? stg->key[g - g0] : 0u;
                const int32_t cnt = valid ? stg->cnt[g - g0] : 0;
                const bool pos = key != 0u;
                if (!use_thr) {
                    take = pos ? cnt : 0;
                } else {
                    // chunks without a key at or above the threshold take nothing
                    if (!__any_sync(kFull, valid && pos && key >= thr)) continue;
                    const bool tie = valid && pos && key == thr;
                    const int32_t tcnt = tie ? cnt : 0;
                    const int32_t tincl = warp_inclusive_scan(tcnt);
                    const int64_t texcl = static_cast<int64_t>(tincl - tcnt) + tie_seen;
                    tie_seen += __shfl_sync(kFull, tincl, 31);
                    if (!pos || key < thr) take = 0;
                    else if (key > thr) take = cnt;
                    else {
                        const int64_t left = keep_thr - texcl;
                        take = left > 0 ? static_cast<int32_t>(left < cnt ? left : cnt) : 0;
                    }
                }
                if (!valid) take = 0;
                if (take > 0) { rel = sd.grel[g]; wg = __uint_as_float(key); }
            } else {
                rel = valid ? sd.grel[g] : 0;
                const int32_t cnt = valid ? sd.gcount[g] : 0;
                wg = valid ? wdir[rel] : 0.0f;
                if constexpr (kSampled) {
                    // Sequential quota arithmetic of flashlog.cu:1505-1531, lane 0.
                    ws.rel[lane] = rel;
                    __syncwarp();
                    if (lane == 0) {
                        int64_t nvalid = (g1 - cb) < 32 ? (g1 - cb) : 32;
                        for (int k = 0; k < nvalid; ++k) {
                            int32_t c = sd.gcount[cb + k];
                            float sc = wdir[ws.rel[k]];
                            int64_t cur = sc > 0.0f ? c : 0;
                            if (cur > 0 && q_spare > 0) {
                                int64_t base = static_cast<int64_t>(fmin(static_cast<double>(c),
                                    floor(static_cast<double>(q_target) * static_cast<double>(sc) / q_wsum)));
                                int64_t spare = static_cast<int64_t>(c) - base;
                                q_prefix += spare;
                                q_capleft -= spare;
                                int64_t cumulative = q_prefix == q_spare ? q_residual
                                    : static_cast<int64_t>(floor(static_cast<double>(q_residual) * static_cast<double>(q_prefix) /
                                                                 static_cast<double>(q_spare) + q_phase));
                                int64_t extra = cumulative - (q_residual - q_left);
                                int64_t lim = spare < q_left ? spare : q_left;
                                extra = extra < lim ? extra : lim;
                                extra = extra > 0 ? extra : 0;
                                extra = extra > (q_left - q_capleft) ? extra : (q_left - q_capleft);
                                q_left -= extra;
                                cur = base + extra;
                            }
                            ws.quota[k] = static_cast<int32_t>(cur);
                        }
                    }
                    __syncwarp();
                    take = valid ? ws.quota[lane] : 0;
                } else if (!skip_nonpos) {
                    take = cnt;
                } else if (kRanked && ranked) {
                    const uint32_t r = valid ? static_cast<uint32_t>(rk[rel]) : kNoRank;
                    take = r == kNoRank ? 0 : (!use_thr || r < thr ? cnt : (r == thr ? static_cast<int32_t>(keep_thr) : 0));
                } else if (!use_thr) {
                    take = wg > 0.0f ? cnt : 0;
                } else {
                    uint32_t key = __float_as_uint(wg);
                    bool pos = wg > 0.0f;
                    bool tie = valid && pos && key == thr;
                    int64_t tcnt = tie ? cnt : 0;
                    int64_t tincl = warp_inclusive_scan(tcnt);
                    int64_t texcl = tincl - tcnt + tie_seen;
                    tie_seen += __shfl_sync(kFull, tincl, 31);
                    if (!pos || key < thr) take = 0;
                    else if (key > thr) take = cnt;
                    else {
                        int64_t left = keep_thr - texcl;
                        take = left > 0 ? static_cast<int32_t>(left < cnt ? left : cnt) : 0;
                    }
                }
                if (!valid) take = 0;
            }
            if (!__any_sync(kFull, take > 0)) continue;
            emit_groups(a, ws, sd, vis, take, take > 0 ? sd.gstart[g] : 0, v * wg, rel + static_cast<int32_t>(off), out,
                        &written, drop_masked, edge_w, edge_score);
        }
    }
    if (!wot_i) {
        if (lane == 0) {
            const int64_t pos = out + written;
            a.fact_dst[pos] = static_cast<int32_t>(src);
            a.fact_val[pos] = v * wrow[a.n - 1];
            a.fact_rel[pos] = static_cast<int16_t>(a.n - 1);
            if (a.fact_m) a.fact_m[pos] = 1.0f;
            if (a.fact_edge) a.fact_edge[pos] = 0;
        }
        written += 1;
    }
    if (lane == 0) a.entry_count[i] = static_cast<int32_t>(written);
    // Slots the entry reserved but did not fill get the destination -1.
    for (int64_t s = out + written + lane; s < a.slot_base[i + 1]; s += 32) a.fact_dst[s] = -1;
}

// Sampled c2: one warp per entry.
__global__ void __launch_bounds__(kExpandWarps * 32, 2) hop_expand_sampled_kernel(ExpandArgs a) {
    __shared__ WarpScratch scratch[kExpandWarps];
    const int wib = threadIdx.x >> 5;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kExpandWarps;
    const int64_t S_live = a.row_ptr[a.rows] < a.S ? a.row_ptr[a.rows] : a.S;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kExpandWarps + wib; i < S_live; i += nwarps)
        expand_entry_warp<true, false>(a, scratch[wib], nullptr, i);
}

// c2 take of the (at most kTeam) groups of one side held one per team lane:
// the threshold by all-pairs comparison of the keys (flashlog.cu:26-63), ties
// at the threshold taken in group order.
__device__ __forceinline__ int32_t team_take(float wg, int32_t cnt, int64_t topk, bool skip_nonpos, unsigned tm,
                                             int tl, int tbase) {
    if (!skip_nonpos) return cnt;
    const bool pos = wg > 0.0f;
    const int64_t c = pos ? cnt : 0;
    int64_t total = c;
#pragma unroll
    for (int o = 1; o < kTeam; o <<= 1) total += __shfl_xor_sync(tm, total, o, kTeam);
    if (topk >= kNoBudget || total <= topk) return pos ? cnt : 0;
    const uint32_t key = pos ? __float_as_uint(wg) : 0u;
    int64_t ge = 0, gt = 0;
#pragma unroll
    for (int j = 0; j < kTeam; ++j) {
        const uint32_t kj = __shfl_sync(tm, key, j, kTeam);
        const int64_t cj = __shfl_sync(tm, c, j, kTeam);
        ge += kj >= key ? cj : 0;
        gt += kj > key ? cj : 0;
    }
    const unsigned q = (__ballot_sync(tm, c > 0 && gt < topk && ge >= topk) >> tbase) & 0xffu;
    const int srcl = __ffs(q) - 1;  // one lane holds the threshold key when the total exceeds the budget
    const uint32_t thr = __shfl_sync(tm, key, srcl, kTeam);
    const int64_t keep = topk - __shfl_sync(tm, gt, srcl, kTeam);
    const int32_t tc = (pos && key == thr) ? cnt : 0;
    int32_t tincl = tc;
#pragma unroll
    for (int o = 1; o < kTeam; o <<= 1) {
        const int32_t u = __shfl_up_sync(tm, tincl, o, kTeam);
        if (tl >= o) tincl += u;
    }
    const int64_t texcl = tincl - tc;
    if (!pos || key < thr) return 0;
    if (key > thr) return cnt;
    const int64_t left = keep - texcl;
    return left > 0 ? static_cast<int32_t>(left < cnt ? left : cnt) : 0;
}

__device__ __forceinline__ int32_t team_incl(int32_t x, unsigned tm, int tl) {
#pragma unroll
    for (int o = 1; o < kTeam; o <<= 1) {
        const int32_t u = __shfl_up_sync(tm, x, o, kTeam);
        if (tl >= o) x += u;
    }
    return x;
}

// One entry with at most kTeam groups on each side, expanded by an 8-lane
// team: both sides' groups are loaded together (lane tl holds group tl of
// each side), then the taken edges of both sides are emitted kTeam at a time
// in canonical order (ori facts, then inv facts).  Returns the fact count.
__device__ __forceinline__ int64_t team_entry(const ExpandArgs &a, const float *wrow, float v, int64_t g0o,
                                              int64_t g1o, int64_t g0i, int64_t g1i, unsigned tm, int tl, int tbase,
                                              int64_t out, bool skip_nonpos, bool drop_masked, bool edge_w,
                                              bool edge_score) {
    const bool vo = tl < (g1o - g0o), vi = tl < (g1i - g0i);
    const int32_t rel_o = vo ? a.ori.grel[g0o + tl] : 0, rel_i = vi ? a.inv.grel[g0i + tl] : 0;
    const int32_t cnt_o = vo ? a.ori.gcount[g0o + tl] : 0, cnt_i = vi ? a.inv.gcount[g0i + tl] : 0;
    const int32_t st_o = vo ? a.ori.gstart[g0o + tl] : 0, st_i = vi ? a.inv.gstart[g0i + tl] : 0;
    const float w_o = vo ? wrow[rel_o] : 0.0f, w_i = vi ? wrow[a.r_size + rel_i] : 0.0f;
    const int32_t take_o = team_take(w_o, cnt_o, a.topk, skip_nonpos, tm, tl, tbase);
    const int32_t take_i = team_take(w_i, cnt_i, a.topk, skip_nonpos, tm, tl, tbase);
    const int32_t incl_o = team_incl(vo ? take_o : 0, tm, tl), incl_i = team_incl(vi ? take_i : 0, tm, tl);
    const int32_t tot_o = __shfl_sync(tm, incl_o, kTeam - 1, kTeam);
    const int32_t tot = tot_o + __shfl_sync(tm, incl_i, kTeam - 1, kTeam);
    const float prod_o = v * w_o, prod_i = v * w_i;
    const int32_t rel_i_abs = rel_i + static_cast<int32_t>(a.r_size);
    int64_t written = 0;
    for (int32_t f0 = 0; f0 < tot; f0 += kTeam) {
        const int32_t f = f0 + tl;
        const bool act = f < tot;
        const bool inv = f >= tot_o;
        const int32_t fs = inv ? f - tot_o : f;
        int ko = 0, ki = 0;  // the group holding fact fs: lanes whose inclusive count is <= fs
#pragma unroll
        for (int j = 0; j < kTeam; ++j) {
            ko += (__shfl_sync(tm, incl_o, j, kTeam) <= fs) ? 1 : 0;
            ki += (__shfl_sync(tm, incl_i, j, kTeam) <= fs) ? 1 : 0;
        }
        ko = ko < kTeam ? ko : kTeam - 1;
        ki = ki < kTeam ? ki : kTeam - 1;
        const int32_t prev_o = __shfl_sync(tm, incl_o, ko > 0 ? ko - 1 : 0, kTeam);
        const int32_t prev_i = __shfl_sync(tm, incl_i, ki > 0 ? ki - 1 : 0, kTeam);
        const int32_t s_o = __shfl_sync(tm, st_o, ko, kTeam), s_i = __shfl_sync(tm, st_i, ki, kTeam);
        const float p_o = __shfl_sync(tm, prod_o, ko, kTeam), p_i = __shfl_sync(tm, prod_i, ki, kTeam);
        const int32_t r_o = __shfl_sync(tm, rel_o, ko, kTeam), r_i = __shfl_sync(tm, rel_i_abs, ki, kTeam);
        bool visible = false;
        int32_t dst = 0, edge = 0;
        float value = 0.0f, m = 1.0f;
        if (act) {
            const Side &sd = inv ? a.inv : a.ori;
            const int64_t p = inv ? static_cast<int64_t>(s_i) + (fs - (ki > 0 ? prev_i : 0))
                                  : static_cast<int64_t>(s_o) + (fs - (ko > 0 ? prev_o : 0));
            fact_mask(a, sd, inv ? a.vis_inv : a.vis_ori, p, drop_masked, edge_w, edge_score, &m, &visible);
            dst = sd.col[p];
            value = (inv ? p_i : p_o) * m;
            if (a.fact_edge) edge = (a.flags & FL_EDGE_POS) ? static_cast<int32_t>(p) : sd.order[p];
        }
        const unsigned ball = (__ballot_sync(tm, act && visible) >> tbase) & 0xffu;
        if (act && visible) {
            const int64_t pos = out + written + __popc(ball & ((1u << tl) - 1u));
            a.fact_dst[pos] = dst;
            a.fact_val[pos] = value;
            a.fact_rel[pos] = static_cast<int16_t>(inv ? r_i : r_o);
            if (a.fact_m) a.fact_m[pos] = m;
            if (a.fact_edge) a.fact_edge[pos] = edge;
        }
        written += __popc(ball);
    }
    return written;
}

// Deterministic c2 (and the all-edges path): four entries per warp in 8-lane
// teams; entries with more than kTeam groups on a side go to the whole warp.
template <bool kRanked>
__global__ void __launch_bounds__(kExpandWarps * 32, kRanked ? 4 : 3) hop_expand_kernel(ExpandArgs a) {
    __shared__ WarpScratch scratch[kExpandWarps];
    extern __shared__ __align__(16) unsigned char stage_raw[];
    constexpr size_t kStageBytes = kRanked ? sizeof(StageRank) : sizeof(StageBuf);
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int team = lane / kTeam, tl = lane % kTeam, tbase = team * kTeam;
    const unsigned tm = 0xffu << tbase;
    const bool skip_nonpos = (a.flags & FL_SKIP_NONPOS_W) != 0;
    const bool drop_masked = (a.flags & FL_DROP_MASKED) != 0;
    const bool edge_w = (a.flags & FL_EDGE_WEIGHT) != 0 && a.edge_weight != nullptr;
    const bool edge_score = (a.flags & FL_EDGE_SCORE) != 0;
    const bool wot_i = (a.flags & FL_WOT_I) != 0;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kExpandWarps;
    const int64_t S_live = a.row_ptr[a.rows] < a.S ? a.row_ptr[a.rows] : a.S;
    // Four entries (one per team) starting at `base`; `which` selects the
    // whole-warp entries (kBigPass), the team entries (kSmallPass) or both.
    auto four = [&](int64_t base, int which) {
        const int64_t i = base + team;
        const bool mine = i < S_live;
        bool small = false, over = false;
        int64_t src = 0, out = 0, end = 0;
        EntryInfo e{0, 0, 0, 0, 0};
        float v = 0.0f;
        if (mine) {
            out = a.slot_base[i];
            end = a.slot_base[i + 1];
            over = a.capacity > 0 && end > a.capacity;
            src = a.ent[i];
            v = a.val[i];
            if (a.info) {
                e = a.info[i];
            } else {
                e.g0o = a.ori.gptr[src]; e.g1o = (a.flags & FL_NO_ORI) ? e.g0o : a.ori.gptr[src + 1];
                e.g0i = a.inv.gptr[src]; e.g1i = (a.flags & FL_NO_INV) ? e.g0i : a.inv.gptr[src + 1];
            }
            // few groups and few facts: a team emits kTeam facts per step, so an
            // entry with many reserved slots is emitted faster by the whole warp
            small = !over && (e.g1o - e.g0o) <= kTeam && (e.g1i - e.g0i) <= kTeam && end - out <= kTeamMaxSlots;
        }
        if (small && which != kBigPass) {
            const int64_t row = a.info ? static_cast<int64_t>(e.row) : find_row(a.row_ptr, a.rows, i);
            const float *wrow = a.w + row * a.n;
            int64_t written = team_entry(a, wrow, v, e.g0o, e.g1o, e.g0i, e.g1i, tm, tl, tbase, out, skip_nonpos,
                                         drop_masked, edge_w, edge_score);
            if (!wot_i) {
                if (tl == 0) {
                    const int64_t pos = out + written;
                    a.fact_dst[pos] = static_cast<int32_t>(src);
                    a.fact_val[pos] = v * wrow[a.n - 1];
                    a.fact_rel[pos] = static_cast<int16_t>(a.n - 1);
                    if (a.fact_m) a.fact_m[pos] = 1.0f;
                    if (a.fact_edge) a.fact_edge[pos] = 0;
                }
                written += 1;
            }
            if (tl == 0) a.entry_count[i] = static_cast<int32_t>(written);
            for (int64_t s = out + written + tl; s < end; s += kTeam) a.fact_dst[s] = -1;
        }
        __syncwarp();
        unsigned big = __ballot_sync(kFull, mine && !small && tl == 0 && which != kSmallPass);
        while (big) {
            const int t = (__ffs(big) - 1) / kTeam;
            big &= big - 1;
            expand_entry_warp<false, kRanked>(a, scratch[wib], stage_raw + wib * kStageBytes, base + t);
        }
    };
    if (a.work != nullptr) {
        // Warps take runs of entries from two queues (counted in entries):
        // first the whole-warp entries, then the team entries, so the
        // kernel's tail is made of short team work; a warp held up by a hub
        // does not hold up the others of its block.  16 entries per grab
        // while more than 64 per resident warp remain, then 4 (guided).
        for (int pass = kBigPass; pass <= kSmallPass; ++pass) {
            int64_t seen = 0;  // this warp's last grab: the queue has passed it
            for (;;) {
                const uint32_t take = (S_live - seen > nwarps * 64) ? 16u : 4u;
                uint32_t c = 0;
                if (lane == 0) c = atomicAdd(a.work + pass, take);
                c = __shfl_sync(kFull, c, 0);
                const int64_t b0 = static_cast<int64_t>(c);
                if (b0 >= S_live) break;
                seen = b0;
                for (int64_t base = b0; base < b0 + take && base < S_live; base += 4) four(base, pass);
            }
        }
    } else {
        for (int64_t base = (static_cast<int64_t>(blockIdx.x) * kExpandWarps + wib) * 4; base < S_live;
             base += nwarps * 4)
            four(base, kBothPasses);
    }
}

// ---------------------------------------------------------------------------
// Row reduction: one CTA per row; facts bucketed by destination in shared memory.
//
// A row's facts occupy the contiguous slot range
// [slot_base[row_ptr[r]], slot_base[row_ptr[r + 1]]) in canonical order; slots
// an entry did not fill hold the destination -1.  The row's destinations are
// counted into at most kKBins bins of 2^shift consecutive entities; the bins
// are cut into chunks of at most kTileK facts.  Each chunk's facts are
// scattered into their bins in shared memory as keys
// ((destination - chunk base) << 32 | row-local slot), so the key order is
// destination order and, within a destination, canonical order.  A fact of
// a bin of at most kRankBinMax facts finds its sorted position by counting
// the smaller keys of its bin (an inverse permutation, inv); larger bins are
// sorted in place by one warp, or by the whole block above kWarpSortMax.
// Then every thread walks a contiguous range of sorted positions: a block
// scan of the destination-run heads gives each run its output index, the
// head sums its run left to right (the reference CPU's order) or picks the
// MAX winner, and each fact gets its output position.  A single bin of more
// than kTileK facts is summed through dense kDenseW-wide windows that stream
// the row in canonical order.
// Rows of at most kRankSortMax slots are sorted in one tile by rank.
// ---------------------------------------------------------------------------
// Threads of a row-reduction CTA (1024: one CTA per SM; 512: two, with
// every tile halved).  The tile sizes scale with it.
#ifndef FL_ROW_THREADS
#define FL_ROW_THREADS 1024
#endif
constexpr int kRThreads = FL_ROW_THREADS;
static_assert(kRThreads == 1024 || kRThreads == 512, "row reduction CTAs of 512 or 1024 threads");
constexpr int kRowCtasPerSm = 1024 / kRThreads;
constexpr int kRWarps = kRThreads / 32;
constexpr int kDigits = 256;
constexpr int kRankSortMax = 128;  // rows of at most this many slots: one tile, sorted by rank
constexpr int kTileD = 6 * kRThreads;   // dense-window sub-tile
constexpr int kDenseW = 4 * kRThreads;  // dense window width (destinations)
constexpr int kLoadK = 4;  // slots per thread per load step
constexpr int kLoadStep = kRThreads * kLoadK;
static_assert(kLoadStep <= 6 * kRThreads, "a load step must fit an empty dense-window sub-tile, or load_range stalls");
constexpr int kKBitsMax = kRThreads == 1024 ? 13 : 12;
constexpr int kKBins = 1 << kKBitsMax;  // destination bins per row (at most)
constexpr int kTileK = 12 * kRThreads;  // facts per chunk
constexpr int kRankBinMax = 512;       // bins up to this size: each fact ranked within its bin
constexpr int kMultiPairs = 2 * kRThreads;  // comparator pairs of the block-wide sort of the larger bins
constexpr int kWarpSortMax = 1024;      // bins up to this size are sorted by one warp
constexpr int kBigBinsMax = kTileK / kWarpSortMax + 1;

struct TileA {
    uint32_t key[kRankSortMax];
    float val[kRankSortMax];
    uint16_t idx[2][kRankSortMax];
};
struct TileK {
    unsigned long long key[kTileK];  // ((destination - chunk base) << 32) | row-local slot
    float val[kTileK];
    uint16_t inv[kTileK];            // sorted position -> tile position
    uint32_t off[kKBins + 1];        // bin starts; the scatter advances off[b] to the bin's end
};
struct TileD {
    uint16_t cnt[kRWarps * kDigits];  // per-warp digit counters of the sub-tile sorts (cleared as uint4)
    uint32_t key[kTileD];
    float val[kTileD];
    uint16_t idx[2][kTileD];
    uint32_t slot[kTileD];
    float acc[kDenseW];
    uint32_t oidx[kDenseW];
    uint32_t touched[kDenseW / 32];
    unsigned long long bkey[kDenseW];  // MAX: winner's (source, triple id)
    uint32_t bslot[kDenseW];           // MAX: winner's row-local slot
};

struct ReduceSmem {
    union {
        TileA a;
        TileK k;
        TileD d;
    } t;
    int64_t scan_scratch[kRWarps + 1];
    float fscratch[kRWarps + 1];
    int chunk_end;
    int big_n;
    int big_bin[kBigBinsMax];
    int32_t win[kTileK / 32];  // per 32 sorted positions: run heads, then their exclusive prefix
    // bins of more than kRankBinMax facts: tile start, size, first comparator pair
    uint16_t mb_beg[kTileK / (kRankBinMax + 1) + 1];
    uint16_t mb_n[kTileK / (kRankBinMax + 1) + 1];
    int32_t mb_pair[kTileK / (kRankBinMax + 1) + 2];
    int mb_count, mb_mmax;
};
static_assert(kTileK / (kRankBinMax + 1) + 1 < kRThreads, "listed bins are scanned one per thread");
static_assert(sizeof(ReduceSmem) <= 227 * 1024, "row reduction shared memory exceeds one CTA's budget");
static_assert(kRowCtasPerSm == 1 || sizeof(ReduceSmem) <= 112 * 1024, "two row-reduction CTAs must fit one SM");
static_assert(offsetof(TileD, cnt) == 0, "digit counters are cleared with 16-byte stores");
static_assert(kTileD <= 65536, "tile indices are 16-bit");
static_assert(kTileK <= 65536, "tile positions are 16-bit");

struct ReduceArgs {
    const int64_t *row_ptr;      // rows of the (selected) state
    int64_t rows;
    const int64_t *slot_base;    // per entry
    const int32_t *fact_dst;
    const float *fact_val;
    int64_t E;
    int32_t *fact_pos;           // may be null
    int32_t *tmp_ent;            // outputs at the row's slot base
    float *tmp_x;
    int64_t *out_count;
    float *out_sum;
    int64_t capacity;            // length of the fact / output buffers
    int32_t *status;             // device status bits (may be null)
    // MAX coalesce (flashlog_kernel.py:399-478): each destination keeps its
    // largest fact; ties go to the smaller source (ori < inv < identity, from
    // the fact's relation column), then to the smaller triple id.  fact_pos
    // gets -1 for the facts that do not win.
    int max_mode;
    int64_t r_size, n;
    const int16_t *fact_rel;
    const int32_t *fact_edge;
    const int32_t *row_order;    // block -> row (a permutation), or null
};

// MAX order of values: fp32 order (mode 1) or the unsigned order of the fp32
// bit patterns (mode 2, the packed CAS-max of the dense path).
__device__ __forceinline__ bool max_greater(int mode, float v, float x) {
    return mode == 2 ? __float_as_uint(v) > __float_as_uint(x) : v > x;
}
__device__ __forceinline__ bool max_equal(int mode, float v, float x) {
    return mode == 2 ? __float_as_uint(v) == __float_as_uint(x) : v == x;
}

// Tie key of a fact for the MAX coalesce: (source, triple id).
__device__ __forceinline__ unsigned long long max_tie_key(const ReduceArgs &a, int64_t slot) {
    if (a.fact_rel == nullptr) return 0ull;  // FL_MAX_VALUE_ONLY: no tie keys
    const int64_t rel = a.fact_rel[slot];
    const unsigned long long src = rel == a.n - 1 ? 2ull : (rel >= a.r_size ? 1ull : 0ull);
    return (src << 32) | static_cast<uint32_t>(a.fact_edge[slot]);
}

__device__ __forceinline__ int bits_for(int64_t width) {  // bits to represent width - 1
    int b = 0;
    while ((int64_t(1) << b) < width) ++b;
    return b;
}

// Stable LSD radix sort of the index permutation idx0[0..n) by key[idx] over
// the low `bits` bits, 8 bits per pass.  idx0 must hold 0..n-1 in load order.
// Returns the buffer holding the sorted permutation.
__device__ uint16_t *lsd_sort(const uint32_t *key, uint16_t *idx0, uint16_t *idx1, int n, int bits, ReduceSmem &sm) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int nw = (n + 255) >> 8;
    nw = nw < 1 ? 1 : (nw > kRWarps ? kRWarps : nw);
    const int per = (((n + nw - 1) / nw) + 31) & ~31;
    const int wlo = warp * per;
    const int whi = (wlo + per) < n ? (wlo + per) : n;  // empty when wlo >= n
    uint16_t *src = idx0, *dst = idx1;
    for (int shift = 0; shift < bits; shift += 8) {
        const uint32_t dmask = (bits - shift) >= 8 ? 255u : ((1u << (bits - shift)) - 1u);
        for (int k = threadIdx.x; k < kDigits * kRWarps / 8; k += kRThreads)
            reinterpret_cast<uint4 *>(sm.t.d.cnt)[k] = make_uint4(0u, 0u, 0u, 0u);
        __syncthreads();
        for (int base = wlo; base < whi; base += 32) {
            const int j = base + lane;
            const bool valid = j < whi;
            const uint32_t d = valid ? (key[src[j]] >> shift) & dmask : 0u;
            const unsigned act = __ballot_sync(kFull, valid);
            if (valid) {
                const unsigned peers = __match_any_sync(act, d);
                if (lane == __ffs(peers) - 1) sm.t.d.cnt[warp * kDigits + d] += static_cast<uint16_t>(__popc(peers));
            }
        }
        __syncthreads();
        {  // exclusive prefix in (digit, warp) order, 8 counters per thread
            int v[8];
            int s = 0;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int q = threadIdx.x * 8 + k;
                v[k] = sm.t.d.cnt[(q & (kRWarps - 1)) * kDigits + (q / kRWarps)];
                s += v[k];
            }
            int64_t tot;
            int run = static_cast<int>(block_exclusive_scan<int64_t>(s, sm.scan_scratch, &tot));
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int q = threadIdx.x * 8 + k;
                sm.t.d.cnt[(q & (kRWarps - 1)) * kDigits + (q / kRWarps)] = static_cast<uint16_t>(run);
                run += v[k];
            }
        }
        __syncthreads();
        for (int base = wlo; base < whi; base += 32) {
            const int j = base + lane;
            const bool valid = j < whi;
            const uint16_t id = valid ? src[j] : 0;
            const uint32_t d = valid ? (key[id] >> shift) & dmask : 0u;
            const unsigned act = __ballot_sync(kFull, valid);
            if (valid) {
                const unsigned peers = __match_any_sync(act, d);
                const uint32_t b = sm.t.d.cnt[warp * kDigits + d];
                dst[b + __popc(peers & lanemask_lt())] = id;
                __syncwarp(act);
                if (lane == __ffs(peers) - 1) sm.t.d.cnt[warp * kDigits + d] = static_cast<uint16_t>(b + __popc(peers));
            }
            __syncwarp();
        }
        __syncthreads();
        uint16_t *t = src; src = dst; dst = t;
    }
    return src;
}

// Emit a sorted tile: positions [0, n) of perm, keys key[perm[p]] ascending
// (destination = lo + key).  Each destination's facts are summed in
// permutation order (canonical order), left to right.  Outputs go to the
// row's output index *written onwards; slot_of(i) is the row-local slot of
// tile element i.  `segs` (n 16-bit entries, free during the emit) gets the
// segment starts.  Returns the block sum of the emitted values.
template <typename SlotOf>
__device__ float emit_tile(const ReduceArgs &a, ReduceSmem &sm, const uint32_t *key, const float *val,
                           const uint16_t *perm, uint16_t *segs, int n, int64_t lo, int64_t s0, int64_t *written,
                           SlotOf slot_of) {
    const int per = (n + kRThreads - 1) / kRThreads;
    const int p0 = threadIdx.x * per;
    const int p1 = (p0 + per) < n ? (p0 + per) : n;
    int heads = 0;
    uint32_t prev = p0 > 0 && p0 < n ? key[perm[p0 - 1]] : 0xffffffffu;
    for (int p = p0; p < p1; ++p) {
        const uint32_t k = key[perm[p]];
        heads += (p == 0 || k != prev) ? 1 : 0;
        prev = k;
    }
    int64_t tot;
    const int64_t ex = block_exclusive_scan<int64_t>(heads, sm.scan_scratch, &tot);
    // every position: its output index into fact_pos; heads: segment starts
    int oi = static_cast<int>(ex) - 1;
    prev = p0 > 0 && p0 < n ? key[perm[p0 - 1]] : 0xffffffffu;
    for (int p = p0; p < p1; ++p) {
        const uint16_t i = perm[p];
        const uint32_t k = key[i];
        if (p == 0 || k != prev) { ++oi; segs[oi] = static_cast<uint16_t>(p); }
        prev = k;
        if (a.fact_pos && !a.max_mode) a.fact_pos[s0 + slot_of(i)] = static_cast<int32_t>(*written + oi);
    }
    const int nseg = static_cast<int>(tot);
    __syncthreads();
    float local = 0.0f;
    for (int sgi = threadIdx.x; sgi < nseg; sgi += kRThreads) {
        const int st = segs[sgi];
        const int en = sgi + 1 < nseg ? segs[sgi + 1] : n;
        const int64_t o = *written + sgi;
        float x = 0.0f;
        if (a.max_mode) {
            uint16_t bi = perm[st];
            x = val[bi];
            if (en - st > 1) {
                unsigned long long bk = max_tie_key(a, s0 + slot_of(bi));
                for (int q = st + 1; q < en; ++q) {
                    const uint16_t i = perm[q];
                    const float v = val[i];
                    if (max_greater(a.max_mode, v, x)) { x = v; bi = i; bk = max_tie_key(a, s0 + slot_of(i)); }
                    else if (max_equal(a.max_mode, v, x)) {
                        const unsigned long long k = max_tie_key(a, s0 + slot_of(i));
                        if (k < bk) { bi = i; bk = k; }
                    }
                }
            }
            if (a.fact_pos)
                for (int q = st; q < en; ++q) {
                    const uint16_t i = perm[q];
                    a.fact_pos[s0 + slot_of(i)] = i == bi ? static_cast<int32_t>(o) : -1;
                }
        } else {
            int q = st;
            for (; q + 4 <= en; q += 4) {  // loads issued ahead of the dependent adds
                const float v0 = val[perm[q]], v1 = val[perm[q + 1]], v2 = val[perm[q + 2]], v3 = val[perm[q + 3]];
                x += v0;
                x += v1;
                x += v2;
                x += v3;
            }
            for (; q < en; ++q) x += val[perm[q]];
        }
        a.tmp_ent[s0 + o] = static_cast<int32_t>(lo + key[perm[st]]);
        a.tmp_x[s0 + o] = x;
        local += x;
    }
    *written += tot;
    return block_sum(local, sm.fscratch);
}

// Stable sort of a tiny tile (n <= kRankSortMax): rank of element i among
// the (key, position) pairs, one pass.
__device__ uint16_t *rank_sort(const uint32_t *key, uint16_t *out, int n) {
    for (int i = threadIdx.x; i < n; i += kRThreads) {
        const uint32_t ki = key[i];
        int r = 0;
        for (int j = 0; j < n; ++j) {
            const uint32_t kj = key[j];
            r += (kj < ki || (kj == ki && j < i)) ? 1 : 0;
        }
        out[r] = static_cast<uint16_t>(i);
    }
    __syncthreads();
    return out;
}

// Sort a loaded tile (idx0 = identity) by key; returns the permutation and
// the other 16-bit buffer in *spare.
__device__ uint16_t *sort_tile(const uint32_t *key, uint16_t *idx0, uint16_t *idx1, int n, int bits, ReduceSmem &sm,
                               uint16_t **spare) {
    uint16_t *perm;
    if (n <= kRankSortMax) perm = rank_sort(key, idx1, n);
    else perm = lsd_sort(key, idx0, idx1, n, bits, sm);
    *spare = perm == idx0 ? idx1 : idx0;
    return perm;
}

// Load, in canonical order, the facts of the row's slot range whose
// destination lies in [lo, hi) into key (dst - lo), val, slot (row-local) and
// idx0 (identity), starting at tile position `pos`.  Stops before a load step
// that would overflow `cap` and returns the slot where it stopped in *next
// (ns when done).  Returns the new tile length.
__device__ int load_range(const ReduceArgs &a, ReduceSmem &sm, int64_t s0, int64_t ns, int64_t from, int64_t lo,
                          int64_t hi, uint32_t *key, float *val, uint32_t *slot, uint16_t *idx0, int pos, int cap,
                          int64_t *next) {
    int64_t fb = from;
    for (; fb < ns; fb += kLoadStep) {
        if (pos + kLoadStep > cap) break;
        int32_t d[kLoadK];
        int c = 0;
#pragma unroll
        for (int k = 0; k < kLoadK; ++k) {
            const int64_t j = fb + threadIdx.x * kLoadK + k;
            d[k] = -1;
            if (j < ns) {
                const int32_t dd = a.fact_dst[s0 + j];
                if (dd >= lo && dd < hi) { d[k] = dd; ++c; }
            }
        }
        int64_t tot;
        const int64_t ex = block_exclusive_scan<int64_t>(c, sm.scan_scratch, &tot);
        int p = pos + static_cast<int>(ex);
#pragma unroll
        for (int k = 0; k < kLoadK; ++k) {
            if (d[k] < 0) continue;
            const int64_t j = fb + threadIdx.x * kLoadK + k;
            key[p] = static_cast<uint32_t>(d[k] - lo);
            val[p] = a.fact_val[s0 + j];
            slot[p] = static_cast<uint32_t>(j);
            idx0[p] = static_cast<uint16_t>(p);
            ++p;
        }
        pos += static_cast<int>(tot);
    }
    *next = fb < ns ? fb : ns;
    __syncthreads();
    return pos;
}

// Dense window [lo, hi), hi - lo <= kDenseW: the window's facts are streamed
// in canonical order in sub-tiles; each sub-tile is stably sorted and added
// into acc[] one destination run at a time, so every destination is summed in
// canonical order.  A second stream writes fact_pos.
__device__ float dense_window(const ReduceArgs &a, ReduceSmem &sm, int64_t s0, int64_t ns, int64_t lo, int64_t hi,
                              int64_t *written) {
    TileD &t = sm.t.d;
    const int W = static_cast<int>(hi - lo);
    const int bits = bits_for(W);
    for (int d = threadIdx.x; d < kDenseW; d += kRThreads) {
        t.acc[d] = a.max_mode ? -INFINITY : 0.0f;
        t.bkey[d] = ~0ull;
        t.bslot[d] = 0xffffffffu;
    }
    for (int d = threadIdx.x; d < kDenseW / 32; d += kRThreads) t.touched[d] = 0u;
    __syncthreads();
    int64_t from = 0;
    while (from < ns) {
        int64_t next;
        const int n = load_range(a, sm, s0, ns, from, lo, hi, t.key, t.val, t.slot, t.idx[0], 0, kTileD, &next);
        from = next;
        if (n == 0) continue;
        uint16_t *spare;
        const uint16_t *perm = sort_tile(t.key, t.idx[0], t.idx[1], n, bits, sm, &spare);
        const int per = (n + kRThreads - 1) / kRThreads;
        const int p0 = threadIdx.x * per;
        const int p1 = (p0 + per) < n ? (p0 + per) : n;
        for (int p = p0; p < p1; ++p) {
            const uint32_t k = t.key[perm[p]];
            if (!(p == 0 || k != t.key[perm[p - 1]])) continue;
            if (a.max_mode) {
                float bv = t.acc[k];
                unsigned long long bk = t.bkey[k];
                uint32_t bs = t.bslot[k];
                for (int q = p; q < n && t.key[perm[q]] == k; ++q) {
                    const uint16_t i = perm[q];
                    const float v = t.val[i];
                    const unsigned long long kk = max_tie_key(a, s0 + t.slot[i]);
                    if (bs == 0xffffffffu || max_greater(a.max_mode, v, bv) || (max_equal(a.max_mode, v, bv) && kk < bk)) {
                        bv = v; bk = kk; bs = t.slot[i];
                    }
                }
                t.acc[k] = bv;
                t.bkey[k] = bk;
                t.bslot[k] = bs;
            } else {
                float accv = t.acc[k];
                for (int q = p; q < n && t.key[perm[q]] == k; ++q) accv += t.val[perm[q]];
                t.acc[k] = accv;
            }
            atomicOr(&t.touched[k >> 5], 1u << (k & 31));
        }
        __syncthreads();
    }
    // Output index of every touched destination (ordered compaction).
    int64_t nout = 0;
    float local = 0.0f;
    for (int base = 0; base < W; base += kRThreads) {
        const int d = base + threadIdx.x;
        const bool hit = d < W && ((t.touched[d >> 5] >> (d & 31)) & 1u);
        int64_t tot;
        const int64_t ex = block_exclusive_scan<int64_t>(hit ? 1 : 0, sm.scan_scratch, &tot);
        if (hit) {
            const int64_t oi = *written + nout + ex;
            t.oidx[d] = static_cast<uint32_t>(oi);
            a.tmp_ent[s0 + oi] = static_cast<int32_t>(lo + d);
            a.tmp_x[s0 + oi] = t.acc[d];
            local += t.acc[d];
        }
        nout += tot;
    }
    __syncthreads();
    if (a.fact_pos)
        for (int64_t j = threadIdx.x; j < ns; j += kRThreads) {
            const int32_t dd = a.fact_dst[s0 + j];
            if (dd >= lo && dd < hi)
                a.fact_pos[s0 + j] = (!a.max_mode || t.bslot[dd - lo] == static_cast<uint32_t>(j))
                                         ? static_cast<int32_t>(t.oidx[dd - lo]) : -1;
        }
    *written += nout;
    const float total = block_sum(local, sm.fscratch);
    return total;
}

// Bucketed row reduction ---------------------------------------------------

__device__ __forceinline__ void cas_kv(unsigned long long *key, float *val, int i, int l) {
    const unsigned long long ki = key[i], kl = key[l];
    if (kl < ki) {
        key[i] = kl;
        key[l] = ki;
        const float t = val[i];
        val[i] = val[l];
        val[l] = t;
    }
}

// Ascending sort of key[0, n) (val alongside) by the bitonic network whose
// comparators all put the smaller key first: the first step of each merge
// compares mirrored positions, the others are half-cleaners.  Comparators
// reaching n or beyond are skipped: those positions stand for +infinity,
// which is already in place.  Threads tid, tid + nt, ... take the
// comparators of a step; sync() separates the steps.
template <typename Sync>
__device__ void bitonic_sort_kv(unsigned long long *key, float *val, int n, int tid, int nt, Sync sync) {
    int m = 1;
    while (m < n) m <<= 1;
    for (int k = 2; k <= m; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            const int lj = 31 - __clz(j);
            for (int q = tid; q < (m >> 1); q += nt) {
                const int i = ((q >> lj) << (lj + 1)) | (q & (j - 1));
                const int l = j == (k >> 1) ? (i ^ (k - 1)) : (i + j);
                if (l < n) cas_kv(key, val, i, l);
            }
            sync();
        }
    }
}

// Bin b of the current chunk: its tile range.
__device__ __forceinline__ void bin_range(const TileK &t, int b, int bl, uint32_t base, int *beg, int *n) {
    const uint32_t e = t.off[b] - base;
    const uint32_t s = b == bl ? 0u : t.off[b - 1] - base;
    *beg = static_cast<int>(s);
    *n = static_cast<int>(e - s);
}

// Destination histogram of the row over nbins bins of 2^shift entities,
// turned into bin starts: off[b] = facts in bins < b (off[nbins] = total).
__device__ void bucket_hist(const ReduceArgs &a, ReduceSmem &sm, int64_t s0, int64_t ns, int shift, int nbins) {
    TileK &t = sm.t.k;
    for (int b = threadIdx.x; b <= nbins; b += kRThreads) t.off[b] = 0u;
    __syncthreads();
    int32_t d[kLoadK];
    auto fetch = [&](int64_t fb) {
#pragma unroll
        for (int k = 0; k < kLoadK; ++k) {
            const int64_t j = fb + k * kRThreads + threadIdx.x;
            d[k] = j < ns ? a.fact_dst[s0 + j] : -1;
        }
    };
    fetch(0);
    for (int64_t fb = 0; fb < ns; fb += kLoadStep) {  // the next step's loads go out before this step's atomics
        int32_t dc[kLoadK];
#pragma unroll
        for (int k = 0; k < kLoadK; ++k) dc[k] = d[k];
        if (fb + kLoadStep < ns) fetch(fb + kLoadStep);
#pragma unroll
        for (int k = 0; k < kLoadK; ++k)
            if (dc[k] >= 0 && static_cast<int64_t>(dc[k]) < a.E) atomicAdd(&t.off[dc[k] >> shift], 1u);
    }
    __syncthreads();
    const int per = (nbins + kRThreads - 1) / kRThreads;  // <= 8
    const int b0 = threadIdx.x * per;
    uint32_t v[kKBins / kRThreads];
    int64_t part = 0;
#pragma unroll
    for (int k = 0; k < kKBins / kRThreads; ++k) {
        v[k] = (k < per && b0 + k < nbins) ? t.off[b0 + k] : 0u;
        part += v[k];
    }
    int64_t tot;
    int64_t run = block_exclusive_scan<int64_t>(part, sm.scan_scratch, &tot);
#pragma unroll
    for (int k = 0; k < kKBins / kRThreads; ++k) {
        if (k < per && b0 + k < nbins) t.off[b0 + k] = static_cast<uint32_t>(run);
        run += v[k];
    }
    if (threadIdx.x == 0) t.off[nbins] = static_cast<uint32_t>(tot);
    __syncthreads();
}

// The row's facts bucketed by destination (see the section comment).
// Returns this thread's share of the row's output sum; *written counts outputs.
__device__ float bucket_row(const ReduceArgs &a, ReduceSmem &sm, int64_t s0, int64_t ns, int64_t *written) {
    TileK &t = sm.t.k;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int kb = 8;  // bins ~ half the slots, 2^8 .. 2^13
    while (kb < kKBitsMax && (int64_t(1) << (kb + 1)) < ns) ++kb;
    const int eb = bits_for(a.E);
    const int shift = eb > kb ? eb - kb : 0;
    const int nbins = static_cast<int>(((a.E - 1) >> shift) + 1);
    float local = 0.0f;
    float dense_sum = 0.0f;
    bucket_hist(a, sm, s0, ns, shift, nbins);
    int start = 0;
    while (start < nbins) {
        if (threadIdx.x == 0) {
            // largest e in (start, nbins] with off[e] - off[start] <= kTileK (bins >= start are untouched)
            const uint32_t base = t.off[start];
            int lo = start, hi = nbins;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (t.off[mid] - base <= static_cast<uint32_t>(kTileK)) lo = mid; else hi = mid - 1;
            }
            sm.chunk_end = lo;  // == start: bin `start` alone exceeds the tile
            sm.big_n = 0;
        }
        __syncthreads();
        const int bl = start;
        const int bh = sm.chunk_end;
        if (bh == bl) {
            // one bin above a tile: dense windows over its entities, then the bin starts again
            const int64_t lo = static_cast<int64_t>(bl) << shift;
            int64_t hi = static_cast<int64_t>(bl + 1) << shift;
            if (hi > a.E) hi = a.E;
            for (int64_t wlo = lo; wlo < hi; wlo += kDenseW) {
                const int64_t whi = (wlo + kDenseW) < hi ? (wlo + kDenseW) : hi;
                dense_sum += dense_window(a, sm, s0, ns, wlo, whi, written);
            }
            __syncthreads();
            bucket_hist(a, sm, s0, ns, shift, nbins);
            start = bl + 1;
            continue;
        }
        const uint32_t base = t.off[bl];
        const int C = static_cast<int>(t.off[bh] - base);  // off[bh] is not advanced by this chunk
        const int64_t cbase = static_cast<int64_t>(bl) << shift;
        __syncthreads();  // every thread has read off[bl], off[bh] before the scatter advances them
        // scatter the chunk's facts into their bins; each step's destinations
        // and values are loaded together, one step ahead of their use
        {
            int32_t d[kLoadK];
            float fv[kLoadK];
            auto fetch = [&](int64_t fb) {
#pragma unroll
                for (int k = 0; k < kLoadK; ++k) {
                    const int64_t j = fb + k * kRThreads + threadIdx.x;
                    d[k] = j < ns ? a.fact_dst[s0 + j] : -1;
                    fv[k] = j < ns ? a.fact_val[s0 + j] : 0.0f;
                }
            };
            fetch(0);
            for (int64_t fb = 0; fb < ns; fb += kLoadStep) {
                int32_t dc[kLoadK];
                float vc[kLoadK];
#pragma unroll
                for (int k = 0; k < kLoadK; ++k) { dc[k] = d[k]; vc[k] = fv[k]; }
                if (fb + kLoadStep < ns) fetch(fb + kLoadStep);
#pragma unroll
                for (int k = 0; k < kLoadK; ++k) {
                    if (dc[k] < 0 || static_cast<int64_t>(dc[k]) >= a.E) continue;
                    const int b = dc[k] >> shift;
                    if (b < bl || b >= bh) continue;
                    const int64_t j = fb + k * kRThreads + threadIdx.x;
                    const uint32_t pos = atomicAdd(&t.off[b], 1u) - base;
                    t.key[pos] = (static_cast<unsigned long long>(dc[k] - cbase) << 32) | static_cast<uint32_t>(j);
                    t.val[pos] = vc[k];
                }
            }
        }
        __syncthreads();
        // sorted positions: by rank within bins of at most kRankBinMax facts ...
        for (int p = threadIdx.x; p < C; p += kRThreads) {
            const unsigned long long k = t.key[p];
            const int b = bl + static_cast<int>((k >> 32) >> shift);
            int beg, n;
            bin_range(t, b, bl, base, &beg, &n);
            if (n > kRankBinMax) continue;
            int r = 0;
            for (int q = beg; q < beg + n; ++q) r += t.key[q] < k ? 1 : 0;
            t.inv[beg + r] = static_cast<uint16_t>(p);
        }
        // ... the larger bins listed ...
        if (threadIdx.x == 0) { sm.mb_count = 0; sm.mb_mmax = 0; }
        __syncthreads();
        for (int bb = bl + warp * 32; bb < bh; bb += kRThreads) {
            const int b = bb + lane;
            int beg = 0, n = 0;
            if (b < bh) bin_range(t, b, bl, base, &beg, &n);
            if (n > kRankBinMax) {
                const int slot = atomicAdd(&sm.mb_count, 1);  // at most kTileK / (kRankBinMax + 1)
                sm.mb_beg[slot] = static_cast<uint16_t>(beg);
                sm.mb_n[slot] = static_cast<uint16_t>(n);
                int m = 1;
                while (m < n) m <<= 1;
                atomicMax(&sm.mb_mmax, m);
            }
        }
        __syncthreads();
        const int nmb = sm.mb_count;
        {  // first comparator pair of each listed bin (m / 2 pairs each; nmb < kRThreads)
            int m = 0;
            if (threadIdx.x < nmb) {
                m = 1;
                while (m < sm.mb_n[threadIdx.x]) m <<= 1;
            }
            int64_t pairs;
            const int64_t first = block_exclusive_scan<int64_t>(m >> 1, sm.scan_scratch, &pairs);
            if (threadIdx.x < nmb) sm.mb_pair[threadIdx.x] = static_cast<int32_t>(first);
            if (threadIdx.x == 0) sm.mb_pair[nmb] = static_cast<int32_t>(pairs);
            __syncthreads();
        }
        const bool multi = sm.mb_pair[nmb] <= kMultiPairs;
        if (multi && nmb > 0) {
            // ... all sorted at once by the block, one bitonic step per barrier: each
            // thread keeps the (at most two) comparator pairs it owns across the steps
            int pb[2], pn[2], pq[2], pm[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int g = threadIdx.x + u * kRThreads;
                pb[u] = 0; pn[u] = 0; pq[u] = -1; pm[u] = 0;
                if (g < sm.mb_pair[nmb]) {
                    int lo = 0, hi = nmb - 1;  // last bin whose first pair is <= g
                    while (lo < hi) {
                        const int mid = (lo + hi + 1) >> 1;
                        if (sm.mb_pair[mid] <= g) lo = mid; else hi = mid - 1;
                    }
                    pb[u] = sm.mb_beg[lo];
                    pn[u] = sm.mb_n[lo];
                    pq[u] = g - sm.mb_pair[lo];
                    pm[u] = 2 * (sm.mb_pair[lo + 1] - sm.mb_pair[lo]);
                }
            }
            const int mmax = sm.mb_mmax;
            for (int k = 2; k <= mmax; k <<= 1) {
                for (int j = k >> 1; j > 0; j >>= 1) {
                    const int lj = 31 - __clz(j);
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        if (pq[u] < 0 || k > pm[u]) continue;  // that bin is sorted after its own stages
                        const int q = pq[u];
                        const int i = ((q >> lj) << (lj + 1)) | (q & (j - 1));
                        const int l = j == (k >> 1) ? (i ^ (k - 1)) : (i + j);
                        if (l < pn[u]) cas_kv(t.key + pb[u], t.val + pb[u], i, l);
                    }
                    __syncthreads();
                }
            }
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                if (pq[u] < 0) continue;
                const int i0 = 2 * pq[u];
                if (i0 < pn[u]) t.inv[pb[u] + i0] = static_cast<uint16_t>(pb[u] + i0);
                if (i0 + 1 < pn[u]) t.inv[pb[u] + i0 + 1] = static_cast<uint16_t>(pb[u] + i0 + 1);
            }
        }
        // (when they hold too many pairs: one warp per bin, above kWarpSortMax the whole block)
        for (int bb = bl + warp * 32; bb < bh && !multi; bb += kRThreads) {
            const int b = bb + lane;
            int beg = 0, n = 0;
            if (b < bh) bin_range(t, b, bl, base, &beg, &n);
            unsigned big = __ballot_sync(kFull, n > kRankBinMax);
            while (big) {
                const int src = __ffs(big) - 1;
                big &= big - 1;
                const int mb = __shfl_sync(kFull, b, src);
                const int mbeg = __shfl_sync(kFull, beg, src);
                const int mn = __shfl_sync(kFull, n, src);
                if (mn > kWarpSortMax) {
                    if (lane == 0) {
                        const int slot = atomicAdd(&sm.big_n, 1);
                        if (slot < kBigBinsMax) sm.big_bin[slot] = mb;
                    }
                    continue;
                }
                bitonic_sort_kv(t.key + mbeg, t.val + mbeg, mn, lane, 32, [] { __syncwarp(); });
                for (int i = lane; i < mn; i += 32) t.inv[mbeg + i] = static_cast<uint16_t>(mbeg + i);
                __syncwarp();
            }
        }
        __syncthreads();
        // each holds more than kWarpSortMax of the chunk's <= kTileK facts: at most kBigBinsMax
        const int nbig = sm.big_n < kBigBinsMax ? sm.big_n : kBigBinsMax;
        for (int k = 0; k < nbig; ++k) {
            int beg, n;
            bin_range(t, sm.big_bin[k], bl, base, &beg, &n);
            bitonic_sort_kv(t.key + beg, t.val + beg, n, threadIdx.x, kRThreads, [] { __syncthreads(); });
            for (int i = threadIdx.x; i < n; i += kRThreads) t.inv[beg + i] = static_cast<uint16_t>(beg + i);
            __syncthreads();
        }
        // destination runs, 32 sorted positions per warp step: heads counted per
        // window, one scan over the windows, then outputs and fact positions
        const int64_t wbase = *written;
        const int nwin = (C + 31) >> 5;
        auto dst_at = [&](int i) { return static_cast<uint32_t>(t.key[t.inv[i]] >> 32); };
        for (int w = warp; w < nwin; w += kRWarps) {
            const int i = w * 32 + lane;
            const uint32_t d = i < C ? dst_at(i) : 0xffffffffu;
            uint32_t dp = __shfl_up_sync(kFull, d, 1);
            if (lane == 0) dp = i > 0 ? dst_at(i - 1) : 0xffffffffu;
            const unsigned hb = __ballot_sync(kFull, i < C && d != dp);
            if (lane == 0) sm.win[w] = static_cast<int32_t>(__popc(hb));
        }
        __syncthreads();
        int64_t tot;
        {
            const int64_t wc = threadIdx.x < nwin ? sm.win[threadIdx.x] : 0;
            const int64_t wex = block_exclusive_scan<int64_t>(wc, sm.scan_scratch, &tot);
            if (threadIdx.x < nwin) sm.win[threadIdx.x] = static_cast<int32_t>(wex);
            __syncthreads();
        }
        for (int w = warp; w < nwin; w += kRWarps) {
            const int i = w * 32 + lane;
            const bool has = i < C;
            int p = 0;
            unsigned long long k = 0;
            uint32_t d = 0xffffffffu;
            if (has) { p = t.inv[i]; k = t.key[p]; d = static_cast<uint32_t>(k >> 32); }
            uint32_t dp = __shfl_up_sync(kFull, d, 1);
            uint32_t dn = __shfl_down_sync(kFull, d, 1);
            if (lane == 0) dp = i > 0 && has ? dst_at(i - 1) : 0xffffffffu;
            if (lane == 31) dn = i + 1 < C ? dst_at(i + 1) : 0xffffffffu;
            const bool head = has && d != dp;
            const unsigned hb = __ballot_sync(kFull, head);
            const int64_t o = wbase + sm.win[w] + __popc(hb & (lanemask_lt() | (1u << lane))) - 1;
            if (head) {
                float x = t.val[p];
                int q = i + 1;
                if (a.max_mode) {
                    int bq = i;
                    if (dn == d) {
                        unsigned long long bk = 0;
                        bool have_bk = false;
                        for (; q < C; ++q) {
                            const int pq = t.inv[q];
                            const unsigned long long kq = t.key[pq];
                            if (static_cast<uint32_t>(kq >> 32) != d) break;
                            const float v = t.val[pq];
                            if (max_greater(a.max_mode, v, x)) {
                                x = v; bq = q; have_bk = false;
                            } else if (max_equal(a.max_mode, v, x)) {
                                if (!have_bk) {
                                    bk = max_tie_key(a, s0 + static_cast<uint32_t>(t.key[t.inv[bq]]));
                                    have_bk = true;
                                }
                                const unsigned long long tk = max_tie_key(a, s0 + static_cast<uint32_t>(kq));
                                if (tk < bk) { bq = q; bk = tk; }
                            }
                        }
                    }
                    if (a.fact_pos)
                        for (int r = i; r < q; ++r)
                            a.fact_pos[s0 + static_cast<uint32_t>(t.key[t.inv[r]])] =
                                r == bq ? static_cast<int32_t>(o) : -1;
                } else if (dn == d) {
                    for (; q + 8 <= C; q += 8) {  // loads issued ahead of the dependent adds
                        int pq[8];
                        uint32_t dq[8];
                        float vq[8];
#pragma unroll
                        for (int u = 0; u < 8; ++u) pq[u] = t.inv[q + u];
#pragma unroll
                        for (int u = 0; u < 8; ++u) { dq[u] = static_cast<uint32_t>(t.key[pq[u]] >> 32); vq[u] = t.val[pq[u]]; }
                        int u = 0;
                        for (; u < 8 && dq[u] == d; ++u) x += vq[u];
                        if (u < 8) { q += u; break; }
                    }
                    for (; q < C && dst_at(q) == d; ++q) x += t.val[t.inv[q]];
                }
                a.tmp_ent[s0 + o] = static_cast<int32_t>(cbase + d);
                a.tmp_x[s0 + o] = x;
                local += x;
            }
            if (has && !a.max_mode && a.fact_pos) a.fact_pos[s0 + static_cast<uint32_t>(k)] = static_cast<int32_t>(o);
        }
        *written = wbase + tot;
        __syncthreads();
        start = bh;
    }
    return local + (threadIdx.x == 0 ? dense_sum : 0.0f);
}

__global__ void __launch_bounds__(kRThreads, kRowCtasPerSm) row_reduce_kernel(ReduceArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    ReduceSmem &sm = *reinterpret_cast<ReduceSmem *>(smem_raw);
    const int64_t r = a.row_order != nullptr ? static_cast<int64_t>(a.row_order[blockIdx.x]) : blockIdx.x;
    if (r >= a.rows) return;
    const int64_t ea = a.row_ptr[r], eb = a.row_ptr[r + 1];
    const int64_t s0 = a.slot_base[ea], s1 = a.slot_base[eb];
    if (s1 > a.capacity) {  // the row's slots lie past the buffers: skip it
        if (threadIdx.x == 0) {
            a.out_count[r] = 0;
            a.out_sum[r] = 0.0f;
            if (a.status) atomicOr(a.status, FL_STATUS_SLOT_OVERFLOW);
        }
        return;
    }
    const int64_t ns = s1 - s0;
    int64_t written = 0;
    float rsum = 0.0f;
    if (ns <= kRankSortMax) {
        // A tiny row: one tile sorted by rank; unused slots get the key E (sorted last).
        TileA &t = sm.t.a;
        const uint32_t sentinel = static_cast<uint32_t>(a.E);
        int valid = 0;
        for (int j = threadIdx.x; j < ns; j += kRThreads) {
            const int32_t d = a.fact_dst[s0 + j];
            const bool ok = d >= 0 && static_cast<int64_t>(d) < a.E;
            t.key[j] = ok ? static_cast<uint32_t>(d) : sentinel;
            t.val[j] = ok ? a.fact_val[s0 + j] : 0.0f;
            t.idx[0][j] = static_cast<uint16_t>(j);
            valid += ok ? 1 : 0;
        }
        const int n = static_cast<int>(block_sum<int64_t>(valid, sm.scan_scratch));
        if (n > 0) {
            const uint16_t *perm = rank_sort(t.key, t.idx[1], static_cast<int>(ns));
            rsum = emit_tile(a, sm, t.key, t.val, perm, t.idx[0], n, 0, s0, &written,
                             [](uint16_t i) { return static_cast<uint32_t>(i); });
        }
    } else {
        rsum = block_sum(bucket_row(a, sm, s0, ns, &written), sm.fscratch);
    }
    if (threadIdx.x == 0) { a.out_count[r] = written; a.out_sum[r] = rsum; }
}

// Compact per-row outputs (at the row's slot base) into a row layout and
// write normalized values.
constexpr int kCompactThreads = 256;
constexpr int kCompactTile = 4 * kCompactThreads;  // outputs per CTA step

// Compact the per-row outputs (written at each row's slot base) into the
// packed row layout and normalize them.  Persistent CTAs each take a
// contiguous run of tiles of kCompactTile consecutive output positions: one
// thread finds the rows holding the tile's first and last output, galloping
// forward from the previous tile's last row, every thread finds its own row
// inside that range, and the copies are coalesced.  The row denominators
// (empty rows included) are written by a strided loop over the rows.
__global__ void __launch_bounds__(kCompactThreads) compact_kernel(
    const int64_t *row_ptr, const int64_t *slot_base, const int64_t *out_row_ptr, int64_t rows, const int32_t *tmp_ent,
    const float *tmp_x, const float *out_sum, float eps, int32_t *out_ent, float *out_x, float *out_y,
    float *out_denom, DropoutArgs drop) {
    __shared__ int64_t span[2];
    if (out_denom)
        for (int64_t r = blockIdx.x * static_cast<int64_t>(kCompactThreads) + threadIdx.x; r < rows;
             r += static_cast<int64_t>(gridDim.x) * kCompactThreads)
            out_denom[r] = out_sum[r];
    const int64_t U = out_row_ptr[rows];
    const uint64_t key = drop.on ? dropout_key(drop) : 0ull;
    // a contiguous run of tiles per CTA: the row of each tile's last output
    // is where the next tile starts looking
    const int64_t tiles = (U + kCompactTile - 1) / kCompactTile;
    const int64_t per = (tiles + gridDim.x - 1) / gridDim.x;
    const int64_t tb = static_cast<int64_t>(blockIdx.x) * per;
    const int64_t te = (tb + per) < tiles ? (tb + per) : tiles;
    if (tb >= te) return;
    auto row_of = [&](int64_t o, int64_t lo) {  // largest r >= lo with out_row_ptr[r] <= o (galloping, then halving)
        int64_t step = 1, hi = lo;
        while (hi + step < rows && out_row_ptr[hi + step] <= o) { hi += step; step <<= 1; }
        lo = hi;
        hi = (hi + step) < rows ? (hi + step) : rows - 1;
        while (lo < hi) {
            const int64_t mid = (lo + hi + 1) >> 1;
            if (out_row_ptr[mid] <= o) lo = mid; else hi = mid - 1;
        }
        return lo;
    };
    if (threadIdx.x == 0) {
        int64_t lo = 0, hi = rows - 1;
        const int64_t o = tb * kCompactTile;
        while (lo < hi) {
            const int64_t mid = (lo + hi + 1) >> 1;
            if (out_row_ptr[mid] <= o) lo = mid; else hi = mid - 1;
        }
        span[1] = lo;
    }
    __syncthreads();
    for (int64_t tile = tb; tile < te; ++tile) {
        const int64_t t0 = tile * kCompactTile;
        const int64_t t1 = (t0 + kCompactTile) < U ? (t0 + kCompactTile) : U;
        if (threadIdx.x == 0) {
            const int64_t ra = row_of(t0, span[1]);
            span[0] = ra;
            span[1] = row_of(t1 - 1, ra);
        }
        __syncthreads();
        const int64_t ra = span[0], rb = span[1];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int64_t o = t0 + k * kCompactThreads + threadIdx.x;
            if (o >= t1) break;
            int64_t lo = ra, hi = rb;
            while (lo < hi) {
                const int64_t mid = (lo + hi + 1) >> 1;
                if (out_row_ptr[mid] <= o) lo = mid; else hi = mid - 1;
            }
            const int64_t r = lo;
            const int64_t src = slot_base[row_ptr[r]] + (o - out_row_ptr[r]);
            const float d = out_sum[r];
            const float x = tmp_x[src];
            out_ent[o] = tmp_ent[src];
            if (out_x) out_x[o] = x;
            if (out_y) {
                float y = x / (d > eps ? d : eps);
                if (drop.on) y *= dropout_factor(drop, key, o);  // the values' training dropout, in place
                out_y[o] = y;
            }
        }
        __syncthreads();  // span[] is rewritten for the next tile
    }
}

// ---------------------------------------------------------------------------
// Backward of one hop (+ normalization).
// ---------------------------------------------------------------------------
constexpr int kBThreads = 256;
constexpr int kSmemRel = 4096;  // relations whose exact grad_w accumulators fit in shared memory
constexpr int64_t kBTeamMax = 32;  // entries with at most this many facts: an 8-lane team each

struct BackwardArgs {
    const int64_t *row_ptr;
    const float *val;
    const float *w;
    int64_t rows, n;
    float eps;
    int normalize;
    const int64_t *slot_base;
    const int32_t *entry_count;
    const int32_t *fact_pos;
    const int16_t *fact_rel;
    const float *fact_m;
    const int64_t *out_row_ptr;
    const float *out_x;
    const float *out_denom;
    const float *g_y;
    float *grad_val;
    float *grad_w;
    unsigned long long *gacc;  // rows * n * 2 exact accumulators when n > kSmemRel
    const int32_t *row_order;  // block -> row (a permutation), or null
};

__global__ void __launch_bounds__(kBThreads, 5) hop_backward_kernel(BackwardArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned long long *sacc = reinterpret_cast<unsigned long long *>(smem_raw);
    __shared__ float fscratch[kBThreads / 32 + 1];
    __shared__ int64_t iscratch[kBThreads / 32 + 1];
    const int64_t r = a.row_order != nullptr ? static_cast<int64_t>(a.row_order[blockIdx.x]) : blockIdx.x;
    if (r >= a.rows) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t oa = a.out_row_ptr[r], ob = a.out_row_ptr[r + 1];
    const int64_t ea = a.row_ptr[r], eb = a.row_ptr[r + 1];
    const bool in_smem = a.n <= kSmemRel;
    unsigned long long *acc = in_smem ? sacc : a.gacc + static_cast<size_t>(r) * a.n * 2;
    for (int64_t c = threadIdx.x; c < 2 * a.n; c += kBThreads) acc[c] = 0ull;
    float d = a.out_denom ? a.out_denom[r] : 1.0f;
    float dd = d > a.eps ? d : a.eps;
    float corr = 0.0f;
    if (a.normalize) {
        float s = 0.0f;
        for (int64_t u = oa + threadIdx.x; u < ob; u += kBThreads) s += a.g_y[u] * a.out_x[u];
        s = block_sum(s, fscratch);
        corr = (d >= a.eps) ? s / (dd * dd) : 0.0f;
    }
    // Bound of |g * v * m| for the fixed-point scale.
    float gmax = 0.0f, vmax = 0.0f, mmax = 1.0f;
    for (int64_t u = oa + threadIdx.x; u < ob; u += kBThreads) {
        float g = a.normalize ? (a.g_y[u] / dd - corr) : a.g_y[u];
        gmax = fmaxf(gmax, fabsf(g));
    }
    int64_t F = 0;
    for (int64_t e = ea + threadIdx.x; e < eb; e += kBThreads) {
        vmax = fmaxf(vmax, fabsf(a.val[e]));
        F += a.entry_count[e];
    }
    if (a.fact_m) {
        float mm = 0.0f;
        for (int64_t e = ea + warp; e < eb; e += kBThreads / 32) {
            const int64_t s0 = a.slot_base[e], cnt = a.entry_count[e];
            for (int64_t f = lane; f < cnt; f += 32) mm = fmaxf(mm, fabsf(a.fact_m[s0 + f]));
        }
        mmax = block_max(mm, fscratch);
    }
    gmax = block_max(gmax, fscratch);
    vmax = block_max(vmax, fscratch);
    F = block_sum(F, iscratch);
    float bound = gmax * vmax * mmax * 1.0001f;
    const int scale = fixed_scale_for(bound, F + 1);
    __syncthreads();
    const float *wrow = a.w + r * a.n;
    // Entries of at most kBTeamMax facts: one 8-lane team each, four per
    // warp; each lane keeps two facts in flight.
    {
        const int team = lane / kTeam, tl = lane % kTeam;
        const unsigned tm = 0xffu << (team * kTeam);
        for (int64_t e0 = ea + (warp * 4); e0 < eb; e0 += kBThreads / 8) {
            const int64_t e = e0 + team;
            int64_t cnt = e < eb ? a.entry_count[e] : 0;
            const bool mine = e < eb && cnt <= kBTeamMax;
            if (mine) {
                const float v = a.val[e];
                const int64_t s0 = a.slot_base[e];
                float gv = 0.0f;
                for (int64_t f0 = 0; f0 < cnt; f0 += 2 * kTeam) {
                    int32_t fp[2];
                    int c[2];
                    float m[2];
#pragma unroll
                    for (int k = 0; k < 2; ++k) {
                        const int64_t f = f0 + k * kTeam + tl;
                        fp[k] = -1;
                        c[k] = 0;
                        m[k] = 1.0f;
                        if (f < cnt) {
                            fp[k] = a.fact_pos[s0 + f];
                            c[k] = a.fact_rel[s0 + f];
                            if (a.fact_m) m[k] = a.fact_m[s0 + f];
                        }
                    }
                    float gy[2];
#pragma unroll
                    for (int k = 0; k < 2; ++k) gy[k] = fp[k] >= 0 ? a.g_y[oa + fp[k]] : 0.0f;
#pragma unroll
                    for (int k = 0; k < 2; ++k) {
                        if (fp[k] < 0) continue;
                        const float g = a.normalize ? (gy[k] / dd - corr) : gy[k];
                        gv += g * wrow[c[k]] * m[k];
                        fixed_atomic_add(acc + 2 * c[k], to_fixed(g * v * m[k], scale));
                    }
                }
#pragma unroll
                for (int o = 1; o < kTeam; o <<= 1) gv += __shfl_xor_sync(tm, gv, o, kTeam);
                if (tl == 0) a.grad_val[e] = gv;
            }
        }
    }
    for (int64_t e = ea + warp; e < eb; e += kBThreads / 32) {
        const int64_t cnt = a.entry_count[e];
        if (cnt <= kBTeamMax) continue;  // taken by a team above
        const float v = a.val[e];
        const int64_t s0 = a.slot_base[e];
        float gv = 0.0f;
        for (int64_t f0 = 0; f0 < cnt; f0 += 128) {  // four facts per lane: the loads go out together
            int32_t fp[4];
            int c[4];
            float m[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int64_t f = f0 + k * 32 + lane;
                fp[k] = -1;
                c[k] = 0;
                m[k] = 1.0f;
                if (f < cnt) {
                    fp[k] = a.fact_pos[s0 + f];
                    c[k] = a.fact_rel[s0 + f];
                    if (a.fact_m) m[k] = a.fact_m[s0 + f];
                }
            }
            float gy[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) gy[k] = fp[k] >= 0 ? a.g_y[oa + fp[k]] : 0.0f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                if (fp[k] < 0) continue;  // an empty slot or a fact that lost a MAX coalesce
                const float g = a.normalize ? (gy[k] / dd - corr) : gy[k];
                gv += g * wrow[c[k]] * m[k];
                fixed_atomic_add(acc + 2 * c[k], to_fixed(g * v * m[k], scale));
            }
        }
        gv = warp_sum(gv);
        if (lane == 0) a.grad_val[e] = gv;
    }
    __syncthreads();
    for (int64_t c = threadIdx.x; c < a.n; c += kBThreads)
        a.grad_w[r * a.n + c] = fixed_to_float(acc[2 * c], acc[2 * c + 1], scale);
}

// Work counts of one hop added to acc: [0] live entries S, [1] relation groups
// of both sides G, [2] facts through graph edges F (entry counts minus the
// identity terms), [3] live outputs U.
__global__ void hop_stats_kernel(const int64_t *row_ptr, int64_t rows, const int32_t *ent, int64_t S, Side ori, Side inv,
                                 const int32_t *entry_count, const int64_t *out_row_ptr, int wot_i,
                                 unsigned long long *acc) {
    __shared__ long long scratch[33];
    const int64_t live = row_ptr[rows] < S ? row_ptr[rows] : S;
    long long g = 0, f = 0;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < live;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t src = ent[i];
        g += (ori.gptr[src + 1] - ori.gptr[src]) + (inv.gptr[src + 1] - inv.gptr[src]);
        f += entry_count[i] - (wot_i ? 0 : 1);
    }
    g = block_sum(g, scratch);
    f = block_sum(f, scratch);
    if (threadIdx.x == 0) {
        atomicAdd(acc + 1, static_cast<unsigned long long>(g));
        atomicAdd(acc + 2, static_cast<unsigned long long>(f));
        if (blockIdx.x == 0) {
            atomicAdd(acc + 0, static_cast<unsigned long long>(live));
            atomicAdd(acc + 3, static_cast<unsigned long long>(out_row_ptr[rows]));
        }
    }
}

// Gradient of learnable edge weights (flashlog_kernel.py:1306-1336 for SUM,
// 1590-1614 for MAX): every edge fact f of a live entry that reached an
// output (fact_pos >= 0, the position within its row's outputs) adds
// g[out_row_ptr[row] + fact_pos] * v * w[row, rel] * m * (1 - sigmoid(ew)) to
// grad_edge[triple id].  One warp per entry, lanes over its facts; the
// identity fact (rel = n - 1) has no edge.  Float atomics, as the
// reference's index_add_.
__global__ void edge_weight_grad_kernel(const int64_t *row_ptr, int64_t rows, int64_t n, const float *val, int64_t S,
                                        const float *w, const int64_t *slot_base, const int32_t *entry_count,
                                        const int32_t *fact_pos, const int16_t *fact_rel, const float *fact_m,
                                        const int32_t *fact_edge, const int64_t *out_row_ptr, const float *g,
                                        const float *edge_weight, float *grad_edge) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
    const int64_t nw = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int64_t S_live = row_ptr[rows] < S ? row_ptr[rows] : S;
    for (int64_t i = warp; i < S_live; i += nw) {
        const int64_t row = find_row(row_ptr, rows, i);
        const float v = val[i];
        const float *wrow = w + row * n;
        const float *grow = g + out_row_ptr[row];
        const int64_t f0 = slot_base[i];
        const int32_t cnt = entry_count[i];
        for (int32_t k = lane; k < cnt; k += 32) {
            const int64_t f = f0 + k;
            const int32_t rel = fact_rel[f];
            const int32_t pos = fact_pos[f];
            if (rel >= n - 1 || pos < 0) continue;
            const int32_t e = fact_edge[f];
            const float score = 1.0f / (1.0f + expf(-edge_weight[e]));
            atomicAdd(grad_edge + e, grow[pos] * v * wrow[rel] * fact_m[f] * (1.0f - score));
        }
    }
}

// x[0, min(n, *live)) = 0, grid-stride.
__global__ void zero_prefix_kernel(float *x, int64_t n, const int64_t *live) {
    const int64_t m = *live < n ? *live : n;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < m;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        x[i] = 0.0f;
}

__global__ void scatter_grad_kernel(const float *grad_sel, const int64_t *src, int64_t n, const int64_t *n_live,
                                    float *grad_full, DropoutArgs d) {
    int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i < n && (n_live == nullptr || i < *n_live)) {
        const int64_t j = src[i];
        // with dropout: the factor of position j, the backward of the full vector's dropout
        grad_full[j] = d.on ? grad_sel[i] * dropout_factor(d, dropout_key(d), j) : grad_sel[i];
    }
}

// ---------------------------------------------------------------------------
// Normalization alone (flashlog.cu:2508-2591): one CTA per row.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) normalize_forward_kernel(const int64_t *row_ptr, const float *x, int64_t rows,
                                                                float eps, float *y, float *denom) {
    __shared__ float part[256];
    const int64_t r = blockIdx.x;
    if (r >= rows) return;
    const int64_t a0 = row_ptr[r], a1 = row_ptr[r + 1];
    // 256 strided partials then a halving tree, as the reference kernel.
    float s = 0.0f;
    for (int64_t i = a0 + threadIdx.x; i < a1; i += 256) s += x[i];
    part[threadIdx.x] = s;
    __syncthreads();
    for (int stride = 128; stride > 0; stride >>= 1) {
        if (threadIdx.x < stride) part[threadIdx.x] += part[threadIdx.x + stride];
        __syncthreads();
    }
    const float raw = part[0];
    if (threadIdx.x == 0) denom[r] = raw;
    const float d = raw >= eps ? raw : eps;
    for (int64_t i = a0 + threadIdx.x; i < a1; i += 256) y[i] = x[i] / d;
}

__global__ void __launch_bounds__(256) normalize_backward_kernel(const int64_t *row_ptr, const float *x,
                                                                 const float *denom, const float *g, int64_t rows,
                                                                 float eps, float *gx) {
    __shared__ float part[256];
    const int64_t r = blockIdx.x;
    if (r >= rows) return;
    const int64_t a0 = row_ptr[r], a1 = row_ptr[r + 1];
    float s = 0.0f;
    for (int64_t i = a0 + threadIdx.x; i < a1; i += 256) s += g[i] * x[i];
    part[threadIdx.x] = s;
    __syncthreads();
    for (int stride = 128; stride > 0; stride >>= 1) {
        if (threadIdx.x < stride) part[threadIdx.x] += part[threadIdx.x + stride];
        __syncthreads();
    }
    const float raw = denom[r];
    const bool active = raw >= eps;
    const float d = active ? raw : eps;
    const float corr = active ? part[0] / (d * d) : 0.0f;
    for (int64_t i = a0 + threadIdx.x; i < a1; i += 256) gx[i] = g[i] / d - corr;
}

// One step of the in-register bitonic network over 32 keys per lane
// (position lane * 32 + e): partners J < 32 apart inside the lane.
template <int J>
__device__ __forceinline__ void rank_step_lane(unsigned long long (&x)[32], int lane, int k) {
#pragma unroll
    for (int e = 0; e < 32; ++e) {
        if (e & J) continue;
        const int f = e | J;
        const bool up = (((lane << 5) | e) & k) == 0;
        const unsigned long long lo = x[e], hi = x[f];
        const bool swap = up ? (lo > hi) : (lo < hi);
        x[e] = swap ? hi : lo;
        x[f] = swap ? lo : hi;
    }
}

// Partners j >= 32 apart: the same slot of lane ^ (j / 32).
__device__ __forceinline__ void rank_step_cross(unsigned long long (&x)[32], int lane, int j, int k) {
    const int pl = j >> 5;
    const bool lower = (lane & pl) == 0;
    const bool up = ((lane << 5) & k) == 0;
    const bool keep_min = lower == up;
#pragma unroll
    for (int e = 0; e < 32; ++e) {
        const unsigned long long y = __shfl_xor_sync(kFull, x[e], pl);
        x[e] = keep_min ? (y < x[e] ? y : x[e]) : (y > x[e] ? y : x[e]);
    }
}

// rel_rank for R <= 1024: one warp per (row, direction).  The 1024 keys
// (padded with the largest key) sit 32 per lane in registers, position
// lane * 32 + e; the bitonic network's steps below 32 compare inside a lane,
// the wider ones across lanes by shuffles: no barriers.
__global__ void __launch_bounds__(256) rel_rank_warp_kernel(const float *w, int64_t n, int64_t R, int64_t pairs,
                                                            const int32_t *rank_row, uint16_t *rank) {
    __shared__ uint16_t staged[8][1024];  // the warp's ranks, written out coalesced
    const int lane = threadIdx.x & 31;
    const int64_t rd = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
    if (rd >= pairs) return;
    const int64_t row = rd >> 1, dir = rd & 1;
    if (rank_row != nullptr && rank_row[row] != row) return;  // shares another row's ranks
    const float *wd = w + row * n + dir * R;
    uint16_t *rk = rank + rd * R;
    uint16_t *srk = staged[threadIdx.x >> 5];
    unsigned long long x[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) {
        const int j = e * 32 + lane;  // any placement: the network sorts all positions
        unsigned long long k = ~0ull;
        if (j < R) {
            const float v = wd[j];
            if (v > 0.0f)
                k = (static_cast<unsigned long long>(0xffffffffu - __float_as_uint(v)) << 32) | static_cast<unsigned>(j);
            else
                srk[j] = static_cast<uint16_t>(kNoRank);
        }
        x[e] = k;
    }
    // the network's loops stay rolled (one copy of each step kind): unrolled
    // whole it outgrows the instruction cache
#pragma unroll 1
    for (int k = 2; k <= 1024; k <<= 1) {
#pragma unroll 1
        for (int j = k >> 1; j > 0; j >>= 1) {
            switch (j) {
                case 1: rank_step_lane<1>(x, lane, k); break;
                case 2: rank_step_lane<2>(x, lane, k); break;
                case 4: rank_step_lane<4>(x, lane, k); break;
                case 8: rank_step_lane<8>(x, lane, k); break;
                case 16: rank_step_lane<16>(x, lane, k); break;
                default: rank_step_cross(x, lane, j, k); break;
            }
        }
    }
#pragma unroll
    for (int e = 0; e < 32; ++e)
        if (x[e] != ~0ull) srk[x[e] & 0xffffu] = static_cast<uint16_t>((lane << 5) | e);
    __syncwarp();
    for (int j = lane; j < R; j += 32) rk[j] = srk[j];
}

// Per (row, direction): rank[j] = the position of relation j in the order
// (w[row, dir * R + j] descending, j ascending) of the relations with w > 0,
// kNoRank for the others; by a bitonic sort of 64-bit keys in shared memory.
// One CTA per (row, direction).
__global__ void __launch_bounds__(1024) rel_rank_kernel(const float *w, int64_t n, int64_t R, int P,
                                                        const int32_t *rank_row, uint16_t *rank) {
    extern __shared__ __align__(16) unsigned long long keys[];
    uint16_t *srk = reinterpret_cast<uint16_t *>(keys + P);  // ranks, written out coalesced
    const int64_t rd = blockIdx.x;
    const int64_t row = rd >> 1, dir = rd & 1;
    if (rank_row != nullptr && rank_row[row] != row) return;  // shares another row's ranks
    const float *wd = w + row * n + dir * R;
    uint16_t *rk = rank + rd * R;
    for (int j = threadIdx.x; j < P; j += blockDim.x) {
        unsigned long long k = ~0ull;
        if (j < R) {
            const float x = wd[j];
            if (x > 0.0f)
                k = (static_cast<unsigned long long>(0xffffffffu - __float_as_uint(x)) << 32) | static_cast<unsigned>(j);
            else
                srk[j] = static_cast<uint16_t>(kNoRank);
        }
        keys[j] = k;
    }
    __syncthreads();
    // Bitonic sort.  With one element per thread (P <= blockDim.x), partners
    // closer than 32 are in the same warp and exchange by shuffles; only the
    // wider stages go through shared memory with block barriers.
    const bool one_per_thread = P <= static_cast<int>(blockDim.x) && P >= 32;
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            if (one_per_thread && j < 32) {
                // finish this k's stages j < 32 in registers
                const int i = threadIdx.x;
                unsigned long long x = i < P ? keys[i] : ~0ull;
                for (int jj = j; jj > 0; jj >>= 1) {
                    const unsigned long long y = __shfl_xor_sync(kFull, x, jj);
                    const bool up = (i & k) == 0;
                    const bool lower = (i & jj) == 0;
                    // the lower index keeps the smaller key when sorting up
                    const bool take_min = (lower == up);
                    x = take_min ? (x < y ? x : y) : (x < y ? y : x);
                }
                if (i < P) keys[i] = x;
                __syncthreads();
                break;
            }
            for (int i = threadIdx.x; i < P; i += blockDim.x) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const unsigned long long a = keys[i], b = keys[ixj];
                    const bool up = (i & k) == 0;
                    if ((a > b) == up) { keys[i] = b; keys[ixj] = a; }
                }
            }
            __syncthreads();
        }
    }
    for (int k = threadIdx.x; k < P; k += blockDim.x) {
        const unsigned long long key = keys[k];
        if (key != ~0ull) srk[key & 0xffffu] = static_cast<uint16_t>(k);
    }
    __syncthreads();
    for (int j = threadIdx.x; j < R; j += blockDim.x) rk[j] = srk[j];
}

}  // namespace

// ===========================================================================
// Host side
// ===========================================================================
static Side make_side(const fl_csr_side &s, const float *mask_csr) {
    Side d;
    d.row_ptr = s.row_ptr; d.col = s.col; d.order = s.order; d.gptr = s.group_ptr;
    d.gstart = s.group_start; d.gcount = s.group_count; d.grel = s.group_rel; d.mask_csr = mask_csr;
    return d;
}

int relation_rank(const float *w, int64_t rows, int64_t r_size, const int32_t *rank_row, uint16_t *rank,
                  cudaStream_t st) {
    FL_REQUIRE(r_size > 0 && r_size <= 16384, "relation ranks support 1..16384 relations per direction");
    int P = 1;
    while (P < r_size) P <<= 1;
    const size_t smem = static_cast<size_t>(P) * (sizeof(unsigned long long) + sizeof(uint16_t));
    static bool attr_set = false;
    if (!attr_set) {
        FL_CUDA(cudaFuncSetAttribute(rel_rank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(16384 * (sizeof(unsigned long long) + sizeof(uint16_t)))));
        attr_set = true;
    }
    if (rows > 0 && r_size <= 1024)
        launch(rel_rank_warp_kernel, static_cast<unsigned>((rows * 2 + 7) / 8), 256, 0, st, w, 2 * r_size + 1, r_size,
               rows * 2, rank_row, rank);
    else if (rows > 0)
        launch(rel_rank_kernel, static_cast<unsigned>(rows * 2), 1024, smem, st, w, 2 * r_size + 1, r_size, P,
               rank_row, rank);
    return check_launch("relation_rank");
}

int row_order(const int64_t *row_ptr, const int64_t *slot_base, int64_t rows, int32_t *order, cudaStream_t st) {
    FL_REQUIRE(rows >= 0 && rows <= kRowOrderMax, "fl_row_order handles at most %d rows (got %lld)", kRowOrderMax,
               static_cast<long long>(rows));
    if (rows == 0) return FL_OK;
    int m = 1;
    while (m < rows) m <<= 1;
    const size_t smem = static_cast<size_t>(m) * sizeof(unsigned long long);
    static bool attr_set = false;
    if (!attr_set) {
        FL_CUDA(cudaFuncSetAttribute(row_order_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(kRowOrderMax * sizeof(unsigned long long))));
        attr_set = true;
    }
    launch(row_order_kernel, 1, 1024, smem, st, row_ptr, slot_base, rows, order);
    return check_launch("row_order");
}

int csr_visibility(const int32_t *order, int64_t m, const uint8_t *mask_triple, uint8_t *vis, cudaStream_t st) {
    if (m > 0) {
        int64_t blocks = (m + 255) / 256;
        const int sms = fl_device_sm_count();
        const int64_t cap = static_cast<int64_t>(sms > 0 ? sms : 148) * 16;
        if (blocks > cap) blocks = cap;
        launch(csr_visibility_kernel, static_cast<unsigned>(blocks), 256, 0, st, order, m, mask_triple, vis);
    }
    return check_launch("csr_visibility");
}

size_t hop_workspace(int64_t rows, int64_t S) {
    size_t s = carve_bytes<int64_t>(S + 1) + scan_workspace(S > rows ? S : rows) + carve_bytes<int64_t>(rows + 1) * 3 +
               carve_bytes<float>(rows + 1);
    return s + 4096;
}

size_t hop_output_tmp_bytes(int64_t total_slots) {
    return carve_bytes<int32_t>(total_slots) + carve_bytes<float>(total_slots);
}

int hop_plan(const fl_hop_params *p, const int64_t *row_ptr, const int32_t *ent, int64_t S, const fl_csr_side &ori,
             const fl_csr_side &inv, int64_t *slot_base, int64_t *total_slots, void *ws, size_t ws_bytes,
             cudaStream_t st) {
    Carve c(ws, ws_bytes);
    int64_t *cap = c.take<int64_t>(S + 1);
    size_t sws = scan_workspace(S);
    void *scan_ws = c.take<char>(sws);
    FL_REQUIRE(cap && scan_ws, "hop workspace too small");
    (void)row_ptr;
    if (S > 0) {
        launch(hop_capacity_kernel, static_cast<unsigned>((S + 255) / 256), 256, 0, st, ent, row_ptr, p->rows, S,
               make_side(ori, nullptr), make_side(inv, nullptr), p->topk_edges, (p->flags & FL_WOT_I) ? 1 : 0,
               ((p->flags & FL_NO_ORI) ? 0 : 1) | ((p->flags & FL_NO_INV) ? 0 : 2), cap,
               reinterpret_cast<EntryInfo *>(p->entry_info));
    }
    int rc = exclusive_scan<int64_t>(cap, S, slot_base, scan_ws, sws, st);
    if (rc) return rc;
    if (total_slots) {
        FL_CUDA(cudaMemcpyAsync(total_slots, slot_base + S, sizeof(int64_t), cudaMemcpyDeviceToHost, st));
        FL_CUDA(cudaStreamSynchronize(st));
    }
    return check_launch("hop_plan");
}

int hop_expand(const fl_hop_params *p, const int64_t *row_ptr, const int32_t *ent, const float *val, int64_t S,
               const float *w, const fl_csr_side &ori, const fl_csr_side &inv, const float *mask_csr_ori,
               const float *mask_csr_inv, const uint8_t *mask_triple, const float *edge_weight,
               const int64_t *slot_base, int32_t *fact_dst, float *fact_val, int16_t *fact_rel, float *fact_m,
               int32_t *entry_count, cudaStream_t st) {
    if (S == 0) return FL_OK;
    ExpandArgs a;
    a.row_ptr = row_ptr; a.ent = ent; a.val = val; a.S = S; a.rows = p->rows; a.n = p->n; a.r_size = p->r_size;
    a.capacity = p->slot_capacity; a.status = p->status;
    a.topk = p->topk_edges; a.flags = p->flags; a.seed = p->sampling_seed; a.L = p->L; a.w = w;
    a.ori = make_side(ori, mask_csr_ori); a.inv = make_side(inv, mask_csr_inv);
    a.mask_triple = mask_triple; a.edge_weight = edge_weight; a.slot_base = slot_base;
    a.vis_ori = p->vis_ori; a.vis_inv = p->vis_inv; a.info = reinterpret_cast<const EntryInfo *>(p->entry_info); a.work = p->work;
    a.rel_rank = p->rel_rank; a.rank_row = p->rank_row; a.fact_edge = p->fact_edge;
    a.rank_bin = static_cast<int32_t>((p->r_size + kRankBins - 1) / kRankBins);
    if (a.rel_rank != nullptr && (a.rank_bin < 1 || a.rank_bin > 32)) a.rel_rank = nullptr;
    a.fact_dst = fact_dst; a.fact_val = fact_val; a.fact_rel = fact_rel; a.fact_m = fact_m; a.entry_count = entry_count;
    int sms = fl_device_sm_count();
    const int64_t per_sm = 3;  // resident CTAs per SM (registers and staging buffers)
    int64_t cap_blocks = static_cast<int64_t>(sms > 0 ? sms : 148) * per_sm * 8;
    if (p->flags & FL_SAMPLED) {
        int64_t blocks = (S + kExpandWarps - 1) / kExpandWarps;
        if (blocks > cap_blocks) blocks = cap_blocks;
        launch(hop_expand_sampled_kernel, static_cast<unsigned>(blocks), kExpandWarps * 32, 0, st, a);
    } else {
        // the rank select needs the ranks and a budget that fits the 16-bit staged counts
        const bool ranked = a.rel_rank != nullptr && a.topk >= 1 && a.topk < 65536;
        int64_t blocks = (S + 4 * kExpandWarps - 1) / (4 * kExpandWarps);
        if (a.work != nullptr) {  // resident blocks drain the work queue (4 per SM with the rank staging)
            FL_CUDA(cudaMemsetAsync(a.work, 0, 2 * sizeof(uint32_t), st));
            cap_blocks = static_cast<int64_t>(sms > 0 ? sms : 148) * (ranked ? 4 : per_sm);
        }
        if (blocks > cap_blocks) blocks = cap_blocks;
        const size_t smem_rank = sizeof(StageRank) * kExpandWarps, smem_radix = sizeof(StageBuf) * kExpandWarps;
        static bool attr_set = false;
        if (!attr_set) {
            FL_CUDA(cudaFuncSetAttribute(hop_expand_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem_rank)));
            FL_CUDA(cudaFuncSetAttribute(hop_expand_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem_radix)));
            attr_set = true;
        }
        if (ranked)
            launch(hop_expand_kernel<true>, static_cast<unsigned>(blocks), kExpandWarps * 32, smem_rank, st, a);
        else
            launch(hop_expand_kernel<false>, static_cast<unsigned>(blocks), kExpandWarps * 32, smem_radix, st, a);
    }
    return check_launch("hop_expand");
}

// Persistent compaction grid: enough CTAs for the output capacity, at most 8 per SM.
static int64_t compact_grid(int64_t rows, int64_t capacity) {
    const int sms = fl_device_sm_count();
    const int64_t cap = static_cast<int64_t>(sms > 0 ? sms : 148) * 8;
    int64_t need = (capacity + kCompactTile - 1) / kCompactTile;
    const int64_t need_rows = (rows + kCompactThreads - 1) / kCompactThreads;
    if (need < need_rows) need = need_rows;
    return need < 1 ? 1 : (need > cap ? cap : need);
}

static int reduce_rows(const int64_t *row_ptr, int64_t rows, int64_t E, const int64_t *slot_base,
                       const int32_t *fact_dst, const float *fact_val, int64_t total_slots, int32_t *fact_pos,
                       float eps, int64_t *out_row_ptr, int32_t *out_ent, float *out_x, float *out_y,
                       float *out_denom, int32_t *status, int max_mode, int64_t r_size, const int16_t *fact_rel,
                       const int32_t *fact_edge, const int32_t *row_order, void *ws, size_t ws_bytes,
                       const fl_dropout *drop, cudaStream_t st) {
    DropoutArgs dargs;
    {
        int rc = dropout_args(drop, &dargs);
        if (rc) return rc;
    }
    FL_REQUIRE(total_slots < (int64_t(1) << 32), "too many facts in one hop (%lld)", static_cast<long long>(total_slots));
    FL_REQUIRE(E < (int64_t(1) << 31), "entity count exceeds int32");
    Carve c(ws, ws_bytes);
    int64_t *out_count = c.take<int64_t>(rows + 1);
    float *out_sum = c.take<float>(rows + 1);
    size_t sws = scan_workspace(rows);
    void *scan_ws = c.take<char>(sws);
    int32_t *tmp_ent = c.take<int32_t>(total_slots > 0 ? total_slots : 1);
    float *tmp_x = c.take<float>(total_slots > 0 ? total_slots : 1);
    FL_REQUIRE(out_count && out_sum && scan_ws && tmp_ent && tmp_x, "row_reduce workspace too small");
    if (rows > 0) {
        ReduceArgs a;
        a.row_ptr = row_ptr; a.rows = rows; a.slot_base = slot_base;
        a.fact_dst = fact_dst; a.fact_val = fact_val; a.E = E; a.fact_pos = fact_pos;
        a.tmp_ent = tmp_ent; a.tmp_x = tmp_x; a.out_count = out_count; a.out_sum = out_sum;
        a.capacity = total_slots; a.status = status;
        a.max_mode = max_mode; a.r_size = r_size; a.n = 2 * r_size + 1; a.fact_rel = fact_rel; a.fact_edge = fact_edge;
        a.row_order = row_order;
        const size_t smem = sizeof(ReduceSmem);
        static bool attr_set = false;
        if (!attr_set) {
            FL_CUDA(cudaFuncSetAttribute(row_reduce_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem)));
            attr_set = true;
        }
        launch(row_reduce_kernel, static_cast<unsigned>(rows), kRThreads, smem, st, a);
        int rc = check_launch("row_reduce");
        if (rc) return rc;
    }
    int rc = exclusive_scan<int64_t>(out_count, rows, out_row_ptr, scan_ws, sws, st);
    if (rc) return rc;
    if (rows > 0)
        launch(compact_kernel, static_cast<unsigned>(compact_grid(rows, total_slots)), kCompactThreads, 0, st, row_ptr,
               slot_base, out_row_ptr, rows, tmp_ent, tmp_x,
               out_sum, eps, out_ent, out_x, out_y, out_denom, dargs);
    return check_launch("row_compact");
}

int row_reduce(const int64_t *row_ptr, int64_t rows, int64_t E, const int64_t *slot_base, const int32_t *entry_count,
               const int32_t *fact_dst, const float *fact_val, int64_t total_slots, int32_t *fact_pos, float eps,
               int64_t *out_row_ptr, int32_t *out_ent, float *out_x, float *out_y, float *out_denom, int32_t *status,
               const int32_t *row_order, void *ws, size_t ws_bytes, const fl_dropout *drop, cudaStream_t st) {
    (void)entry_count;  // unfilled slots carry the destination -1
    return reduce_rows(row_ptr, rows, E, slot_base, fact_dst, fact_val, total_slots, fact_pos, eps, out_row_ptr,
                       out_ent, out_x, out_y, out_denom, status, 0, 0, nullptr, nullptr, row_order, ws, ws_bytes, drop,
                       st);
}

int row_reduce_max(const int64_t *row_ptr, int64_t rows, int64_t E, int64_t r_size, const int64_t *slot_base,
                   const int32_t *fact_dst, const float *fact_val, const int16_t *fact_rel, const int32_t *fact_edge,
                   int64_t total_slots, int32_t *fact_pos, int64_t *out_row_ptr, int32_t *out_ent, float *out_x,
                   int max_mode, bool value_only, int32_t *status, void *ws, size_t ws_bytes, cudaStream_t st) {
    FL_REQUIRE(max_mode == 1 || max_mode == 2, "bad MAX mode");
    if (value_only) {
        fact_rel = nullptr;
        fact_edge = nullptr;
    } else {
        FL_REQUIRE(fact_rel != nullptr && fact_edge != nullptr,
                   "the MAX reduction needs fact relations and triple ids (or FL_MAX_VALUE_ONLY)");
    }
    return reduce_rows(row_ptr, rows, E, slot_base, fact_dst, fact_val, total_slots, fact_pos, 1e-7f, out_row_ptr,
                       out_ent, out_x, nullptr, nullptr, status, max_mode, r_size, fact_rel, fact_edge, nullptr, ws,
                       ws_bytes, nullptr, st);
}

size_t row_reduce_workspace(int64_t rows, int64_t total_slots) {
    return carve_bytes<int64_t>(rows + 1) + carve_bytes<float>(rows + 1) + scan_workspace(rows) +
           hop_output_tmp_bytes(total_slots) + 4096;
}

size_t hop_backward_workspace(int64_t rows, int64_t n) {
    return n > kSmemRel ? carve_bytes<unsigned long long>(static_cast<size_t>(rows) * n * 2) : 256;
}

int hop_backward(const fl_hop_params *p, const int64_t *row_ptr, const float *val, int64_t S, const float *w,
                 const int64_t *slot_base, const int32_t *entry_count, const int32_t *fact_pos, const int16_t *fact_rel,
                 const float *fact_m, const int64_t *out_row_ptr, const float *out_x, const float *out_denom,
                 const float *g_y, float *grad_val, float *grad_w, void *ws, size_t ws_bytes, cudaStream_t st) {
    (void)S;
    BackwardArgs a;
    a.row_ptr = row_ptr; a.val = val; a.w = w; a.rows = p->rows; a.n = p->n; a.eps = p->eps;
    a.normalize = (p->flags & FL_NO_NORMALIZE) ? 0 : 1;
    a.slot_base = slot_base; a.entry_count = entry_count; a.fact_pos = fact_pos; a.fact_rel = fact_rel;
    a.fact_m = fact_m; a.out_row_ptr = out_row_ptr; a.out_x = out_x; a.out_denom = out_denom; a.g_y = g_y;
    a.grad_val = grad_val; a.grad_w = grad_w; a.gacc = nullptr; a.row_order = p->row_order;
    size_t smem = 0;
    if (p->n > kSmemRel) {
        Carve c(ws, ws_bytes);
        a.gacc = c.take<unsigned long long>(static_cast<size_t>(p->rows) * p->n * 2);
        FL_REQUIRE(a.gacc != nullptr, "hop backward workspace too small");
    } else {
        smem = static_cast<size_t>(p->n) * 2 * sizeof(unsigned long long);
        static bool attr_set = false;
        if (!attr_set) {
            FL_CUDA(cudaFuncSetAttribute(hop_backward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmemRel * 2 * sizeof(unsigned long long))));
            attr_set = true;
        }
    }
    if (p->rows > 0)
        launch(hop_backward_kernel, static_cast<unsigned>(p->rows), kBThreads, smem, st, a);
    return check_launch("hop_backward");
}

int normalize_forward(const int64_t *row_ptr, const float *x, int64_t rows, float eps, float *y, float *denom,
                      cudaStream_t st) {
    if (rows > 0) launch(normalize_forward_kernel, static_cast<unsigned>(rows), 256, 0, st, row_ptr, x, rows, eps, y, denom);
    return check_launch("normalize_forward");
}

int normalize_backward(const int64_t *row_ptr, const float *x, const float *denom, const float *g, int64_t rows,
                       float eps, float *gx, cudaStream_t st) {
    if (rows > 0)
        launch(normalize_backward_kernel, static_cast<unsigned>(rows), 256, 0, st, row_ptr, x, denom, g, rows, eps, gx);
    return check_launch("normalize_backward");
}

int hop_stats(const int64_t *row_ptr, int64_t rows, const int32_t *ent, int64_t S, const fl_csr_side &ori,
              const fl_csr_side &inv, const int32_t *entry_count, const int64_t *out_row_ptr, int wot_i, int64_t *acc,
              cudaStream_t st) {
    const int sms = fl_device_sm_count();
    int64_t blocks = (S + 255) / 256;
    const int64_t cap = static_cast<int64_t>(sms > 0 ? sms : 148) * 4;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    launch(hop_stats_kernel, static_cast<unsigned>(blocks), 256, 0, st, row_ptr, rows, ent, S, make_side(ori, nullptr),
           make_side(inv, nullptr), entry_count, out_row_ptr, wot_i, reinterpret_cast<unsigned long long *>(acc));
    return check_launch("hop_stats");
}

int edge_weight_grad(const fl_hop_params *p, const int64_t *row_ptr, const float *val, int64_t S, const float *w,
                     const int64_t *slot_base, const int32_t *entry_count, const int32_t *fact_pos,
                     const int16_t *fact_rel, const float *fact_m, const int32_t *fact_edge,
                     const int64_t *out_row_ptr, const float *g, const float *edge_weight, float *grad_edge,
                     cudaStream_t st) {
    FL_REQUIRE(p != nullptr && S >= 0, "edge_weight_grad: bad arguments");
    FL_REQUIRE(slot_base && entry_count && fact_pos && fact_rel && fact_m && fact_edge && out_row_ptr && g &&
                   edge_weight && grad_edge,
               "edge_weight_grad needs the recorded facts (positions, relations, masks, triple ids)");
    if (S == 0) return FL_OK;
    const int sms = fl_device_sm_count();
    int64_t blocks = (S + 7) / 8;
    const int64_t cap = static_cast<int64_t>(sms > 0 ? sms : 148) * 8;
    if (blocks > cap) blocks = cap;
    launch(edge_weight_grad_kernel, static_cast<unsigned>(blocks), 256, 0, st, row_ptr, p->rows, p->n, val, S, w,
           slot_base, entry_count, fact_pos, fact_rel, fact_m, fact_edge, out_row_ptr, g, edge_weight, grad_edge);
    return check_launch("edge_weight_grad");
}

int zero_prefix(float *x, int64_t n, const int64_t *live, cudaStream_t st) {
    if (n <= 0) return FL_OK;
    if (live == nullptr) {
        FL_CUDA(cudaMemsetAsync(x, 0, static_cast<size_t>(n) * sizeof(float), st));
        return FL_OK;
    }
    const int sms = fl_device_sm_count();
    int64_t blocks = (n + 255) / 256;
    const int64_t cap = static_cast<int64_t>(sms > 0 ? sms : 148) * 8;
    if (blocks > cap) blocks = cap;
    launch(zero_prefix_kernel, static_cast<unsigned>(blocks), 256, 0, st, x, n, live);
    return check_launch("zero_prefix");
}

int scatter_grad(const float *grad_sel, const int64_t *src, int64_t n_sel, const int64_t *n_live, float *grad_full,
                 int64_t n_full, const int64_t *full_live, const fl_dropout *drop, cudaStream_t st) {
    DropoutArgs d;
    int rc = dropout_args(drop, &d);
    if (rc) return rc;
    rc = zero_prefix(grad_full, n_full, full_live, st);
    if (rc) return rc;
    if (n_sel > 0)
        launch(scatter_grad_kernel, static_cast<unsigned>((n_sel + 255) / 256), 256, 0, st, grad_sel, src, n_sel, n_live,
               grad_full, d);
    return check_launch("scatter_grad");
}

}  // namespace fl
