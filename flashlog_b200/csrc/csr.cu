// csr.cu -- CSR build on the device.
//
// Same output as the reference builder (flashlog_kernel/source/csr.cpp:12-69):
// edges ordered by (source, relation, edge id) -- the result of its two
// stable counting passes -- with row_ptr, columns, edge_rel, order (CSR
// position -> edge id), per-source relation groups (group_ptr, group_rel,
// group_start, group_count).  Here the order comes from a stable LSD radix
// sort of key = source * relations + relation over 8-bit digits: per pass a
// tile histogram, a digit-major scan and a stable in-tile scatter that ranks
// equal digits with warp match operations.
#include "common.cuh"
#include "scan.cuh"

namespace fl {
namespace {

constexpr int kCThreads = 512;
constexpr int kCWarps = kCThreads / 32;
constexpr int kCItems = 8;                       // rows of 32 per warp
constexpr int kCTile = kCThreads * kCItems;      // 4096 keys per tile

__global__ void make_keys_kernel(const int64_t *src, const int64_t *rel, int64_t m, int64_t relations,
                                 uint64_t *key, uint32_t *idx) {
    int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= m) return;
    key[i] = static_cast<uint64_t>(src[i]) * static_cast<uint64_t>(relations) + static_cast<uint64_t>(rel[i]);
    idx[i] = static_cast<uint32_t>(i);
}

__global__ void __launch_bounds__(kCThreads) tile_hist_kernel(const uint64_t *key, int64_t m, int shift, int64_t ntiles,
                                                              int32_t *hist) {
    __shared__ uint32_t h[256];
    for (int d = threadIdx.x; d < 256; d += kCThreads) h[d] = 0;
    __syncthreads();
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kCTile;
    for (int k = 0; k < kCItems; ++k) {
        int64_t i = base + static_cast<int64_t>(k) * kCThreads + threadIdx.x;
        if (i < m) atomicAdd(&h[(key[i] >> shift) & 255u], 1u);
    }
    __syncthreads();
    for (int d = threadIdx.x; d < 256; d += kCThreads) hist[static_cast<int64_t>(d) * ntiles + blockIdx.x] = h[d];
}

__global__ void __launch_bounds__(kCThreads) tile_scatter_kernel(const uint64_t *key_in, const uint32_t *idx_in,
                                                                 int64_t m, int shift, int64_t ntiles,
                                                                 const int64_t *offs, uint64_t *key_out,
                                                                 uint32_t *idx_out) {
    __shared__ uint32_t wh[kCWarps][256];
    __shared__ int64_t tile_off[256];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t base = static_cast<int64_t>(blockIdx.x) * kCTile + static_cast<int64_t>(warp) * (32 * kCItems);
    for (int d = lane; d < 256; d += 32) wh[warp][d] = 0;
    for (int d = threadIdx.x; d < 256; d += kCThreads) tile_off[d] = offs[static_cast<int64_t>(d) * ntiles + blockIdx.x];
    __syncwarp();
    for (int k = 0; k < kCItems; ++k) {
        int64_t i = base + k * 32 + lane;
        if (i < m) atomicAdd(&wh[warp][(key_in[i] >> shift) & 255u], 1u);
    }
    __syncthreads();
    // per-warp exclusive offsets within the tile (warp-major per digit)
    for (int d = threadIdx.x; d < 256; d += kCThreads) {
        uint32_t run = 0;
        for (int w = 0; w < kCWarps; ++w) { uint32_t c = wh[w][d]; wh[w][d] = run; run += c; }
    }
    __syncthreads();
    for (int k = 0; k < kCItems; ++k) {
        int64_t i = base + k * 32 + lane;
        bool valid = i < m;
        uint64_t kk = valid ? key_in[i] : 0ull;
        uint32_t d = static_cast<uint32_t>((kk >> shift) & 255u);
        unsigned act = __ballot_sync(kFull, valid);
        if (valid) {
            unsigned peers = __match_any_sync(act, d);
            int rank = __popc(peers & lanemask_lt());
            uint32_t wb = wh[warp][d];
            int64_t pos = tile_off[d] + wb + rank;
            key_out[pos] = kk;
            idx_out[pos] = idx_in[i];
            __syncwarp(act);
            if (lane == __ffs(peers) - 1) wh[warp][d] = wb + __popc(peers);
        }
        __syncwarp();
    }
}

__global__ void gather_kernel(const uint32_t *order, const int64_t *dst, const int64_t *rel, int64_t m,
                              int32_t *order_out, int32_t *col, int16_t *edge_rel) {
    int64_t j = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (j >= m) return;
    uint32_t i = order[j];
    order_out[j] = static_cast<int32_t>(i);
    col[j] = static_cast<int32_t>(dst[i]);
    edge_rel[j] = static_cast<int16_t>(rel[i]);
}

__global__ void flags_kernel(const uint64_t *key, int64_t m, int32_t *flag) {
    int64_t j = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (j < m) flag[j] = (j == 0 || key[j] != key[j - 1]) ? 1 : 0;
}

__global__ void src_hist_kernel(const int64_t *src, int64_t m, int32_t *cnt) {
    int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i < m) atomicAdd(&cnt[src[i]], 1);
}

__global__ void groups_kernel(const uint64_t *key, const int32_t *flag, const int64_t *gid, int64_t m,
                              int64_t relations, int32_t *gstart, int16_t *grel, int32_t *gsrc_cnt) {
    int64_t j = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (j >= m || !flag[j]) return;
    int64_t g = gid[j];
    gstart[g] = static_cast<int32_t>(j);
    grel[g] = static_cast<int16_t>(key[j] % static_cast<uint64_t>(relations));
    atomicAdd(&gsrc_cnt[key[j] / static_cast<uint64_t>(relations)], 1);
}

__global__ void group_count_kernel(const int32_t *gstart, int64_t G, int64_t m, int32_t *gcount) {
    int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (g < G) gcount[g] = static_cast<int32_t>((g + 1 < G ? gstart[g + 1] : m) - gstart[g]);
}

__global__ void narrow_kernel(const int64_t *in, int64_t n, int32_t *out) {
    int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i < n) out[i] = static_cast<int32_t>(in[i]);
}

__global__ void validate_kernel(const int64_t *src, const int64_t *dst, const int64_t *rel, int64_t m, int64_t nodes,
                                int64_t relations, int *bad) {
    int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= m) return;
    if (src[i] < 0 || src[i] >= nodes || dst[i] < 0 || dst[i] >= nodes || rel[i] < 0 || rel[i] >= relations)
        atomicExch(bad, 1);
}

inline unsigned grid_for(int64_t n, int t) { return static_cast<unsigned>((n + t - 1) / t); }

}  // namespace

size_t csr_build_workspace(int64_t m, int64_t nodes) {
    const int64_t ntiles = (m + kCTile - 1) / kCTile;
    const int64_t big = m > nodes + 1 ? m : nodes + 1;
    return 2 * carve_bytes<uint64_t>(m + 1) + 2 * carve_bytes<uint32_t>(m + 1) +
           carve_bytes<int32_t>(256 * ntiles + 1) + carve_bytes<int64_t>(256 * ntiles + 1) +
           carve_bytes<int32_t>(big + 1) + carve_bytes<int64_t>(big + 1) + carve_bytes<int32_t>(nodes + 1) +
           scan_workspace(256 * ntiles > big ? 256 * ntiles : big) + 4096;
}

int csr_build_side(const int64_t *src, const int64_t *dst, const int64_t *rel, int64_t m, int64_t nodes,
                   int64_t relations, int32_t *row_ptr, int32_t *col, int16_t *edge_rel, int32_t *order,
                   int32_t *group_ptr, int16_t *group_rel, int32_t *group_start, int32_t *group_count,
                   int64_t *n_groups, void *ws, size_t ws_bytes, cudaStream_t st) {
    FL_REQUIRE(m >= 0 && nodes >= 0 && nodes <= INT32_MAX && m <= INT32_MAX,
               "CSR requires equal 1D arrays and int32-sized graph");
    FL_REQUIRE(relations >= 0 && relations <= 32768, "CSR relation ID outside supported range");
    const int64_t ntiles = (m + kCTile - 1) / kCTile;
    const int64_t big = m > nodes + 1 ? m : nodes + 1;
    Carve c(ws, ws_bytes);
    uint64_t *ka = c.take<uint64_t>(m + 1), *kb = c.take<uint64_t>(m + 1);
    uint32_t *ia = c.take<uint32_t>(m + 1), *ib = c.take<uint32_t>(m + 1);
    int32_t *hist = c.take<int32_t>(256 * ntiles + 1);
    int64_t *offs = c.take<int64_t>(256 * ntiles + 1);
    int32_t *tmp32 = c.take<int32_t>(big + 1);
    int64_t *tmp64 = c.take<int64_t>(big + 1);
    int32_t *gsrc_cnt = c.take<int32_t>(nodes + 1);
    const size_t sws = scan_workspace(256 * ntiles > big ? 256 * ntiles : big);
    void *scan_ws = c.take<char>(sws);
    FL_REQUIRE(ka && kb && ia && ib && hist && offs && tmp32 && tmp64 && gsrc_cnt && scan_ws, "CSR workspace too small");
    if (m == 0) {
        FL_CUDA(cudaMemsetAsync(row_ptr, 0, (nodes + 1) * sizeof(int32_t), st));
        FL_CUDA(cudaMemsetAsync(group_ptr, 0, (nodes + 1) * sizeof(int32_t), st));
        *n_groups = 0;
        return FL_OK;
    }
    const int64_t rels = relations > 0 ? relations : 1;
    // Reject out-of-range ids before any scatter (csr.cpp:19-22).
    int *bad = reinterpret_cast<int *>(tmp32);
    int bad_host = 0;
    FL_CUDA(cudaMemsetAsync(bad, 0, sizeof(int), st));
    launch(validate_kernel, grid_for(m, 256), 256, 0, st, src, dst, rel, m, nodes, relations, bad);
    FL_CUDA(cudaMemcpyAsync(&bad_host, bad, sizeof(int), cudaMemcpyDeviceToHost, st));
    FL_CUDA(cudaStreamSynchronize(st));
    FL_REQUIRE(!bad_host, "CSR entity or relation ID outside supported range");
    launch(make_keys_kernel, grid_for(m, 256), 256, 0, st, src, rel, m, rels, ka, ia);
    const uint64_t max_key = static_cast<uint64_t>(nodes > 0 ? nodes : 1) * static_cast<uint64_t>(rels);
    int bits = 0;
    while (bits < 64 && (uint64_t(1) << bits) < max_key) ++bits;
    for (int shift = 0; shift < bits; shift += 8) {
        launch(tile_hist_kernel, static_cast<unsigned>(ntiles), kCThreads, 0, st, ka, m, shift, ntiles, hist);
        int rc = exclusive_scan<int32_t>(hist, 256 * ntiles, offs, scan_ws, sws, st);
        if (rc) return rc;
        launch(tile_scatter_kernel, static_cast<unsigned>(ntiles), kCThreads, 0, st, ka, ia, m, shift, ntiles, offs, kb, ib);
        uint64_t *tk = ka; ka = kb; kb = tk;
        uint32_t *ti = ia; ia = ib; ib = ti;
    }
    launch(gather_kernel, grid_for(m, 256), 256, 0, st, ia, dst, rel, m, order, col, edge_rel);
    // row_ptr from source counts
    FL_CUDA(cudaMemsetAsync(tmp32, 0, (nodes + 1) * sizeof(int32_t), st));
    launch(src_hist_kernel, grid_for(m, 256), 256, 0, st, src, m, tmp32);
    int rc = exclusive_scan<int32_t>(tmp32, nodes, tmp64, scan_ws, sws, st);
    if (rc) return rc;
    launch(narrow_kernel, grid_for(nodes + 1, 256), 256, 0, st, tmp64, nodes + 1, row_ptr);
    // groups
    launch(flags_kernel, grid_for(m, 256), 256, 0, st, ka, m, tmp32);
    rc = exclusive_scan<int32_t>(tmp32, m, tmp64, scan_ws, sws, st);
    if (rc) return rc;
    FL_CUDA(cudaMemcpyAsync(n_groups, tmp64 + m, sizeof(int64_t), cudaMemcpyDeviceToHost, st));
    FL_CUDA(cudaStreamSynchronize(st));
    const int64_t G = *n_groups;
    FL_CUDA(cudaMemsetAsync(gsrc_cnt, 0, (nodes + 1) * sizeof(int32_t), st));
    launch(groups_kernel, grid_for(m, 256), 256, 0, st, ka, tmp32, tmp64, m, rels, group_start, group_rel, gsrc_cnt);
    launch(group_count_kernel, grid_for(G, 256), 256, 0, st, group_start, G, m, group_count);
    rc = exclusive_scan<int32_t>(gsrc_cnt, nodes, tmp64, scan_ws, sws, st);
    if (rc) return rc;
    launch(narrow_kernel, grid_for(nodes + 1, 256), 256, 0, st, tmp64, nodes + 1, group_ptr);
    return check_launch("csr_build_side");
}

}  // namespace fl
