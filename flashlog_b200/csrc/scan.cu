// scan.cu -- device-wide exclusive scan of int64 counts (three phases).
#include "common.cuh"
#include "scan.cuh"

namespace fl {

namespace {
constexpr int kScanThreads = 1024;
constexpr int kScanItems = 4;
constexpr int kScanTile = kScanThreads * kScanItems;

template <typename In>
__global__ void __launch_bounds__(kScanThreads) scan_tile_sums(const In *in, int64_t n, int64_t *tile_sums) {
    __shared__ int64_t scratch[kScanThreads / 32 + 1];
    int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile;
    int64_t s = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        int64_t i = base + static_cast<int64_t>(k) * kScanThreads + threadIdx.x;
        if (i < n) s += static_cast<int64_t>(in[i]);
    }
    s = block_sum(s, scratch);
    if (threadIdx.x == 0) tile_sums[blockIdx.x] = s;
}

__global__ void __launch_bounds__(kScanThreads) scan_tile_offsets(int64_t *tile_sums, int64_t tiles, int64_t *total) {
    __shared__ int64_t scratch[kScanThreads / 32 + 1];
    int64_t carry = 0;
    for (int64_t b = 0; b < tiles; b += kScanThreads) {
        int64_t i = b + threadIdx.x;
        int64_t v = i < tiles ? tile_sums[i] : 0;
        int64_t tot;
        int64_t ex = block_exclusive_scan(v, scratch, &tot);
        if (i < tiles) tile_sums[i] = carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0 && total) *total = carry;
}

template <typename In>
__global__ void __launch_bounds__(kScanThreads) scan_apply(const In *in, int64_t n, const int64_t *tile_offsets,
                                                           int64_t *out) {
    __shared__ int64_t scratch[kScanThreads / 32 + 1];
    int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile;
    // Each thread owns kScanItems consecutive elements.
    int64_t v[kScanItems];
    int64_t s = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        int64_t i = base + static_cast<int64_t>(threadIdx.x) * kScanItems + k;
        v[k] = i < n ? static_cast<int64_t>(in[i]) : 0;
        s += v[k];
    }
    int64_t tot;
    int64_t ex = block_exclusive_scan(s, scratch, &tot) + tile_offsets[blockIdx.x];
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        int64_t i = base + static_cast<int64_t>(threadIdx.x) * kScanItems + k;
        if (i < n) out[i] = ex;
        ex += v[k];
    }
    if (blockIdx.x == gridDim.x - 1 && threadIdx.x == kScanThreads - 1) out[n] = ex;
}
// Arrays of at most kSmallTiles tiles: one block walks the tiles in order,
// carrying the running total (one launch instead of three).
constexpr int64_t kSmallTiles = 4;

template <typename In>
__global__ void __launch_bounds__(kScanThreads) scan_small(const In *in, int64_t n, int64_t *out) {
    __shared__ int64_t scratch[kScanThreads / 32 + 1];
    int64_t carry = 0;
    for (int64_t base = 0; base < n; base += kScanTile) {
        int64_t v[kScanItems];
        int64_t s = 0;
#pragma unroll
        for (int k = 0; k < kScanItems; ++k) {
            const int64_t i = base + static_cast<int64_t>(threadIdx.x) * kScanItems + k;
            v[k] = i < n ? static_cast<int64_t>(in[i]) : 0;
            s += v[k];
        }
        int64_t tot;
        int64_t ex = block_exclusive_scan(s, scratch, &tot) + carry;
#pragma unroll
        for (int k = 0; k < kScanItems; ++k) {
            const int64_t i = base + static_cast<int64_t>(threadIdx.x) * kScanItems + k;
            if (i < n) out[i] = ex;
            ex += v[k];
        }
        carry += tot;
    }
    if (threadIdx.x == 0) out[n] = carry;
}
}  // namespace

size_t scan_workspace(int64_t n) {
    int64_t tiles = (n + kScanTile - 1) / kScanTile;
    return carve_bytes<int64_t>(static_cast<size_t>(tiles + 1) + 1);
}

template <typename In>
int exclusive_scan(const In *in, int64_t n, int64_t *out, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (n <= 0) {
        FL_CUDA(cudaMemsetAsync(out, 0, sizeof(int64_t), st));
        return FL_OK;
    }
    int64_t tiles = (n + kScanTile - 1) / kScanTile;
    if (tiles <= kSmallTiles) {
        launch(scan_small<In>, 1, kScanThreads, 0, st, in, n, out);
        return check_launch("exclusive_scan");
    }
    Carve c(ws, ws_bytes);
    int64_t *tile = c.take<int64_t>(static_cast<size_t>(tiles + 1));
    FL_REQUIRE(tile != nullptr, "scan workspace too small");
    launch(scan_tile_sums<In>, static_cast<unsigned>(tiles), kScanThreads, 0, st, in, n, tile);
    launch(scan_tile_offsets, 1, kScanThreads, 0, st, tile, tiles, nullptr);
    launch(scan_apply<In>, static_cast<unsigned>(tiles), kScanThreads, 0, st, in, n, tile, out);
    return check_launch("exclusive_scan");
}

template int exclusive_scan<int64_t>(const int64_t *, int64_t, int64_t *, void *, size_t, cudaStream_t);
template int exclusive_scan<int32_t>(const int32_t *, int64_t, int64_t *, void *, size_t, cudaStream_t);

}  // namespace fl
