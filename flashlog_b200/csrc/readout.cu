// readout.cu -- channel readout of the final state at each query's target.
//
// The sparse DRUM models sum the channels of the last state
// (sum_sp_3d, src/model_DRUM_kernel_sp.py:22-28) and the loss reads the
// score of each query's target entity (log_loss_common_sp, src/utils.py:36-47).
// One thread per query binary-searches its target in each channel row (the
// entities of a row are sorted) and adds the channels in order, as the
// coalesce of the summed sparse tensor does.  The backward writes the score
// gradient to the entries it read and zeros elsewhere.
#include "common.cuh"
#include "hop.cuh"

namespace fl {
namespace {

__device__ __forceinline__ int64_t find_entity(const int32_t *ent, int64_t a, int64_t b, int64_t e) {
    while (a < b) {
        const int64_t mid = a + ((b - a) >> 1);
        if (ent[mid] < e) a = mid + 1; else b = mid;
    }
    return a;
}

__global__ void readout_kernel(const int64_t *row_ptr, const int32_t *ent, const float *val, int64_t N,
                               const int64_t *targets, int64_t Q, float *scores) {
    const int64_t q = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (q >= Q) return;
    const int64_t t = targets[q];
    float s = 0.0f;
    for (int64_t l = 0; l < N; ++l) {
        const int64_t r = q * N + l, a = row_ptr[r], b = row_ptr[r + 1];
        const int64_t k = find_entity(ent, a, b, t);
        if (k < b && ent[k] == t) s += val[k];
    }
    scores[q] = s;
}

__global__ void readout_backward_kernel(const int64_t *row_ptr, const int32_t *ent, int64_t N, const int64_t *targets,
                                        int64_t Q, const float *g, float *grad_val) {
    const int64_t q = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (q >= Q) return;
    const int64_t t = targets[q];
    for (int64_t l = 0; l < N; ++l) {
        const int64_t r = q * N + l, a = row_ptr[r], b = row_ptr[r + 1];
        const int64_t k = find_entity(ent, a, b, t);
        if (k < b && ent[k] == t) grad_val[k] = g[q];
    }
}

// SplitMix64 output function (G. Steele, D. Lea, C. Flood, "Fast splittable
// pseudorandom number generators", OOPSLA 2014): a bijective 64-bit mix, so
// keep bits are a pure function of (seed, counter, subseq, position).
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// y[i] = x[i] * (keep(i) ? scale : 0) for i < min(n, *live); keep(i) iff the
// high 32 bits of splitmix64(key + i) reach `cut` (= p * 2^32).  The same
// call on a gradient applies the same mask, which is the backward.
__global__ void value_dropout_kernel(const float *x, float *y, int64_t n, const int64_t *live, uint64_t seed,
                                     const int64_t *counter, uint64_t subseq, uint64_t cut, float scale) {
    int64_t m = n;
    if (live != nullptr && *live < m) m = *live;
    const uint64_t c = counter != nullptr ? static_cast<uint64_t>(*counter) : 0ull;
    const uint64_t key = splitmix64(seed ^ splitmix64((c << 16) | subseq));
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < m;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const bool keep = (splitmix64(key + static_cast<uint64_t>(i)) >> 32) >= cut;
        y[i] = x[i] * (keep ? scale : 0.0f);  // a dropped entry is x * 0, as in torch
    }
}

}  // namespace

int value_dropout(const float *x, float *y, int64_t n, const int64_t *live, double p, uint64_t seed,
                  const int64_t *counter, uint64_t subseq, cudaStream_t st) {
    FL_REQUIRE(n >= 0 && p >= 0.0 && p <= 1.0 && subseq < 65536, "value_dropout: need n >= 0, 0 <= p <= 1 and "
               "subseq < 65536");
    if (n == 0) return FL_OK;
    const uint64_t cut = p >= 1.0 ? (1ull << 32) : static_cast<uint64_t>(p * 4294967296.0);
    // torch's rounding: the keep probability in float, its reciprocal rounded to float
    const float scale = p >= 1.0 ? 0.0f : static_cast<float>(1.0 / static_cast<double>(static_cast<float>(1.0 - p)));
    const int sms = fl_device_sm_count();
    int64_t blocks = (n + 255) / 256;
    const int64_t cap = static_cast<int64_t>(sms > 0 ? sms : 148) * 8;
    if (blocks > cap) blocks = cap;
    launch(value_dropout_kernel, static_cast<unsigned>(blocks), 256, 0, st, x, y, n, live, seed, counter, subseq, cut,
           scale);
    return check_launch("value_dropout");
}

int readout(const int64_t *row_ptr, const int32_t *ent, const float *val, int64_t N, const int64_t *targets, int64_t Q,
            float *scores, cudaStream_t st) {
    if (Q > 0)
        launch(readout_kernel, static_cast<unsigned>((Q + 127) / 128), 128, 0, st, row_ptr, ent, val, N, targets, Q,
               scores);
    return check_launch("readout");
}

int readout_backward(const int64_t *row_ptr, const int32_t *ent, int64_t N, const int64_t *targets, int64_t Q,
                     const float *g, float *grad_val, int64_t n_val, const int64_t *val_live, cudaStream_t st) {
    int rc = zero_prefix(grad_val, n_val, val_live, st);
    if (rc) return rc;
    if (Q > 0)
        launch(readout_backward_kernel, static_cast<unsigned>((Q + 127) / 128), 128, 0, st, row_ptr, ent, N, targets,
               Q, g, grad_val);
    return check_launch("readout_backward");
}

}  // namespace fl
