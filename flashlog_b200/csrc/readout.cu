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
                                        int64_t Q, const float *g, float *grad_val, DropoutArgs d) {
    const int64_t q = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (q >= Q) return;
    const int64_t t = targets[q];
    const uint64_t key = d.on ? dropout_key(d) : 0ull;
    for (int64_t l = 0; l < N; ++l) {
        const int64_t r = q * N + l, a = row_ptr[r], b = row_ptr[r + 1];
        const int64_t k = find_entity(ent, a, b, t);
        if (k < b && ent[k] == t) grad_val[k] = d.on ? g[q] * dropout_factor(d, key, k) : g[q];
    }
}

// y[i] = x[i] * (keep(i) ? scale : 0) for i < min(n, *live): the keep bits of
// common.cuh.  The same call on a gradient applies the same mask, which is
// the backward.
__global__ void value_dropout_kernel(const float *x, float *y, int64_t n, const int64_t *live, DropoutArgs d) {
    int64_t m = n;
    if (live != nullptr && *live < m) m = *live;
    const uint64_t key = dropout_key(d);
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < m;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] = x[i] * dropout_factor(d, key, i);  // a dropped entry is x * 0, as in torch
}

}  // namespace

int dropout_args(const fl_dropout *drop, DropoutArgs *out) {
    *out = DropoutArgs{0, 0, 0, nullptr, 1.0f, 0};
    if (drop == nullptr) return FL_OK;
    const double p = drop->p;
    FL_REQUIRE(p >= 0.0 && p <= 1.0 && drop->subseq < 65536, "dropout: need 0 <= p <= 1 and subseq < 65536");
    out->seed = drop->seed;
    out->subseq = drop->subseq;
    out->counter = drop->counter;
    out->cut = p >= 1.0 ? (1ull << 32) : static_cast<uint64_t>(p * 4294967296.0);
    // torch's rounding: the keep probability in float, its reciprocal rounded to float
    out->scale = p >= 1.0 ? 0.0f : static_cast<float>(1.0 / static_cast<double>(static_cast<float>(1.0 - p)));
    out->on = 1;
    return FL_OK;
}

int value_dropout(const float *x, float *y, int64_t n, const int64_t *live, double p, uint64_t seed,
                  const int64_t *counter, uint64_t subseq, cudaStream_t st) {
    FL_REQUIRE(n >= 0, "value_dropout: n < 0");
    const fl_dropout drop{p, seed, counter, subseq};
    DropoutArgs d;
    int rc = dropout_args(&drop, &d);
    if (rc) return rc;
    if (n == 0) return FL_OK;
    const int sms = fl_device_sm_count();
    int64_t blocks = (n + 255) / 256;
    const int64_t cap = static_cast<int64_t>(sms > 0 ? sms : 148) * 8;
    if (blocks > cap) blocks = cap;
    launch(value_dropout_kernel, static_cast<unsigned>(blocks), 256, 0, st, x, y, n, live, d);
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
                     const float *g, float *grad_val, int64_t n_val, const int64_t *val_live, const fl_dropout *drop,
                     cudaStream_t st) {
    DropoutArgs d;
    int rc = dropout_args(drop, &d);
    if (rc) return rc;
    rc = zero_prefix(grad_val, n_val, val_live, st);
    if (rc) return rc;
    if (Q > 0)
        launch(readout_backward_kernel, static_cast<unsigned>((Q + 127) / 128), 128, 0, st, row_ptr, ent, N, targets,
               Q, g, grad_val, d);
    return check_launch("readout_backward");
}

}  // namespace fl
