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

}  // namespace

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
