// masks.cu -- CSR-ordered edge masks and gradient alignment on the row layout.
//
// fl_csr_mask is prepare_csr_masks / apply_mask_cuda of the reference
// (flashlog_kernel/flashlog_kernel.py:225-255, flashlog.cu:1286-1340): per CSR
// position p, mask[order[p]] times, with learnable edge weights, the logistic
// sigmoid of weight[order[p]].
//
// fl_align_rows gives the upstream gradient of a hop's output at the output's
// own coordinates.  Both the output and the gradient are row layouts (rows
// b * L + l, entities ascending per row), so every output entity is looked up
// by binary search inside its own row of the gradient; coordinates missing
// from the gradient get 0.
#include <math.h>

#include "common.cuh"

namespace fl {
namespace {

template <typename MaskT>
__global__ void csr_mask_kernel(const MaskT *mask, const int32_t *order, int64_t m, const float *weight,
                                float *out) {
    for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; p < m;
         p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = order[p];
        float v = static_cast<float>(mask[t]);
        if (weight != nullptr) v *= 1.0f / (1.0f + expf(-weight[t]));
        out[p] = v;
    }
}

__global__ void align_rows_kernel(const int64_t *out_b, const int64_t *out_l, const int64_t *out_e, int64_t n,
                                  int64_t L, int64_t rows, const int64_t *g_row_ptr, const int32_t *g_ent,
                                  const float *g_val, float *out) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = out_b[i] * L + out_l[i];
        float v = 0.0f;
        if (r >= 0 && r < rows) {
            int64_t lo = g_row_ptr[r], hi = g_row_ptr[r + 1];
            const int64_t e = out_e[i];
            while (lo < hi) {  // first position with entity >= e
                const int64_t mid = lo + ((hi - lo) >> 1);
                if (g_ent[mid] < e) lo = mid + 1; else hi = mid;
            }
            if (lo < g_row_ptr[r + 1] && g_ent[lo] == e) v = g_val[lo];
        }
        out[i] = v;
    }
}

unsigned grid_for(int64_t n, int threads) {
    int64_t b = (n + threads - 1) / threads;
    const int64_t cap = 148 * 16;
    return static_cast<unsigned>(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace

int csr_mask(const void *mask, int mask_kind, const int32_t *order, int64_t m, const float *weight, float *out,
             cudaStream_t st) {
    FL_REQUIRE(m >= 0 && (m == 0 || (mask && order && out)), "fl_csr_mask: bad arguments");
    FL_REQUIRE(mask_kind == FL_MASK_U8 || mask_kind == FL_MASK_F32, "fl_csr_mask: mask kind must be u8 or f32");
    if (m == 0) return FL_OK;
    if (mask_kind == FL_MASK_U8)
        launch(csr_mask_kernel<uint8_t>, grid_for(m, 256), 256, 0, st, static_cast<const uint8_t *>(mask), order, m,
               weight, out);
    else
        launch(csr_mask_kernel<float>, grid_for(m, 256), 256, 0, st, static_cast<const float *>(mask), order, m,
               weight, out);
    return check_launch("csr_mask");
}

int align_rows(const int64_t *out_b, const int64_t *out_l, const int64_t *out_e, int64_t n, int64_t L, int64_t rows,
               const int64_t *g_row_ptr, const int32_t *g_ent, const float *g_val, float *out, cudaStream_t st) {
    FL_REQUIRE(n >= 0 && L > 0 && rows >= 0, "fl_align_rows: bad shape");
    FL_REQUIRE(n == 0 || (out_b && out_l && out_e && g_row_ptr && out), "fl_align_rows: null pointer");
    if (n == 0) return FL_OK;
    launch(align_rows_kernel, grid_for(n, 256), 256, 0, st, out_b, out_l, out_e, n, L, rows, g_row_ptr, g_ent, g_val,
           out);
    return check_launch("align_rows");
}

}  // namespace fl
