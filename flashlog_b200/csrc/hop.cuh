// hop.cuh -- internal entry points of the propagation kernels.
#pragma once
#include "common.cuh"

namespace fl {
size_t hop_workspace(int64_t rows, int64_t S);
size_t row_reduce_workspace(int64_t rows, int64_t total_slots);
size_t hop_backward_workspace(int64_t rows, int64_t n);
size_t topc_workspace(int64_t rows, int64_t S);

int hop_plan(const fl_hop_params *p, const int64_t *row_ptr, const int32_t *ent, int64_t S, const fl_csr_side &ori,
             const fl_csr_side &inv, int64_t *slot_base, int64_t *total_slots, void *ws, size_t ws_bytes,
             cudaStream_t st);
int relation_rank(const float *w, int64_t rows, int64_t r_size, const int32_t *rank_row, uint16_t *rank,
                  cudaStream_t st);
int row_order(const int64_t *row_ptr, const int64_t *slot_base, int64_t rows, int32_t *order, cudaStream_t st);
int csr_visibility(const int32_t *order, int64_t m, const uint8_t *mask_triple, uint8_t *vis, cudaStream_t st);
int hop_expand(const fl_hop_params *p, const int64_t *row_ptr, const int32_t *ent, const float *val, int64_t S,
               const float *w, const fl_csr_side &ori, const fl_csr_side &inv, const float *mask_csr_ori,
               const float *mask_csr_inv, const uint8_t *mask_triple, const float *edge_weight,
               const int64_t *slot_base, int32_t *fact_dst, float *fact_val, int16_t *fact_rel, float *fact_m,
               int32_t *entry_count, cudaStream_t st);
int row_reduce_max(const int64_t *row_ptr, int64_t rows, int64_t E, int64_t r_size, const int64_t *slot_base,
                   const int32_t *fact_dst, const float *fact_val, const int16_t *fact_rel, const int32_t *fact_edge,
                   int64_t total_slots, int32_t *fact_pos, int64_t *out_row_ptr, int32_t *out_ent, float *out_x,
                   int max_mode, bool value_only, int32_t *status, void *ws, size_t ws_bytes, cudaStream_t st);
int row_reduce(const int64_t *row_ptr, int64_t rows, int64_t E, const int64_t *slot_base, const int32_t *entry_count,
               const int32_t *fact_dst, const float *fact_val, int64_t total_slots, int32_t *fact_pos, float eps,
               int64_t *out_row_ptr, int32_t *out_ent, float *out_x, float *out_y, float *out_denom, int32_t *status,
               const int32_t *row_order, void *ws, size_t ws_bytes, const fl_dropout *drop, cudaStream_t st);
int hop_backward(const fl_hop_params *p, const int64_t *row_ptr, const float *val, int64_t S, const float *w,
                 const int64_t *slot_base, const int32_t *entry_count, const int32_t *fact_pos, const int16_t *fact_rel,
                 const float *fact_m, const int64_t *out_row_ptr, const float *out_x, const float *out_denom,
                 const float *g_y, float *grad_val, float *grad_w, void *ws, size_t ws_bytes, cudaStream_t st);
int normalize_forward(const int64_t *row_ptr, const float *x, int64_t rows, float eps, float *y, float *denom,
                      cudaStream_t st);
int normalize_backward(const int64_t *row_ptr, const float *x, const float *denom, const float *g, int64_t rows,
                       float eps, float *gx, cudaStream_t st);
int zero_prefix(float *x, int64_t n, const int64_t *live, cudaStream_t st);
int edge_weight_grad(const fl_hop_params *p, const int64_t *row_ptr, const float *val, int64_t S, const float *w,
                     const int64_t *slot_base, const int32_t *entry_count, const int32_t *fact_pos,
                     const int16_t *fact_rel, const float *fact_m, const int32_t *fact_edge,
                     const int64_t *out_row_ptr, const float *g, const float *edge_weight, float *grad_edge,
                     cudaStream_t st);
int hop_stats(const int64_t *row_ptr, int64_t rows, const int32_t *ent, int64_t S, const fl_csr_side &ori,
              const fl_csr_side &inv, const int32_t *entry_count, const int64_t *out_row_ptr, int wot_i, int64_t *acc,
              cudaStream_t st);
int scatter_grad(const float *grad_sel, const int64_t *src, int64_t n_sel, const int64_t *n_live, float *grad_full,
                 int64_t n_full, const int64_t *full_live, const fl_dropout *drop, cudaStream_t st);
int topc_select(const int64_t *row_ptr, const int32_t *ent, const float *val, int64_t rows, int64_t S, int64_t c1,
                const double *noise, int64_t *out_row_ptr, int32_t *out_ent, float *out_val, int64_t *out_src,
                int64_t out_capacity, int32_t *status, void *ws, size_t ws_bytes, cudaStream_t st);
int topc_candidates(const int64_t *row_ptr, const float *val, int64_t rows, int64_t S, int64_t c1,
                    int64_t *n_candidates, void *ws, size_t ws_bytes, cudaStream_t st);
}  // namespace fl
