// Launchers of the MoE layer kernels (host side of each .cu file).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#define TMOE_WT_Q4K 0
#define TMOE_WT_Q6K 1

namespace tmoe {

// route.cu
cudaError_t launch_rms_norm(const float *x, const float *norm_w, float eps, int64_t T, int H,
                            float *out, cudaStream_t st);
// The router logits; when q8_qs != NULL (and router_fuses_q8(H)) also the Q8_K rows of xn.
cudaError_t launch_router_logits(const float *xn, const float *rw, int64_t T, int H, int E, float *logits,
                                 int8_t *q8_qs, float *q8_d, int16_t *q8_bs, cudaStream_t st);
bool router_fuses_q8(int H);
cudaError_t launch_softmax_topk(const float *logits, int64_t T, int E, int k, int32_t *ids,
                                float *w, float *probs, cudaStream_t st);
cudaError_t launch_quantize_q8k(const float *x, int64_t rows, int K, const int32_t *valid,
                                int8_t *qs, float *d, int16_t *bsums, cudaStream_t st);

// dispatch.cu
size_t sort_pairs_smem(int n_slots);
cudaError_t launch_sort_pairs(const int32_t *ids, int n_pairs, int n_slots, int32_t *counts,
                              int32_t *offsets, int32_t *perm, int32_t *active, int32_t *n_active,
                              int *err, cudaStream_t st);
// Fused softmax/top-k + optional EP map + dispatch for T*k <= ROUTE_FUSED_MAX_PAIRS.
#define ROUTE_FUSED_MAX_PAIRS 4096
bool route_dispatch_fits(int64_t T, int k, int E, int n_slots);
cudaError_t launch_route_dispatch(const float *logits, int T, int E, int k, const int32_t *table, int n_table,
                                  int32_t *ids_out, float *w_out, int32_t *mapped, int n_slots, int32_t *counts,
                                  int32_t *offsets, int32_t *perm, int32_t *active, int32_t *n_active, int *err,
                                  cudaStream_t st);
cudaError_t launch_map_ids(const int32_t *ids, int64_t n, const int32_t *table, int64_t n_table,
                           int32_t *out, cudaStream_t st);
cudaError_t launch_zero_invalid_rows(const int32_t *ids, int64_t n_pairs, int n_slots, int N,
                                     float *out, cudaStream_t st);
cudaError_t launch_combine(const float *dout, const int32_t *ids, const float *w, int64_t T, int k,
                           int H, int n_slots, float *out, cudaStream_t st);

// quant.cu
cudaError_t launch_quantize(int wt, const float *x, int64_t nblocks, uint8_t *out, cudaStream_t st);
cudaError_t launch_dequantize(int wt, const uint8_t *in, int64_t n, float *out, cudaStream_t st);

// gemv.cu
struct GemvArgs {
    const uint8_t *w0;  // gate (or the single matrix)
    const uint8_t *w1;  // up (GATEUP only)
    size_t nb1_0, nb2_0, nb1_1, nb2_1;
    int K;  // columns, multiple of 256
    int N;  // rows per expert
    const int8_t *xq;  // Q8_K activations, SoA rows of K
    const float *xd;
    const int16_t *xb;
    const float *xf;   // or f32 activation rows, quantised to Q8_K while staged (xq/xd/xb unused)
    int x_div;  // activation row of pair p = p / x_div
    const int32_t *perm, *offsets, *active, *n_active;
    int n_slots;     // experts in the weight tensors (active ids are checked against it)
    int max_active;  // the grid was sized for at most this many active experts
    int n_pairs;     // pair rows of perm / out
    float *out;  // [pairs][N]
    int *err;
    // filled by the launcher
    int tiles;
    int n_stages;
    uint32_t stage_bytes;
    int tokcap;      // activation rows staged in shared memory at a time
    int row_stride;  // shared-memory row (Q4_K) or 8-row group (Q6_K) stride
    int mat_stride;  // shared-memory bytes of one matrix of a stage
};
// Rows per work item of the GEMV for K columns and N rows per expert; 0 if N does not fit.
int gemv_rows_per_item(int wt, int K, int N);
cudaError_t launch_gemv(int wt, bool gateup, const GemvArgs &a, int max_items, int sm_count,
                        cudaStream_t st);

}  // namespace tmoe
