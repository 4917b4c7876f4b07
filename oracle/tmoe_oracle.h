/*
 * tmoe_oracle.h -- CPU restatement of Tetraeder's Qwen3-MoE layer hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path in
 * tetraeder_b200/csrc and the timed CPU baseline of bench.py.  Nothing in the
 * product links or calls it.
 *
 * What it restates (reference paths relative to the tetraeder project root):
 *   - router():           crates/model/src/qwen3moe.rs:2871-2890
 *                         (rms_norm * ffn_norm, mul_mat(gate_inp), soft_max,
 *                          argsort_top_k, get_rows, sum_rows, clamp, div)
 *   - weighted_experts(): crates/model/src/qwen3moe.rs:2899-2914
 *                         (mul_mat_id up, gate, swiglu_split, mul_mat_id down,
 *                          mul by the router weights)
 *   - sum_experts():      crates/model/src/qwen3moe.rs:2917-2923
 *                         (fold of adds in choice order)
 *   - mul_mat_id with id -1 = no weights read, exact zero row:
 *                         patches/0004-cuda-mul-mat-id-skip-negative.patch:1-10,
 *                         crates/ggml-sys/tests/mul_mat_id_skip.rs:170-191
 *   - the per-expert pair order (token-major, choice-minor):
 *                         crates/model/src/qwen3moe.rs:2126-2150 (group_pairs)
 *   - the EP id map (local slot or -1):
 *                         crates/model/src/qwen3moe_shard.rs:617-626,1043-1050
 *
 * The arithmetic of ggml itself (llama.cpp tag b12426, commit fc504f91, the
 * reference's vendor/PIN) is a third-party dependency that is not present in
 * the reference tree.  Its published algorithms are restated here:
 *   - Q4_K / Q6_K block formats and dequantisation (ggml-quants.c
 *     dequantize_row_q4_K / q6_K; pinned against gguf-py's
 *     gguf.quants.Q4_K/Q6_K.dequantize_blocks, bit for bit, in tests/);
 *   - the Q8_K activation quantiser (ggml quantize_row_q8_K_ref: per 256-block
 *     amax, iscale = -127/max, round-to-nearest-even, clamp to 127, 16 block
 *     sums, d = 1/iscale);
 *   - the K-quant x Q8_K dot (vec_dot_q4_K_q8_K / vec_dot_q6_K_q8_K): integer
 *     sub-block sums scaled by the super-block scales.
 * The Q4_K / Q6_K quantisers below are OUR OWN fits of the block formats (not
 * ggml's search).  The kernels and this oracle read the same bytes, so that
 * does not affect parity.
 *
 * Pinning.  Pinned to the reference or an independent decoder: the Q4_K / Q6_K
 * block decoders (bit for bit against gguf-py golden vectors), the pair order
 * and the -1 row semantics (the properties of the reference's own tests,
 * qwen3moe.rs:2954-3070 and mul_mat_id_skip.rs), and the Q8_K dot against the
 * reference's f64 error bound (iqk_kernels.rs:128-147).  Parity unpinned: the
 * expert-product arithmetic against ggml itself -- ggml is not in the tree and
 * the reference holds no golden MoE outputs, so that restatement follows the
 * published algorithm only.
 *
 * Canonical orders.  Selected expert ids must be bit-exact between this oracle
 * and the CUDA path, so every floating-point step that feeds the top-k is done
 * in one fixed order of IEEE operations that both sides follow
 * (tmo_router_dot, tmo_exp_canon, tmo_softmax_topk).  The library is built
 * with -ffp-contract=off so that only the explicit fmaf() calls fuse.
 */
#ifndef TMOE_ORACLE_H
#define TMOE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (ggml.h enum ggml_type) for the types this path handles. */
#define TMO_TYPE_F32 0
#define TMO_TYPE_F16 1
#define TMO_TYPE_Q4_K 12
#define TMO_TYPE_Q6_K 14
#define TMO_TYPE_Q8_K 15

#define TMO_QK_K 256
#define TMO_Q4K_BYTES 144 /* f16 d, f16 dmin, 12 B scales/mins, 128 B nibbles */
#define TMO_Q6K_BYTES 210 /* 128 B low nibbles, 64 B high bits, 16 int8 scales, f16 d */
#define TMO_Q8K_BYTES 292 /* f32 d, 256 int8, 16 int16 block sums */

/* Dot-product numerics of the expert products. */
#define TMO_MODE_Q8K 0 /* activations through Q8_K, integer block sums (the ggml CPU path) */
#define TMO_MODE_F64 1 /* dequantised weights x Q8_K round-tripped activations, f64 sum */

typedef struct {
    float d;
    int8_t qs[TMO_QK_K];
    int16_t bsums[TMO_QK_K / 16];
} tmo_block_q8k;

/* --- half precision ---------------------------------------------------- */
float tmo_f16_to_f32(uint16_t h);
uint16_t tmo_f32_to_f16(float f); /* round to nearest even */

/* --- block formats ----------------------------------------------------- */
size_t tmo_row_size(int type, int64_t ncols);
/* Quantise nrows x ncols f32 (ncols % 256 == 0).  Our own fit. */
void tmo_quantize_q4k(const float *x, void *out, int64_t nrows, int64_t ncols);
void tmo_quantize_q6k(const float *x, void *out, int64_t nrows, int64_t ncols);
void tmo_dequantize(int type, const void *in, float *out, int64_t n);
void tmo_quantize_q8k(const float *x, tmo_block_q8k *y, int64_t n);
void tmo_dequantize_q8k(const tmo_block_q8k *y, float *x, int64_t n);

/* One weight row (ncols) against one Q8_K activation row. */
float tmo_vec_dot_q4k_q8k(int64_t ncols, const void *w, const tmo_block_q8k *x);
float tmo_vec_dot_q6k_q8k(int64_t ncols, const void *w, const tmo_block_q8k *x);
/* The same two dots with AVX2 byte multiply-adds (bit-identical results). */
float tmo_vec_dot_q4k_q8k_simd(int64_t ncols, const void *w, const tmo_block_q8k *x);
float tmo_vec_dot_q6k_q8k_simd(int64_t ncols, const void *w, const tmo_block_q8k *x);
/* One Q4_K / Q6_K row against nc (1..TMO_COLS) Q8_K rows xs[c]: out[c] bit for bit the scalar dots'. */
#define TMO_COLS 8
void tmo_dot_cols(int type, int64_t ncols, const void *w, const tmo_block_q8k *const *xs, int nc, float *out);

/* --- canonical router arithmetic (bit-exact with the CUDA path) --------- */
/* e^x for finite x <= 0 (Cody-Waite reduction by ln 2, degree-7 Taylor). */
float tmo_exp_canon(float x);
/* dot(w, x) over n f32: lane l of 32 accumulates the elements whose index i has
 * (i / 4) % 32 == l in increasing i with fmaf from 0; then a butterfly sum over
 * lane distances 16, 8, 4, 2, 1. */
float tmo_router_dot(const float *w, const float *x, int64_t n);
/* ggml rms_norm (f64 sum of squares) times an optional norm weight, canonical order. */
void tmo_rms_norm(const float *x, const float *norm_w, float eps, float *out, int64_t n);
/* softmax over E logits, top-k (descending prob, ties -> lower index), renormalised weights. */
void tmo_softmax_topk(const float *logits, int E, int k, float *probs_out, int32_t *ids, float *w);

/* --- the path ---------------------------------------------------------- */
/* logits[t][e] = tmo_router_dot(router_w + e*H, xn + t*H, H). */
void tmo_router_logits(const float *xn, const float *router_w, int64_t T, int64_t H, int64_t E,
                       float *logits);

/* Full router: optional rms_norm (norm_w may be NULL: plain rms_norm; use_norm 0: x used as is),
 * logits from router_w (or taken from `logits_in` when router_w is NULL), softmax, top-k, weights.
 * xn_out, logits_out may be NULL. */
void tmo_route(const float *x, int64_t T, int64_t H, int64_t E, int k, int use_norm,
               const float *norm_w, float eps, const float *router_w, const float *logits_in,
               float *xn_out, float *logits_out, int32_t *ids, float *w);

/* Map ids through table[E] (-1 = not local); ids < 0 stay -1. */
void tmo_map_ids(const int32_t *ids, int64_t n, const int32_t *table, int64_t E, int32_t *out);

/* Per-expert pairs, token-major choice-minor; ids < 0 excluded.
 * counts[E], offsets[E+1], perm[n_pairs] (pair index t*k+j), returns the number of valid pairs. */
int64_t tmo_sort_pairs(const int32_t *ids, int64_t T, int k, int64_t E, int32_t *counts,
                       int32_t *offsets, int32_t *perm);

/* ggml mul_mat_id: W stacked [E][N rows][K] of `type` (row stride nb1, expert stride nb2 bytes),
 * b f32 [T][b1][K] (b1 == 1 or n_used), ids [T][n_used] (< 0: zero row),
 * out f32 [T][n_used][N].  mode TMO_MODE_Q8K or TMO_MODE_F64.  nthreads <= 0: all. */
int tmo_mul_mat_id(int type, const void *W, size_t nb1, size_t nb2, int64_t K, int64_t N, int64_t E,
                   const float *b, int64_t b1, int64_t T, const int32_t *ids, int n_used, float *out,
                   int mode, int nthreads);

/* weighted_experts + sum_experts for given ids and weights:
 * out[t] = sum_j (w[t][j] * down(silu(gate x_t) * up x_t)) in choice order. */
int tmo_experts(const float *x, int64_t T, int64_t H, int64_t I, int64_t E, int k,
                const int32_t *ids, const float *w, int gate_type, const void *gate, size_t gate_nb1,
                size_t gate_nb2, int up_type, const void *up, size_t up_nb1, size_t up_nb2,
                int down_type, const void *down, size_t down_nb1, size_t down_nb2, float *out,
                float *act_out, int mode, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
