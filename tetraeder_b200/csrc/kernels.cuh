// Launchers of the MoE layer kernels (host side of each .cu file).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#define TMOE_WT_Q4K 0
#define TMOE_WT_Q6K 1
#define TMOE_WT_Q6KR 2  // Q6_K in 8-row fragment order (TMOE_Q6R_UNIT); Q8_K activations as for Q6_K

struct tmoe_comm;

namespace tmoe {

// While a PdlScope(true) lives on this thread, launch_k launches with programmatic stream
// serialization: the kernel may start during its predecessor's tail (see pdl_wait in common.cuh).
struct PdlScope {
    bool prev;
    explicit PdlScope(bool on);
    ~PdlScope();
};
bool pdl_on();

template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    if (pdl_on()) {
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// ep.cu: in-place sum of n floats over the communicator's ranks (stream-ordered); TMOE_OK or
// TMOE_E_COMM with a message.
int ep_allreduce_sum(tmoe_comm *c, float *buf, size_t n, cudaStream_t st, char *msg, size_t msg_len);
int ep_comm_device(const tmoe_comm *c);
int ep_comm_ranks(const tmoe_comm *c, int *rank);
struct EpBuf {
    const void *send;  // [nranks][bytes_per_peer]
    void *recv;        // [nranks][bytes_per_peer]
    size_t bytes_per_peer;
};
int ep_allgather_bytes(tmoe_comm *c, const void *send, void *recv, size_t bytes, cudaStream_t st, char *msg,
                       size_t msg_len);
// copy_self: also copy this rank's own block send -> recv (false when the producer wrote it in place)
int ep_alltoall(tmoe_comm *c, const EpBuf *bufs, int nbufs, cudaStream_t st, char *msg, size_t msg_len,
                bool copy_self = true);
// ep_a2a.cu: the token dispatch and combine of the all-to-all mode (see ep_a2a.cu)
cudaError_t launch_ep_pack(const int32_t *ids, const float *w, const float *x, int T, int k, int H, int per, int g,
                           int cap, int self, int32_t *row_of, int32_t *s_ids, float *s_w, int32_t *r_ids,
                           float *r_w, int32_t *s_tok, int32_t *counts, float *s_x, float *r_x, cudaStream_t st);
cudaError_t launch_ep_combine(const float *ret, const float *part, int self, const int32_t *row_of, int T, int H,
                              int g, int cap, float *out, cudaStream_t st);
// The exchange over peer memory (ep_a2a.cu): every rank's receive buffers, mapped into this
// process (this rank's own included), and its arrival counters flags[2][g]: [0][p] counts the
// dispatch messages rank p has finished writing here, [1][p] its returns.
constexpr int EP_MAX_PEERS = 8;
struct EpPeers {
    int32_t *r_ids[EP_MAX_PEERS];
    float *r_w[EP_MAX_PEERS];
    float *r_x[EP_MAX_PEERS];
    float *ret[EP_MAX_PEERS];
    int *flags[EP_MAX_PEERS];
};
// ctl: this rank's counters: [0..1] messages sent per direction, [2..3] CTA tallies of the
// writing kernels (zero between calls), [4..] seen[2][g] (messages consumed per direction, peer).
cudaError_t launch_ep_dispatch_p2p(const int32_t *ids, const float *w, const float *x, int T, int k, int H, int per,
                                   int g, int cap, int self, const EpPeers &P, int32_t *row_of, int32_t *s_tok,
                                   int32_t *counts, int *ctl, cudaStream_t st);
cudaError_t launch_ep_return_p2p(const float *part, const int32_t *r_ids, int k, int H, int g, int cap, int self,
                                 const EpPeers &P, int *ctl, cudaStream_t st);
// Waits (bounded) until every peer's next message of direction `dir` has arrived; on a timeout
// latches TMOE_DEV_ERR_TIMEOUT in err and returns.
cudaError_t launch_ep_wait(int dir, int g, int self, const int *flags, int *ctl, int *err, cudaStream_t st);

// Q8_K rows as the expert GEMV reads them: qs int8 [rows][K], d f32 [rows][K/256], and per
// super-block the activation sums over the weight type's sub-blocks (32 elements for Q4_K, 16 for
// Q6_K), split exactly as B = 64 * hi + lo, lo in [0, 64): bl (u8 bytes) / bh (s8 bytes)
// [rows][K/256][nbw] words, nbw = 2 (Q4_K) or 4 (Q6_K).
struct Q8Rows {
    int8_t *qs;
    float *d;
    uint32_t *bl, *bh;
    int wt;  // the consumer's weight type: TMOE_WT_Q4K, TMOE_WT_Q6K or TMOE_WT_Q6KR
};
inline int q8_nbw(int wt) { return wt == TMOE_WT_Q4K ? 2 : 4; }
// Where element e (0..255) of a Q8_K block sits in the stored block.  Q6_K consumers: the MMA
// fragment order (m16n8k16 per 16-element sub-block, thread t4 of a column holding elements
// 4 t4 .. 4 t4 + 3 of each), e = 16 s + 4 t4 + c -> 64 t4 + 4 s + c, so that the thread's operand
// bytes of the whole block are 64 contiguous bytes (four 16-byte loads instead of sixteen 4-byte
// ones).  Q4_K consumers: element order (a thread's 8-byte operands are already contiguous; the
// same reordering measured slower there: C2 T = 64 gate/up 64.8 us against 60.6).
__host__ __device__ inline int q8_frag_pos(int wt, int e) {
    if (wt == TMOE_WT_Q4K) return e;
    return 64 * ((e >> 2) & 3) + 4 * (e >> 4) + (e & 3);
}

// route.cu
cudaError_t launch_rms_norm(const float *x, const float *norm_w, float eps, int64_t T, int H, float *out,
                            cudaStream_t st);
// The router logits; with q8 (non-NULL, router_fuses_q8(H, T)) also the Q8_K rows of xn.
cudaError_t launch_router_logits(const float *xn, const float *rw, int64_t T, int H, int E, float *logits,
                                 const Q8Rows *q8, int *err, cudaStream_t st);
bool router_fuses_q8(int H, int64_t T);
cudaError_t launch_softmax_topk(const float *logits, int64_t T, int E, int k, int32_t *ids, float *w, float *probs,
                                cudaStream_t st);
// Q8_K of rows of K f32; rows whose valid entry is negative are skipped (valid may be NULL).
cudaError_t launch_quantize_q8k(const float *x, int64_t rows, int K, const int32_t *valid, const Q8Rows &out,
                                cudaStream_t st);
// bf16 [n] -> f32 [n] (exact; n % 8 == 0 and 16-byte aligned pointers use 16-byte accesses)
cudaError_t launch_widen_bf16(const uint16_t *x, int64_t n, float *out, cudaStream_t st);

// dispatch.cu
size_t sort_pairs_smem(int n_slots);
// The dispatch also zeroes `counters` (n_counters ints: the GEMV work counters; may be NULL).
// active: the experts with pairs, {e, offsets[e], offsets[e + 1], 0} each, n_active[0] of them.
// With scratch (sort_scratch_ints(n_pairs, n_slots) ints) and many pairs the sort runs over many CTAs
// (the same permutation); otherwise in one CTA.
size_t sort_scratch_ints(int64_t n_pairs, int n_slots);
cudaError_t launch_sort_pairs(const int32_t *ids, int n_pairs, int n_slots, int32_t *counts, int32_t *offsets,
                              int32_t *perm, int4 *active, int32_t *n_active, int *counters, int n_counters,
                              int *err, cudaStream_t st, int32_t *scratch = nullptr, size_t scratch_ints = 0);
// Fused softmax/top-k + optional EP map + dispatch for T*k <= ROUTE_FUSED_MAX_PAIRS.
#define ROUTE_FUSED_MAX_PAIRS 4096
bool route_dispatch_fits(int64_t T, int k, int E, int n_slots);
cudaError_t launch_route_dispatch(const float *logits, int T, int E, int k, const int32_t *table, int n_table,
                                  int32_t *ids_out, float *w_out, int32_t *mapped, int n_slots, int32_t *counts,
                                  int32_t *offsets, int32_t *perm, int4 *active, int32_t *n_active,
                                  int *counters, int n_counters, int *err, cudaStream_t st);
// The decode regime's routing in one launch (logits + Q8_K of x + top-k + map + dispatch) when
// route_fused_fits; done: route_fused_tiles(...) + 1 ints, zero before the first launch.
bool route_fused_fits(int64_t T, int k, int E, int H, int n_slots);
int route_fused_tiles(int64_t T, int k, int E, int H, int n_slots);
cudaError_t launch_route_fused(const float *x, const float *rw, int T, int H, int E, int k, const Q8Rows *q8,
                               float *logits, const int32_t *table, int n_table, int32_t *ids_out, float *w_out,
                               int32_t *mapped, int n_slots, int32_t *counts, int32_t *offsets, int32_t *perm,
                               int4 *active, int32_t *n_active, int *counters, int n_counters, int *done, int *err,
                               cudaStream_t st);
cudaError_t launch_map_ids(const int32_t *ids, int64_t n, const int32_t *table, int64_t n_table, int32_t *out,
                           cudaStream_t st);
cudaError_t launch_zero_invalid_rows(const int32_t *ids, int64_t n_pairs, int n_slots, int N, float *out,
                                     cudaStream_t st);
cudaError_t launch_combine(const float *dout, const int32_t *ids, const float *w, int64_t T, int k, int H,
                           int n_slots, float *out, cudaStream_t st);
cudaError_t launch_wait_flag(const int32_t *flag, int32_t value, uint64_t limit_ns, int *err, cudaStream_t st);

// quant.cu
cudaError_t launch_quantize(int wt, const float *x, int64_t nblocks, uint8_t *out, cudaStream_t st);
cudaError_t launch_dequantize(int wt, const uint8_t *in, int64_t n, float *out, cudaStream_t st);
// Q6_K matrices (n_mats x n_rows rows, nb1 / nb2 apart) into 8-row fragment order, contiguous at dst.
cudaError_t launch_prepack_q6k(const uint8_t *src, size_t nb1, size_t nb2, int64_t n_rows, int K, int64_t n_mats,
                               uint8_t *dst, cudaStream_t st);
// out[i][:K] = row rows[i] of W (ggml type 0 F32, 1 F16, 12 Q4_K, 14 Q6_K; n_rows_w rows nb1 apart);
// a row outside [0, n_rows_w) gives zeros and latches TMOE_DEV_ERR_BADID in err.
cudaError_t launch_get_rows(int32_t type, const uint8_t *W, size_t nb1, int K, int64_t n_rows_w, const int32_t *rows,
                            int64_t n, float *out, int *err, cudaStream_t st);
// model.cu: the decode step around the MoE layer
cudaError_t launch_rope_neox(float *x, const int32_t *pos, int64_t n_tok, int n_head, int head_dim, int n_rot,
                             float freq_base, cudaStream_t st);
cudaError_t launch_qk_norm_rope(float *q, float *k, const float *qw, const float *kw, const int32_t *pos, int64_t T,
                                int n_head, int n_kv, int d, int n_rot, float freq_base, float eps, cudaStream_t st);
int attn_splits(int B, int n_kv, int n_ctx, int sm_count);
size_t attn_scratch_floats(int B, int n_head, int head_dim, int n_kv, int n_ctx, int sm_count);
cudaError_t launch_attn_decode(const float *q, const float *k, const float *v, __half *kc, __half *vc,
                               const int32_t *pos, int B, int n_head, int n_kv, int head_dim, int n_ctx, float scale,
                               float *part, float *out, int sm_count, int *err, cudaStream_t st);
cudaError_t launch_attn_prefill(const float *q, const float *k, const float *v, __half *kc, __half *vc, int seq,
                                int pos0, int S, int n_head, int n_kv, int head_dim, int n_ctx, float scale, float *out,
                                cudaStream_t st);
cudaError_t launch_add(const float *a, const float *b, float *out, int64_t n, cudaStream_t st);
cudaError_t launch_dense_prep(int T, int group, int ks, int4 *active, int32_t *n_active, int32_t *perm, int *counters,
                              int n_counters, cudaStream_t st);
cudaError_t launch_splitk_sum(const float *part, int64_t T, int N, int ks, float *out, cudaStream_t st);
cudaError_t launch_argmax(const float *x, int64_t rows, int64_t n, int32_t *out, cudaStream_t st);

// gemv.cu
struct GemvArgs {
    const uint8_t *w0;  // gate (or the single matrix)
    const uint8_t *w1;  // up (GATEUP only)
    size_t nb1_0, nb2_0, nb1_1, nb2_1;
    int K;  // columns, multiple of 256
    int N;  // rows per expert
    // Q8_K activation rows (Q8Rows layout for this weight type); the row of pair p is p / x_div
    const int8_t *xq;
    const float *xd;
    const uint32_t *xbl, *xbh;
    int x_div;
    const int32_t *perm;   // 16 bytes past the last pair are readable (bulk copies round up)
    const int4 *active;    // {e, first pair, end pair, 0} per active expert (launch_sort_pairs)
    const int32_t *n_active;
    int n_slots;     // experts in the weight tensors (active ids are checked against it)
    int max_active;  // the grid was sized for at most this many active experts
    int n_pairs;     // pair rows of perm / out
    int *work;       // work counter, zero at launch (the dispatch kernels zero it)
    float *out;      // [pairs][N]
    int *err;
    // the dispatch data (n_active, active, perm, work) were written two or more launches back, so
    // that under programmatic launch the kernel may read them and issue its first weight fills
    // before it waits for its predecessor (non-gate/up only)
    int early;
    // filled by the launcher
    int tiles;         // items per active expert
    int chunk_blocks;  // super-blocks per fill
    int n_chunks;      // fills per row span of K
    int row_stride;    // shared-memory bytes per fill row
    int slot_bytes;    // shared-memory bytes per slot (16 rows, then the pass's pair indices)
    int wbytes;        // weight bytes of a slot
    int d_slots;       // slots per warp
    int spread;        // items dealt one per warp over the whole grid (few items)
    uint64_t tiles_m, xdiv_m;  // ceil(2^40 / tiles), ceil(2^40 / x_div): exact division of n < 2^24
};
// prefill.cu: the grouped tcgen05 GEMMs of the large-batch regime (see prefill.cu)
bool prefill_fits(int H, int I);
// n_valid (device, may be NULL): rows past it (no dispatched pair) are skipped.
cudaError_t launch_prep_rows(const float *src, const int32_t *perm, int n_rows, const int32_t *n_valid, int x_div,
                             int K, __half *dst, cudaStream_t st);
cudaError_t launch_dequant_f16(int wt, const uint8_t *w, size_t nb2, int N, int K, const int4 *active,
                               const int32_t *n_active, int max_active, __half *dst, cudaStream_t st);
cudaError_t launch_prefill_gemm(bool swiglu, const __half *A, int n_rows, int K, const __half *b0, const __half *b1,
                                int n_slots, int N, const int4 *active, const int32_t *n_active, int max_active,
                                int *tile_start, const int32_t *perm, float *out, int *err, int sm_count,
                                cudaStream_t st);

// n_valid (device, may be NULL): the dispatched pairs; sorted rows past it are not gathered.
// tokens_ready: aq_t / ad_t / ab_t already hold these T tokens (an earlier chunk of the same call).
cudaError_t launch_prep_gateup_a(const float *x, int T, const int32_t *perm, int n_rows, const int32_t *n_valid,
                                 int x_div, int K, __half *aq_t, float *ad_t, __half *ab_t, __half *aq, float *ad,
                                 __half *ab, bool tokens_ready, cudaStream_t st);
cudaError_t launch_prefill_gateup(const __half *aq, const float *ad, const __half *ab, int n_rows, int K, int I,
                                  const uint8_t *gate, const uint8_t *up, size_t nb1, size_t nb2_gate,
                                  size_t nb2_up, const int4 *active, const int32_t *n_active, int max_active,
                                  int *tile_start, float *act, int *err, int sm_count, cudaStream_t st);

// slots.cu: the expert-slot cache of one layer on the device (see slots.cu)
struct SlotsDev {
    int n_expert, max_slots, max_chunks;
    int32_t *owner;               // [max_slots] expert in the slot, -1 free
    unsigned long long *stamp;    // [max_slots] LRU stamps
    int32_t *slot_of;             // [n_expert] slot of a resident expert, -1 otherwise
    uint8_t *pinned;              // [n_expert]
    int32_t *active;              // [1] slots in use
    unsigned long long *meta;     // [4] clock, hits, misses, bypasses
    unsigned long long *counts;   // [n_expert] routed pairs since creation
    int32_t *n_chunks;            // [1] chunks of the last step
    int32_t *map;                 // [max_chunks][n_expert] slot of the chunk's experts, -1 others
    int2 *loads;                  // [max_chunks][max_slots] (expert, slot) of the chunk's misses
    int32_t *n_loads;             // [max_chunks]
};
struct SlotCopy {  // gate, up, down: the host store (mapped device addresses) and the slot tensors
    const uint8_t *src[3];
    size_t src_nb2[3];
    uint8_t *dst[3];
    size_t dst_nb2[3];
    size_t bytes[3];  // bytes of one expert's matrix, a multiple of 16
};
bool slots_fit(int n_expert, int max_slots);
cudaError_t launch_slot_plan(const int32_t *ids, int n_pairs, const SlotsDev &s, int *err, cudaStream_t st);
cudaError_t launch_slot_lookup_list(const int32_t *list, int n, const SlotsDev &s, int *err, cudaStream_t st);
cudaError_t launch_slot_page(const SlotsDev &s, int chunk, const SlotCopy &cp, int sm_count, cudaStream_t st);
// The overlapped miss path (see slots.cu): host store -> staging (load index order, ebytes per
// expert), and staging -> the loads' slots.
cudaError_t launch_slot_stage(const SlotsDev &s, int chunk, const SlotCopy &cp, uint8_t *staging, size_t ebytes,
                              cudaStream_t st);
cudaError_t launch_slot_unstage(const SlotsDev &s, int chunk, const SlotCopy &cp, const uint8_t *staging,
                                size_t ebytes, int sm_count, cudaStream_t st);

// Rows per work item of the GEMV for K columns and N rows per expert; 0 if N does not fit.
int gemv_rows_per_item(int wt, int K, int N);
cudaError_t launch_gemv(int wt, bool gateup, const GemvArgs &a, int max_items, int sm_count, cudaStream_t st);

}  // namespace tmoe
