/*
 * tmoe.h -- C ABI of the B200-native Qwen3-MoE layer hot path (router -> dispatch ->
 * Q4_K/Q6_K SwiGLU experts -> weighted combine, optional expert parallelism).
 *
 * The entry points replace, for the MoE layer of Tetraeder's own Qwen3-MoE builder
 * (`--engine moe`), the ggml graph ops that crates/ggml-sys forwards today.  Paths below are
 * relative to the tetraeder project root:
 *
 *   tmoe_mul_mat_id   <- Context::mul_mat_id            crates/ggml-sys/src/ggml/context.rs:322-336
 *   tmoe_route        <- router()                       crates/model/src/qwen3moe.rs:2871-2890
 *                        (soft_max :279, argsort_top_k :290, get_rows :231, sum_rows,
 *                         clamp, div of context.rs)
 *   tmoe_experts      <- weighted_experts() + sum_experts()
 *                                                       crates/model/src/qwen3moe.rs:2899-2923
 *   tmoe_layer        <- moe_ffn() / the router+experts window of build_step
 *                                                       crates/model/src/qwen3moe.rs:2892-2896
 *   tmoe_map_ids      <- the EP id remap get_rows(map, ids)
 *                                                       crates/model/src/qwen3moe_shard.rs:1043-1050
 *   tmoe_ep_*         <- the EP combine b.reduce -> Executor::all_reduce -> Comm::all_reduce
 *                        crates/model/src/qwen3moe_shard.rs:1051-1056,
 *                        crates/executor/src/exec.rs:326-351, crates/ggml-sys/src/comm.rs:69-87
 *                        (tmoe_ep_a2a_layer: the same partial sums, tokens dispatched all-to-all)
 *   tmoe_slots_*      <- LayerSlots                     crates/memory/src/slots.rs:67-262
 *                        and Streamer::make_resident    crates/model/src/experts.rs:1492-1543
 *   tmoe_streamed_layer <- the streamed step's readback, plan, uploads and chunk groups
 *                        crates/model/src/qwen3moe.rs:1829,2021-2050; experts.rs:644-662
 *
 * Conventions (the same as ggml's, so a binding passes ggml tensor data pointers through):
 *   - tensors are row-major with ne[0] fastest; an expert weight tensor is
 *     [ne0 = K, ne1 = N rows, ne2 = experts or slots], row r of expert e at byte
 *     e*nb2 + r*nb1.  gate/up are [H, I, E], down is [I, H, E];
 *   - type ids are ggml's: 12 = Q4_K, 14 = Q6_K;
 *   - ids are int32 [T][k] (token-major); an id < 0 means "no expert": nothing is read and the
 *     row is exactly zero (patches/0004-cuda-mul-mat-id-skip-negative.patch:1-10);
 *   - every pointer argument of a compute call is a device pointer; `stream` is a cudaStream_t
 *     (NULL = the legacy default stream).  Calls are stream-ordered and do not block the host.
 *
 * Errors: every call returns TMOE_OK (0) or a negative TMOE_E* code and never aborts; the
 * message is kept per handle (tmoe_last_error).  Device-side faults of the kernels' own bounded
 * waits are latched in a device flag and reported by tmoe_check().
 * Threading: a handle is used from one host thread at a time (one handle per model thread,
 * like the reference's non-Send builder).  Workspace is owned by the handle, sized at create,
 * and shared by its calls: issue a handle's calls on one stream, or order the streams (an event
 * or a synchronisation) between calls on different ones.
 */
#ifndef TMOE_H
#define TMOE_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TMOE_API __attribute__((visibility("default")))
#else
#define TMOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define TMOE_OK 0
#define TMOE_E_INVALID -1   /* bad argument or shape */
#define TMOE_E_CUDA -2      /* a CUDA runtime call failed */
#define TMOE_E_NOMEM -3     /* device allocation failed */
#define TMOE_E_UNSUPPORTED -4
#define TMOE_E_DEVICE -5    /* a kernel reported an error (timeout of a bounded wait) */
#define TMOE_E_COMM -6      /* NCCL failure */
#define TMOE_E_NOTFOUND -7  /* a GGUF key or tensor that the file does not have */

#define TMOE_TYPE_Q4_K 12
#define TMOE_TYPE_Q6_K 14
/* Q6_K in this library's 8-row fragment order, made from Q6_K matrices by tmoe_prepack (not a
 * ggml type; the value is outside ggml's range).  Accepted for the expert tensors (tmoe_config's
 * types, tmoe_mul_mat_id); its row size, nb1 and nb2 are those of the ggml matrix it was made from. */
#define TMOE_TYPE_Q6_K_R8 270

typedef struct tmoe_handle tmoe_handle;

typedef struct {
    int32_t n_embd;        /* H */
    int32_t n_ff;          /* I, moe_intermediate */
    int32_t n_expert;      /* E, router width (global expert count) */
    int32_t n_expert_used; /* k */
    int32_t gate_type;     /* ggml type ids */
    int32_t up_type;
    int32_t down_type;
    int32_t max_tokens;    /* T the workspace is sized for */
    int32_t device;        /* CUDA ordinal */
    float rms_eps;         /* rms_norm epsilon of the router's ffn_norm */
} tmoe_config;

/* Stacked or slot expert tensors, device pointers into caller-owned buffers (never copied). */
typedef struct {
    const void *gate;
    const void *up;
    const void *down;
    size_t gate_nb1, gate_nb2; /* row and expert strides in bytes */
    size_t up_nb1, up_nb2;
    size_t down_nb1, down_nb2;
    int32_t n_slots; /* experts (or slots) in the tensors; ids must be < n_slots */
} tmoe_expert_tensors;

/* Returns the ABI version (major * 100 + minor). */
TMOE_API int tmoe_version(void);

TMOE_API int tmoe_create(const tmoe_config *cfg, tmoe_handle **out);
TMOE_API void tmoe_destroy(tmoe_handle *h);
/* Message of the last failed call on this handle ("" if none).  NULL handle: the last
 * create failure of this thread. */
TMOE_API const char *tmoe_last_error(const tmoe_handle *h);
/* Synchronises `stream`, then reads and clears the device error flag. */
TMOE_API int tmoe_check(tmoe_handle *h, void *stream);

/* Holds `stream` until *flag == value, on the device, under the kernels' bounded-wait rule: after
 * limit_ns nanoseconds (<= 0 or above one second: one second) the wait gives up, latches the
 * handle's device error flag and lets the stream go on, so the next tmoe_check returns
 * TMOE_E_DEVICE and the context stays usable.  `flag` is a device address: a word in device
 * memory or in pinned, device-mapped host memory that the host writes (a host watchdog's gate on
 * a step).  It must not be a word that another kernel on the same device is to set: kernels that
 * wait on one another are not guaranteed to run at the same time.  No counterpart in the
 * reference, whose executor waits on the host (crates/executor/src/exec.rs:164-177); this is the
 * device side of the same rule, and the way to see a bounded device wait run out without a fault. */
TMOE_API int tmoe_wait_flag(tmoe_handle *h, void *stream, const int32_t *flag, int32_t value, int64_t limit_ns);

/* ggml mul_mat_id: out[t][j][:] = W[ids[t][j]] . b[t][b1 == 1 ? 0 : j][:]  (f32 [T][n_used][N]).
 * W: [K, N, n_w] of `type` (Q4_K, Q6_K or Q6_K_R8, K % 256 == 0) with strides nb1/nb2;
 * b: f32 [T][b1][K], b1 == 1 or n_used; activations go through Q8_K as on ggml's CPU path.
 * Its scratch is the handle's, allocated by tmoe_create for T * b1 and T * n_used up to
 * max_tokens * n_expert_used and K up to max(n_embd, n_ff); a call beyond that returns
 * TMOE_E_INVALID.  The call allocates nothing and does not synchronise. */
TMOE_API int tmoe_mul_mat_id(tmoe_handle *h, void *stream, int32_t type, const void *W, size_t nb1,
                    size_t nb2, int64_t K, int64_t N, int64_t n_w, const float *b, int64_t b1,
                    const int32_t *ids, int64_t n_used, int64_t T, float *out);

/* tmoe_mul_mat_id without any device allocation (no counterpart in the reference: an addition
 * for callers that cannot allocate during the call -- code that runs under a fixed device-memory
 * budget, or where a cudaMalloc would synchronise the device in the middle of a step).  The same
 * arguments, arithmetic and results as tmoe_mul_mat_id; its scratch (the Q8_K rows of b, the
 * dispatch buffers) lives in a 2 MiB module-global device array instead of the handle's growable
 * buffer.  Limit: with rows = T * b1, P = T * n_used and nbw = 2 for Q4_K, 4 for Q6_K, the scratch
 * is rows*K*(1 + (4 + 8*nbw)/256) + 4*P + 16 bytes in five parts, each rounded up to 256 bytes,
 * plus 25,344 bytes of per-slot tables and counters, and it must fit in 2 MiB (2,097,152 bytes);
 * e.g. T <= 233 at K = 8192 for Q4_K with b1 = 1 and n_used = 8.  Larger calls return
 * TMOE_E_INVALID.
 * The first call on a device looks the array up (cudaGetSymbolAddress), so make it before any
 * stream capture; the address is then cached per device, and a cudaDeviceReset invalidates it
 * (do not use this entry point after resetting the device in the same process).  The array is
 * shared by every handle of the process on that device: overlapping calls (on different
 * streams, or from different threads) race on it and must be ordered by the caller. */
TMOE_API int tmoe_mul_mat_id_noalloc(tmoe_handle *h, void *stream, int32_t type, const void *W, size_t nb1,
                                     size_t nb2, int64_t K, int64_t N, int64_t n_w, const float *b, int64_t b1,
                                     const int32_t *ids, int64_t n_used, int64_t T, float *out);

/* router(): optional xn = rms_norm(x, eps) * norm_w (use_norm != 0; norm_w may be NULL),
 * logits = router_w . xn (router_w f32 [E][H], the ggml [H, E] gate_inp) or the given
 * `logits` f32 [T][E] when router_w is NULL; probs = softmax; ids = top-k (descending, ties to
 * the lower index); w = sel / clamp(sum sel, 6.1035156e-5).  ids_out int32 [T][k], w_out f32
 * [T][k]; xn_out f32 [T][H] and logits_out f32 [T][E] may be NULL. */
TMOE_API int tmoe_route(tmoe_handle *h, void *stream, const float *x, int64_t T, int32_t use_norm,
               const float *norm_w, const float *router_w, const float *logits, int32_t *ids_out,
               float *w_out, float *xn_out, float *logits_out);

/* weighted_experts() + sum_experts(): out[t] = sum_j w[t][j] * down(silu(gate xn_t) * up xn_t)
 * over the choices j in order; ids are slot ids of `wts` (< 0: no contribution). */
TMOE_API int tmoe_experts(tmoe_handle *h, void *stream, const float *xn, int64_t T, const int32_t *ids,
                 const float *w, const tmoe_expert_tensors *wts, float *out);

/* route + (optional id map) + experts in one call.  id_map int32 [E] (device) maps global
 * expert ids to slots of `wts` or -1 (NULL: identity).  ids_out / w_out may be NULL.
 * The layer's kernels are launched with programmatic stream serialization: each may start while
 * the kernel before it runs, and waits for it before reading its outputs.  Two reads happen
 * before that wait: the routing kernel stages router_w, and the down products start loading
 * `wts->down`.  So a kernel that writes router_w or the expert tensors must not be the one
 * launched on the stream right before this call (a copy, an event or any other kernel in between
 * is enough).  While profile() is on, the kernels launch one after another. */
TMOE_API int tmoe_layer(tmoe_handle *h, void *stream, const float *x, int64_t T, int32_t use_norm,
               const float *norm_w, const float *router_w, const float *logits,
               const int32_t *id_map, const tmoe_expert_tensors *wts, float *out,
               int32_t *ids_out, float *w_out);
/* tmoe_layer with bf16 activations x [T][H], for a caller whose hidden state is bf16.  The rows
 * are widened to f32, which is exact, into the handle's workspace, and then the layer runs as
 * tmoe_layer on them, so the results equal tmoe_layer's on the f32 values bit for bit.  `out`
 * stays f32. */
TMOE_API int tmoe_layer_bf16(tmoe_handle *h, void *stream, const uint16_t *x, int64_t T, int32_t use_norm,
                             const float *norm_w, const float *router_w, const float *logits,
                             const int32_t *id_map, const tmoe_expert_tensors *wts, float *out,
                             int32_t *ids_out, float *w_out);

/* --- expert parallelism (qwen3moe_shard.rs:1038-1056) ----------------------------------------
 * A communicator over the ranks of an expert-parallel group, one rank per GPU (NCCL).  Rank 0
 * makes an id (tmoe_comm_unique_id), the caller hands its bytes to every rank (e.g. through
 * torch.distributed or a store), and every rank calls tmoe_comm_init with it.  Host waits on the
 * communicator give up after timeout_s seconds (TMOE_E_COMM; the communicator is then aborted).
 * Errors of these calls: tmoe_comm_last_error() of the calling thread. */
typedef struct tmoe_comm tmoe_comm;
#define TMOE_COMM_ID_BYTES 128
TMOE_API int tmoe_comm_unique_id(void *id_out);
TMOE_API int tmoe_comm_init(const void *id, int32_t nranks, int32_t rank, int32_t device, double timeout_s,
                            tmoe_comm **out);
/* Ends the communicator at once (a host watchdog's call when a peer died); it is then unusable. */
TMOE_API int tmoe_comm_abort(tmoe_comm *c);
TMOE_API void tmoe_comm_destroy(tmoe_comm *c);
TMOE_API const char *tmoe_comm_last_error(void);

/* The reference's EP layer: every rank passes the same tokens x, its id_map (global expert id ->
 * slot of its own `wts`, or -1 for experts held elsewhere) and its expert tensors; each rank
 * computes tmoe_layer over its experts and the partial outputs are summed across the ranks
 * (the all-reduce of qwen3moe_shard.rs:1056), so that every rank ends with the full `out`.
 * Every rank must make the same calls in the same order; a rank whose local layer fails still
 * takes part in the sum and then returns the error. */
TMOE_API int tmoe_ep_layer(tmoe_handle *h, void *stream, tmoe_comm *comm, const float *x, int64_t T,
                           int32_t use_norm, const float *norm_w, const float *router_w, const float *logits,
                           const int32_t *id_map, const tmoe_expert_tensors *wts, float *out, int32_t *ids_out,
                           float *w_out);

/* --- expert slots and the streamed layer step --------------------------------------------------
 * The expert-slot cache of one MoE layer (LayerSlots, crates/memory/src/slots.rs:67-262) with its
 * table on the device, and the streamed step of `--expert-slots N < E` (qwen3moe.rs:2021-2050,
 * Streamer::plan experts.rs:644-662, make_resident experts.rs:1507-1543).  The reference reads the
 * ids back to the host every layer (qwen3moe.rs:1829) and plans there; here the plan (distinct
 * experts in order of first appearance, residents first, chunks of the slot count, one LRU lookup
 * per expert) runs in one CTA on the device, and a copy kernel pages each miss in from the host
 * store, so the step is stream-ordered with no host round trip.
 * `slots`: device slot tensors (n_slots = the slot count); `store`: the layer's E experts in pinned
 * host memory (cudaHostAlloc / cudaHostRegister, i.e. device-mapped), the same row layout
 * (nb1) as the slots.  The cache keeps both pointers; neither is copied.  One cache per layer;
 * calls on a cache are stream-ordered like the handle's.  With more experts than slots the cache
 * also owns a staging area of (slot count) experts of device memory and a side stream: the misses
 * of chunks after the first are paged in there while the earlier chunk computes. */
typedef struct tmoe_slots tmoe_slots;
TMOE_API int tmoe_slots_create(tmoe_handle *h, const tmoe_expert_tensors *slots, const tmoe_expert_tensors *store,
                               tmoe_slots **out);
TMOE_API void tmoe_slots_destroy(tmoe_slots *s);
/* Chunk passes of a streamed step: ceil(E / slot count). */
TMOE_API int tmoe_slots_max_chunks(const tmoe_slots *s);
/* make_resident (experts.rs:1492): looks up the n (<= slot count) listed experts (host array) in
 * order and pages their misses in.  A lookup that finds every slot pinned sets the device error
 * (tmoe_check: TMOE_E_INVALID, "no free expert slot (all pinned)"). */
TMOE_API int tmoe_slots_make_resident(tmoe_slots *s, void *stream, const int32_t *experts, int32_t n);
/* set_hot_set (slots.rs:189-207) then make_resident of the pinned experts that are not resident,
 * in increasing id (refresh_hot_set, experts.rs:1549-1566).  Synchronises `stream`. */
TMOE_API int tmoe_slots_set_hot_set(tmoe_slots *s, void *stream, const int32_t *hot, int32_t n);
/* Synchronising reads: owner[slot count] (expert per slot, -1 free), stats[3] = hits, misses,
 * bypasses, counts[E] = routed pairs per expert since creation; any may be NULL. */
TMOE_API int tmoe_slots_state(tmoe_slots *s, void *stream, int32_t *owner, int64_t *stats, int64_t *counts);
/* Synchronising read of the last step's plan: n_chunks; map int32 [max_chunks][E] (slot of each
 * expert of the chunk, -1 others); loads int32 [max_chunks][slot count][2] (expert, slot) of each
 * chunk's misses; n_loads [max_chunks]; any may be NULL. */
TMOE_API int tmoe_slots_last_plan(tmoe_slots *s, void *stream, int32_t *n_chunks, int32_t *map, int32_t *loads,
                                  int32_t *n_loads);
/* The streamed layer step: tmoe_route, the device plan, then per chunk: page its misses in (chunk 0
 * straight into its slots; later chunks into the staging area on the side stream, overlapping the
 * previous chunk's compute, then moved into their slots), compute its pairs from the slot tensors
 * (dout rows of the chunk's pairs), and finally one combine of all pairs in choice order -- the same
 * per-pair arithmetic as tmoe_layer on resident experts. */
TMOE_API int tmoe_streamed_layer(tmoe_handle *h, void *stream, tmoe_slots *s, const float *x, int64_t T,
                                 int32_t use_norm, const float *norm_w, const float *router_w, const float *logits,
                                 float *out, int32_t *ids_out, float *w_out);

/* Expert parallelism with token dispatch/combine over an all-to-all (the mode beside the reference's
 * all-reduce), for ranks that hold different tokens: rank r holds experts [r*E/g, (r+1)*E/g) in `wts`
 * (n_slots = E/g) and its own T tokens (T <= max_tokens / g; create the handle with max_tokens = g x the
 * tokens per rank, since it computes the rows the other ranks send). Each token is sent once to every rank
 * that holds one of its choices; that rank computes its experts' pairs and combines them in choice order
 * (the reference's per-rank partial, qwen3moe_shard.rs:1043-1056), sends the partial row back, and the
 * token's rank adds the partials in rank order. Messages have a fixed capacity of max_tokens / g rows per
 * peer (no host readback). Every rank must make the same calls in the same order; a rank whose routing fails
 * still takes both exchange steps. Exchange: the first call with a communicator maps every rank's exchange
 * buffers into every rank (CUDA IPC; host-synchronous, so not under stream capture), and from then on the
 * messages are written straight into the peers' buffers over NVLink with counted arrivals (a wait that runs
 * out after 1 s latches TMOE_DEV_ERR_TIMEOUT, reported by tmoe_check). With g > 8, or if any rank cannot map
 * a peer, the ranks exchange through NCCL instead. A rank must not destroy its handle while another rank is
 * still inside a call with it. */
TMOE_API int tmoe_ep_a2a_layer(tmoe_handle *h, void *stream, tmoe_comm *comm, const float *x, int64_t T,
                               int32_t use_norm, const float *norm_w, const float *router_w, const float *logits,
                               const tmoe_expert_tensors *wts, float *out, int32_t *ids_out, float *w_out);

/* ids' = table[ids] for ids in [0, n_table), else -1 (the EP expert_map lookup). */
TMOE_API int tmoe_map_ids(tmoe_handle *h, void *stream, const int32_t *ids, int64_t n,
                 const int32_t *table, int64_t n_table, int32_t *out);

/* The per-expert dispatch of `ids` int32 [T][k] over n_slots experts (a4 of the path, the row
 * mapping of ggml's mul_mat_id): counts[n_slots], offsets[n_slots + 1] and perm[] holding, for
 * each expert in increasing order, its pair indices t*k + j in increasing order (token-major,
 * choice-minor: crates/model/src/qwen3moe.rs:2126-2150 group_pairs).  Ids outside
 * [0, n_slots) are skipped; perm must hold T*k entries (offsets[n_slots] are written). */
TMOE_API int tmoe_dispatch(tmoe_handle *h, void *stream, const int32_t *ids, int64_t T,
                           int32_t n_slots, int32_t *counts, int32_t *offsets, int32_t *perm);

/* quant::quantize (crates/ggml-sys/src/quant.rs:52) for Q4_K / Q6_K on the device: nrows x ncols
 * f32 (ncols % 256 == 0) -> nrows * row_size bytes.  This library's own fit of the formats, not
 * ggml's search; the bytes are deterministic.  Errors: tmoe_last_error(NULL). */
TMOE_API int tmoe_quantize(int32_t type, const float *x, int64_t nrows, int64_t ncols, void *out,
                           void *stream);
/* quant::to_f32 (crates/ggml-sys/src/quant.rs:19) for Q4_K / Q6_K: n values (n % 256 == 0). */
TMOE_API int tmoe_dequantize(int32_t type, const void *in, int64_t n, float *out, void *stream);

/* The optional, explicit repack that the boundary allows (weights are never repacked implicitly;
 * the reference keeps expert weights unrepacked, docs/adr/0039): n_mats Q6_K matrices of n_rows
 * rows (n_rows % 8 == 0) and K columns (K % 256 == 0, K <= 16384), rows nb1 bytes apart and matrices nb2 apart,
 * are written to dst (16-byte aligned, n_mats * n_rows * row size bytes, not overlapping src) as
 * TMOE_TYPE_Q6_K_R8: per matrix, n_rows / 8 row groups of K / 256 units of 1680 bytes, the same
 * bytes rearranged so that the expert GEMV reads them with aligned, conflict-free vector loads and
 * fills one super-block at a time.  The results of every product are bit for bit those of the Q6_K
 * matrix it came from.  type must be TMOE_TYPE_Q6_K.  Stream-ordered; errors: tmoe_last_error(NULL). */
TMOE_API int tmoe_prepack(int32_t type, const void *src, size_t nb1, size_t nb2, int64_t n_rows, int64_t K,
                          int64_t n_mats, void *dst, void *stream);

/* The decode step around the MoE layer (config 3: the full Qwen3-MoE model, attention() of
 * crates/model/src/attn.rs:246-405 and build_step of qwen3moe.rs:2777-2870), as stream-ordered
 * ops on a handle (its error flag and SM count); the projections are tmoe_mul_mat_id with one
 * expert.  Device pointers throughout.
 *   tmoe_get_rows    <- Context::get_rows (context.rs:231): out[i] = row rows[i] of W as f32 (ggml
 *                       type 0 F32, 1 F16, 12 Q4_K, 14 Q6_K; rows nb1 apart); a row outside
 *                       [0, n_rows_w) gives zeros and latches the device error (tmoe_check)
 *   tmoe_rms_norm    <- rms_norm (:274) times w (NULL: none), over `rows` rows of n
 *   tmoe_rope_neox   <- rope_ext (:343) in NeoX mode, in place on x [n_tok][n_head][head_dim],
 *                       token t at position pos[t], the first n_rot dims rotated
 *   tmoe_attn_decode <- set_rows (:238) of the new K/V rows into F16 caches [B][n_ctx][n_kv]
 *                       [head_dim] at pos[b], then flash_attn_ext (:368) of one query per sequence
 *                       over its positions 0..pos[b]: q [B][n_head][head_dim] (n_head a multiple
 *                       of n_kv, at most 8 query heads per KV head; head_dim 64 or 128), k/v
 *                       [B][n_kv][head_dim], out [B][n_head][head_dim]; scratch of
 *                       tmoe_attn_decode_scratch_bytes
 *   tmoe_attn_prefill <- the multi-token form of the same two ops (attention_seqs, attn.rs:269-302,
 *                       one sequence): the S new K/V rows k/v [S][n_kv][head_dim] go to positions
 *                       pos0 .. pos0+S-1 of sequence `seq` of the caches [n_seq][n_ctx][n_kv]
 *                       [head_dim], then query i of q [S][n_head][head_dim] attends to positions
 *                       0 .. pos0+i (the causal mask of a prefill) -> out [S][n_head][head_dim];
 *                       no scratch
 *   tmoe_add         <- add (:243);  tmoe_argmax: the first index of each row's maximum */
/* Context::mul_mat (context.rs) of one Q4_K/Q6_K matrix W [N rows of K] and x f32 [T][K] ->
 * out [T][N], on the decode GEMV.  reuse_x != 0: x is the activations of the previous
 * tmoe_mul_mat call on this handle with the same K, T and weight family (Q4_K or Q6_K), whose Q8_K
 * rows are reused (the Q, K and V projections of one normalised input).  The workspace is sized on
 * first use: make a first call outside a stream capture.  It belongs to the handle, so calls that
 * may run at the same time (on different streams) need a handle each. */
TMOE_API int tmoe_mul_mat(tmoe_handle *h, void *stream, int32_t type, const void *W, size_t nb1, int64_t K, int64_t N,
                          const float *x, int64_t T, int32_t reuse_x, float *out);
TMOE_API int tmoe_get_rows(tmoe_handle *h, void *stream, int32_t type, const void *W, size_t nb1, int64_t K,
                           int64_t n_rows_w, const int32_t *rows, int64_t n, float *out);
TMOE_API int tmoe_rms_norm(tmoe_handle *h, void *stream, const float *x, const float *w, float eps, int64_t rows,
                           int64_t n, float *out);
TMOE_API int tmoe_rope_neox(tmoe_handle *h, void *stream, float *x, const int32_t *pos, int64_t n_tok, int32_t n_head,
                            int32_t head_dim, int32_t n_rot, float freq_base);
/* The two per-head norms and the two RoPEs of attention() (attn.rs:320-325) in one launch:
 * q [T][n_head][head_dim] = rope(rms_norm(q) * q_norm), k [T][n_kv][head_dim] likewise with k_norm
 * (head_dim a multiple of 32, at most 128). */
TMOE_API int tmoe_qk_norm_rope(tmoe_handle *h, void *stream, float *q, float *k, const float *q_norm,
                               const float *k_norm, const int32_t *pos, int64_t T, int32_t n_head, int32_t n_kv,
                               int32_t head_dim, int32_t n_rot, float freq_base, float eps);
TMOE_API int64_t tmoe_attn_decode_scratch_bytes(tmoe_handle *h, int32_t B, int32_t n_head, int32_t n_kv,
                                                int32_t head_dim, int32_t n_ctx);
TMOE_API int tmoe_attn_decode(tmoe_handle *h, void *stream, const float *q, const float *k, const float *v,
                              void *k_cache, void *v_cache, const int32_t *pos, int32_t B, int32_t n_head,
                              int32_t n_kv, int32_t head_dim, int32_t n_ctx, float scale, void *scratch, float *out);
TMOE_API int tmoe_attn_prefill(tmoe_handle *h, void *stream, const float *q, const float *k, const float *v,
                               void *k_cache, void *v_cache, int32_t seq, int32_t n_seq, int32_t pos0, int32_t S,
                               int32_t n_head, int32_t n_kv, int32_t head_dim, int32_t n_ctx, float scale, float *out);
TMOE_API int tmoe_add(tmoe_handle *h, void *stream, const float *a, const float *b, float *out, int64_t n);
TMOE_API int tmoe_argmax(tmoe_handle *h, void *stream, const float *x, int64_t rows, int64_t n, int32_t *out);

/* GGUF model files (crates/model/src/gguf.rs; the loader of load_weights, qwen3moe.rs:2498-2584).
 *   tmoe_gguf_open        <- Gguf::open (gguf.rs:236-296): the header, metadata and tensor index of a
 *                            file, or of every shard of a split model opened from its first shard
 *                            (<prefix>-00001-of-0000N.gguf); GGUF version 3 only
 *   tmoe_gguf_kv          <- Gguf::get/str/u64/f32 (gguf.rs:409-450): integers widen to u64 / i64,
 *                            floats to f64, arrays keep their length only
 *   tmoe_gguf_tensor_info <- Gguf::tensor (gguf.rs:452): name, ggml type, ne[4], shard, absolute
 *                            byte offset in the shard file, bytes
 *   tmoe_gguf_read/load   <- the reads of load_weights: bytes [offset, offset + nbytes) of a tensor
 *                            (an expert slab is nbytes / ne[2] long, TensorInfo::slab gguf.rs:76-86)
 *                            into host memory, or into device memory of `device` through pinned
 *                            bounce buffers on `stream` (returns when the copies are done)
 * Errors: TMOE_E_INVALID (bad file, bad range), TMOE_E_UNSUPPORTED (version), TMOE_E_NOTFOUND
 * (missing key), TMOE_E_CUDA; the message is tmoe_gguf_last_error() (per thread).  Strings
 * returned stay valid until tmoe_gguf_close. */
typedef struct tmoe_gguf tmoe_gguf;
#define TMOE_GGUF_U64 0
#define TMOE_GGUF_I64 1
#define TMOE_GGUF_F64 2
#define TMOE_GGUF_BOOL 3 /* in u: 0 or 1 */
#define TMOE_GGUF_STR 4
#define TMOE_GGUF_ARRAY 5 /* in n: the length */
TMOE_API int tmoe_gguf_open(const char *path, tmoe_gguf **out);
TMOE_API void tmoe_gguf_close(tmoe_gguf *g);
TMOE_API const char *tmoe_gguf_last_error(void);
TMOE_API int32_t tmoe_gguf_n_shards(const tmoe_gguf *g);
TMOE_API int64_t tmoe_gguf_n_kv(const tmoe_gguf *g);
TMOE_API int tmoe_gguf_kv_key(const tmoe_gguf *g, int64_t i, const char **key);
TMOE_API int tmoe_gguf_kv(const tmoe_gguf *g, const char *key, int32_t *kind, uint64_t *u, int64_t *i, double *f,
                          const char **s, uint64_t *n);
TMOE_API int64_t tmoe_gguf_n_tensors(const tmoe_gguf *g);
/* index of the tensor, or -1 */
TMOE_API int64_t tmoe_gguf_find_tensor(const tmoe_gguf *g, const char *name);
TMOE_API int tmoe_gguf_tensor_info(const tmoe_gguf *g, int64_t i, const char **name, int32_t *type, int64_t *ne,
                                   int32_t *shard, uint64_t *offset, uint64_t *nbytes);
/* ggml's block size (elements) and bytes per block of a type id */
TMOE_API int tmoe_gguf_type_size(int32_t type, int32_t *block_elems, int32_t *block_bytes);
TMOE_API int tmoe_gguf_read(const tmoe_gguf *g, int64_t tensor, uint64_t offset, uint64_t nbytes, void *dst);
TMOE_API int tmoe_gguf_load(const tmoe_gguf *g, int64_t tensor, uint64_t offset, uint64_t nbytes, void *dst,
                            int32_t device, void *stream);

/* Routing traces, the tetraeder-routing v1 format (crates/memory/src/replay/trace.rs): a JSON
 * header line (TraceHeader), then records of a layer step's routed ids (and optional predictions)
 * or of a hot-set refresh.  For replaying recorded routing into the layer.
 *   tmoe_trace_open/next/ids <- TraceReader (trace.rs:225-330): the header is parsed and checked
 *     (format and version, id_bytes = 1 for n_expert <= 256 else 2, n_used > 0, one expert_bytes
 *     entry per layer); tmoe_trace_next returns 1 with a record, 0 at a clean end of file, a
 *     negative code on a truncated or corrupt record (more than 2^20 tokens, an id >= n_expert, an
 *     unknown kind), after which the reader stays failed; tmoe_trace_ids copies the current step's
 *     routed (which = 0), predicted (1) or depth-2 predicted (2) ids, n_tokens * n_used int32
 *     token-major
 *   tmoe_trace_create/write_step/write_refresh/finish <- TraceWriter (trace.rs:120-200): the header
 *     is given as JSON, checked and written back as serde_json writes it; ids outside
 *     [0, n_expert) are an error and nothing of that record is written
 * Errors: TMOE_E_INVALID, TMOE_E_NOTFOUND (no profile / no predictions); message:
 * tmoe_trace_last_error() (per thread). */
typedef struct tmoe_trace tmoe_trace;
typedef struct tmoe_trace_writer tmoe_trace_writer;
typedef struct {
    uint32_t version, n_layer, n_expert, n_used, id_bytes, vram_slots, ram_slots, prefetch_depth, ubatch;
    int32_t has_profile;
} tmoe_trace_info;
#define TMOE_TRACE_STEP 0
#define TMOE_TRACE_REFRESH 1
TMOE_API int tmoe_trace_open(const char *path, tmoe_trace **out);
TMOE_API void tmoe_trace_close(tmoe_trace *t);
TMOE_API const char *tmoe_trace_last_error(void);
TMOE_API int tmoe_trace_header(const tmoe_trace *t, tmoe_trace_info *info);
/* the header line as read; the string fields format, model, hot_source, prompt_hash */
TMOE_API const char *tmoe_trace_header_json(const tmoe_trace *t);
TMOE_API const char *tmoe_trace_header_str(const tmoe_trace *t, const char *field);
TMOE_API int tmoe_trace_expert_bytes(const tmoe_trace *t, uint64_t *out);
TMOE_API int tmoe_trace_profile(const tmoe_trace *t, int64_t *rows, int64_t *cols, uint64_t *out);
TMOE_API int tmoe_trace_next(tmoe_trace *t, int32_t *kind, uint32_t *step, int32_t *layer, uint32_t *n_tokens,
                             int32_t *flags);
TMOE_API int tmoe_trace_ids(const tmoe_trace *t, int32_t which, int32_t *out);
TMOE_API int tmoe_trace_create(const char *path, const char *header_json, tmoe_trace_writer **out);
TMOE_API int tmoe_trace_write_step(tmoe_trace_writer *w, uint32_t step, int32_t layer, uint32_t n_tokens,
                                   const int32_t *ids, const int32_t *predicted, const int32_t *predicted2);
TMOE_API int tmoe_trace_write_refresh(tmoe_trace_writer *w, uint32_t step);
TMOE_API int tmoe_trace_finish(tmoe_trace_writer *w);

/* Per-kernel device timing of this handle's calls (the StepProfile phase timers of
 * crates/model/src/qwen3moe.rs:69-107, narrowed to the layer's kernels).  While enabled, every
 * kernel launch is bracketed by CUDA events on its stream; tmoe_profile_collect synchronises,
 * adds the elapsed times to per-phase totals and writes the totals (ms) and launch counts to
 * arrays of TMOE_N_PHASES entries (either may be NULL).  Enabling resets the totals.  At most
 * 64 launches are recorded between two collects.  Phase ids: */
#define TMOE_PHASE_RMS_NORM 0
#define TMOE_PHASE_ROUTER_LOGITS 1
#define TMOE_PHASE_TOPK 2
#define TMOE_PHASE_MAP_IDS 3
#define TMOE_PHASE_DISPATCH 4
#define TMOE_PHASE_QUANT_X 5
#define TMOE_PHASE_GATE_UP 6
#define TMOE_PHASE_QUANT_ACT 7
#define TMOE_PHASE_DOWN 8
#define TMOE_PHASE_COMBINE 9
#define TMOE_PHASE_SLOT_PLAN 10 /* the device slot planner of tmoe_streamed_layer */
#define TMOE_PHASE_SLOT_PAGE 11 /* paging misses in from the host store */
#define TMOE_N_PHASES 12
TMOE_API int tmoe_profile_enable(tmoe_handle *h, int32_t enable);
TMOE_API int tmoe_profile_collect(tmoe_handle *h, double *ms_out, int64_t *count_out);

#ifdef __cplusplus
}
#endif
#endif /* TMOE_H */
