// C ABI of the MoE layer hot path (include/tmoe.h): handle, workspace and the launch sequences
// route -> dispatch -> gate/up (+SwiGLU) -> Q8_K of the activation -> down -> combine.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/tmoe.h"
#include "common.cuh"
#include "kernels.cuh"

namespace {

constexpr int kMaxSlots = 1024;
constexpr int kCounters = 4;
// Pairs (T * k) from which the expert products run as grouped tcgen05 GEMMs instead of the
// decode GEMV; handles sized for fewer pairs carry no prefill buffers.  The GEMV's time grows
// with the tokens per expert, while the GEMMs cost about a full M tile per active expert however
// few rows it has.  On a Qwen3-30B-shaped layer (128 experts, top-8) the two meet between
// 4096 pairs (GEMV 470 us, GEMMs 583 us) and 8192 (GEMV 784 us, GEMMs 581 us).
constexpr int64_t kPrefillMinPairs = 6144;
// Tokens from which tmoe_mul_mat runs as one tcgen05 GEMM over fp16-dequantised weights instead of
// the decode GEMV (a prompt's projections; decode batches stay on the GEMV's exact integer sums).
constexpr int64_t kDenseGemmMinTokens = 512;
thread_local std::string g_create_error;

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

struct tmoe_handle {
    tmoe_config cfg{};
    int sm_count = 0;
    void *ws = nullptr;
    size_t ws_bytes = 0;
    // tmoe_mul_mat: its workspace, and which activations its Q8_K rows hold (for reuse_x)
    void *dense_ws = nullptr;
    size_t dense_ws_bytes = 0;
    const float *dense_x = nullptr;
    int dense_wt = -1;
    int64_t dense_k = 0, dense_t = 0;
    bool dense_nosplit = false;  // the GEMV took no tensor map over a matrix's K slices
    bool dense_a16 = false;      // the fp16 A rows of dense_x are in the workspace (the GEMM path)
    // routing
    float *logits = nullptr;
    int32_t *ids = nullptr;
    float *w = nullptr;
    int32_t *mapped = nullptr;
    int32_t *counts = nullptr, *offsets = nullptr, *perm = nullptr, *n_active = nullptr;
    int4 *active = nullptr;
    // activations: Q8_K of the layer input (read by gate/up) and of the SwiGLU output (read by down)
    float *xn = nullptr;
    float *x32 = nullptr;  // bf16 layer inputs widened to f32 (tmoe_layer_bf16)
    int8_t *xq = nullptr;
    float *xd = nullptr;
    uint32_t *xbl = nullptr, *xbh = nullptr;
    float *act = nullptr;
    int8_t *aq = nullptr;
    float *ad = nullptr;
    uint32_t *abl = nullptr, *abh = nullptr;
    float *dout = nullptr;
    // prefill (grouped GEMM) buffers: fp16 A rows of the two GEMMs, fp16 weights, tile tables
    __half *a2 = nullptr, *w16_down = nullptr, *aq16 = nullptr, *ab16 = nullptr, *aq16_t = nullptr, *ab16_t = nullptr;
    float *ad16 = nullptr, *ad16_t = nullptr;  // d of the A rows' Q8_K blocks (sorted rows, token rows)
    int *tile_start = nullptr, *tile_start2 = nullptr;
    int *counters = nullptr;    // GEMV work counters
    int32_t *sort_scratch = nullptr;  // per-chunk expert counts of the many-CTA dispatch
    size_t sort_scratch_ints = 0;
    int *route_done = nullptr;  // the fused routing kernel's tile counters (zero between calls)
    int *err = nullptr;
    // exchange buffers of the all-to-all EP mode (allocated on its first call; see tmoe_ep_a2a_layer)
    struct A2A {
        void *mem = nullptr;
        size_t bytes = 0;
        int g = 0, cap = 0;
        int32_t *row_of = nullptr, *s_ids = nullptr, *r_ids = nullptr, *s_tok = nullptr, *counts = nullptr;
        float *s_w = nullptr, *r_w = nullptr, *s_x = nullptr, *r_x = nullptr, *part = nullptr, *ret = nullptr;
        // the exchange over peer memory: arrival counters (written by the peers), this rank's
        // counters, every rank's buffers mapped here (peer_base: the IPC mappings to close)
        int *flags = nullptr, *ctl = nullptr;
        const tmoe_comm *comm = nullptr;
        bool p2p = false;
        void *peer_base[tmoe::EP_MAX_PEERS] = {};
        tmoe::EpPeers peers{};
    } a2a;
    // scratch of tmoe_mul_mat_id, sized at create for max_tokens * n_expert_used rows of
    // K = max(n_embd, n_ff) in the larger (Q6_K) Q8_K layout
    void *op_ws = nullptr;
    size_t op_ws_bytes = 0;
    std::string last_error;
    // per-kernel timing (tmoe_profile_*)
    struct Prof {
        bool on = false;
        static constexpr int kRing = 128;
        cudaEvent_t ev[kRing] = {};
        int phase[kRing / 2] = {};
        int n = 0;  // events recorded since the last collect
        double ms[TMOE_N_PHASES] = {};
        int64_t count[TMOE_N_PHASES] = {};
    } prof;
};

struct tmoe_slots {
    tmoe_handle *h = nullptr;
    tmoe::SlotsDev dev{};
    tmoe::SlotCopy copy{};
    tmoe_expert_tensors slot_wts{};
    void *mem = nullptr;
    int32_t *list = nullptr;  // device copy of a make_resident list
    int active = 0;           // host mirror of the slots in use (LayerSlots::active)
    // the overlapped miss path: staging for one chunk's loads, the side stream that pages them in,
    // and per chunk the events of "staged" (side -> main) and "moved into the slots" (main -> side)
    uint8_t *staging = nullptr;
    size_t ebytes = 0;
    cudaStream_t side = nullptr;
    std::vector<cudaEvent_t> ev_staged, ev_moved;
    cudaEvent_t ev_plan = nullptr;
};

namespace {

int fail(tmoe_handle *h, int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    if (h)
        h->last_error = buf;
    else
        g_create_error = buf;
    return code;
}

int cuda_fail(tmoe_handle *h, cudaError_t e, const char *what) {
    return fail(h, TMOE_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

// Brackets one kernel launch with timing events when profiling is on.
struct PhaseMark {
    tmoe_handle *h;
    cudaStream_t st;
    int slot = -1;
    PhaseMark(tmoe_handle *h_, cudaStream_t st_, int phase) : h(h_), st(st_) {
        auto &p = h->prof;
        if (!p.on || p.n + 2 > tmoe_handle::Prof::kRing) return;
        slot = p.n;
        p.phase[slot / 2] = phase;
        cudaEventRecord(p.ev[slot], st);
        p.n += 2;
    }
    ~PhaseMark() {
        if (slot >= 0) cudaEventRecord(h->prof.ev[slot + 1], st);
    }
};

bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

bool is_kquant(int t) { return t == TMOE_TYPE_Q4_K || t == TMOE_TYPE_Q6_K; }
// The expert products also take Q6_K in 8-row fragment order (tmoe_prepack).
bool is_expert_type(int t) { return is_kquant(t) || t == TMOE_TYPE_Q6_K_R8; }
int wt_of(int t) {
    return t == TMOE_TYPE_Q4_K ? TMOE_WT_Q4K : t == TMOE_TYPE_Q6_K_R8 ? TMOE_WT_Q6KR : TMOE_WT_Q6K;
}
// Bytes per row (for Q6_K_R8: per row of the ggml matrix it was made from; the matrix has as many)
size_t row_size(int t, int64_t K) {
    return (size_t)(K / TMOE_QK) * (t == TMOE_TYPE_Q4_K ? TMOE_Q4K_BYTES : TMOE_Q6K_BYTES);
}

// Carves the workspace out of one allocation; returns the bytes needed when base == nullptr.
size_t carve(tmoe_handle *h, char *base) {
    const tmoe_config &c = h->cfg;
    const size_t T = (size_t)c.max_tokens, k = (size_t)c.n_expert_used, P = T * k;
    const size_t H = (size_t)c.n_embd, I = (size_t)c.n_ff, E = (size_t)c.n_expert;
    size_t off = 0;
    auto take = [&](size_t bytes) -> char * {
        char *p = base ? base + off : nullptr;
        off = align_up(off + bytes, 256);
        return p;
    };
    h->logits = (float *)take(T * E * 4);
    h->ids = (int32_t *)take(P * 4);
    h->w = (float *)take(P * 4);
    h->mapped = (int32_t *)take(P * 4);
    h->counts = (int32_t *)take(kMaxSlots * 4);
    h->offsets = (int32_t *)take((kMaxSlots + 1) * 4);
    h->active = (int4 *)take(kMaxSlots * 16);
    h->n_active = (int32_t *)take(4);
    h->perm = (int32_t *)take(P * 4 + 16);  // + the GEMV's bulk-copy round-up
    const size_t nbg = (size_t)tmoe::q8_nbw(wt_of(c.gate_type)), nbd = (size_t)tmoe::q8_nbw(wt_of(c.down_type));
    h->xn = (float *)take(T * H * 4);
    h->x32 = (float *)take(T * H * 4);
    h->xq = (int8_t *)take(T * H);
    h->xd = (float *)take(T * (H / 256) * 4);
    h->xbl = (uint32_t *)take(T * (H / 256) * nbg * 4);
    h->xbh = (uint32_t *)take(T * (H / 256) * nbg * 4);
    h->act = (float *)take(P * I * 4);
    h->aq = (int8_t *)take(P * I);
    h->ad = (float *)take(P * (I / 256) * 4);
    h->abl = (uint32_t *)take(P * (I / 256) * nbd * 4);
    h->abh = (uint32_t *)take(P * (I / 256) * nbd * 4);
    h->dout = (float *)take(P * H * 4);
    if ((int64_t)P >= kPrefillMinPairs && tmoe::prefill_fits((int)H, (int)I)) {
        h->a2 = (__half *)take(P * I * 2);
        h->w16_down = (__half *)take(E * H * I * 2);
        h->tile_start = (int *)take((kMaxSlots + 1) * 4);
        h->tile_start2 = (int *)take((kMaxSlots + 1) * 4);
        h->aq16 = (__half *)take(P * H * 2);
        h->ad16 = (float *)take(P * (H / 256) * 4);
        h->ab16 = (__half *)take(P * (H / 256) * 16 * 2);
        h->aq16_t = (__half *)take(T * H * 2);
        h->ad16_t = (float *)take(T * (H / 256) * 4);
        h->ab16_t = (__half *)take(T * (H / 256) * 16 * 2);
    }
    h->counters = (int *)take(kCounters * 4);
    h->sort_scratch_ints = tmoe::sort_scratch_ints(P, kMaxSlots);
    h->sort_scratch = (int32_t *)take(h->sort_scratch_ints * 4);
    h->route_done = (int *)take((T / 4 + 2) * 4);
    h->err = (int *)take(4);
    return off;
}

int check_tensors(tmoe_handle *h, const tmoe_expert_tensors *t) {
    const tmoe_config &c = h->cfg;
    if (!t || !t->gate || !t->up || !t->down) return fail(h, TMOE_E_INVALID, "expert tensors missing");
    if (t->n_slots <= 0 || t->n_slots > kMaxSlots)
        return fail(h, TMOE_E_INVALID, "n_slots %d out of range (1..%d)", t->n_slots, kMaxSlots);
    const size_t gr = row_size(c.gate_type, c.n_embd), ur = row_size(c.up_type, c.n_embd),
                 dr = row_size(c.down_type, c.n_ff);
    if (t->gate_nb1 != gr || t->up_nb1 != ur || t->down_nb1 != dr)
        return fail(h, TMOE_E_UNSUPPORTED, "expert rows must be contiguous (nb1 == row size)");
    if (t->gate_nb2 < gr * (size_t)c.n_ff || t->up_nb2 < ur * (size_t)c.n_ff ||
        t->down_nb2 < dr * (size_t)c.n_embd)
        return fail(h, TMOE_E_INVALID, "expert stride smaller than one expert");
    if (((uintptr_t)t->gate | (uintptr_t)t->up | (uintptr_t)t->down) & 15u)
        return fail(h, TMOE_E_INVALID, "expert tensors must be 16-byte aligned");
    if ((t->gate_nb2 | t->up_nb2 | t->down_nb2) & 15u)
        return fail(h, TMOE_E_INVALID, "expert strides must be multiples of 16 bytes");
    return TMOE_OK;
}

// The down product of the large-batch regime as a grouped tcgen05 GEMM: A2 = Q8_K round trip of
// the SwiGLU activations in expert-sorted order, as fp16; fp16 copies of the active experts'
// down rows; dout[pair] = A2 . down^T.  (gate/up stay on the integer MMA path: their outputs feed
// the Q8_K quantisation of the activations, and fp16 operands there move enough values across a
// Q8_K rounding boundary to leave the north-star max-abs bound.)
cudaError_t prefill_down(tmoe_handle *h, cudaStream_t st, int64_t P, const tmoe_expert_tensors *t, int max_active,
                         bool act_sorted) {
    const tmoe_config &c = h->cfg;
    const int H = c.n_embd, I = c.n_ff;
    cudaError_t e = tmoe::launch_prep_rows(h->act, act_sorted ? nullptr : h->perm, (int)P, h->offsets + t->n_slots, 1,
                                           I, h->a2, st);
    if (e == cudaSuccess)
        e = tmoe::launch_dequant_f16(wt_of(c.down_type), (const uint8_t *)t->down, t->down_nb2, H, I, h->active,
                                     h->n_active, max_active, h->w16_down, st);
    if (e == cudaSuccess)
        e = tmoe::launch_prefill_gemm(false, h->a2, (int)P, I, h->w16_down, nullptr, c.n_expert, H, h->active,
                                      h->n_active, max_active, h->tile_start, h->perm, h->dout, h->err, h->sm_count,
                                      st);
    return e;
}

// a4-a8 on `ids` (already slot ids) and `w`.  dispatched: the dispatch buffers (counts, offsets,
// perm, active, zeroed work counters) already hold this call's dispatch; x_quantized: the Q8_K
// rows of xn are already in h->xq/xd/xbl/xbh; combine: fold the pair rows into `out` (else they
// stay in h->dout); a16_ready: the large-batch regime's per-token fp16 Q8_K rows of xn
// (h->aq16_t/ad16_t/ab16_t) are already there, from an earlier chunk of the same layer call.
int run_experts(tmoe_handle *h, cudaStream_t st, const float *xn, int64_t T, const int32_t *ids, const float *w,
                const tmoe_expert_tensors *t, float *out, bool dispatched, bool x_quantized, bool combine = true,
                bool a16_ready = false) {
    const tmoe_config &c = h->cfg;
    const int k = c.n_expert_used, H = c.n_embd, I = c.n_ff;
    const int64_t P = T * k;
    const int wg = wt_of(c.gate_type), wd = wt_of(c.down_type);
    cudaError_t e;
    // the expert kernels overlap their predecessors' tails (programmatic dependent launch) unless
    // profile()'s per-kernel events sit between them
    tmoe::PdlScope pdl(!h->prof.on);
    if (!dispatched) {
        {
            PhaseMark pm(h, st, TMOE_PHASE_DISPATCH);
            e = tmoe::launch_sort_pairs(ids, (int)P, t->n_slots, h->counts, h->offsets, h->perm, h->active,
                                        h->n_active, h->counters, kCounters, h->err, st, h->sort_scratch,
                                        h->sort_scratch_ints);
        }
        if (e != cudaSuccess) return cuda_fail(h, e, "sort_pairs");
    }
    const int max_active = (int)(P < t->n_slots ? P : t->n_slots);
    const bool prefill = P >= kPrefillMinPairs && h->a2 && t->n_slots <= c.n_expert;
    if (prefill && wg == TMOE_WT_Q4K) {
        // gate/up as exact grouped tcgen05 GEMMs (rows in expert-sorted order), then the down GEMM
        {
            PhaseMark pm(h, st, TMOE_PHASE_QUANT_X);
            e = tmoe::launch_prep_gateup_a(xn, (int)T, h->perm, (int)P, h->offsets + t->n_slots, k, H, h->aq16_t,
                                           h->ad16_t, h->ab16_t, h->aq16, h->ad16, h->ab16, a16_ready, st);
        }
        if (e != cudaSuccess) return cuda_fail(h, e, "prefill gate/up rows");
        {
            PhaseMark pm(h, st, TMOE_PHASE_GATE_UP);
            e = tmoe::launch_prefill_gateup(h->aq16, h->ad16, h->ab16, (int)P, H, I, (const uint8_t *)t->gate,
                                            (const uint8_t *)t->up, t->gate_nb1, t->gate_nb2, t->up_nb2, h->active,
                                            h->n_active, max_active, h->tile_start2, h->act, h->err, h->sm_count, st);
        }
        if (e != cudaSuccess) return cuda_fail(h, e, "prefill gate/up");
        {
            PhaseMark pm(h, st, TMOE_PHASE_DOWN);
            e = prefill_down(h, st, P, t, max_active, true);
        }
        if (e != cudaSuccess) return cuda_fail(h, e, "prefill down");
        if (!combine) return TMOE_OK;
        {
            PhaseMark pm(h, st, TMOE_PHASE_COMBINE);
            e = tmoe::launch_combine(h->dout, ids, w, T, k, H, t->n_slots, out, st);
        }
        if (e != cudaSuccess) return cuda_fail(h, e, "combine");
        return TMOE_OK;
    }
    if (!x_quantized) {
        {
            PhaseMark pm(h, st, TMOE_PHASE_QUANT_X);
            e = tmoe::launch_quantize_q8k(xn, T, H, nullptr, tmoe::Q8Rows{h->xq, h->xd, h->xbl, h->xbh, wg}, st);
        }
        if (e != cudaSuccess) return cuda_fail(h, e, "quantize x");
    }
    tmoe::GemvArgs g{};
    g.w0 = (const uint8_t *)t->gate;
    g.w1 = (const uint8_t *)t->up;
    g.nb1_0 = t->gate_nb1, g.nb2_0 = t->gate_nb2, g.nb1_1 = t->up_nb1, g.nb2_1 = t->up_nb2;
    g.K = H, g.N = I;
    g.xq = h->xq, g.xd = h->xd, g.xbl = h->xbl, g.xbh = h->xbh, g.x_div = k;
    g.perm = h->perm, g.active = h->active, g.n_active = h->n_active;
    g.n_slots = t->n_slots, g.max_active = max_active, g.n_pairs = (int)P, g.work = h->counters + 0;
    g.out = h->act, g.err = h->err;
    {
        PhaseMark pm(h, st, TMOE_PHASE_GATE_UP);
        e = tmoe::launch_gemv(wg, true, g, max_active, h->sm_count, st);
    }
    if (e != cudaSuccess) return cuda_fail(h, e, "gate/up gemv");
    if (prefill) {
        {
            PhaseMark pm(h, st, TMOE_PHASE_DOWN);
            e = prefill_down(h, st, P, t, max_active, false);
        }
        if (e != cudaSuccess) return cuda_fail(h, e, "prefill down");
        if (!combine) return TMOE_OK;
        {
            PhaseMark pm(h, st, TMOE_PHASE_COMBINE);
            e = tmoe::launch_combine(h->dout, ids, w, T, k, H, t->n_slots, out, st);
        }
        if (e != cudaSuccess) return cuda_fail(h, e, "combine");
        return TMOE_OK;
    }
    {
        PhaseMark pm(h, st, TMOE_PHASE_QUANT_ACT);
        e = tmoe::launch_quantize_q8k(h->act, P, I, ids, tmoe::Q8Rows{h->aq, h->ad, h->abl, h->abh, wd}, st);
    }
    if (e != cudaSuccess) return cuda_fail(h, e, "quantize act");
    tmoe::GemvArgs d{};
    d.w0 = (const uint8_t *)t->down;
    d.nb1_0 = t->down_nb1, d.nb2_0 = t->down_nb2;
    d.K = I, d.N = H;
    d.xq = h->aq, d.xd = h->ad, d.xbl = h->abl, d.xbh = h->abh, d.x_div = 1;
    d.perm = h->perm, d.active = h->active, d.n_active = h->n_active;
    d.n_slots = t->n_slots, d.max_active = max_active, d.n_pairs = (int)P, d.work = h->counters + 1;
    d.out = h->dout, d.err = h->err, d.early = 1;  // the dispatch is three launches back
    {
        PhaseMark pm(h, st, TMOE_PHASE_DOWN);
        e = tmoe::launch_gemv(wd, false, d, max_active, h->sm_count, st);
    }
    if (e != cudaSuccess) return cuda_fail(h, e, "down gemv");
    if (!combine) return TMOE_OK;
    {
        PhaseMark pm(h, st, TMOE_PHASE_COMBINE);
        e = tmoe::launch_combine(h->dout, ids, w, T, k, H, t->n_slots, out, st);
    }
    if (e != cudaSuccess) return cuda_fail(h, e, "combine");
    return TMOE_OK;
}

// Scratch of one mul_mat_id call: the Q8_K rows of b (qs, d, the split sub-block sums) and the
// dispatch buffers, each part rounded up to 256 bytes.  In bytes, with nbw = 2 (Q4_K) or 4 (Q6_K):
// rows*K*(1 + (4 + 8*nbw)/256) + 4*P + about 25 KiB of per-slot tables, plus the rounding.
struct MmidLayout {
    size_t q = 0, d = 0, bl = 0, bh = 0, cnt = 0, off = 0, act = 0, na = 0, perm = 0, work = 0, need = 0;
    MmidLayout(int wt, int64_t rows, int64_t K, int64_t P) {
        auto lay = [&](size_t bytes) {
            const size_t o = need;
            need = align_up(need + bytes, 256);
            return o;
        };
        const size_t nbw = (size_t)tmoe::q8_nbw(wt), nb = (size_t)(K / 256);
        q = lay((size_t)rows * (size_t)K), d = lay((size_t)rows * nb * 4);
        bl = lay((size_t)rows * nb * nbw * 4), bh = lay((size_t)rows * nb * nbw * 4);
        cnt = lay(kMaxSlots * 4), off = lay((kMaxSlots + 1) * 4), act = lay(kMaxSlots * 16), na = lay(4);
        perm = lay((size_t)P * 4 + 16), work = lay(kCounters * 4);
    }
};

// The argument checks of both mul_mat_id entry points.  T, n_used and K are bounded before any
// size is formed from them, so no product below can wrap.
int check_mmid(tmoe_handle *h, int32_t type, const void *W, size_t nb1, size_t nb2, int64_t K, int64_t N,
               int64_t n_w, const float *b, int64_t b1, const int32_t *ids, int64_t n_used, int64_t T,
               const float *out) {
    if (!is_expert_type(type))
        return fail(h, TMOE_E_UNSUPPORTED, "mul_mat_id type %d (need Q4_K, Q6_K or Q6_K_R8)", type);
    if (K <= 0 || K % 256 || K > (1 << 20) || N <= 0 || N > (1 << 20) || n_w <= 0 || n_w > kMaxSlots ||
        n_used <= 0 || n_used > kMaxSlots || T < 0 || T > (1 << 24) || T * n_used > (1 << 30) ||
        (b1 != 1 && b1 != n_used))
        return fail(h, TMOE_E_INVALID, "bad mul_mat_id shape");
    if (!W || !b || !ids || !out) return fail(h, TMOE_E_INVALID, "null tensor");
    if (!aligned16(b)) return fail(h, TMOE_E_INVALID, "b must be 16-byte aligned");
    if (nb1 != row_size(type, K)) return fail(h, TMOE_E_UNSUPPORTED, "rows must be contiguous (nb1 == row size)");
    if (((uintptr_t)W & 15u) || (nb2 & 15u)) return fail(h, TMOE_E_INVALID, "W and nb2 must be 16-byte aligned");
    if (!tmoe::gemv_rows_per_item(wt_of(type), (int)K, (int)N))
        return fail(h, TMOE_E_UNSUPPORTED, "N=%lld rows per expert fit no GEMV row tile (multiples of 16 or 32)",
                    (long long)N);
    return TMOE_OK;
}

// The launches of a checked mul_mat_id call, its scratch (layout L) at `base`.
int run_mmid(tmoe_handle *h, cudaStream_t st, int wt, const void *W, size_t nb1, size_t nb2, int64_t K, int64_t N,
             int64_t n_w, const float *b, int64_t b1, const int32_t *ids, int64_t n_used, int64_t T, float *out,
             const MmidLayout &L, char *base) {
    const int64_t P = T * n_used, rows = T * b1;
    int8_t *q = (int8_t *)(base + L.q);
    float *d = (float *)(base + L.d);
    uint32_t *bl = (uint32_t *)(base + L.bl), *bh = (uint32_t *)(base + L.bh);
    int32_t *cnt = (int32_t *)(base + L.cnt), *offs = (int32_t *)(base + L.off), *na = (int32_t *)(base + L.na),
            *perm = (int32_t *)(base + L.perm);
    int4 *act = (int4 *)(base + L.act);
    int *work = (int *)(base + L.work);
    cudaError_t e;
    if ((e = tmoe::launch_sort_pairs(ids, (int)P, (int)n_w, cnt, offs, perm, act, na, work, kCounters, h->err, st)) !=
        cudaSuccess)
        return cuda_fail(h, e, "sort_pairs");
    if ((e = tmoe::launch_quantize_q8k(b, rows, (int)K, nullptr, tmoe::Q8Rows{q, d, bl, bh, wt}, st)) != cudaSuccess)
        return cuda_fail(h, e, "quantize b");
    if ((e = tmoe::launch_zero_invalid_rows(ids, P, (int)n_w, (int)N, out, st)) != cudaSuccess)
        return cuda_fail(h, e, "zero rows");
    tmoe::GemvArgs g{};
    g.w0 = (const uint8_t *)W;
    g.nb1_0 = nb1, g.nb2_0 = nb2;
    g.K = (int)K, g.N = (int)N;
    g.xq = q, g.xd = d, g.xbl = bl, g.xbh = bh, g.x_div = b1 == 1 ? (int)n_used : 1;
    const int max_active = (int)(P < n_w ? P : n_w);
    g.perm = perm, g.active = act, g.n_active = na;
    g.n_slots = (int)n_w, g.max_active = max_active, g.n_pairs = (int)P, g.work = work;
    g.out = out, g.err = h->err;
    if ((e = tmoe::launch_gemv(wt, false, g, max_active, h->sm_count, st)) != cudaSuccess)
        return cuda_fail(h, e, "mul_mat_id gemv");
    return TMOE_OK;
}

// Unmaps the peers' all-to-all buffers.
void close_peers(tmoe_handle::A2A &A) {
    for (auto &b : A.peer_base)
        if (b) cudaIpcCloseMemHandle(b), b = nullptr;
    A.p2p = false;
    A.comm = nullptr;
}

// Maps every rank's all-to-all buffers into this process for the exchange over peer memory (one
// collective step of all the communicator's ranks, on the first call with this communicator and
// buffer size): the ranks exchange their CUDA IPC handles and layouts with an all-gather, open
// the peers' handles, and take the path only if every rank mapped every peer and all layouts are
// the same; otherwise they keep the NCCL exchange.  Host-synchronous; returns TMOE_OK either way,
// or an error of the all-gather.
struct PeerInfo {
    cudaIpcMemHandle_t handle;
    uint64_t bytes;
    int32_t g, cap, k, H, ok;
    char pad[128 - sizeof(cudaIpcMemHandle_t) - 8 - 20];
};
static_assert(sizeof(PeerInfo) == 128, "peer info");

int setup_peers(tmoe_handle *h, tmoe_comm *comm, int g, int rank, cudaStream_t st) {
    auto &A = h->a2a;
    const tmoe_config &c = h->cfg;
    close_peers(A);
    A.comm = comm;
    // the counters start from zero on every rank before any rank can write to another
    if (cudaMemset(A.flags, 0, (size_t)((char *)A.ctl - (char *)A.flags) + (size_t)(4 + 2 * g) * 4) != cudaSuccess) {
        cudaGetLastError();
        return fail(h, TMOE_E_CUDA, "all-to-all counters");
    }
    PeerInfo mine{};
    mine.ok = g <= tmoe::EP_MAX_PEERS && cudaIpcGetMemHandle(&mine.handle, A.mem) == cudaSuccess;
    cudaGetLastError();
    mine.bytes = A.bytes, mine.g = g, mine.cap = A.cap, mine.k = c.n_expert_used, mine.H = c.n_embd;
    void *dev = nullptr;
    if (cudaMalloc(&dev, sizeof(PeerInfo) * (g + 1) + 8 * (g + 1)) != cudaSuccess)
        return fail(h, TMOE_E_NOMEM, "peer exchange scratch");
    std::vector<PeerInfo> all(g);
    char msg[256];
    int rc = TMOE_OK;
    int ok = 0;
    if (cudaMemcpy(dev, &mine, sizeof mine, cudaMemcpyHostToDevice) != cudaSuccess)
        rc = fail(h, TMOE_E_CUDA, "peer exchange copy");
    if (rc == TMOE_OK) {
        rc = tmoe::ep_allgather_bytes(comm, dev, (char *)dev + sizeof(PeerInfo), sizeof(PeerInfo), st, msg, sizeof msg);
        if (rc) rc = fail(h, rc, "%s", msg);
    }
    if (rc == TMOE_OK && (cudaStreamSynchronize(st) != cudaSuccess ||
                          cudaMemcpy(all.data(), (char *)dev + sizeof(PeerInfo), sizeof(PeerInfo) * g,
                                     cudaMemcpyDeviceToHost) != cudaSuccess))
        rc = fail(h, TMOE_E_CUDA, "peer exchange read-back");
    if (rc == TMOE_OK) {
        ok = 1;
        for (int p = 0; p < g; p++)
            if (!all[p].ok || all[p].bytes != mine.bytes || all[p].g != g || all[p].cap != mine.cap ||
                all[p].k != mine.k || all[p].H != mine.H)
                ok = 0;
        for (int p = 0; p < g && ok; p++) {
            if (p == rank) continue;
            if (cudaIpcOpenMemHandle(&A.peer_base[p], all[p].handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                A.peer_base[p] = nullptr;
                ok = 0;
            }
        }
        // every rank must take the same path: the minimum of the ranks' results
        int *oks = (int *)((char *)dev + sizeof(PeerInfo) * (g + 1));
        if (cudaMemcpy(oks, &ok, 4, cudaMemcpyHostToDevice) != cudaSuccess) rc = fail(h, TMOE_E_CUDA, "peer status");
        if (rc == TMOE_OK) {
            rc = tmoe::ep_allgather_bytes(comm, oks, oks + 1, 4, st, msg, sizeof msg);
            if (rc) rc = fail(h, rc, "%s", msg);
        }
        std::vector<int> all_ok(g, 0);
        if (rc == TMOE_OK && (cudaStreamSynchronize(st) != cudaSuccess ||
                              cudaMemcpy(all_ok.data(), oks + 1, 4 * g, cudaMemcpyDeviceToHost) != cudaSuccess))
            rc = fail(h, TMOE_E_CUDA, "peer status read-back");
        for (int p = 0; p < g; p++)
            if (!all_ok[p]) ok = 0;
    }
    cudaFree(dev);
    if (rc != TMOE_OK || !ok) {
        for (auto &b : A.peer_base)
            if (b) cudaIpcCloseMemHandle(b), b = nullptr;
        A.p2p = false;
        return rc;
    }
    auto at = [&](int p, const void *local) -> char * {
        const size_t off = (size_t)((const char *)local - (const char *)A.mem);
        return (char *)(p == rank ? A.mem : A.peer_base[p]) + off;
    };
    for (int p = 0; p < g; p++) {
        A.peers.r_ids[p] = (int32_t *)at(p, A.r_ids);
        A.peers.r_w[p] = (float *)at(p, A.r_w);
        A.peers.r_x[p] = (float *)at(p, A.r_x);
        A.peers.ret[p] = (float *)at(p, A.ret);
        A.peers.flags[p] = (int *)at(p, A.flags);
    }
    A.p2p = true;
    return TMOE_OK;
}

}  // namespace

extern "C" {

int tmoe_version(void) { return 100; }

int tmoe_create(const tmoe_config *cfg, tmoe_handle **out) {
    if (!cfg || !out) return fail(nullptr, TMOE_E_INVALID, "null argument");
    *out = nullptr;
    const tmoe_config &c = *cfg;
    if (c.n_embd <= 0 || c.n_ff <= 0 || c.n_expert <= 0 || c.n_expert_used <= 0 || c.max_tokens <= 0)
        return fail(nullptr, TMOE_E_INVALID, "non-positive dimension in config");
    if (c.n_embd % 256 || c.n_ff % 256)
        return fail(nullptr, TMOE_E_INVALID, "n_embd and n_ff must be multiples of 256 (K-quant super-blocks)");
    if (c.n_expert > 256 || c.n_expert_used > 32 || c.n_expert_used > c.n_expert)
        return fail(nullptr, TMOE_E_INVALID, "n_expert <= 256 and n_expert_used <= min(32, n_expert) required");
    if (!is_expert_type(c.gate_type) || !is_expert_type(c.up_type) || !is_expert_type(c.down_type))
        return fail(nullptr, TMOE_E_UNSUPPORTED, "expert types must be Q4_K (12), Q6_K (14) or Q6_K_R8 (%d)",
                    TMOE_TYPE_Q6_K_R8);
    if (c.gate_type != c.up_type)
        return fail(nullptr, TMOE_E_UNSUPPORTED, "gate and up must share a type");
    if ((int64_t)c.max_tokens * c.n_expert_used > (1 << 30))
        return fail(nullptr, TMOE_E_INVALID, "max_tokens * n_expert_used too large");
    DeviceGuard dg(c.device);
    if (!dg.ok) return fail(nullptr, TMOE_E_CUDA, "cudaSetDevice(%d) failed", c.device);
    tmoe_handle *h = new tmoe_handle();
    h->cfg = c;
    if (cudaDeviceGetAttribute(&h->sm_count, cudaDevAttrMultiProcessorCount, c.device) != cudaSuccess) {
        delete h;
        return fail(nullptr, TMOE_E_CUDA, "cannot query the SM count");
    }
    if (!tmoe::gemv_rows_per_item(wt_of(c.gate_type), c.n_embd, c.n_ff) ||
        !tmoe::gemv_rows_per_item(wt_of(c.down_type), c.n_ff, c.n_embd)) {
        delete h;
        return fail(nullptr, TMOE_E_UNSUPPORTED, "row counts must be multiples of the GEMV row tile");
    }
    h->ws_bytes = carve(h, nullptr);
    cudaError_t e = cudaMalloc(&h->ws, h->ws_bytes);
    if (e != cudaSuccess) {
        delete h;
        return fail(nullptr, TMOE_E_NOMEM, "cudaMalloc(%zu) failed: %s", h->ws_bytes, cudaGetErrorString(e));
    }
    carve(h, (char *)h->ws);
    {
        const int64_t P = (int64_t)c.max_tokens * c.n_expert_used;
        const MmidLayout L(TMOE_WT_Q6K, P, c.n_embd > c.n_ff ? c.n_embd : c.n_ff, P);
        if ((e = cudaMalloc(&h->op_ws, L.need)) != cudaSuccess) {
            cudaFree(h->ws);
            delete h;
            return fail(nullptr, TMOE_E_NOMEM, "cudaMalloc(%zu) failed: %s", L.need, cudaGetErrorString(e));
        }
        h->op_ws_bytes = L.need;
    }
    e = cudaMemset(h->ws, 0, h->ws_bytes);  // the error flag and the routing counters start at zero
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(h->ws);
        cudaFree(h->op_ws);
        delete h;
        return fail(nullptr, TMOE_E_CUDA, "cudaMemset: %s", cudaGetErrorString(e));
    }
    *out = h;
    return TMOE_OK;
}

void tmoe_destroy(tmoe_handle *h) {
    if (!h) return;
    DeviceGuard dg(h->cfg.device);
    if (h->ws) cudaFree(h->ws);
    if (h->op_ws) cudaFree(h->op_ws);
    if (h->dense_ws) cudaFree(h->dense_ws);
    close_peers(h->a2a);
    if (h->a2a.mem) cudaFree(h->a2a.mem);
    for (auto &ev : h->prof.ev)
        if (ev) cudaEventDestroy(ev);
    delete h;
}

int tmoe_wait_flag(tmoe_handle *h, void *stream, const int32_t *flag, int32_t value, int64_t limit_ns) {
    if (!h) return TMOE_E_INVALID;
    if (!flag || ((uintptr_t)flag & 3u)) return fail(h, TMOE_E_INVALID, "flag must be a 4-byte aligned pointer");
    const uint64_t lim = limit_ns <= 0 || (uint64_t)limit_ns > TMOE_WAIT_LIMIT_NS ? TMOE_WAIT_LIMIT_NS
                                                                                  : (uint64_t)limit_ns;
    DeviceGuard dg(h->cfg.device);
    // a pinned host word is read through its device-mapped address; pageable memory is refused
    cudaPointerAttributes at{};
    cudaError_t e = cudaPointerGetAttributes(&at, flag);
    if (e != cudaSuccess) return cuda_fail(h, e, "wait flag: pointer attributes");
    const int32_t *dflag = flag;
    if (at.type == cudaMemoryTypeHost) {
        if (!at.devicePointer) return fail(h, TMOE_E_INVALID, "wait flag: the host word is not device-mapped");
        dflag = (const int32_t *)at.devicePointer;
    } else if (at.type != cudaMemoryTypeDevice && at.type != cudaMemoryTypeManaged) {
        return fail(h, TMOE_E_INVALID, "wait flag: the word must be device memory or pinned host memory");
    }
    e = tmoe::launch_wait_flag(dflag, value, lim, h->err, (cudaStream_t)stream);
    return e == cudaSuccess ? TMOE_OK : cuda_fail(h, e, "wait flag");
}

const char *tmoe_last_error(const tmoe_handle *h) {
    return h ? h->last_error.c_str() : g_create_error.c_str();
}

int tmoe_check(tmoe_handle *h, void *stream) {
    if (!h) return TMOE_E_INVALID;
    DeviceGuard dg(h->cfg.device);
    cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(h, e, "stream synchronize");
    int flag = 0;
    if ((e = cudaMemcpy(&flag, h->err, sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess)
        return cuda_fail(h, e, "read error flag");
    if (flag) {
        cudaMemset(h->err, 0, sizeof(int));
        if (flag == TMOE_DEV_ERR_BADID) return fail(h, TMOE_E_INVALID, "an expert id was >= n_slots");
        if (flag == TMOE_DEV_ERR_NOSLOT) return fail(h, TMOE_E_INVALID, "no free expert slot (all pinned)");
        return fail(h, TMOE_E_DEVICE, "a kernel gave up on a bounded wait (code %d)", flag);
    }
    return TMOE_OK;
}

int tmoe_route(tmoe_handle *h, void *stream, const float *x, int64_t T, int32_t use_norm,
               const float *norm_w, const float *router_w, const float *logits, int32_t *ids_out,
               float *w_out, float *xn_out, float *logits_out) {
    if (!h) return TMOE_E_INVALID;
    const tmoe_config &c = h->cfg;
    if (T < 0 || T > c.max_tokens) return fail(h, TMOE_E_INVALID, "T=%lld outside [0, max_tokens]", (long long)T);
    if (!ids_out || !w_out) return fail(h, TMOE_E_INVALID, "ids_out and w_out are required");
    if (!router_w && !logits) return fail(h, TMOE_E_INVALID, "need router_w or logits");
    if ((router_w || use_norm) && !x) return fail(h, TMOE_E_INVALID, "x is required");
    if (!aligned16(x) || !aligned16(router_w) || !aligned16(xn_out))
        return fail(h, TMOE_E_INVALID, "x, router_w and xn_out must be 16-byte aligned");
    if (T == 0) return TMOE_OK;
    DeviceGuard dg(c.device);
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e;
    const float *xs = x;
    if (use_norm) {
        float *dst = xn_out ? xn_out : h->xn;
        {
            PhaseMark pm(h, st, TMOE_PHASE_RMS_NORM);
            e = tmoe::launch_rms_norm(x, norm_w, c.rms_eps, T, c.n_embd, dst, st);
        }
        if (e != cudaSuccess) return cuda_fail(h, e, "rms_norm");
        xs = dst;
    } else if (xn_out && x) {
        if ((e = cudaMemcpyAsync(xn_out, x, sizeof(float) * T * c.n_embd, cudaMemcpyDeviceToDevice, st)) !=
            cudaSuccess)
            return cuda_fail(h, e, "copy xn");
    }
    const float *lg = logits;
    if (router_w) {
        float *dst = logits_out ? logits_out : h->logits;
        {
            PhaseMark pm(h, st, TMOE_PHASE_ROUTER_LOGITS);
            e = tmoe::launch_router_logits(xs, router_w, T, c.n_embd, c.n_expert, dst, nullptr, h->err, st);
        }
        if (e != cudaSuccess) return cuda_fail(h, e, "router logits");
        lg = dst;
    } else if (logits_out) {
        if ((e = cudaMemcpyAsync(logits_out, logits, sizeof(float) * T * c.n_expert, cudaMemcpyDeviceToDevice,
                                 st)) != cudaSuccess)
            return cuda_fail(h, e, "copy logits");
    }
    {
        PhaseMark pm(h, st, TMOE_PHASE_TOPK);
        e = tmoe::launch_softmax_topk(lg, T, c.n_expert, c.n_expert_used, ids_out, w_out, nullptr, st);
    }
    if (e != cudaSuccess) return cuda_fail(h, e, "softmax/top-k");
    return TMOE_OK;
}

int tmoe_experts(tmoe_handle *h, void *stream, const float *xn, int64_t T, const int32_t *ids,
                 const float *w, const tmoe_expert_tensors *wts, float *out) {
    if (!h) return TMOE_E_INVALID;
    const tmoe_config &c = h->cfg;
    if (T < 0 || T > c.max_tokens) return fail(h, TMOE_E_INVALID, "T=%lld outside [0, max_tokens]", (long long)T);
    if (!xn || !ids || !w || !out) return fail(h, TMOE_E_INVALID, "null tensor");
    if (!aligned16(xn) || !aligned16(out)) return fail(h, TMOE_E_INVALID, "xn and out must be 16-byte aligned");
    int rc = check_tensors(h, wts);
    if (rc) return rc;
    if (T == 0) return TMOE_OK;
    DeviceGuard dg(c.device);
    return run_experts(h, (cudaStream_t)stream, xn, T, ids, w, wts, out, false, false);
}

int tmoe_layer(tmoe_handle *h, void *stream, const float *x, int64_t T, int32_t use_norm, const float *norm_w,
               const float *router_w, const float *logits, const int32_t *id_map, const tmoe_expert_tensors *wts,
               float *out, int32_t *ids_out, float *w_out) {
    if (!h) return TMOE_E_INVALID;
    const tmoe_config &c = h->cfg;
    if (T < 0 || T > c.max_tokens) return fail(h, TMOE_E_INVALID, "T=%lld outside [0, max_tokens]", (long long)T);
    if (!x || !out) return fail(h, TMOE_E_INVALID, "null tensor");
    if (!router_w && !logits) return fail(h, TMOE_E_INVALID, "need router_w or logits");
    if (!aligned16(x) || !aligned16(out) || !aligned16(router_w))
        return fail(h, TMOE_E_INVALID, "x, out and router_w must be 16-byte aligned");
    int rc = check_tensors(h, wts);
    if (rc) return rc;
    if (T == 0) return TMOE_OK;
    DeviceGuard dg(c.device);
    tmoe::PdlScope pdl(!h->prof.on);  // its kernels overlap their predecessors' tails (programmatic launch)
    cudaStream_t st = (cudaStream_t)stream;
    const int k = c.n_expert_used;
    int32_t *ids = ids_out ? ids_out : h->ids;
    float *w = w_out ? w_out : h->w;
    cudaError_t e;
    const float *xn = x;
    if (use_norm) {
        {
            PhaseMark pm(h, st, TMOE_PHASE_RMS_NORM);
            e = tmoe::launch_rms_norm(x, norm_w, c.rms_eps, T, c.n_embd, h->xn, st);
        }
        if (e != cudaSuccess) return cuda_fail(h, e, "rms_norm");
        xn = h->xn;
    }
    // logits (and, fused, the Q8_K rows of xn)
    bool x_quantized = false;
    const float *lg = logits;
    if (router_w && tmoe::route_fused_fits(T, k, c.n_expert, c.n_embd, wts->n_slots)) {
        // decode regime: logits + Q8_K of xn + top-k + id map + dispatch in one launch
        const tmoe::Q8Rows q8{h->xq, h->xd, h->xbl, h->xbh, wt_of(c.gate_type)};
        {
            PhaseMark pm(h, st, TMOE_PHASE_ROUTER_LOGITS);
            e = tmoe::launch_route_fused(xn, router_w, (int)T, c.n_embd, c.n_expert, k, &q8, h->logits, id_map,
                                         c.n_expert, ids, w, h->mapped, wts->n_slots, h->counts, h->offsets,
                                         h->perm, h->active, h->n_active, h->counters, kCounters, h->route_done,
                                         h->err, st);
        }
        if (e != cudaSuccess) return cuda_fail(h, e, "fused routing");
        return run_experts(h, st, xn, T, h->mapped, w, wts, out, true, true);
    }
    if (router_w) {
        x_quantized = tmoe::router_fuses_q8(c.n_embd, T);
        const tmoe::Q8Rows q8{h->xq, h->xd, h->xbl, h->xbh, wt_of(c.gate_type)};
        {
            PhaseMark pm(h, st, TMOE_PHASE_ROUTER_LOGITS);
            e = tmoe::launch_router_logits(xn, router_w, T, c.n_embd, c.n_expert, h->logits,
                                           x_quantized ? &q8 : nullptr, h->err, st);
        }
        if (e != cudaSuccess) return cuda_fail(h, e, "router logits");
        lg = h->logits;
    }
    const int32_t *used = ids;
    bool dispatched = false;
    if (tmoe::route_dispatch_fits(T, k, c.n_expert, wts->n_slots)) {
        // decode regime: softmax/top-k + id map + dispatch in one kernel
        {
            PhaseMark pm(h, st, TMOE_PHASE_TOPK);
            e = tmoe::launch_route_dispatch(lg, (int)T, c.n_expert, k, id_map, c.n_expert, ids, w, h->mapped,
                                            wts->n_slots, h->counts, h->offsets, h->perm, h->active, h->n_active,
                                            h->counters, kCounters, h->err, st);
        }
        if (e != cudaSuccess) return cuda_fail(h, e, "route/dispatch");
        used = h->mapped;
        dispatched = true;
    } else {
        {
            PhaseMark pm(h, st, TMOE_PHASE_TOPK);
            e = tmoe::launch_softmax_topk(lg, T, c.n_expert, k, ids, w, nullptr, st);
        }
        if (e != cudaSuccess) return cuda_fail(h, e, "softmax/top-k");
        if (id_map) {
            {
                PhaseMark pm(h, st, TMOE_PHASE_MAP_IDS);
                e = tmoe::launch_map_ids(ids, T * k, id_map, c.n_expert, h->mapped, st);
            }
            if (e != cudaSuccess) return cuda_fail(h, e, "map ids");
            used = h->mapped;
        }
    }
    return run_experts(h, st, xn, T, used, w, wts, out, dispatched, x_quantized);
}

int tmoe_layer_bf16(tmoe_handle *h, void *stream, const uint16_t *x, int64_t T, int32_t use_norm, const float *norm_w,
                    const float *router_w, const float *logits, const int32_t *id_map, const tmoe_expert_tensors *wts,
                    float *out, int32_t *ids_out, float *w_out) {
    if (!h) return TMOE_E_INVALID;
    const tmoe_config &c = h->cfg;
    if (T < 0 || T > c.max_tokens) return fail(h, TMOE_E_INVALID, "T=%lld outside [0, max_tokens]", (long long)T);
    if (!x) return fail(h, TMOE_E_INVALID, "null tensor");
    if (!aligned16(x)) return fail(h, TMOE_E_INVALID, "x must be 16-byte aligned");
    if (T == 0) return tmoe_layer(h, stream, h->x32, 0, use_norm, norm_w, router_w, logits, id_map, wts, out, ids_out,
                                  w_out);
    DeviceGuard dg(c.device);
    const cudaError_t e = tmoe::launch_widen_bf16(x, T * c.n_embd, h->x32, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(h, e, "widen bf16");
    return tmoe_layer(h, stream, h->x32, T, use_norm, norm_w, router_w, logits, id_map, wts, out, ids_out, w_out);
}

int tmoe_ep_layer(tmoe_handle *h, void *stream, tmoe_comm *comm, const float *x, int64_t T, int32_t use_norm,
                  const float *norm_w, const float *router_w, const float *logits, const int32_t *id_map,
                  const tmoe_expert_tensors *wts, float *out, int32_t *ids_out, float *w_out) {
    if (!h) return TMOE_E_INVALID;
    const tmoe_config &c = h->cfg;
    if (!comm) return fail(h, TMOE_E_INVALID, "null communicator");
    if (tmoe::ep_comm_device(comm) != c.device)
        return fail(h, TMOE_E_INVALID, "communicator device %d != handle device %d", tmoe::ep_comm_device(comm),
                    c.device);
    // the arguments the sum needs; anything else that fails below still joins the sum
    if (T < 0 || T > c.max_tokens) return fail(h, TMOE_E_INVALID, "T=%lld outside [0, max_tokens]", (long long)T);
    if (!out) return fail(h, TMOE_E_INVALID, "null tensor");
    if (T == 0) return TMOE_OK;
    const int rc = tmoe_layer(h, stream, x, T, use_norm, norm_w, router_w, logits, id_map, wts, out, ids_out, w_out);
    DeviceGuard dg(c.device);
    char msg[256];
    const int rc2 = tmoe::ep_allreduce_sum(comm, out, (size_t)T * c.n_embd, (cudaStream_t)stream, msg, sizeof msg);
    if (rc) return rc;
    if (rc2) return fail(h, rc2, "%s", msg);
    return TMOE_OK;
}

int tmoe_ep_a2a_layer(tmoe_handle *h, void *stream, tmoe_comm *comm, const float *x, int64_t T, int32_t use_norm,
                      const float *norm_w, const float *router_w, const float *logits, const tmoe_expert_tensors *wts,
                      float *out, int32_t *ids_out, float *w_out) {
    if (!h) return TMOE_E_INVALID;
    const tmoe_config &c = h->cfg;
    if (!comm) return fail(h, TMOE_E_INVALID, "null communicator");
    if (tmoe::ep_comm_device(comm) != c.device)
        return fail(h, TMOE_E_INVALID, "communicator device %d != handle device %d", tmoe::ep_comm_device(comm),
                    c.device);
    int rank = 0;
    const int g = tmoe::ep_comm_ranks(comm, &rank);
    const int cap = c.max_tokens / g, k = c.n_expert_used, H = c.n_embd, E = c.n_expert;
    if (E % g) return fail(h, TMOE_E_INVALID, "%d experts do not split over %d ranks", E, g);
    if (cap < 1) return fail(h, TMOE_E_INVALID, "max_tokens %d < %d ranks", c.max_tokens, g);
    if (T < 0 || T > cap) return fail(h, TMOE_E_INVALID, "T=%lld outside [0, max_tokens / ranks = %d]", (long long)T, cap);
    if (!out || !x) return fail(h, TMOE_E_INVALID, "null tensor");
    if (!aligned16(x) || !aligned16(out)) return fail(h, TMOE_E_INVALID, "x and out must be 16-byte aligned");
    int rc = check_tensors(h, wts);
    if (rc) return rc;
    if (wts->n_slots != E / g) return fail(h, TMOE_E_INVALID, "wts hold %d experts, the rank's share is %d",
                                          wts->n_slots, E / g);
    DeviceGuard dg(c.device);
    cudaStream_t st = (cudaStream_t)stream;
    auto &A = h->a2a;
    if (A.g != g || A.cap != cap) {  // the exchange buffers of this rank count
        close_peers(A);
        if (A.mem) cudaFree(A.mem), A.mem = nullptr;
        const size_t ni = (size_t)g * cap, rows_x = ni * H * 4;
        const size_t bytes = align_up(ni * 4, 256) * 2 /* row_of, s_tok */ + align_up((size_t)g * 4, 256) +
                             align_up(ni * k * 4, 256) * 4 /* ids, w both ways */ + align_up(rows_x, 256) * 4 +
                             align_up((size_t)2 * g * 4, 256) + align_up((size_t)(4 + 2 * g) * 4, 256);
        if (cudaMalloc(&A.mem, bytes) != cudaSuccess) {
            cudaGetLastError();
            A.g = A.cap = 0;
            return fail(h, TMOE_E_NOMEM, "all-to-all buffers (%zu bytes)", bytes);
        }
        uint8_t *p = (uint8_t *)A.mem;
        auto take = [&](size_t n) {
            void *r = p;
            p += align_up(n, 256);
            return r;
        };
        A.row_of = (int32_t *)take(ni * 4), A.s_tok = (int32_t *)take(ni * 4), A.counts = (int32_t *)take(g * 4);
        A.s_ids = (int32_t *)take(ni * k * 4), A.r_ids = (int32_t *)take(ni * k * 4);
        A.s_w = (float *)take(ni * k * 4), A.r_w = (float *)take(ni * k * 4);
        A.s_x = (float *)take(rows_x), A.r_x = (float *)take(rows_x);
        A.part = (float *)take(rows_x), A.ret = (float *)take(rows_x);
        A.flags = (int *)take((size_t)2 * g * 4), A.ctl = (int *)take((size_t)(4 + 2 * g) * 4);
        if (cudaMemset(A.flags, 0, (size_t)((char *)p - (char *)A.flags)) != cudaSuccess) {
            cudaGetLastError();
            return fail(h, TMOE_E_CUDA, "all-to-all counters");
        }
        A.bytes = bytes;
        A.g = g, A.cap = cap;
    }
    if (A.comm != comm) {  // map the peers' buffers (every rank of the communicator takes this step)
        const int r = setup_peers(h, comm, g, rank, st);
        if (r != TMOE_OK) return r;
    }
    int32_t *ids = ids_out ? ids_out : h->ids;
    float *w = w_out ? w_out : h->w;
    // route this rank's tokens and pack the messages; on a failure the rank still takes both
    // exchange steps, with messages that carry no rows
    cudaError_t e = cudaSuccess;
    if (T && router_w && tmoe::route_fused_fits(T, k, E, H, E)) {
        // decode batches: the fused routing kernel (logits, top-k and a dispatch the exchange does not
        // use, in one launch), the same ids and weights as tmoe_route's two kernels
        if (use_norm) e = tmoe::launch_rms_norm(x, norm_w, c.rms_eps, T, H, h->xn, st);
        if (e == cudaSuccess) {
            PhaseMark pm(h, st, TMOE_PHASE_ROUTER_LOGITS);
            e = tmoe::launch_route_fused(use_norm ? h->xn : x, router_w, (int)T, H, E, k, nullptr, h->logits, nullptr,
                                         E, ids, w, h->mapped, E, h->counts, h->offsets, h->perm, h->active,
                                         h->n_active, h->counters, kCounters, h->route_done, h->err, st);
        }
        rc = e == cudaSuccess ? TMOE_OK : cuda_fail(h, e, "fused routing");
    } else {
        rc = T ? tmoe_route(h, stream, x, T, use_norm, norm_w, router_w, logits, ids, w, use_norm ? h->xn : nullptr,
                            nullptr)
               : TMOE_OK;
    }
    const float *xn = use_norm ? h->xn : x;
    if (A.p2p) {
        // the exchange over peer memory: the messages written into the peers' buffers, a bounded
        // wait for theirs, the experts, the partial rows written back, a bounded wait, the combine;
        // the kernels overlap their predecessors' tails (programmatic launch)
        tmoe::PdlScope pdl(!h->prof.on);
        {
            PhaseMark pm(h, st, TMOE_PHASE_MAP_IDS);
            e = tmoe::launch_ep_dispatch_p2p(ids, w, xn, rc == TMOE_OK ? (int)T : 0, k, H, E / g, g, cap, rank,
                                             A.peers, A.row_of, A.s_tok, A.counts, A.ctl, st);
        }
        if (e == cudaSuccess) e = tmoe::launch_ep_wait(0, g, rank, A.flags, A.ctl, h->err, st);
        if (e != cudaSuccess) return cuda_fail(h, e, "all-to-all dispatch over peer memory");
        const int rc3 = run_experts(h, st, A.r_x, (int64_t)g * cap, A.r_ids, A.r_w, wts, A.part, false, false);
        if (rc3 != TMOE_OK) cudaMemsetAsync(A.part, 0, (size_t)g * cap * H * 4, st);
        e = tmoe::launch_ep_return_p2p(A.part, A.r_ids, k, H, g, cap, rank, A.peers, A.ctl, st);
        if (e == cudaSuccess) e = tmoe::launch_ep_wait(1, g, rank, A.flags, A.ctl, h->err, st);
        if (e != cudaSuccess) return cuda_fail(h, e, "all-to-all return over peer memory");
        if (rc) return rc;
        if (rc3) return rc3;
        if (T) {
            PhaseMark pm(h, st, TMOE_PHASE_COMBINE);
            e = tmoe::launch_ep_combine(A.ret, A.part, rank, A.row_of, (int)T, H, g, cap, out, st);
        }
        return e == cudaSuccess ? TMOE_OK : cuda_fail(h, e, "all-to-all combine");
    }
    if (rc == TMOE_OK && T) {
        PhaseMark pm(h, st, TMOE_PHASE_MAP_IDS);
        e = tmoe::launch_ep_pack(ids, w, xn, (int)T, k, H, E / g, g, cap, rank, A.row_of, A.s_ids, A.s_w, A.r_ids,
                                 A.r_w, A.s_tok, A.counts, A.s_x, A.r_x, st);
        if (e != cudaSuccess) rc = cuda_fail(h, e, "all-to-all pack");
    }
    if (rc != TMOE_OK || T == 0) {  // no rows: -1 ids in every message, this rank's own one included
        cudaMemsetAsync(A.s_ids, 0xff, (size_t)g * cap * k * 4, st);
        cudaMemsetAsync(A.r_ids + (size_t)rank * cap * k, 0xff, (size_t)cap * k * 4, st);
    }
    char msg[256];
    const size_t nk = (size_t)cap * k * 4;
    const tmoe::EpBuf out_bufs[3] = {{A.s_ids, A.r_ids, nk}, {A.s_w, A.r_w, nk}, {A.s_x, A.r_x, (size_t)cap * H * 4}};
    // the pack wrote this rank's own message into the receive buffers already
    int rc2 = tmoe::ep_alltoall(comm, out_bufs, 3, st, msg, sizeof msg, false);
    if (rc2) return fail(h, rc2, "%s", msg);
    // this rank's experts over every received row (rows of other ranks' tokens), combined per row
    // in choice order: the partial sums of the reference's EP mode
    const int rc3 = run_experts(h, st, A.r_x, (int64_t)g * cap, A.r_ids, A.r_w, wts, A.part, false, false);
    if (rc3 != TMOE_OK) cudaMemsetAsync(A.part, 0, (size_t)g * cap * H * 4, st);
    const tmoe::EpBuf back = {A.part, A.ret, (size_t)cap * H * 4};
    rc2 = tmoe::ep_alltoall(comm, &back, 1, st, msg, sizeof msg, false);  // own partials: read from A.part
    if (rc2) return fail(h, rc2, "%s", msg);
    if (rc) return rc;
    if (rc3) return rc3;
    if (T) {
        PhaseMark pm(h, st, TMOE_PHASE_COMBINE);
        e = tmoe::launch_ep_combine(A.ret, A.part, rank, A.row_of, (int)T, H, g, cap, out, st);
    }
    return e == cudaSuccess ? TMOE_OK : cuda_fail(h, e, "all-to-all combine");
}

int tmoe_map_ids(tmoe_handle *h, void *stream, const int32_t *ids, int64_t n, const int32_t *table,
                 int64_t n_table, int32_t *out) {
    if (!h) return TMOE_E_INVALID;
    if (n < 0 || n_table < 0 || (n > 0 && (!ids || !table || !out)))
        return fail(h, TMOE_E_INVALID, "bad map_ids arguments");
    DeviceGuard dg(h->cfg.device);
    cudaError_t e = tmoe::launch_map_ids(ids, n, table, n_table, out, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(h, e, "map ids");
    return TMOE_OK;
}

int tmoe_mul_mat_id(tmoe_handle *h, void *stream, int32_t type, const void *W, size_t nb1, size_t nb2,
                    int64_t K, int64_t N, int64_t n_w, const float *b, int64_t b1, const int32_t *ids,
                    int64_t n_used, int64_t T, float *out) {
    if (!h) return TMOE_E_INVALID;
    const int rc = check_mmid(h, type, W, nb1, nb2, K, N, n_w, b, b1, ids, n_used, T, out);
    if (rc != TMOE_OK) return rc;
    const MmidLayout L(wt_of(type), T * b1, K, T * n_used);
    if (L.need > h->op_ws_bytes)
        return fail(h, TMOE_E_INVALID,
                    "mul_mat_id needs %zu bytes of scratch for T=%lld, b1=%lld, K=%lld, n_used=%lld; the handle's "
                    "holds %zu (sized at create for T*b1 and T*n_used up to max_tokens*n_expert_used and K up to "
                    "max(n_embd, n_ff))",
                    L.need, (long long)T, (long long)b1, (long long)K, (long long)n_used, h->op_ws_bytes);
    if (T == 0) return TMOE_OK;
    DeviceGuard dg(h->cfg.device);
    return run_mmid(h, (cudaStream_t)stream, wt_of(type), W, nb1, nb2, K, N, n_w, b, b1, ids, n_used, T, out, L,
                    (char *)h->op_ws);
}

int tmoe_mul_mat(tmoe_handle *h, void *stream, int32_t type, const void *W, size_t nb1, int64_t K, int64_t N,
                 const float *x, int64_t T, int32_t reuse_x, float *out) {
    if (!h) return TMOE_E_INVALID;
    if (!is_kquant(type)) return fail(h, TMOE_E_UNSUPPORTED, "mul_mat type %d (need Q4_K or Q6_K)", type);
    if (K <= 0 || K % 256 || N <= 0 || T < 0 || T > (1 << 24)) return fail(h, TMOE_E_INVALID, "bad mul_mat shape");
    if (T == 0) return TMOE_OK;
    if (!W || !x || !out) return fail(h, TMOE_E_INVALID, "null tensor");
    if (!aligned16(x)) return fail(h, TMOE_E_INVALID, "x must be 16-byte aligned");
    const int wt = wt_of(type);
    if (nb1 != row_size(type, K)) return fail(h, TMOE_E_UNSUPPORTED, "rows must be contiguous (nb1 == row size)");
    if ((uintptr_t)W & 15u) return fail(h, TMOE_E_INVALID, "W must be 16-byte aligned");
    if (!tmoe::gemv_rows_per_item(wt, (int)K, (int)N))
        return fail(h, TMOE_E_UNSUPPORTED, "N=%lld rows fit no GEMV row tile (multiples of 16)", (long long)N);
    const bool reuse = reuse_x != 0;
    if (reuse && (h->dense_x != x || h->dense_wt != wt || h->dense_k != K || h->dense_t != T))
        return fail(h, TMOE_E_INVALID, "reuse_x: the last quantised activations are not these (x, K, T, weight family)");
    DeviceGuard dg(h->cfg.device);
    tmoe::PdlScope pdl(!h->prof.on);  // overlap with the kernel before (programmatic launch)
    cudaStream_t st = (cudaStream_t)stream;
    size_t need = 0;
    auto lay = [&](size_t bytes) {
        size_t o = need;
        need = align_up(need + bytes, 256);
        return o;
    };
    if (T >= kDenseGemmMinTokens && N % 256 == 0 && N <= (1 << 20)) {
        // A prompt-sized batch: the matrix dequantised to fp16 once and one tcgen05 GEMM over all rows
        // (x through the same Q8_K round trip, then fp16), the large-batch MoE path's down GEMM with
        // one expert and the rows in place.  fp16 weights are its only departure from the GEMV's sums.
        const size_t o_a = lay((size_t)T * K * 2), o_w = lay((size_t)N * K * 2), o_act = lay(16), o_na = lay(4),
                     o_ts = lay(16), o_perm = lay((size_t)T * 4);
        cudaError_t e;
        if (need > h->dense_ws_bytes) {
            if (reuse) return fail(h, TMOE_E_INVALID, "reuse_x before the workspace exists");
            if (h->dense_ws) {
                cudaStreamSynchronize(st);
                cudaFree(h->dense_ws);
                h->dense_ws = nullptr;
                h->dense_ws_bytes = 0;
                h->dense_x = nullptr;
            }
            if ((e = cudaMalloc(&h->dense_ws, need)) != cudaSuccess)
                return fail(h, TMOE_E_NOMEM, "cudaMalloc(%zu): %s", need, cudaGetErrorString(e));
            h->dense_ws_bytes = need;
        }
        char *base = (char *)h->dense_ws;
        __half *a16 = (__half *)(base + o_a), *w16 = (__half *)(base + o_w);
        int4 *act = (int4 *)(base + o_act);
        int32_t *na = (int32_t *)(base + o_na);
        int *ts = (int *)(base + o_ts);
        int32_t *perm = (int32_t *)(base + o_perm);
        if (!(reuse && h->dense_a16)) {
            if ((e = tmoe::launch_prep_rows(x, nullptr, (int)T, nullptr, 1, (int)K, a16, st)) != cudaSuccess)
                return cuda_fail(h, e, "mul_mat rows");
            h->dense_x = x, h->dense_wt = wt, h->dense_k = K, h->dense_t = T, h->dense_a16 = true;
        }
        // one active "expert" (the matrix) over rows [0, T)
        if ((e = tmoe::launch_dense_prep((int)T, (int)T, 1, act, na, perm, nullptr, 0, st)) != cudaSuccess)
            return cuda_fail(h, e, "mul_mat tile table");
        if ((e = tmoe::launch_dequant_f16(wt, (const uint8_t *)W, 0, (int)N, (int)K, act, na, 1, w16, st)) !=
            cudaSuccess)
            return cuda_fail(h, e, "mul_mat dequant");
        if ((e = tmoe::launch_prefill_gemm(false, a16, (int)T, (int)K, w16, nullptr, 1, (int)N, act, na, 1, ts,
                                           nullptr, out, h->err, h->sm_count, st)) != cudaSuccess)
            return cuda_fail(h, e, "mul_mat gemm");
        return TMOE_OK;
    }
    const size_t nbw = (size_t)tmoe::q8_nbw(wt);
    const size_t o_q = lay((size_t)T * K), o_d = lay((size_t)T * (K / 256) * 4);
    const size_t o_bl = lay((size_t)T * (K / 256) * nbw * 4), o_bh = lay((size_t)T * (K / 256) * nbw * 4);
    // token groups, each an active entry of the matrix: 16 tokens (one pass of the GEMV's two-group
    // kernel) from 64 tokens on, fewer below, so that small batches still spread over the SMs
    // (C3 decode at 16 sequences: 10.7 ms per step against 12.0 with one group)
    // A matrix well beyond L2 (the output head) takes the batch as one entry instead: its token
    // passes over a row tile then follow one another and re-read the tile from L2, where separate
    // groups would each stream the whole matrix from HBM.
    const int kGroup = (size_t)N * nb1 > (64u << 20) ? (int)T : T >= 64 ? 16 : T >= 16 ? 4 : 1;
    const int n_groups = (int)((T + kGroup - 1) / kGroup);
    // Q4_K: split K in ks slices (each at least one two-super-block fill) while the items (row tiles x
    // groups x slices) would leave warps idle; the slices' partial outputs are then added in order.
    const int nb = (int)(K / 256);
    int ks = 1;
    if (wt == TMOE_WT_Q4K && N % 4 == 0 && !h->dense_nosplit)
        while (nb % (2 * ks) == 0 && nb / (2 * ks) >= 2 && (N / 16) * n_groups * ks < 8LL * h->sm_count &&
               T * 2 * ks < (1 << 24))
            ks *= 2;
    const size_t o_act = lay((size_t)n_groups * ks * 16), o_na = lay(4), o_perm = lay((size_t)T * ks * 4 + 16),
                 o_work = lay(kCounters * 4), o_part = ks > 1 ? lay((size_t)T * ks * N * 4) : 0;
    cudaError_t e;
    if (need > h->dense_ws_bytes) {  // grows on first use (outside any stream capture)
        if (reuse) return fail(h, TMOE_E_INVALID, "reuse_x before the workspace exists");
        if (h->dense_ws) {
            cudaStreamSynchronize(st);
            cudaFree(h->dense_ws);
            h->dense_ws = nullptr;
            h->dense_ws_bytes = 0;
        }
        if ((e = cudaMalloc(&h->dense_ws, need)) != cudaSuccess)
            return fail(h, TMOE_E_NOMEM, "cudaMalloc(%zu): %s", need, cudaGetErrorString(e));
        h->dense_ws_bytes = need;
    }
    char *base = (char *)h->dense_ws;
    int8_t *q = (int8_t *)(base + o_q);
    float *d = (float *)(base + o_d);
    uint32_t *bl = (uint32_t *)(base + o_bl), *bh = (uint32_t *)(base + o_bh);
    int4 *act = (int4 *)(base + o_act);
    int32_t *na = (int32_t *)(base + o_na), *perm = (int32_t *)(base + o_perm);
    int *work = (int *)(base + o_work);
    float *part = (float *)(base + o_part);
    if (!reuse) {
        if ((e = tmoe::launch_quantize_q8k(x, T, (int)K, nullptr, tmoe::Q8Rows{q, d, bl, bh, wt}, st)) != cudaSuccess)
            return cuda_fail(h, e, "quantize x");
        h->dense_x = x, h->dense_wt = wt, h->dense_k = K, h->dense_t = T, h->dense_a16 = false;
    }
    for (;;) {
        if ((e = tmoe::launch_dense_prep((int)T, kGroup, ks, act, na, perm, work, kCounters, st)) != cudaSuccess)
            return cuda_fail(h, e, "mul_mat prep");
        tmoe::GemvArgs g{};
        g.w0 = (const uint8_t *)W;
        g.nb1_0 = nb1, g.nb2_0 = ks > 1 ? nb1 / ks : align_up(nb1 * (size_t)N, 16);
        g.K = (int)(K / ks), g.N = (int)N;
        g.xq = q, g.xd = d, g.xbl = bl, g.xbh = bh, g.x_div = 1;
        g.perm = perm, g.active = act, g.n_active = na;
        g.n_slots = ks, g.max_active = n_groups * ks, g.n_pairs = (int)(T * ks), g.work = work;
        g.out = ks > 1 ? part : out, g.err = h->err;
        e = tmoe::launch_gemv(wt, false, g, n_groups * ks, h->sm_count, st);
        if (e == cudaErrorInvalidValue && ks > 1) {  // no tensor map over the slices: unsplit from now on
            cudaGetLastError();
            h->dense_nosplit = true;
            ks = 1;
            continue;
        }
        if (e != cudaSuccess) return cuda_fail(h, e, "mul_mat gemv");
        break;
    }
    if (ks > 1 && (e = tmoe::launch_splitk_sum(part, T, (int)N, ks, out, st)) != cudaSuccess)
        return cuda_fail(h, e, "mul_mat split-K sum");
    return TMOE_OK;
}

}  // extern "C"

namespace {

// Scratch of tmoe_mul_mat_id_noalloc: module-global device memory, so that the call allocates
// nothing.  One array per device (per CUDA context), shared by every handle of the process.
constexpr size_t kNoAllocScratchBytes = 2u << 20;  // 2 MiB
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device, looked up once per device (the
// lookup may load the module there).  The cache entries are atomics, so threads making their first
// call on a device at the same time only repeat the lookup.  A cudaDeviceReset unloads the module
// and leaves the cached address stale; the header says not to use the entry point after one.
cudaError_t noalloc_scratch(int dev, char **out) {
    static std::atomic<char *> addr[64];
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    char *p = addr[dev].load(std::memory_order_acquire);
    if (!p) {
        void *q = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&q, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        p = (char *)q;
        addr[dev].store(p, std::memory_order_release);
    }
    *out = p;
    return cudaSuccess;
}

}  // namespace

extern "C" {

int tmoe_mul_mat_id_noalloc(tmoe_handle *h, void *stream, int32_t type, const void *W, size_t nb1, size_t nb2,
                            int64_t K, int64_t N, int64_t n_w, const float *b, int64_t b1, const int32_t *ids,
                            int64_t n_used, int64_t T, float *out) {
    if (!h) return TMOE_E_INVALID;
    const int rc = check_mmid(h, type, W, nb1, nb2, K, N, n_w, b, b1, ids, n_used, T, out);
    if (rc != TMOE_OK) return rc;
    // the same layout as tmoe_mul_mat_id's scratch, placed in the static array
    const MmidLayout L(wt_of(type), T * b1, K, T * n_used);
    if (L.need > kNoAllocScratchBytes)
        return fail(h, TMOE_E_INVALID,
                    "mul_mat_id_noalloc needs %zu bytes of scratch for T=%lld, b1=%lld, K=%lld, n_used=%lld; the static "
                    "scratch holds %zu (use tmoe_mul_mat_id)",
                    L.need, (long long)T, (long long)b1, (long long)K, (long long)n_used, kNoAllocScratchBytes);
    if (T == 0) return TMOE_OK;
    DeviceGuard dg(h->cfg.device);
    char *base = nullptr;
    const cudaError_t e = noalloc_scratch(h->cfg.device, &base);
    if (e != cudaSuccess) return cuda_fail(h, e, "cudaGetSymbolAddress(noalloc scratch)");
    // nothing in the scratch needs to start at zero: the dispatch kernel writes counts, offsets,
    // the active list and perm, and zeroes the GEMV work counters, before the GEMV reads them
    return run_mmid(h, (cudaStream_t)stream, wt_of(type), W, nb1, nb2, K, N, n_w, b, b1, ids, n_used, T, out, L,
                    base);
}

int tmoe_dispatch(tmoe_handle *h, void *stream, const int32_t *ids, int64_t T, int32_t n_slots,
                  int32_t *counts, int32_t *offsets, int32_t *perm) {
    if (!h) return TMOE_E_INVALID;
    const tmoe_config &c = h->cfg;
    if (T < 0 || T > c.max_tokens) return fail(h, TMOE_E_INVALID, "T=%lld outside [0, max_tokens]", (long long)T);
    if (n_slots <= 0 || n_slots > kMaxSlots) return fail(h, TMOE_E_INVALID, "n_slots %d out of range", n_slots);
    if (!ids || !counts || !offsets || !perm) return fail(h, TMOE_E_INVALID, "null tensor");
    DeviceGuard dg(c.device);
    cudaError_t e = tmoe::launch_sort_pairs(ids, (int)(T * c.n_expert_used), n_slots, counts, offsets, perm,
                                            h->active, h->n_active, nullptr, 0, h->err, (cudaStream_t)stream,
                                            h->sort_scratch, h->sort_scratch_ints);
    if (e != cudaSuccess) return cuda_fail(h, e, "sort_pairs");
    return TMOE_OK;
}

int tmoe_quantize(int32_t type, const float *x, int64_t nrows, int64_t ncols, void *out, void *stream) {
    if (!is_kquant(type)) return fail(nullptr, TMOE_E_UNSUPPORTED, "quantize type %d", type);
    if (nrows < 0 || ncols <= 0 || ncols % 256) return fail(nullptr, TMOE_E_INVALID, "ncols must be a multiple of 256");
    if (nrows == 0) return TMOE_OK;
    if (!x || !out) return fail(nullptr, TMOE_E_INVALID, "null tensor");
    cudaError_t e = tmoe::launch_quantize(wt_of(type), x, nrows * (ncols / 256), (uint8_t *)out, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "quantize");
    return TMOE_OK;
}

int tmoe_dequantize(int32_t type, const void *in, int64_t n, float *out, void *stream) {
    if (!is_kquant(type)) return fail(nullptr, TMOE_E_UNSUPPORTED, "dequantize type %d", type);
    if (n < 0 || n % 256) return fail(nullptr, TMOE_E_INVALID, "n must be a multiple of 256");
    if (n == 0) return TMOE_OK;
    if (!in || !out) return fail(nullptr, TMOE_E_INVALID, "null tensor");
    cudaError_t e = tmoe::launch_dequantize(wt_of(type), (const uint8_t *)in, n, out, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "dequantize");
    return TMOE_OK;
}

int tmoe_prepack(int32_t type, const void *src, size_t nb1, size_t nb2, int64_t n_rows, int64_t K, int64_t n_mats,
                 void *dst, void *stream) {
    if (type != TMOE_TYPE_Q6_K)
        return fail(nullptr, TMOE_E_UNSUPPORTED, "prepack type %d (only Q6_K has a packed layout)", type);
    // (K <= 16384: a row group of 8 rows is staged in shared memory, 13,440 bytes per 1024 columns)
    if (n_rows < 0 || n_mats < 0 || K <= 0 || K % 256 || K > 16384 || n_rows % 8 || n_rows > (1ll << 30) ||
        n_mats > 65535)
        return fail(nullptr, TMOE_E_INVALID,
                    "prepack needs K a multiple of 256 up to 16384, rows a multiple of 8, at most 65535 matrices");
    if (n_rows == 0 || n_mats == 0) return TMOE_OK;
    if (!src || !dst) return fail(nullptr, TMOE_E_INVALID, "null tensor");
    const size_t rb = row_size(type, K);
    if (nb1 < rb || (n_mats > 1 && nb2 < (size_t)n_rows * nb1))
        return fail(nullptr, TMOE_E_INVALID, "rows or matrices overlap (nb1 < row size or nb2 < rows * nb1)");
    if (!aligned16(dst)) return fail(nullptr, TMOE_E_INVALID, "dst must be 16-byte aligned");
    const uintptr_t s0 = (uintptr_t)src, s1 = s0 + (size_t)(n_mats - 1) * nb2 + (size_t)(n_rows - 1) * nb1 + rb;
    const uintptr_t d0 = (uintptr_t)dst, d1 = d0 + (size_t)n_mats * n_rows * rb;
    if (s0 < d1 && d0 < s1) return fail(nullptr, TMOE_E_INVALID, "src and dst overlap");
    const cudaError_t e = tmoe::launch_prepack_q6k((const uint8_t *)src, nb1, nb2, n_rows, (int)K, n_mats,
                                                   (uint8_t *)dst, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "prepack");
    return TMOE_OK;
}

// ---------------------------------------------------------------- the decode step's other ops
int tmoe_get_rows(tmoe_handle *h, void *stream, int32_t type, const void *W, size_t nb1, int64_t K, int64_t n_rows_w,
                  const int32_t *rows, int64_t n, float *out) {
    if (!h) return TMOE_E_INVALID;
    if (type != 0 && type != 1 && !is_kquant(type)) return fail(h, TMOE_E_UNSUPPORTED, "get_rows type %d", type);
    if (K <= 0 || K > (1 << 30) || (is_kquant(type) && K % 256) || n < 0 || n_rows_w <= 0)
        return fail(h, TMOE_E_INVALID, "bad get_rows shape");
    const size_t rb = type == 0 ? (size_t)K * 4 : type == 1 ? (size_t)K * 2 : row_size(type, K);
    if (nb1 < rb) return fail(h, TMOE_E_INVALID, "row stride %zu below the row size %zu", nb1, rb);
    if (n == 0) return TMOE_OK;
    if (!W || !rows || !out) return fail(h, TMOE_E_INVALID, "null tensor");
    DeviceGuard dg(h->cfg.device);
    tmoe::PdlScope pdl(!h->prof.on);  // overlap with the kernel before (programmatic launch)
    cudaError_t e = tmoe::launch_get_rows(type, (const uint8_t *)W, nb1, (int)K, n_rows_w, rows, n, out, h->err,
                                          (cudaStream_t)stream);
    return e == cudaSuccess ? TMOE_OK : cuda_fail(h, e, "get_rows");
}

int tmoe_rms_norm(tmoe_handle *h, void *stream, const float *x, const float *w, float eps, int64_t rows, int64_t n,
                  float *out) {
    if (!h) return TMOE_E_INVALID;
    if (rows < 0 || n <= 0 || n > (1 << 30)) return fail(h, TMOE_E_INVALID, "bad rms_norm shape");
    if (rows == 0) return TMOE_OK;
    if (!x || !out) return fail(h, TMOE_E_INVALID, "null tensor");
    DeviceGuard dg(h->cfg.device);
    tmoe::PdlScope pdl(!h->prof.on);  // overlap with the kernel before (programmatic launch)
    cudaError_t e = tmoe::launch_rms_norm(x, w, eps, rows, (int)n, out, (cudaStream_t)stream);
    return e == cudaSuccess ? TMOE_OK : cuda_fail(h, e, "rms_norm");
}

int tmoe_rope_neox(tmoe_handle *h, void *stream, float *x, const int32_t *pos, int64_t n_tok, int32_t n_head,
                   int32_t head_dim, int32_t n_rot, float freq_base) {
    if (!h) return TMOE_E_INVALID;
    if (n_tok < 0 || n_head <= 0 || head_dim <= 0 || n_rot <= 0 || n_rot > head_dim || n_rot % 2 || freq_base <= 0)
        return fail(h, TMOE_E_INVALID, "bad rope shape");
    if (n_tok == 0) return TMOE_OK;
    if (!x || !pos) return fail(h, TMOE_E_INVALID, "null tensor");
    DeviceGuard dg(h->cfg.device);
    tmoe::PdlScope pdl(!h->prof.on);  // overlap with the kernel before (programmatic launch)
    cudaError_t e = tmoe::launch_rope_neox(x, pos, n_tok, n_head, head_dim, n_rot, freq_base, (cudaStream_t)stream);
    return e == cudaSuccess ? TMOE_OK : cuda_fail(h, e, "rope");
}

int tmoe_qk_norm_rope(tmoe_handle *h, void *stream, float *q, float *k, const float *q_norm, const float *k_norm,
                      const int32_t *pos, int64_t T, int32_t n_head, int32_t n_kv, int32_t head_dim, int32_t n_rot,
                      float freq_base, float eps) {
    if (!h) return TMOE_E_INVALID;
    if (T < 0 || n_head <= 0 || n_kv <= 0 || head_dim <= 0 || head_dim > 128 || head_dim % 32 || n_rot <= 0 ||
        n_rot > head_dim || n_rot % 2 || freq_base <= 0)
        return fail(h, TMOE_E_INVALID, "bad qk_norm_rope shape (head_dim a multiple of 32 up to 128)");
    if (T == 0) return TMOE_OK;
    if (!q || !k || !q_norm || !k_norm || !pos) return fail(h, TMOE_E_INVALID, "null tensor");
    DeviceGuard dg(h->cfg.device);
    tmoe::PdlScope pdl(!h->prof.on);  // overlap with the kernel before (programmatic launch)
    cudaError_t e = tmoe::launch_qk_norm_rope(q, k, q_norm, k_norm, pos, T, n_head, n_kv, head_dim, n_rot, freq_base,
                                              eps, (cudaStream_t)stream);
    return e == cudaSuccess ? TMOE_OK : cuda_fail(h, e, "qk_norm_rope");
}

int64_t tmoe_attn_decode_scratch_bytes(tmoe_handle *h, int32_t B, int32_t n_head, int32_t n_kv, int32_t head_dim,
                                       int32_t n_ctx) {
    if (!h || B < 0 || n_head <= 0 || n_kv <= 0 || head_dim <= 0 || n_ctx <= 0) return TMOE_E_INVALID;
    return (int64_t)(tmoe::attn_scratch_floats(B, n_head, head_dim, n_kv, n_ctx, h->sm_count) * 4);
}

int tmoe_attn_decode(tmoe_handle *h, void *stream, const float *q, const float *k, const float *v, void *k_cache,
                     void *v_cache, const int32_t *pos, int32_t B, int32_t n_head, int32_t n_kv, int32_t head_dim,
                     int32_t n_ctx, float scale, void *scratch, float *out) {
    if (!h) return TMOE_E_INVALID;
    if (B < 0 || n_kv <= 0 || n_head % n_kv || n_head / n_kv > 8 || (head_dim != 64 && head_dim != 128) || n_ctx <= 0)
        return fail(h, TMOE_E_UNSUPPORTED, "attention shape: %d heads over %d KV heads of %d (up to 8 heads per KV "
                                           "head, head_dim 64 or 128)", n_head, n_kv, head_dim);
    if (B == 0) return TMOE_OK;
    if (!q || !k || !v || !k_cache || !v_cache || !pos || !scratch || !out) return fail(h, TMOE_E_INVALID, "null tensor");
    if (((uintptr_t)k_cache | (uintptr_t)v_cache) & 15u) return fail(h, TMOE_E_INVALID, "caches must be 16-byte aligned");
    DeviceGuard dg(h->cfg.device);
    tmoe::PdlScope pdl(!h->prof.on);  // overlap with the kernel before (programmatic launch)
    cudaError_t e = tmoe::launch_attn_decode(q, k, v, (__half *)k_cache, (__half *)v_cache, pos, B, n_head, n_kv,
                                             head_dim, n_ctx, scale, (float *)scratch, out, h->sm_count, h->err,
                                             (cudaStream_t)stream);
    return e == cudaSuccess ? TMOE_OK : cuda_fail(h, e, "attention");
}

int tmoe_attn_prefill(tmoe_handle *h, void *stream, const float *q, const float *k, const float *v, void *k_cache,
                      void *v_cache, int32_t seq, int32_t n_seq, int32_t pos0, int32_t S, int32_t n_head, int32_t n_kv,
                      int32_t head_dim, int32_t n_ctx, float scale, float *out) {
    if (!h) return TMOE_E_INVALID;
    if (n_kv <= 0 || n_head <= 0 || n_head % n_kv || n_head > 65535 || (head_dim != 64 && head_dim != 128))
        return fail(h, TMOE_E_UNSUPPORTED, "attention shape: %d heads over %d KV heads of %d (head_dim 64 or 128)",
                    n_head, n_kv, head_dim);
    if (S < 0 || n_seq <= 0 || seq < 0 || seq >= n_seq || pos0 < 0 || n_ctx <= 0 || (int64_t)pos0 + S > n_ctx)
        return fail(h, TMOE_E_INVALID, "prefill of %d tokens at position %d of sequence %d: caches hold %d sequences "
                                       "of %d positions", S, pos0, seq, n_seq, n_ctx);
    if (S == 0) return TMOE_OK;
    if (!q || !k || !v || !k_cache || !v_cache || !out) return fail(h, TMOE_E_INVALID, "null tensor");
    if (((uintptr_t)k_cache | (uintptr_t)v_cache | (uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15u)
        return fail(h, TMOE_E_INVALID, "q, k, v, out and the caches must be 16-byte aligned");
    DeviceGuard dg(h->cfg.device);
    const cudaError_t e = tmoe::launch_attn_prefill(q, k, v, (__half *)k_cache, (__half *)v_cache, seq, pos0, S, n_head,
                                                    n_kv, head_dim, n_ctx, scale, out, (cudaStream_t)stream);
    return e == cudaSuccess ? TMOE_OK : cuda_fail(h, e, "prefill attention");
}

int tmoe_add(tmoe_handle *h, void *stream, const float *a, const float *b, float *out, int64_t n) {
    if (!h) return TMOE_E_INVALID;
    if (n < 0) return fail(h, TMOE_E_INVALID, "bad add size");
    if (n == 0) return TMOE_OK;
    if (!a || !b || !out) return fail(h, TMOE_E_INVALID, "null tensor");
    DeviceGuard dg(h->cfg.device);
    tmoe::PdlScope pdl(!h->prof.on);  // overlap with the kernel before (programmatic launch)
    cudaError_t e = tmoe::launch_add(a, b, out, n, (cudaStream_t)stream);
    return e == cudaSuccess ? TMOE_OK : cuda_fail(h, e, "add");
}

int tmoe_argmax(tmoe_handle *h, void *stream, const float *x, int64_t rows, int64_t n, int32_t *out) {
    if (!h) return TMOE_E_INVALID;
    if (rows < 0 || n <= 0 || n > 0x7fffffff) return fail(h, TMOE_E_INVALID, "bad argmax shape");
    if (rows == 0) return TMOE_OK;
    if (!x || !out) return fail(h, TMOE_E_INVALID, "null tensor");
    DeviceGuard dg(h->cfg.device);
    tmoe::PdlScope pdl(!h->prof.on);  // overlap with the kernel before (programmatic launch)
    cudaError_t e = tmoe::launch_argmax(x, rows, n, out, (cudaStream_t)stream);
    return e == cudaSuccess ? TMOE_OK : cuda_fail(h, e, "argmax");
}

int tmoe_profile_enable(tmoe_handle *h, int32_t enable) {
    if (!h) return TMOE_E_INVALID;
    DeviceGuard dg(h->cfg.device);
    auto &p = h->prof;
    if (enable && !p.ev[0]) {
        for (auto &ev : p.ev) {
            cudaError_t e = cudaEventCreate(&ev);
            if (e != cudaSuccess) return cuda_fail(h, e, "cudaEventCreate");
        }
    }
    p.on = enable != 0;
    p.n = 0;
    for (int i = 0; i < TMOE_N_PHASES; i++) p.ms[i] = 0.0, p.count[i] = 0;
    return TMOE_OK;
}

int tmoe_profile_collect(tmoe_handle *h, double *ms_out, int64_t *count_out) {
    if (!h) return TMOE_E_INVALID;
    DeviceGuard dg(h->cfg.device);
    auto &p = h->prof;
    for (int i = 0; i + 1 < p.n; i += 2) {
        cudaError_t e = cudaEventSynchronize(p.ev[i + 1]);
        if (e != cudaSuccess) return cuda_fail(h, e, "cudaEventSynchronize");
        float ms = 0.f;
        if ((e = cudaEventElapsedTime(&ms, p.ev[i], p.ev[i + 1])) != cudaSuccess)
            return cuda_fail(h, e, "cudaEventElapsedTime");
        p.ms[p.phase[i / 2]] += ms;
        p.count[p.phase[i / 2]] += 1;
    }
    p.n = 0;
    for (int i = 0; i < TMOE_N_PHASES; i++) {
        if (ms_out) ms_out[i] = p.ms[i];
        if (count_out) count_out[i] = p.count[i];
    }
    return TMOE_OK;
}

// ------------------------------------------------------------------ expert slots (a10)
int tmoe_slots_create(tmoe_handle *h, const tmoe_expert_tensors *slots, const tmoe_expert_tensors *store,
                      tmoe_slots **out) {
    if (!h || !out || !store) return h ? fail(h, TMOE_E_INVALID, "null argument") : TMOE_E_INVALID;
    *out = nullptr;
    const tmoe_config &c = h->cfg;
    int rc = check_tensors(h, slots);
    if (rc) return rc;
    const int E = c.n_expert, S = slots->n_slots;
    if (store->n_slots != E) return fail(h, TMOE_E_INVALID, "the store must hold all %d experts", E);
    if (!tmoe::slots_fit(E, S)) return fail(h, TMOE_E_UNSUPPORTED, "E=%d / %d slots not supported", E, S);
    if (store->gate_nb1 != slots->gate_nb1 || store->up_nb1 != slots->up_nb1 || store->down_nb1 != slots->down_nb1)
        return fail(h, TMOE_E_INVALID, "store and slot rows differ (nb1)");
    const size_t bytes[3] = {slots->gate_nb1 * (size_t)c.n_ff, slots->up_nb1 * (size_t)c.n_ff,
                             slots->down_nb1 * (size_t)c.n_embd};
    const void *src[3] = {store->gate, store->up, store->down};
    const size_t src_nb2[3] = {store->gate_nb2, store->up_nb2, store->down_nb2};
    const size_t dst_nb2[3] = {slots->gate_nb2, slots->up_nb2, slots->down_nb2};
    uint8_t *dst[3] = {(uint8_t *)slots->gate, (uint8_t *)slots->up, (uint8_t *)slots->down};
    DeviceGuard dg(c.device);
    tmoe_slots *sl = new tmoe_slots;
    sl->h = h;
    sl->slot_wts = *slots;
    for (int m = 0; m < 3; m++) {
        if ((bytes[m] & 15) || (src_nb2[m] & 15) || src_nb2[m] < bytes[m] || ((uintptr_t)src[m] & 15)) {
            delete sl;
            return fail(h, TMOE_E_INVALID, "store matrices must be 16-byte aligned multiples of 16 bytes");
        }
        void *dp = nullptr;  // the mapped device address of the pinned store
        if (cudaHostGetDevicePointer(&dp, const_cast<void *>(src[m]), 0) != cudaSuccess || !dp) {
            cudaGetLastError();
            delete sl;
            return fail(h, TMOE_E_INVALID, "the expert store must be pinned (device-mapped) host memory");
        }
        sl->copy.src[m] = (const uint8_t *)dp;
        sl->copy.src_nb2[m] = src_nb2[m];
        sl->copy.dst[m] = dst[m];
        sl->copy.dst_nb2[m] = dst_nb2[m];
        sl->copy.bytes[m] = bytes[m];
    }
    const int MC = (E + S - 1) / S;
    // one allocation: stamps and meta/counts first (8-byte), then the int arrays
    const size_t n8 = (size_t)S + 4 + E, n4 = (size_t)S + E + 1 + 1 + (size_t)MC * E + (size_t)MC * S * 2 + MC + E,
                 nbytes = n8 * 8 + n4 * 4 + E + 64;
    if (cudaMalloc(&sl->mem, nbytes) != cudaSuccess) {
        cudaGetLastError();
        delete sl;
        return fail(h, TMOE_E_NOMEM, "slot tables (%zu bytes)", nbytes);
    }
    uint8_t *p = (uint8_t *)sl->mem;
    tmoe::SlotsDev &d = sl->dev;
    d.n_expert = E, d.max_slots = S, d.max_chunks = MC;
    d.stamp = (unsigned long long *)p, p += (size_t)S * 8;
    d.meta = (unsigned long long *)p, p += 4 * 8;
    d.counts = (unsigned long long *)p, p += (size_t)E * 8;
    d.loads = (int2 *)p, p += (size_t)MC * S * 8;
    d.owner = (int32_t *)p, p += (size_t)S * 4;
    d.slot_of = (int32_t *)p, p += (size_t)E * 4;
    d.active = (int32_t *)p, p += 4;
    d.n_chunks = (int32_t *)p, p += 4;
    d.map = (int32_t *)p, p += (size_t)MC * E * 4;
    d.n_loads = (int32_t *)p, p += (size_t)MC * 4;
    sl->list = (int32_t *)p, p += (size_t)E * 4;
    d.pinned = p;
    // initial state: nothing resident, no pins, every slot active
    cudaError_t e = cudaMemset(sl->mem, 0, nbytes);
    if (e == cudaSuccess) e = cudaMemset(d.owner, 0xff, (size_t)S * 4);
    if (e == cudaSuccess) e = cudaMemset(d.slot_of, 0xff, (size_t)E * 4);
    if (e == cudaSuccess) e = cudaMemset(d.map, 0xff, (size_t)MC * E * 4);
    if (e == cudaSuccess) e = cudaMemcpy(d.active, &S, 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(sl->mem);
        delete sl;
        return cuda_fail(h, e, "slot tables init");
    }
    sl->active = S;
    if (MC > 1) {  // chunks after the first are paged in on a side stream while the first computes
        sl->ebytes = bytes[0] + bytes[1] + bytes[2];
        bool ok = cudaMalloc(&sl->staging, (size_t)S * sl->ebytes) == cudaSuccess &&
                  cudaStreamCreateWithFlags(&sl->side, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaEventCreateWithFlags(&sl->ev_plan, cudaEventDisableTiming) == cudaSuccess;
        sl->ev_staged.assign(MC, nullptr), sl->ev_moved.assign(MC, nullptr);
        for (int i = 0; ok && i < MC; i++)
            ok = cudaEventCreateWithFlags(&sl->ev_staged[i], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&sl->ev_moved[i], cudaEventDisableTiming) == cudaSuccess;
        if (!ok) {
            cudaGetLastError();
            tmoe_slots_destroy(sl);
            return fail(h, TMOE_E_NOMEM, "staging of the miss path (%zu bytes)", (size_t)S * sl->ebytes);
        }
    }
    *out = sl;
    return TMOE_OK;
}

void tmoe_slots_destroy(tmoe_slots *s) {
    if (!s) return;
    DeviceGuard dg(s->h->cfg.device);
    if (s->side) cudaStreamSynchronize(s->side);
    for (cudaEvent_t ev : s->ev_staged)
        if (ev) cudaEventDestroy(ev);
    for (cudaEvent_t ev : s->ev_moved)
        if (ev) cudaEventDestroy(ev);
    if (s->ev_plan) cudaEventDestroy(s->ev_plan);
    if (s->side) cudaStreamDestroy(s->side);
    if (s->staging) cudaFree(s->staging);
    cudaFree(s->mem);
    delete s;
}

int tmoe_slots_max_chunks(const tmoe_slots *s) { return s ? s->dev.max_chunks : TMOE_E_INVALID; }

int tmoe_slots_make_resident(tmoe_slots *s, void *stream, const int32_t *experts, int32_t n) {
    if (!s) return TMOE_E_INVALID;
    tmoe_handle *h = s->h;
    if (n < 0 || n > s->dev.max_slots || (n && !experts))
        return fail(h, TMOE_E_INVALID, "make_resident of %d experts (at most the %d slots)", n, s->dev.max_slots);
    if (n == 0) return TMOE_OK;
    DeviceGuard dg(h->cfg.device);
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e = cudaMemcpyAsync(s->list, experts, (size_t)n * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = tmoe::launch_slot_lookup_list(s->list, n, s->dev, h->err, st);
    if (e == cudaSuccess) e = tmoe::launch_slot_page(s->dev, 0, s->copy, h->sm_count, st);
    return e == cudaSuccess ? TMOE_OK : cuda_fail(h, e, "make_resident");
}

int tmoe_slots_set_hot_set(tmoe_slots *s, void *stream, const int32_t *hot, int32_t n) {
    if (!s) return TMOE_E_INVALID;
    tmoe_handle *h = s->h;
    const int E = s->dev.n_expert;
    if (n < 0 || (n && !hot)) return fail(h, TMOE_E_INVALID, "bad hot set");
    std::vector<uint8_t> pinned(E, 0);
    int count = 0;
    for (int i = 0; i < n; i++) {
        const int e = hot[i];
        if (count < s->active && e >= 0 && e < E && !pinned[e]) pinned[e] = 1, count++;
    }
    DeviceGuard dg(h->cfg.device);
    cudaStream_t st = (cudaStream_t)stream;
    std::vector<int32_t> slot_of(E);
    cudaError_t e = cudaMemcpyAsync(s->dev.pinned, pinned.data(), E, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(slot_of.data(), s->dev.slot_of, (size_t)E * 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(h, e, "set_hot_set");
    std::vector<int32_t> missing;
    for (int x = 0; x < E; x++)
        if (pinned[x] && slot_of[x] < 0) missing.push_back(x);
    const int rc = tmoe_slots_make_resident(s, stream, missing.data(), (int32_t)missing.size());
    if (rc) return rc;
    return cudaStreamSynchronize(st) == cudaSuccess ? TMOE_OK : cuda_fail(h, cudaGetLastError(), "set_hot_set");
}

int tmoe_slots_state(tmoe_slots *s, void *stream, int32_t *owner, int64_t *stats, int64_t *counts) {
    if (!s) return TMOE_E_INVALID;
    tmoe_handle *h = s->h;
    DeviceGuard dg(h->cfg.device);
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e = cudaStreamSynchronize(st);
    unsigned long long meta[4];
    if (e == cudaSuccess && owner)
        e = cudaMemcpy(owner, s->dev.owner, (size_t)s->dev.max_slots * 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(meta, s->dev.meta, sizeof meta, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && counts)
        e = cudaMemcpy(counts, s->dev.counts, (size_t)s->dev.n_expert * 8, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(h, e, "slot state");
    if (stats)
        for (int i = 0; i < 3; i++) stats[i] = (int64_t)meta[i + 1];
    return TMOE_OK;
}

int tmoe_slots_last_plan(tmoe_slots *s, void *stream, int32_t *n_chunks, int32_t *map, int32_t *loads,
                         int32_t *n_loads) {
    if (!s) return TMOE_E_INVALID;
    tmoe_handle *h = s->h;
    const tmoe::SlotsDev &d = s->dev;
    DeviceGuard dg(h->cfg.device);
    cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e == cudaSuccess && n_chunks) e = cudaMemcpy(n_chunks, d.n_chunks, 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && map)
        e = cudaMemcpy(map, d.map, (size_t)d.max_chunks * d.n_expert * 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && loads)
        e = cudaMemcpy(loads, d.loads, (size_t)d.max_chunks * d.max_slots * 8, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && n_loads) e = cudaMemcpy(n_loads, d.n_loads, (size_t)d.max_chunks * 4, cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? TMOE_OK : cuda_fail(h, e, "last plan");
}

int tmoe_streamed_layer(tmoe_handle *h, void *stream, tmoe_slots *s, const float *x, int64_t T, int32_t use_norm,
                        const float *norm_w, const float *router_w, const float *logits, float *out,
                        int32_t *ids_out, float *w_out) {
    if (!h || !s || s->h != h) return h ? fail(h, TMOE_E_INVALID, "slot cache of another handle") : TMOE_E_INVALID;
    const tmoe_config &c = h->cfg;
    if (!x || !out) return fail(h, TMOE_E_INVALID, "null tensor");
    if (!aligned16(out)) return fail(h, TMOE_E_INVALID, "out must be 16-byte aligned");
    int32_t *ids = ids_out ? ids_out : h->ids;
    float *w = w_out ? w_out : h->w;
    int rc = tmoe_route(h, stream, x, T, use_norm, norm_w, router_w, logits, ids, w, use_norm ? h->xn : nullptr,
                        nullptr);
    if (rc || T == 0) return rc;
    DeviceGuard dg(c.device);
    cudaStream_t st = (cudaStream_t)stream;
    const float *xn = use_norm ? h->xn : x;
    const int k = c.n_expert_used, E = c.n_expert;
    const int64_t P = T * k;
    cudaError_t e;
    {
        PhaseMark pm(h, st, TMOE_PHASE_SLOT_PLAN);
        e = tmoe::launch_slot_plan(ids, (int)P, s->dev, h->err, st);
    }
    if (e != cudaSuccess) return cuda_fail(h, e, "slot plan");
    // Chunk 0's misses are paged straight into their slots.  Chunk c >= 1 is paged from the host
    // store into the staging area on the side stream while chunk c - 1 computes, then moved into
    // its slots right before it computes (its slots may be chunk c - 1's).  The events are enqueued
    // in dependency order, so the schedule holds under stream capture too.  Chunks >= 1 reuse
    // chunk 0's Q8_K rows of xn.
    const int MC = s->dev.max_chunks;
    const bool overlap = s->side != nullptr;
    if (overlap) {
        if ((e = cudaEventRecord(s->ev_plan, st)) == cudaSuccess &&
            (e = cudaStreamWaitEvent(s->side, s->ev_plan, 0)) == cudaSuccess &&
            (e = tmoe::launch_slot_stage(s->dev, 1, s->copy, s->staging, s->ebytes, s->side)) == cudaSuccess)
            e = cudaEventRecord(s->ev_staged[1], s->side);
        if (e != cudaSuccess) return cuda_fail(h, e, "staging");
    }
    for (int ch = 0; ch < MC; ch++) {
        if (ch == 0 || !overlap) {
            PhaseMark pm(h, st, TMOE_PHASE_SLOT_PAGE);
            e = tmoe::launch_slot_page(s->dev, ch, s->copy, h->sm_count, st);
        } else {
            if ((e = cudaStreamWaitEvent(st, s->ev_staged[ch], 0)) == cudaSuccess) {
                PhaseMark pm(h, st, TMOE_PHASE_SLOT_PAGE);
                e = tmoe::launch_slot_unstage(s->dev, ch, s->copy, s->staging, s->ebytes, h->sm_count, st);
            }
            if (e == cudaSuccess && ch + 1 < MC) {  // the staging is free again: the next chunk's pages
                if ((e = cudaEventRecord(s->ev_moved[ch], st)) == cudaSuccess &&
                    (e = cudaStreamWaitEvent(s->side, s->ev_moved[ch], 0)) == cudaSuccess &&
                    (e = tmoe::launch_slot_stage(s->dev, ch + 1, s->copy, s->staging, s->ebytes, s->side)) ==
                        cudaSuccess)
                    e = cudaEventRecord(s->ev_staged[ch + 1], s->side);
            }
        }
        if (e != cudaSuccess) return cuda_fail(h, e, "slot paging");
        {
            PhaseMark pm(h, st, TMOE_PHASE_MAP_IDS);
            e = tmoe::launch_map_ids(ids, P, s->dev.map + (size_t)ch * E, E, h->mapped, st);
        }
        if (e != cudaSuccess) return cuda_fail(h, e, "chunk map");
        rc = run_experts(h, st, xn, T, h->mapped, w, &s->slot_wts, out, false, ch > 0, false, ch > 0);
        if (rc) return rc;
    }
    {
        PhaseMark pm(h, st, TMOE_PHASE_COMBINE);
        e = tmoe::launch_combine(h->dout, ids, w, T, k, c.n_embd, E, out, st);
    }
    return e == cudaSuccess ? TMOE_OK : cuda_fail(h, e, "combine");
}

}  // extern "C"
