// Token-to-expert dispatch: per-expert counts, offsets and the stable permutation of pairs
// (token-major, choice-minor within each expert: qwen3moe.rs:2126-2150 group_pairs, the order
// ggml's mul_mat_id row mapping visits), the EP id map (qwen3moe_shard.rs:1043-1050), the fused
// top-k + map + dispatch kernel of the decode regime, and the weighted combine in choice order
// (qwen3moe.rs:2912-2923).
#include "common.cuh"
#include "kernels.cuh"
#include "q8k.cuh"
#include "route.cuh"

namespace tmoe {

static thread_local bool g_pdl = false;
PdlScope::PdlScope(bool on) : prev(g_pdl) { g_pdl = on; }
PdlScope::~PdlScope() { g_pdl = prev; }
bool pdl_on() { return g_pdl; }

constexpr int SORT_WARPS = 32;

// The dispatch of n_pairs ids (ids may live in shared memory) by one CTA of 1024 threads.  Warp w
// owns the contiguous pair segment [w*seg, (w+1)*seg):
//   1. per-warp histograms in shared memory;
//   2. per expert, an exclusive scan over the warps plus the expert offset gives each warp its
//      first slot for that expert;
//   3. each warp walks its segment in order, 32 pairs at a time; __match_any_sync ranks the lanes
//      of equal expert, so the scatter is stable.
// ids outside [0, n_slots) are not dispatched; ids >= n_slots also latch TMOE_DEV_ERR_BADID.
// Also writes the increasing list of experts with pairs (n_active[0] of them) with their pair
// ranges: active[i] = {e, offsets[e], offsets[e + 1], 0}.
// NW: the warps of the CTA.  sh: NW * n_slots + n_slots + 65 ints of shared memory; n_slots <= 1024.
template <int NW>
__device__ void sort_pairs_cta(const int32_t *ids, int n_pairs, int n_slots, int32_t *__restrict__ counts,
                               int32_t *__restrict__ offsets, int32_t *__restrict__ perm,
                               int4 *__restrict__ active, int32_t *__restrict__ n_active, int *counters,
                               int n_counters, int *err, int32_t *sh) {
    int32_t *hist = sh;                         // [NW][n_slots]
    int32_t *offs = sh + NW * n_slots;  // [n_slots + 1], then the chunk totals
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (counters && (int)threadIdx.x < n_counters) counters[threadIdx.x] = 0;  // work counters of the GEMVs
    for (int i = threadIdx.x; i < NW * n_slots; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    int seg = (n_pairs + NW - 1) / NW;
    seg = (seg + 31) & ~31;
    const int p0 = warp * seg, p1 = min(n_pairs, p0 + seg);
    bool bad = false;
    for (int p = p0 + lane; p < p1; p += 32) {
        const int e = ids[p];
        if (e >= n_slots) bad = true;
        if (e >= 0 && e < n_slots) atomicAdd(&hist[warp * n_slots + e], 1);
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) latch_error(err, TMOE_DEV_ERR_BADID);
    __syncthreads();
    for (int e = threadIdx.x; e < n_slots; e += blockDim.x) {
        int run = 0;
        for (int w = 0; w < NW; w++) {
            const int c = hist[w * n_slots + e];
            hist[w * n_slots + e] = run;
            run += c;
        }
        counts[e] = run;
        offs[e] = run;
    }
    __syncthreads();
    // Exclusive scan of the counts and the active list, 32 experts per warp step: each chunk's
    // inclusive scan and its pair and active totals first, then every chunk adds the totals of the
    // chunks before it (n_slots <= 32 * 32).
    int32_t *ctot = offs + n_slots + 1;  // [32] pair totals, then [32] active-expert totals
    const int nch = (n_slots + 31) >> 5;
    const unsigned lt = (1u << lane) - 1u;
    for (int c = warp; c < nch; c += NW) {
        const int e = 32 * c + lane;
        const int v = e < n_slots ? offs[e] : 0;
        int inc = v;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, inc, off);
            if (lane >= off) inc += o;
        }
        const unsigned m = __ballot_sync(0xffffffffu, v > 0);
        if (e < n_slots) offs[e] = inc;
        if (lane == 31) {
            ctot[c] = inc;
            ctot[32 + c] = __popc(m);
        }
    }
    __syncthreads();
    for (int c = warp; c < nch; c += NW) {
        int base = 0, abase = 0;
        for (int j = 0; j < c; j++) {
            base += ctot[j];
            abase += ctot[32 + j];
        }
        const int e = 32 * c + lane;
        const int inc = e < n_slots ? offs[e] : 0;
        const int prev = __shfl_up_sync(0xffffffffu, inc, 1);
        const int v = e < n_slots ? inc - (lane ? prev : 0) : 0;
        const unsigned m = __ballot_sync(0xffffffffu, v > 0);
        const int start = base + inc - v;
        if (e < n_slots) {
            offs[e] = start;
            offsets[e] = start;
            if (v > 0) active[abase + __popc(m & lt)] = make_int4(e, start, start + v, 0);
        }
        if (c == nch - 1 && lane == 0) {
            offs[n_slots] = base + ctot[c];
            offsets[n_slots] = base + ctot[c];
            n_active[0] = abase + ctot[32 + c];
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < n_slots; e += blockDim.x)
        for (int w = 0; w < NW; w++) hist[w * n_slots + e] += offs[e];
    __syncthreads();
    for (int base = p0; base < p1; base += 32) {
        const int p = base + lane;
        const int e = p < p1 ? ids[p] : -1;
        const bool ok = e >= 0 && e < n_slots;
        const unsigned peers = __match_any_sync(0xffffffffu, ok ? e : -1);
        if (ok) perm[hist[warp * n_slots + e] + __popc(peers & lt)] = p;
        __syncwarp();
        if (ok && (peers & lt) == 0) hist[warp * n_slots + e] += __popc(peers);
        __syncwarp();
    }
}

// The same dispatch for a few pairs (n_pairs and n_slots at most NT, the CTA's threads), by
// ranking instead of histograms: thread e counts expert e's pairs and the valid pairs of the
// experts below it (its offset), and thread p puts pair p after them and after the earlier pairs
// of its own expert -- the stable order of sort_pairs_cta.  sids: the ids in shared memory.
// sh: n_slots + NT / 32 ints.
constexpr int SMALL_SORT_PAIRS = 64;  // the batches of one token tile at top-8

template <int NT>
__device__ void sort_pairs_small(const int32_t *sids, int n_pairs, int n_slots, int32_t *__restrict__ counts,
                                 int32_t *__restrict__ offsets, int32_t *__restrict__ perm,
                                 int4 *__restrict__ active, int32_t *__restrict__ n_active, int *counters,
                                 int n_counters, int *err, int32_t *sh) {
    int32_t *offs = sh;            // [n_slots]
    int32_t *wtot = sh + n_slots;  // [NT / 32] experts with pairs, per warp
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (counters && tid < n_counters) counters[tid] = 0;  // work counters of the GEMVs
    const int e = tid;
    int c = 0, below = 0;
    if (e < n_slots) {
        for (int q = 0; q < n_pairs; q++) {
            const int f = sids[q];
            c += f == e;
            below += f >= 0 && f < e;
        }
        counts[e] = c;
        offsets[e] = below;
        offs[e] = below;
        if (e == n_slots - 1) offsets[n_slots] = below + c;
    }
    const unsigned m = __ballot_sync(0xffffffffu, e < n_slots && c > 0);
    if (lane == 0) wtot[warp] = __popc(m);
    const bool bad = tid < n_pairs && sids[tid] >= n_slots;
    if (__any_sync(0xffffffffu, bad) && lane == 0) latch_error(err, TMOE_DEV_ERR_BADID);
    __syncthreads();
    int base = 0, total = 0;
    for (int w = 0; w < NT / 32; w++) {
        base += w < warp ? wtot[w] : 0;
        total += wtot[w];
    }
    if (e < n_slots && c > 0) active[base + __popc(m & ((1u << lane) - 1u))] = make_int4(e, below, below + c, 0);
    if (tid == 0) n_active[0] = total;
    if (tid < n_pairs) {
        const int f = sids[tid];
        if (f >= 0 && f < n_slots) {
            int r = 0;
            for (int q = 0; q < tid; q++) r += sids[q] == f;
            perm[offs[f] + r] = tid;
        }
    }
}

__global__ void __launch_bounds__(1024) sort_pairs_kernel(const int32_t *__restrict__ ids, int n_pairs, int n_slots,
                                                          int32_t *__restrict__ counts, int32_t *__restrict__ offsets,
                                                          int32_t *__restrict__ perm, int4 *__restrict__ active,
                                                          int32_t *__restrict__ n_active, int *counters, int n_counters,
                                                          int *err) {
    extern __shared__ int32_t sh[];
    if (n_pairs <= SMALL_SORT_PAIRS && n_slots <= SORT_WARPS * 32) {
        int32_t *sid = sh;  // [n_pairs], then the ranking's scratch
        if ((int)threadIdx.x < n_pairs) sid[threadIdx.x] = ids[threadIdx.x];
        __syncthreads();
        sort_pairs_small<SORT_WARPS * 32>(sid, n_pairs, n_slots, counts, offsets, perm, active, n_active, counters,
                                          n_counters, err, sh + SMALL_SORT_PAIRS);
        return;
    }
    sort_pairs_cta<SORT_WARPS>(ids, n_pairs, n_slots, counts, offsets, perm, active, n_active, counters, n_counters,
                               err, sh);
}

// The same dispatch for many pairs, over CTAs of SORT_CHUNK consecutive pairs: each chunk counts its
// pairs per expert; one CTA turns the counts into offsets (and the active list) and each chunk's
// first slot per expert; each chunk then scatters its pairs in order, ranked per warp as in
// sort_pairs_cta.  Pairs of an expert end up in increasing pair order, exactly as one CTA sorts
// them.  scratch: n_chunks * n_slots ints.
constexpr int SORT_CHUNK = 2048;  // 64 pairs per warp

__global__ void __launch_bounds__(1024) sort_hist_kernel(const int32_t *__restrict__ ids, int n_pairs, int n_slots,
                                                         int32_t *__restrict__ chunk, int *err) {
    extern __shared__ int32_t hc[];  // [n_slots]
    for (int e = threadIdx.x; e < n_slots; e += blockDim.x) hc[e] = 0;
    __syncthreads();
    const int p0 = blockIdx.x * SORT_CHUNK, p1 = min(n_pairs, p0 + SORT_CHUNK);
    bool bad = false;
    for (int p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
        const int e = ids[p];
        if (e >= n_slots) bad = true;
        if (e >= 0 && e < n_slots) atomicAdd(&hc[e], 1);
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) latch_error(err, TMOE_DEV_ERR_BADID);
    __syncthreads();
    for (int e = threadIdx.x; e < n_slots; e += blockDim.x) chunk[(int64_t)blockIdx.x * n_slots + e] = hc[e];
}

__global__ void __launch_bounds__(1024) sort_scan_kernel(int n_chunks, int n_slots, int32_t *__restrict__ chunk,
                                                         int32_t *__restrict__ counts, int32_t *__restrict__ offsets,
                                                         int4 *__restrict__ active, int32_t *__restrict__ n_active,
                                                         int *counters, int n_counters) {
    extern __shared__ int32_t offs[];  // [n_slots + 1]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (counters && (int)threadIdx.x < n_counters) counters[threadIdx.x] = 0;  // work counters of the GEMVs
    for (int e = threadIdx.x; e < n_slots; e += blockDim.x) {  // each chunk's first slot within its expert
        int run = 0;
        for (int c = 0; c < n_chunks; c++) {
            const int v = chunk[(int64_t)c * n_slots + e];
            chunk[(int64_t)c * n_slots + e] = run;
            run += v;
        }
        counts[e] = run;
        offs[e] = run;
    }
    __syncthreads();
    if (warp == 0) {  // exclusive scan of the counts, 32 experts per step
        int carry = 0;
        for (int base = 0; base < n_slots; base += 32) {
            const int e = base + lane;
            const int c = e < n_slots ? offs[e] : 0;
            int inc = c;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int o = __shfl_up_sync(0xffffffffu, inc, off);
                if (lane >= off) inc += o;
            }
            if (e < n_slots) offs[e] = carry + inc - c;
            carry += __shfl_sync(0xffffffffu, inc, 31);
        }
        if (lane == 0) offs[n_slots] = carry;
    }
    __syncthreads();
    for (int e = threadIdx.x; e <= n_slots; e += blockDim.x) offsets[e] = offs[e];
    if (warp == 0) {
        int na = 0;
        for (int base = 0; base < n_slots; base += 32) {
            const int e = base + lane;
            const bool has = e < n_slots && (offs[e + 1] - offs[e]) > 0;
            const unsigned m = __ballot_sync(0xffffffffu, has);
            if (has) active[na + __popc(m & ((1u << lane) - 1u))] = make_int4(e, offs[e], offs[e + 1], 0);
            na += __popc(m);
        }
        if (lane == 0) n_active[0] = na;
    }
    for (int e = threadIdx.x; e < n_slots; e += blockDim.x)
        for (int c = 0; c < n_chunks; c++) chunk[(int64_t)c * n_slots + e] += offs[e];
}

__global__ void __launch_bounds__(1024) sort_scatter_kernel(const int32_t *__restrict__ ids, int n_pairs, int n_slots,
                                                            const int32_t *__restrict__ chunk,
                                                            int32_t *__restrict__ perm) {
    extern __shared__ int32_t hw[];  // [32 warps][n_slots]
    constexpr int NW = 32, SEG = SORT_CHUNK / NW;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < NW * n_slots; i += blockDim.x) hw[i] = 0;
    __syncthreads();
    const int c0 = blockIdx.x * SORT_CHUNK;
    const int p0 = c0 + warp * SEG, p1 = min(n_pairs, p0 + SEG);
    for (int p = p0 + lane; p < p1; p += 32) {
        const int e = ids[p];
        if (e >= 0 && e < n_slots) atomicAdd(&hw[warp * n_slots + e], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < n_slots; e += blockDim.x) {  // warp w's first slot: the chunk's + earlier warps'
        int run = chunk[(int64_t)blockIdx.x * n_slots + e];
        for (int w = 0; w < NW; w++) {
            const int v = hw[w * n_slots + e];
            hw[w * n_slots + e] = run;
            run += v;
        }
    }
    __syncthreads();
    const unsigned lt = (1u << lane) - 1u;
    for (int base = p0; base < p1; base += 32) {
        const int p = base + lane;
        const int e = p < p1 ? ids[p] : -1;
        const bool ok = e >= 0 && e < n_slots;
        const unsigned peers = __match_any_sync(0xffffffffu, ok ? e : -1);
        if (ok) perm[hw[warp * n_slots + e] + __popc(peers & lt)] = p;
        __syncwarp();
        if (ok && (peers & lt) == 0) hw[warp * n_slots + e] += __popc(peers);
        __syncwarp();
    }
}

size_t sort_scratch_ints(int64_t n_pairs, int n_slots) {
    return (size_t)((n_pairs + SORT_CHUNK - 1) / SORT_CHUNK) * (size_t)n_slots;
}

// Decode regime (T*k <= ROUTE_FUSED_MAX_PAIRS): softmax/top-k of every token, the optional EP
// map, and the dispatch of the (mapped) ids, in one CTA of 1024 threads.  ids_out / w_out get the
// router's choices; mapped gets the ids the experts see (= ids_out without a table).
template <int MAXPER>
__global__ void __launch_bounds__(1024) route_dispatch_kernel(const float *__restrict__ logits, int T, int E, int k,
                                                              const int32_t *__restrict__ table, int n_table,
                                                              int32_t *__restrict__ ids_out, float *__restrict__ w_out,
                                                              int32_t *__restrict__ mapped, int n_slots,
                                                              int32_t *__restrict__ counts, int32_t *__restrict__ offsets,
                                                              int32_t *__restrict__ perm, int4 *__restrict__ active,
                                                              int32_t *__restrict__ n_active, int *counters,
                                                              int n_counters, int *err) {
    extern __shared__ int32_t sh[];
    int32_t *sid = sh;  // [T*k] mapped ids
    int32_t *sort_sh = sh + ((T * k + 3) & ~3);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int t = warp; t < T; t += 32) {
        int id;
        float wt;
        topk_token<MAXPER>(logits + (int64_t)t * E, E, k, nullptr, id, wt);
        if (lane < k) {
            const int m = table ? ((id >= 0 && id < n_table) ? table[id] : -1) : id;
            ids_out[t * k + lane] = id;
            w_out[t * k + lane] = wt;
            mapped[t * k + lane] = m;
            sid[t * k + lane] = m;
        }
    }
    __syncthreads();
    sort_pairs_cta<SORT_WARPS>(sid, T * k, n_slots, counts, offsets, perm, active, n_active, counters, n_counters,
                               err, sort_sh);
}

// The decode regime's whole routing in one launch: router logits, Q8_K of x, softmax/top-k, the
// optional EP map and the dispatch.  CTA (i, j) of a (ceil(E/8), ceil(T/TT)) grid:
//  1. stages TT token rows of x and 8 expert rows of the router matrix into shared memory with
//     bulk copies.  Warps 0-3 compute those logits in the canonical dot order (the same arithmetic
//     as router_logits_kernel: bit-identical logits), warp w the 4 experts 4 (w & 1) .. and the
//     token half w >> 1, each thread holding 4 x TT/2 sums, so that a staged word feeds several
//     products; warps 4-7 write the Q8_K rows of x, spread over the tile's CTAs;
//  2. the last CTA of token tile j (a counter per tile, taken with an acquire-release atomic; no
//     CTA waits on another) reads the tile's logits back and runs top-k, one warp per token;
//  3. with one token tile that CTA goes on to dispatch the pairs, whose ids it holds; with several,
//     the last tile to finish (a second counter) reads all the ids back and dispatches them.
// done: gridDim.y + 1 ints, zero before the first launch (the kernel leaves them zero).
constexpr int FR_WARPS = 8;      // warps per CTA, and experts per CTA
constexpr int FR_DOT_WARPS = 4;  // the warps that compute logits (2 expert halves x 2 token halves)

__device__ __forceinline__ int atomic_add_acq_rel(int *p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

template <int TT, int MAXPER>
__global__ void __launch_bounds__(FR_WARPS * 32) route_fused_kernel(
    const float *__restrict__ x, const float *__restrict__ rw, int T, int H, int E, int k, Q8Rows q8,
    float *__restrict__ logits, const int32_t *__restrict__ table, int n_table, int32_t *__restrict__ ids_out,
    float *__restrict__ w_out, int32_t *__restrict__ mapped, int n_slots, int32_t *__restrict__ counts,
    int32_t *__restrict__ offsets, int32_t *__restrict__ perm, int4 *__restrict__ active,
    int32_t *__restrict__ n_active, int *counters, int n_counters, int *done, int *err) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ uint64_t bar_s;
    __shared__ int flag_s;
    uint64_t *bar = &bar_s;
    int *flag = &flag_s;
    float *xs = reinterpret_cast<float *>(sm);  // [TT][H]
    float *ws = xs + TT * H;                    // [FR_WARPS][H]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e0 = blockIdx.x * FR_WARPS, t0 = blockIdx.y * TT;
    const int nt = min(TT, T - t0), ne = min(FR_WARPS, E - e0);
    const int H4 = H / 4;
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    const uint32_t row = (uint32_t)H * 4u;
    if (threadIdx.x == 0) {  // the router rows are not written by the kernel before: staged before the wait
        mbar_arrive_expect_tx(bar, (uint32_t)(nt + ne) * row);
        for (int j = 0; j < ne; j++) bulk_g2s(ws + j * H, rw + (int64_t)(e0 + j) * H, row, bar);
    }
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0)
        for (int j = 0; j < nt; j++) bulk_g2s(xs + j * H, x + (int64_t)(t0 + j) * H, row, bar);
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(bar, 0))) {
        // nothing else may run on this tile: the copies may still be in flight
        if (lane == 0) latch_error(err, TMOE_DEV_ERR_TIMEOUT);
        if (threadIdx.x == 0) mbar_wait_bounded(bar, 0);
    }
    const float4 *xs4 = reinterpret_cast<const float4 *>(xs);
    if (warp >= FR_DOT_WARPS) {
        if (q8.qs) {  // Q8_K of the staged rows: one warp per (token, 256-block)
            constexpr int QW = FR_WARPS - FR_DOT_WARPS;
            const int nb = H / TMOE_QK;
            for (int u = blockIdx.x * QW + warp - FR_DOT_WARPS; u < nt * nb; u += gridDim.x * QW) {
                const int j = u / nb, b = u % nb;
                const float4 a0 = xs4[j * H4 + b * 64 + 2 * lane], a1 = xs4[j * H4 + b * 64 + 2 * lane + 1];
                const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                uint2 q;
                float d;
                int s16;
                q8k_block_warp(v, q, d, s16);
                q8k_store_warp(q8, t0 + j, H, b, q, d, s16);
            }
        }
    } else {
        // canonical dot: lane l takes elements 128m + 4l .. 4l+3 in m order, then a butterfly
        constexpr int TK = TT >= 2 ? TT / 2 : 1;
        const int eg = 4 * (warp & 1), tg = TK * (warp >> 1);
        if (tg < nt) {
            const float4 *w4 = reinterpret_cast<const float4 *>(ws + eg * H);
            float acc[4][TK];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < TK; j++) acc[i][j] = 0.0f;
            for (int m = 0; m < H / 128; m++) {
                float4 w[4];
#pragma unroll
                for (int i = 0; i < 4; i++) w[i] = w4[i * H4 + 32 * m + lane];
#pragma unroll
                for (int j = 0; j < TK; j++) {
                    const float4 xv = xs4[(tg + j) * H4 + 32 * m + lane];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        acc[i][j] = __fmaf_rn(w[i].x, xv.x, acc[i][j]);
                        acc[i][j] = __fmaf_rn(w[i].y, xv.y, acc[i][j]);
                        acc[i][j] = __fmaf_rn(w[i].z, xv.z, acc[i][j]);
                        acc[i][j] = __fmaf_rn(w[i].w, xv.w, acc[i][j]);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < TK; j++) {
                    const float sv = butterfly_f32(acc[i][j]);
                    if (lane == 0 && eg + i < ne && tg + j < nt) logits[(int64_t)(t0 + tg + j) * E + e0 + eg + i] = sv;
                }
        }
    }
    // 2. the last CTA of this token tile: top-k of its tokens
    __syncthreads();
    if (threadIdx.x == 0) *flag = atomic_add_acq_rel(&done[blockIdx.y], 1) == (int)gridDim.x - 1;
    __syncthreads();
    if (!*flag) return;
    float *lgs = xs;  // [TT][E], the staged rows are no longer needed
    const int n_pairs = T * k;
    int32_t *sid = reinterpret_cast<int32_t *>(lgs + TT * E);  // [n_pairs], then the sort's scratch
    for (int i = threadIdx.x; i < nt * E; i += blockDim.x) lgs[i] = __ldcg(logits + (int64_t)t0 * E + i);
    __syncthreads();
    if (warp < nt) {
        const int t = t0 + warp;
        int id;
        float wt;
        topk_token<MAXPER>(lgs + warp * E, E, k, nullptr, id, wt);
        if (lane < k) {
            const int m = table ? ((id >= 0 && id < n_table) ? table[id] : -1) : id;
            ids_out[t * k + lane] = id;
            w_out[t * k + lane] = wt;
            mapped[t * k + lane] = m;
            sid[t * k + lane] = m;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) done[blockIdx.y] = 0;  // every CTA of this tile has counted
    // 3. the dispatch of all pairs: here with one token tile, else by the last tile to finish
    if (gridDim.y > 1) {
        if (threadIdx.x == 0) *flag = atomic_add_acq_rel(&done[gridDim.y], 1) == (int)gridDim.y - 1;
        __syncthreads();
        if (!*flag) return;
        for (int i = threadIdx.x; i < n_pairs; i += blockDim.x) sid[i] = __ldcg(mapped + i);
        __syncthreads();
    }
    if (n_pairs <= SMALL_SORT_PAIRS && n_slots <= FR_WARPS * 32)
        sort_pairs_small<FR_WARPS * 32>(sid, n_pairs, n_slots, counts, offsets, perm, active, n_active, counters,
                                        n_counters, err, sid + ((n_pairs + 3) & ~3));
    else
        sort_pairs_cta<FR_WARPS>(sid, n_pairs, n_slots, counts, offsets, perm, active, n_active, counters,
                                 n_counters, err, sid + ((n_pairs + 3) & ~3));
    if (threadIdx.x == 0 && gridDim.y > 1) done[gridDim.y] = 0;
}

__global__ void map_ids_kernel(const int32_t *__restrict__ ids, int64_t n, const int32_t *__restrict__ table,
                               int64_t n_table, int32_t *__restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int e = ids[i];
    out[i] = (e >= 0 && e < n_table) ? table[e] : -1;
}

// Zero the output rows of pairs with no expert (id < 0 or >= n_slots).
__global__ void zero_invalid_rows_kernel(const int32_t *__restrict__ ids, int64_t n_pairs, int n_slots, int N,
                                         float *__restrict__ out) {
    const int64_t p = blockIdx.x;
    if (p >= n_pairs) return;
    const int e = ids[p];
    if (e >= 0 && e < n_slots) return;
    float *o = out + p * N;
    for (int i = threadIdx.x; i < N; i += blockDim.x) o[i] = 0.0f;
}

// out[t][h] = ((m_0 + m_1) + m_2) + ...  with m_j = d[t*k+j][h] * w[t][j], d = 0 for no expert
// (ctx.mul(experts, w) then the fold of sum_experts).  One thread per 4 outputs; all of the token's
// ids, weights and rows are loaded before the fold.
template <int KMAX>
__global__ void combine_kernel(const float *__restrict__ dout, const int32_t *__restrict__ ids,
                               const float *__restrict__ w, int64_t T, int k, int H, int n_slots,
                               float *__restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i >= T * H) return;
    const int64_t t = i / H;
    const int h = (int)(i % H);
    int e[KMAX];
    float wj[KMAX];
    float4 d[KMAX];
#pragma unroll
    for (int j = 0; j < KMAX; j++) {
        if (j < k) {
            e[j] = __ldg(ids + t * k + j);
            wj[j] = __ldg(w + t * k + j);
        }
    }
#pragma unroll
    for (int j = 0; j < KMAX; j++) {
        d[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j < k && e[j] >= 0 && e[j] < n_slots) d[j] = __ldg(reinterpret_cast<const float4 *>(dout + (t * k + j) * H + h));
    }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < KMAX; j++) {
        if (j >= k) break;
        const float4 m = make_float4(__fmul_rn(d[j].x, wj[j]), __fmul_rn(d[j].y, wj[j]), __fmul_rn(d[j].z, wj[j]),
                                     __fmul_rn(d[j].w, wj[j]));
        acc = j == 0 ? m
                     : make_float4(__fadd_rn(acc.x, m.x), __fadd_rn(acc.y, m.y), __fadd_rn(acc.z, m.z),
                                   __fadd_rn(acc.w, m.w));
    }
    *reinterpret_cast<float4 *>(out + i) = acc;
}

// ------------------------------------------------------------------ launchers
size_t sort_pairs_smem(int n_slots) { return sizeof(int32_t) * ((size_t)SORT_WARPS * n_slots + n_slots + 65); }

template <typename KernT>
static cudaError_t set_smem_once(KernT kern, size_t smem, int *cache) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (smem > 48 * 1024 && (int)smem > cache[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        cache[dev] = (int)smem;
    }
    return cudaSuccess;
}

cudaError_t launch_sort_pairs(const int32_t *ids, int n_pairs, int n_slots, int32_t *counts, int32_t *offsets,
                              int32_t *perm, int4 *active, int32_t *n_active, int *counters, int n_counters,
                              int *err, cudaStream_t st, int32_t *scratch, size_t scratch_ints) {
    const int n_chunks = (n_pairs + SORT_CHUNK - 1) / SORT_CHUNK;
    if (scratch && n_chunks >= 4 && scratch_ints >= sort_scratch_ints(n_pairs, n_slots)) {
        static int cache_s[64] = {};
        const size_t smem_s = (size_t)32 * n_slots * 4;
        cudaError_t e = set_smem_once(sort_scatter_kernel, smem_s, cache_s);
        if (e != cudaSuccess) return e;
        sort_hist_kernel<<<n_chunks, 1024, (size_t)n_slots * 4, st>>>(ids, n_pairs, n_slots, scratch, err);
        sort_scan_kernel<<<1, 1024, (size_t)(n_slots + 1) * 4, st>>>(n_chunks, n_slots, scratch, counts, offsets,
                                                                      active, n_active, counters, n_counters);
        sort_scatter_kernel<<<n_chunks, 1024, smem_s, st>>>(ids, n_pairs, n_slots, scratch, perm);
        return cudaGetLastError();
    }
    const size_t smem = sort_pairs_smem(n_slots);
    static int cache[64] = {};
    cudaError_t e = set_smem_once(sort_pairs_kernel, smem, cache);
    if (e != cudaSuccess) return e;
    sort_pairs_kernel<<<1, 1024, smem, st>>>(ids, n_pairs, n_slots, counts, offsets, perm, active, n_active, counters,
                                             n_counters, err);
    return cudaGetLastError();
}

bool route_dispatch_fits(int64_t T, int k, int E, int n_slots) {
    return T * k <= ROUTE_FUSED_MAX_PAIRS && E <= 256 && n_slots <= 256;
}

cudaError_t launch_route_dispatch(const float *logits, int T, int E, int k, const int32_t *table, int n_table,
                                  int32_t *ids_out, float *w_out, int32_t *mapped, int n_slots, int32_t *counts,
                                  int32_t *offsets, int32_t *perm, int4 *active, int32_t *n_active,
                                  int *counters, int n_counters, int *err, cudaStream_t st) {
    const size_t smem = sizeof(int32_t) * ((size_t)((T * k + 3) & ~3)) + sort_pairs_smem(n_slots);
    static int cache[4][64] = {};
#define TMOE_RD(MP, CI)                                                                                        \
    do {                                                                                                       \
        cudaError_t e = set_smem_once(route_dispatch_kernel<MP>, smem, cache[CI]);                             \
        if (e != cudaSuccess) return e;                                                                        \
        route_dispatch_kernel<MP><<<1, 1024, smem, st>>>(logits, T, E, k, table, n_table, ids_out, w_out,      \
                                                         mapped, n_slots, counts, offsets, perm, active,      \
                                                         n_active, counters, n_counters, err);                 \
    } while (0)
    if (E <= 32)
        TMOE_RD(1, 0);
    else if (E <= 64)
        TMOE_RD(2, 1);
    else if (E <= 128)
        TMOE_RD(4, 2);
    else if (E <= 256)
        TMOE_RD(8, 3);
    else
        return cudaErrorInvalidValue;
#undef TMOE_RD
    return cudaGetLastError();
}

static size_t route_fused_smem(int tt, int H, int E, int T, int k, int n_slots) {
    const size_t staged = (size_t)(tt + FR_WARPS) * H * 4;
    const size_t sorting =
        4 * ((size_t)tt * E + (size_t)((T * k + 3) & ~3) + (size_t)FR_WARPS * n_slots + n_slots + 65);
    return staged > sorting ? staged : sorting;
}

// Tokens per CTA: the batch itself below 8 tokens (rounded up to a power of two, so that a CTA
// computes no dot products of empty token rows: at T = 1 a tile of 8 did eight times the work),
// else 8, or 4 when 8 staged rows do not fit.
static int route_fused_tt(int H, int E, int T, int k, int n_slots) {
    int want = 8;
    while (want > 1 && want / 2 >= T) want /= 2;
    for (int tt = want; tt >= (want < 4 ? want : 4); tt >>= 1)
        if (route_fused_smem(tt, H, E, T, k, n_slots) <= 200 * 1024) return tt;
    return 0;
}

bool route_fused_fits(int64_t T, int k, int E, int H, int n_slots) {
    return route_dispatch_fits(T, k, E, n_slots) && H % 128 == 0 && route_fused_tt(H, E, (int)T, k, n_slots) > 0;
}

int route_fused_tiles(int64_t T, int k, int E, int H, int n_slots) {
    const int tt = route_fused_tt(H, E, (int)T, k, n_slots);
    return tt ? (int)((T + tt - 1) / tt) : 0;
}

cudaError_t launch_route_fused(const float *x, const float *rw, int T, int H, int E, int k, const Q8Rows *q8,
                               float *logits, const int32_t *table, int n_table, int32_t *ids_out, float *w_out,
                               int32_t *mapped, int n_slots, int32_t *counts, int32_t *offsets, int32_t *perm,
                               int4 *active, int32_t *n_active, int *counters, int n_counters, int *done, int *err,
                               cudaStream_t st) {
    const int tt = route_fused_tt(H, E, T, k, n_slots);
    if (!tt || !route_dispatch_fits(T, k, E, n_slots)) return cudaErrorInvalidValue;
    const size_t smem = route_fused_smem(tt, H, E, T, k, n_slots);
    const dim3 grid((E + FR_WARPS - 1) / FR_WARPS, (T + tt - 1) / tt);
    const Q8Rows none{nullptr, nullptr, nullptr, nullptr, 0};
    const Q8Rows qq = q8 ? *q8 : none;
    static int cache[16][64] = {};
#define TMOE_RF(TTV, MP, CI)                                                                                   \
    do {                                                                                                       \
        cudaError_t e = set_smem_once(route_fused_kernel<TTV, MP>, smem, cache[CI]);                           \
        if (e != cudaSuccess) return e;                                                                        \
        e = launch_k(route_fused_kernel<TTV, MP>, grid, FR_WARPS * 32, smem, st,                                \
            x, rw, T, H, E, k, qq, logits, table, n_table, ids_out, w_out, mapped, n_slots, counts, offsets,    \
            perm, active, n_active, counters, n_counters, done, err);                                           \
        if (e != cudaSuccess) return e;                                                                        \
    } while (0)
    const int mp = E <= 32 ? 1 : E <= 64 ? 2 : E <= 128 ? 4 : 8;
#define TMOE_RF_TT(TTV, C0)                      \
    do {                                         \
        if (mp == 1) TMOE_RF(TTV, 1, C0);        \
        else if (mp == 2) TMOE_RF(TTV, 2, C0 + 1); \
        else if (mp == 4) TMOE_RF(TTV, 4, C0 + 2); \
        else TMOE_RF(TTV, 8, C0 + 3);            \
    } while (0)
    if (tt == 8) TMOE_RF_TT(8, 0);
    else if (tt == 4) TMOE_RF_TT(4, 4);
    else if (tt == 2) TMOE_RF_TT(2, 8);
    else TMOE_RF_TT(1, 12);
#undef TMOE_RF_TT
#undef TMOE_RF
    return cudaGetLastError();
}

cudaError_t launch_map_ids(const int32_t *ids, int64_t n, const int32_t *table, int64_t n_table, int32_t *out,
                           cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    map_ids_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(ids, n, table, n_table, out);
    return cudaGetLastError();
}

cudaError_t launch_zero_invalid_rows(const int32_t *ids, int64_t n_pairs, int n_slots, int N, float *out,
                                     cudaStream_t st) {
    if (n_pairs <= 0) return cudaSuccess;
    zero_invalid_rows_kernel<<<(unsigned)n_pairs, 128, 0, st>>>(ids, n_pairs, n_slots, N, out);
    return cudaGetLastError();
}

// One thread holds the stream until *flag == value (a flag the host writes into pinned, device-mapped
// memory, or a device word), with the kernels' bounded-wait rule: it gives up after limit_ns of
// %globaltimer, latches TMOE_DEV_ERR_TIMEOUT and returns, so the stream moves on and the context
// stays usable.  The backoff keeps the polling thread to a few loads per microsecond.
__global__ void wait_flag_kernel(const volatile int32_t *flag, int32_t value, uint64_t limit_ns, int *err) {
    const uint64_t t0 = globaltimer_ns();
    uint32_t nap = 32;
    while (*flag != value) {
        if (globaltimer_ns() - t0 > limit_ns) {
            latch_error(err, TMOE_DEV_ERR_TIMEOUT);
            return;
        }
        __nanosleep(nap);
        if (nap < 2048) nap *= 2;
    }
    __threadfence_system();  // what the writer stored before the flag is visible to later kernels
}

cudaError_t launch_wait_flag(const int32_t *flag, int32_t value, uint64_t limit_ns, int *err, cudaStream_t st) {
    wait_flag_kernel<<<1, 1, 0, st>>>(flag, value, limit_ns, err);
    return cudaGetLastError();
}

cudaError_t launch_combine(const float *dout, const int32_t *ids, const float *w, int64_t T, int k, int H,
                           int n_slots, float *out, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    const int64_t n4 = T * H / 4;
    const unsigned grid = (unsigned)((n4 + 127) / 128);
    cudaError_t e;
    if (k <= 8)
        e = launch_k(combine_kernel<8>, grid, 128, 0, st, dout, ids, w, T, k, H, n_slots, out);
    else if (k <= 16)
        e = launch_k(combine_kernel<16>, grid, 128, 0, st, dout, ids, w, T, k, H, n_slots, out);
    else
        e = launch_k(combine_kernel<32>, grid, 128, 0, st, dout, ids, w, T, k, H, n_slots, out);
    return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace tmoe
