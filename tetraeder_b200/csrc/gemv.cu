// Expert products for the decode regime (few tokens per expert): HBM-bound dequant-GEMV over
// Q4_K / Q6_K rows with Q8_K activations, the arithmetic of ggml's CPU mul_mat_id path
// (vec_dot_q4_K_q8_K / vec_dot_q6_K_q8_K): per sub-block an exact integer dot times the
// sub-block's integer scale, summed per super-block, then scaled by d*dx (and for Q4_K minus
// dmin*dx * sum_s m_s * B_s, B_s the activation's sub-block sum).
//
// The sub-block dots run on the tensor cores as warp-level integer MMAs, 16 weight rows x 8
// tokens per instruction: m16n8k32 for Q4_K's 32-element sub-blocks and m16n8k16 for Q6_K's
// 16-element ones.  The int32 fragments come back to registers after every sub-block, which is
// what the per-sub-block scales need (an accumulator that stays in TMEM across K cannot take
// them); the scaling is a few integer multiply-adds per fragment.  The sub-block sum terms (the
// Q4_K mins, the Q6_K -32 bias) are two more small MMAs per super-block.
//
// Work: items = (active expert, tile of RT rows), expert-major.  Each CTA's producer thread
// takes items in chunks from a global counter (dynamic balancing: items differ in token count),
// streams their weight rows into a ring of shared-memory stages with 1D bulk TMA copies
// (cp.async.bulk ... mbarrier::complete_tx; Q4_K one copy per row into rows padded for
// conflict-free fragment loads, Q6_K one copy per 8 rows since a 630-byte row is not a multiple
// of 16 bytes) and publishes the item index with the stage.  Eight consumer warps: warp (wr, wk)
// multiplies row tile wr over the wk-th slice of K, reading the tokens' Q8_K rows straight from
// global memory (L1/L2-resident); the WK slices are summed in a fixed order through shared
// memory.  gate/up: both matrices share the stage and the activation loads, and the result is
// silu(g) * u (swiglu_split).
#include "common.cuh"
#include "kernels.cuh"

namespace tmoe {

constexpr int GEMV_NW = 8;  // consumer warps
constexpr int GEMV_THREADS = 32 * (GEMV_NW + 1);
constexpr int GEMV_MAX_STAGES = 12;
constexpr int GEMV_BAR_BYTES = 256;  // mbarriers and the per-stage item indices
constexpr int TOKG = 8;              // tokens per MMA (the n of m16n8)
constexpr int GEMV_CHUNK = 2;        // items taken from the work counter at a time
constexpr uint32_t NIB = 0x0f0f0f0fu;

template <int WT>
struct Fmt;
template <>
struct Fmt<TMOE_WT_Q4K> {
    static constexpr int block_bytes = TMOE_Q4K_BYTES;
    static constexpr int sub = 32;        // elements per sub-block
    static constexpr int tile_rows = 16;  // rows of one warp tile
    static constexpr int nbw = 2;         // split-sum words per super-block
};
template <>
struct Fmt<TMOE_WT_Q6K> {
    static constexpr int block_bytes = TMOE_Q6K_BYTES;
    static constexpr int sub = 16;
    static constexpr int tile_rows = 32;  // an even-row and an odd-row MMA
    static constexpr int nbw = 4;
};

// Integer MMAs (warp-level, A 16 x k row-major, B k x 8 col-major, int32 accumulators from 0).
#define TMOE_MMA_K32(AT, BT)                                                                                     \
    __device__ __forceinline__ void mma_k32_##AT##BT(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,         \
                                                     uint32_t a3, uint32_t b0, uint32_t b1) {                   \
        asm volatile("mma.sync.aligned.m16n8k32.row.col.s32." #AT "." #BT                                        \
                     ".s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"                           \
                     : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])                                            \
                     : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));                           \
    }
#define TMOE_MMA_K16(AT, BT)                                                                                     \
    __device__ __forceinline__ void mma_k16_##AT##BT(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {      \
        asm volatile("mma.sync.aligned.m16n8k16.row.col.s32." #AT "." #BT                                        \
                     ".s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"                                         \
                     : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])                                            \
                     : "r"(a0), "r"(a1), "r"(b0), "r"(0));                                                      \
    }
TMOE_MMA_K32(u8, s8)
TMOE_MMA_K16(u8, s8)
TMOE_MMA_K16(u8, u8)
TMOE_MMA_K16(s8, s8)
TMOE_MMA_K16(s8, u8)

__device__ __forceinline__ int ubyte(uint32_t w, int i) { return (int)__byte_perm(w, 0u, 0x4440u | (uint32_t)i); }
__device__ __forceinline__ int sbyte(uint32_t w, int i) { return ((int)(w << (24 - 8 * i))) >> 24; }

__device__ __forceinline__ uint2 ldg64(const void *p) { return __ldg(reinterpret_cast<const uint2 *>(p)); }
__device__ __forceinline__ uint32_t ldg32(const void *p) { return __ldg(reinterpret_cast<const uint32_t *>(p)); }

// The activation rows of one 8-token group, as a thread sees them: column g (its B operand) and
// columns 2*t4, 2*t4+1 (its accumulator fragments).
struct XCols {
    const int8_t *qs_g;                 // Q8_K values of column g
    const uint32_t *bl_g, *bh_g;        // split sub-block sums of column g
    const float *d_0, *d_1;             // d of columns 2*t4 and 2*t4+1
};

// Fragment i of an m16n8 tile: MMA row g (i < 2) or g + 8 (i >= 2), token 2*t4 + (i & 1) of
// the 8-token group (g = lane / 4, t4 = lane % 4).
//
// Q4_K: 16 rows at m0 / m1 (row stride rs), super-blocks [b0, b1).
//  - Inside a sub-block the k order is permuted identically for both operands (thread t4 holds
//    elements 8*t4 .. 8*t4+7 of the 32), so each operand is one 8-byte load, and one load of the
//    nibble bytes serves sub-blocks 2j (low nibbles) and 2j+1 (high nibbles).
//  - The high nibbles go to the MMA in place (byte & 0xf0 = 16 * q, unsigned): those products
//    are 16 times too large and the super-block's sum of them is shifted right by 4, exactly.
//  - The 6-bit scales and mins are unpacked once per row and super-block into byte-packed words.
//  - The min term sum_s m_s * B_s is itself two small MMAs (k = 16: 8 sub-blocks and 8 zeros):
//    mins x lo bytes + 64 * (mins x hi bytes).
template <int NMAT>
__device__ __forceinline__ void q4_dot(const uint8_t *m0, const uint8_t *m1, int rs, const XCols &x, int b0, int b1,
                                       float (&acc)[NMAT][4]) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
    const uint8_t *ra[NMAT], *rb[NMAT];
    ra[0] = m0 + (size_t)g * rs;
    rb[0] = m0 + (size_t)(g + 8) * rs;
    if constexpr (NMAT == 2) {
        ra[1] = m1 + (size_t)g * rs;
        rb[1] = m1 + (size_t)(g + 8) * rs;
    }
    for (int b = b0; b < b1; b++) {
        // activation operands of the whole super-block first (global / L1)
        uint2 xl[4], xh[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            xl[j] = ldg64(x.qs_g + 256 * b + 64 * j + 8 * t4);
            xh[j] = ldg64(x.qs_g + 256 * b + 64 * j + 32 + 8 * t4);
        }
        const uint32_t bl = t4 < 2 ? __ldg(x.bl_g + 2 * b + t4) : 0u;
        const uint32_t bh = t4 < 2 ? __ldg(x.bh_g + 2 * b + t4) : 0u;
        const float dx0 = __ldg(x.d_0 + b), dx1 = __ldg(x.d_1 + b);
        uint32_t sca[NMAT][2], scb[NMAT][2], mna[NMAT][2], mnb[NMAT][2];
        float da[NMAT], ma[NMAT], db[NMAT], mb[NMAT];
#pragma unroll
        for (int m = 0; m < NMAT; m++) {
            const uint4 ha = *reinterpret_cast<const uint4 *>(ra[m] + b * TMOE_Q4K_BYTES);
            const uint4 hb = *reinterpret_cast<const uint4 *>(rb[m] + b * TMOE_Q4K_BYTES);
            sca[m][0] = ha.y & 0x3f3f3f3fu;
            sca[m][1] = (ha.w & 0x0f0f0f0fu) | ((ha.y >> 2) & 0x30303030u);
            mna[m][0] = ha.z & 0x3f3f3f3fu;
            mna[m][1] = ((ha.w >> 4) & 0x0f0f0f0fu) | ((ha.z >> 2) & 0x30303030u);
            scb[m][0] = hb.y & 0x3f3f3f3fu;
            scb[m][1] = (hb.w & 0x0f0f0f0fu) | ((hb.y >> 2) & 0x30303030u);
            mnb[m][0] = hb.z & 0x3f3f3f3fu;
            mnb[m][1] = ((hb.w >> 4) & 0x0f0f0f0fu) | ((hb.z >> 2) & 0x30303030u);
            da[m] = h2f((uint16_t)(ha.x & 0xffffu));
            ma[m] = h2f((uint16_t)(ha.x >> 16));
            db[m] = h2f((uint16_t)(hb.x & 0xffffu));
            mb[m] = h2f((uint16_t)(hb.x >> 16));
        }
        int il[NMAT][4], ih[NMAT][4];
#pragma unroll
        for (int m = 0; m < NMAT; m++)
#pragma unroll
            for (int i = 0; i < 4; i++) il[m][i] = ih[m][i] = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) {
#pragma unroll
            for (int m = 0; m < NMAT; m++) {
                const uint2 wa = *reinterpret_cast<const uint2 *>(ra[m] + b * TMOE_Q4K_BYTES + 16 + 32 * j + 8 * t4);
                const uint2 wb = *reinterpret_cast<const uint2 *>(rb[m] + b * TMOE_Q4K_BYTES + 16 + 32 * j + 8 * t4);
                int dl[4], dh[4];
                mma_k32_u8s8(dl, wa.x & NIB, wb.x & NIB, wa.y & NIB, wb.y & NIB, xl[j].x, xl[j].y);
                mma_k32_u8s8(dh, wa.x & ~NIB, wb.x & ~NIB, wa.y & ~NIB, wb.y & ~NIB, xh[j].x, xh[j].y);
                const int bi = 2 * (j & 1);
                const int sla = ubyte(sca[m][j >> 1], bi), sha = ubyte(sca[m][j >> 1], bi + 1);
                const int slb = ubyte(scb[m][j >> 1], bi), shb = ubyte(scb[m][j >> 1], bi + 1);
                il[m][0] += sla * dl[0];
                il[m][1] += sla * dl[1];
                il[m][2] += slb * dl[2];
                il[m][3] += slb * dl[3];
                ih[m][0] += sha * dh[0];
                ih[m][1] += sha * dh[1];
                ih[m][2] += shb * dh[2];
                ih[m][3] += shb * dh[3];
            }
        }
#pragma unroll
        for (int m = 0; m < NMAT; m++) {
            const uint32_t a0 = t4 == 0 ? mna[m][0] : (t4 == 1 ? mna[m][1] : 0u);
            const uint32_t a1 = t4 == 0 ? mnb[m][0] : (t4 == 1 ? mnb[m][1] : 0u);
            int ml[4], mh[4];
            mma_k16_u8u8(ml, a0, a1, bl);
            mma_k16_u8s8(mh, a0, a1, bh);
            const float dd[4] = {da[m] * dx0, da[m] * dx1, db[m] * dx0, db[m] * dx1};
            const float dm[4] = {ma[m] * dx0, ma[m] * dx1, mb[m] * dx0, mb[m] * dx1};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int isum = il[m][i] + (ih[m][i] >> 4), msum = ml[i] + 64 * mh[i];
                acc[m][i] += __fmul_rn(dd[i], (float)isum) - __fmul_rn(dm[i], (float)msum);
            }
        }
    }
}

// Q6_K rows sit in 8-row groups (row_bytes = 210 * nb apart, group stride gs, a multiple of 4).
// A warp tile is 32 rows: the even rows form one MMA, the odd rows another, so that word
// alignment is uniform across each MMA's rows: a block starts 2 bytes off a word boundary iff
// row * nb + block is odd, and those words are realigned with a funnel shift.  Thread t4 holds
// elements 4*t4 .. 4*t4+3 of a 16-element sub-block.  Per half block (8 sub-blocks) and row: 4
// nibble words (each serving a low and a high nibble sub-block), 2 high-bit words (each serving
// four sub-blocks) and 2 scale words; only halves that meet the warp's slice are loaded.  The raw
// 6-bit values go to the MMA unsigned; the -32 bias is applied as -32 * sum_s sc_s * B_s, and
// that sum is two small MMAs (k = 16 = the block's sub-blocks, outside the slice zeroed).
__device__ __forceinline__ uint32_t ld32_mis(const uint8_t *p, bool mis) {
    if (!mis) return *reinterpret_cast<const uint32_t *>(p);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(p - 2);
    return __funnelshift_r(w[0], w[1], 16);
}

struct Q6Half {
    uint32_t ql[4], qh[2], sc[2];
};

__device__ __forceinline__ void q6_load_half(const uint8_t *blk, int h, int t4, bool mis, Q6Half &q) {
#pragma unroll
    for (int i = 0; i < 4; i++) q.ql[i] = ld32_mis(blk + 64 * h + 16 * i + 4 * t4, mis);
#pragma unroll
    for (int i = 0; i < 2; i++) q.qh[i] = ld32_mis(blk + 128 + 32 * h + 16 * i + 4 * t4, mis);
    q.sc[0] = ld32_mis(blk + 192 + 8 * h, mis);
    q.sc[1] = ld32_mis(blk + 196 + 8 * h, mis);
}

// Unsigned 6-bit values of sub-block sl8 (0..7 within the half, a constant after unrolling).
__device__ __forceinline__ uint32_t q6_vals(const Q6Half &q, int sl8) {
    const uint32_t lo = (q.ql[sl8 & 3] >> (sl8 >= 4 ? 4 : 0)) & NIB;
    const uint32_t hi = ((q.qh[sl8 & 1] >> (2 * (sl8 >> 1))) & 0x03030303u) << 4;
    return lo | hi;
}

template <int NMAT>
__device__ __forceinline__ void q6_dot(const uint8_t *m0, const uint8_t *m1, int gs, int row_bytes, int nb, int rbase,
                                       const XCols &x, int s0, int s1, float (&acc)[NMAT][2][4]) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
    for (int b = s0 >> 4; b * 16 < s1; b++) {
        const int lo = max(s0 - 16 * b, 0), hi = min(s1 - 16 * b, 16);
        uint32_t keep = 0;  // the token's sums for sub-blocks 4*t4 .. 4*t4+3, outside [lo, hi) zeroed
#pragma unroll
        for (int i = 0; i < 4; i++)
            if (4 * t4 + i >= lo && 4 * t4 + i < hi) keep |= 0xffu << (8 * i);
        const uint32_t bl = __ldg(x.bl_g + 4 * b + t4) & keep, bh = __ldg(x.bh_g + 4 * b + t4) & keep;
        const float dx0 = __ldg(x.d_0 + b), dx1 = __ldg(x.d_1 + b);
        uint32_t xw[16];
#pragma unroll
        for (int s = 0; s < 16; s++) xw[s] = (s >= lo && s < hi) ? ldg32(x.qs_g + 16 * (16 * b + s) + 4 * t4) : 0u;
#pragma unroll
        for (int p = 0; p < 2; p++) {  // p = 0: even rows, 1: odd rows
            const bool mis = ((p == 1) && (nb & 1)) != (bool)(b & 1);
            const int r_a = rbase + 2 * g + p, r_b = r_a + 16;
#pragma unroll
            for (int m = 0; m < NMAT; m++) {
                const uint8_t *mat = m == 0 ? m0 : m1;
                const uint8_t *ba = mat + (size_t)(r_a >> 3) * gs + (size_t)(r_a & 7) * row_bytes + b * TMOE_Q6K_BYTES;
                const uint8_t *bb = mat + (size_t)(r_b >> 3) * gs + (size_t)(r_b & 7) * row_bytes + b * TMOE_Q6K_BYTES;
                int isum[4] = {0, 0, 0, 0};
                uint32_t sca[4] = {0u, 0u, 0u, 0u}, scb[4] = {0u, 0u, 0u, 0u};
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    if (hi <= 8 * h || lo >= 8 * h + 8) continue;
                    Q6Half qa, qb;
                    q6_load_half(ba, h, t4, mis, qa);
                    q6_load_half(bb, h, t4, mis, qb);
                    sca[2 * h] = qa.sc[0], sca[2 * h + 1] = qa.sc[1];
                    scb[2 * h] = qb.sc[0], scb[2 * h + 1] = qb.sc[1];
#pragma unroll
                    for (int sl8 = 0; sl8 < 8; sl8++) {
                        const int s = 8 * h + sl8;
                        if (s < lo || s >= hi) continue;
                        int d[4];
                        mma_k16_u8s8(d, q6_vals(qa, sl8), q6_vals(qb, sl8), xw[s]);
                        const int ca = sbyte(qa.sc[sl8 >> 2], sl8 & 3), cb = sbyte(qb.sc[sl8 >> 2], sl8 & 3);
                        isum[0] += ca * d[0];
                        isum[1] += ca * d[1];
                        isum[2] += cb * d[2];
                        isum[3] += cb * d[3];
                    }
                }
                // scale word t4 of each row (selected without indexing the register arrays)
                const uint32_t wa = t4 == 0 ? sca[0] : t4 == 1 ? sca[1] : t4 == 2 ? sca[2] : sca[3];
                const uint32_t wb = t4 == 0 ? scb[0] : t4 == 1 ? scb[1] : t4 == 2 ? scb[2] : scb[3];
                int cl[4], ch[4];
                mma_k16_s8u8(cl, wa, wb, bl);
                mma_k16_s8s8(ch, wa, wb, bh);
                const float fa = h2f(*reinterpret_cast<const uint16_t *>(ba + 208));
                const float fb = h2f(*reinterpret_cast<const uint16_t *>(bb + 208));
                const float dd[4] = {fa * dx0, fa * dx1, fb * dx0, fb * dx1};
#pragma unroll
                for (int i = 0; i < 4; i++)
                    acc[m][p][i] += __fmul_rn(dd[i], (float)(isum[i] - 32 * (cl[i] + 64 * ch[i])));
            }
        }
    }
}

__device__ __forceinline__ float silu_mul(float g, float u) { return (g / (1.0f + expf(-g))) * u; }

// Named barrier 1 over the consumer warps, returning the AND of `ok` over them.  Each warp
// reconverges first (__syncwarp: lanes leave the polling loop on different iterations) and the
// non-.aligned barrier form is used.
__device__ __forceinline__ bool consumers_all(bool ok) {
    __syncwarp();
    uint32_t r;
    asm volatile(
        "{ .reg .pred p, q; setp.ne.u32 p, %1, 0; barrier.red.and.pred q, 1, %2, p; selp.u32 %0, 1, 0, q; }"
        : "=r"(r)
        : "r"((uint32_t)ok), "n"(GEMV_NW * 32)
        : "memory");
    return r != 0;
}

// Consumer protocol, per published item: one bounded wait on the stage, then exactly one
// consumers_all per 8-token group (a skipped item or the end marker: exactly one).  A warp whose
// wait gave up still takes part (ok = false), so every warp leaves on the same barrier.
template <int WT, bool GATEUP, int WK, int MINB>
__global__ void __launch_bounds__(GEMV_THREADS, MINB) gemv_kernel(const GemvArgs a) {
    constexpr int WR = GEMV_NW / WK;
    constexpr int TR = Fmt<WT>::tile_rows;
    constexpr int RT = WR * TR;
    constexpr int NMAT = GATEUP ? 2 : 1;
    constexpr int NBW = Fmt<WT>::nbw;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + GEMV_MAX_STAGES;
    int *sitem = reinterpret_cast<int *>(empty + GEMV_MAX_STAGES);
    uint8_t *stage0 = smem + GEMV_BAR_BYTES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NS = a.n_stages, K = a.K;
    const int nb = K / TMOE_QK;
    const int row_bytes = Fmt<WT>::block_bytes * nb;
    const int rstride = a.row_stride;  // Q4_K: padded row stride; Q6_K: 8-row group stride
    const int mat_bytes = a.mat_stride;
    float *red0 = reinterpret_cast<float *>(stage0 + (size_t)NS * a.stage_bytes);  // [2][NMAT][WK][RT][TOKG]
    constexpr int RED = NMAT * WK * RT * TOKG;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], GEMV_NW);
        }
        fence_barrier_init();
    }
    __syncthreads();
    // Dispatch data are checked before they become addresses: an active count above the grid's
    // sizing or an expert outside [0, n_slots) latches TMOE_DEV_ERR_BADID; such an item is
    // published (so the pipeline stays in step) but loads and computes nothing.
    int na = a.n_active[0];
    if (na > a.max_active || na < 0) {
        if (threadIdx.x == 0 && blockIdx.x == 0) latch_error(a.err, TMOE_DEV_ERR_BADID);
        na = na < 0 ? 0 : a.max_active;
    }
    const int n_items = na * a.tiles;

    if (warp == GEMV_NW) {  // producer
        if (lane == 0) {
            int next = 0, lim = 0;
            for (int it = 0;; ++it) {
                const int s = it % NS;
                if (it >= NS && !mbar_wait_bounded(&empty[s], ((it / NS) - 1) & 1)) {
                    latch_error(a.err, TMOE_DEV_ERR_TIMEOUT);
                    break;  // the consumers' bounded waits end them
                }
                if (next >= lim) {
                    next = atomicAdd(a.work, GEMV_CHUNK);
                    lim = next + GEMV_CHUNK;
                }
                const int item = next < n_items ? next++ : -1;
                sitem[s] = item;
                if (item < 0) {  // end marker
                    mbar_arrive_expect_tx(&full[s], 0u);
                    break;
                }
                const int e = a.active[item / a.tiles];
                const int r0 = (item % a.tiles) * RT;
                uint8_t *dst = stage0 + (size_t)s * a.stage_bytes;
                if (e < 0 || e >= a.n_slots) {
                    latch_error(a.err, TMOE_DEV_ERR_BADID);
                    mbar_arrive_expect_tx(&full[s], 0u);
                    continue;
                }
                mbar_arrive_expect_tx(&full[s], (uint32_t)(NMAT * RT * row_bytes));
#pragma unroll
                for (int m = 0; m < NMAT; m++) {
                    const uint8_t *src = (m == 0 ? a.w0 + (size_t)e * a.nb2_0 : a.w1 + (size_t)e * a.nb2_1) +
                                         (size_t)r0 * row_bytes;
                    uint8_t *d = dst + (size_t)m * mat_bytes;
                    if constexpr (WT == TMOE_WT_Q4K) {
                        for (int r = 0; r < RT; r++)
                            bulk_g2s(d + (size_t)r * rstride, src + (size_t)r * row_bytes, (uint32_t)row_bytes,
                                     &full[s]);
                    } else {
                        for (int gq = 0; gq < RT / 8; gq++)
                            bulk_g2s(d + (size_t)gq * rstride, src + (size_t)gq * 8 * row_bytes,
                                     (uint32_t)(8 * row_bytes), &full[s]);
                    }
                }
            }
        }
        return;
    }

    const int wr = warp / WK, wk = warp % WK;
    const int n_sub = K / Fmt<WT>::sub;
    const int ks0 = (n_sub * wk) / WK, ks1 = (n_sub * (wk + 1)) / WK;  // sub-block slice
    const int ctid = threadIdx.x;
    const int g = lane >> 2, t4 = lane & 3;
    int rbuf = 0;  // reduction buffer (two, alternating: one barrier per reduction)
    for (int it = 0;; ++it) {
        const int s = it % NS;
        const bool ok = mbar_wait_bounded(&full[s], (it / NS) & 1);
        __syncwarp();
        const int item = ok ? sitem[s] : -1;
        if (item < 0) {  // end (or this warp gave up): leave on one barrier
            if (!consumers_all(ok)) latch_error(a.err, TMOE_DEV_ERR_TIMEOUT);
            break;
        }
        const int e = a.active[item / a.tiles];
        const int r0 = (item % a.tiles) * RT;
        const uint8_t *st = stage0 + (size_t)s * a.stage_bytes;
        const bool e_ok = e >= 0 && e < a.n_slots;
        int beg = e_ok ? a.offsets[e] : 0, end = e_ok ? a.offsets[e + 1] : 0;
        if (beg < 0 || end > a.n_pairs || end < beg) beg = end = 0;
        if (beg == end) {  // nothing to compute
            if (lane == 0) mbar_arrive(&empty[s]);
            if (!consumers_all(true)) break;
            continue;
        }
        bool abort = false;
        for (int tg = beg; tg < end; tg += TOKG) {
            const int ntok = min(TOKG, end - tg);
            // this thread's columns: g (B operand), 2*t4 and 2*t4+1 (fragments); past the
            // group's end, the first token stands in (those columns are never written)
            const int pg = a.perm[tg + (g < ntok ? g : 0)];
            const int p0 = a.perm[tg + (2 * t4 < ntok ? 2 * t4 : 0)];
            const int p1 = a.perm[tg + (2 * t4 + 1 < ntok ? 2 * t4 + 1 : 0)];
            const int64_t xg = (pg >= 0 && pg < a.n_pairs ? pg : 0) / a.x_div;
            const int64_t x0 = (p0 >= 0 && p0 < a.n_pairs ? p0 : 0) / a.x_div;
            const int64_t x1 = (p1 >= 0 && p1 < a.n_pairs ? p1 : 0) / a.x_div;
            const XCols xc{a.xq + xg * K, a.xbl + xg * nb * NBW, a.xbh + xg * nb * NBW, a.xd + x0 * nb, a.xd + x1 * nb};
            float *red = red0 + (size_t)rbuf * RED;
            if constexpr (WT == TMOE_WT_Q4K) {
                float acc[NMAT][4];
#pragma unroll
                for (int m = 0; m < NMAT; m++) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.0f;
                q4_dot<NMAT>(st + (size_t)(wr * TR) * rstride, st + mat_bytes + (size_t)(wr * TR) * rstride, rstride,
                             xc, ks0 / 8, ks1 / 8, acc);
#pragma unroll
                for (int m = 0; m < NMAT; m++) {
                    float *rd = red + ((size_t)(m * WK + wk) * RT) * TOKG;
                    const int rA = wr * TR + g, rB = rA + 8;
                    *reinterpret_cast<float2 *>(rd + (size_t)rA * TOKG + 2 * t4) = make_float2(acc[m][0], acc[m][1]);
                    *reinterpret_cast<float2 *>(rd + (size_t)rB * TOKG + 2 * t4) = make_float2(acc[m][2], acc[m][3]);
                }
            } else {
                float acc[NMAT][2][4];
#pragma unroll
                for (int m = 0; m < NMAT; m++)
#pragma unroll
                    for (int p = 0; p < 2; p++)
#pragma unroll
                        for (int i = 0; i < 4; i++) acc[m][p][i] = 0.0f;
                q6_dot<NMAT>(st, st + mat_bytes, rstride, row_bytes, nb, wr * TR, xc, ks0, ks1, acc);
                // MMA row g -> tile row 2g, row g+8 -> 2g+16; the odd-row MMA one row below
#pragma unroll
                for (int m = 0; m < NMAT; m++) {
                    float *rd = red + ((size_t)(m * WK + wk) * RT) * TOKG;
#pragma unroll
                    for (int p = 0; p < 2; p++) {
                        const int rA = wr * TR + 2 * g + p, rB = rA + 16;
                        *reinterpret_cast<float2 *>(rd + (size_t)rA * TOKG + 2 * t4) =
                            make_float2(acc[m][p][0], acc[m][p][1]);
                        *reinterpret_cast<float2 *>(rd + (size_t)rB * TOKG + 2 * t4) =
                            make_float2(acc[m][p][2], acc[m][p][3]);
                    }
                }
            }
            if (tg + TOKG >= end) {  // last read of the stage
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
            if (!consumers_all(true)) {  // the partial sums of every warp are in `red`
                abort = true;
                break;
            }
            // sum the WK slices in order and write the (row, token) outputs
            for (int o = ctid; o < RT * TOKG; o += 32 * GEMV_NW) {
                const int row = o / TOKG, tk = o % TOKG;
                if (tk >= ntok) continue;
                float v0 = 0.0f, v1 = 0.0f;
#pragma unroll
                for (int k = 0; k < WK; k++) {
                    v0 += red[((size_t)k * RT + row) * TOKG + tk];
                    if constexpr (GATEUP) v1 += red[((size_t)(WK + k) * RT + row) * TOKG + tk];
                }
                const int pp = a.perm[tg + tk];
                if (pp >= 0 && pp < a.n_pairs) a.out[(int64_t)pp * a.N + r0 + row] = GATEUP ? silu_mul(v0, v1) : v0;
            }
            rbuf ^= 1;
        }
        if (abort) break;
    }
}

// ------------------------------------------------------------------ launcher
constexpr uint32_t GEMV_SMEM_1CTA = 226 * 1024;
constexpr uint32_t GEMV_SMEM_2CTA = 110 * 1024;

// Warps along K (a power of two dividing the eight consumer warps): Q4_K whole super-blocks per
// warp (WK divides nb); Q6_K preferably at least 12 sub-blocks per warp.  The item's row count
// (8 / WK row tiles) must divide N; if it does not, more warps go along K.  0: no split fits.
template <int WT>
static int choose_wk(int K, int N) {
    const int nb = K / TMOE_QK, n_sub = K / Fmt<WT>::sub;
    int wk = 1;
    if (WT == TMOE_WT_Q4K) {
        for (int c = 8; c >= 1; c >>= 1)
            if (nb % c == 0) {
                wk = c;
                break;
            }
    } else {
        for (int c = 8; c >= 1; c >>= 1)
            if (c == 1 || (n_sub % c == 0 && n_sub / c >= 12)) {
                wk = c;
                break;
            }
    }
    for (; wk <= 8; wk *= 2) {
        if (WT == TMOE_WT_Q4K && nb % wk != 0) continue;
        const int rt = (GEMV_NW / wk) * Fmt<WT>::tile_rows;
        if (N % rt == 0) return wk;
    }
    return 0;
}

template <int WT>
static int rows_per_item(int K, int N) {
    const int wk = choose_wk<WT>(K, N);
    return wk ? (GEMV_NW / wk) * Fmt<WT>::tile_rows : 0;
}

template <typename KernT>
static cudaError_t set_smem_once(KernT kern, size_t smem, int *cache) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if ((int)smem > cache[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        cache[dev] = (int)smem;
    }
    return cudaSuccess;
}

template <int WT, bool GATEUP, int WK>
static cudaError_t launch_one(const GemvArgs &args_in, int max_items, int sm_count, cudaStream_t st) {
    GemvArgs a = args_in;
    constexpr int RT = (GEMV_NW / WK) * Fmt<WT>::tile_rows;
    constexpr int NMAT = GATEUP ? 2 : 1;
    const int row_bytes = Fmt<WT>::block_bytes * (a.K / TMOE_QK);
    if (WT == TMOE_WT_Q4K) {
        // a multiple of 16 B with (stride / 4) % 32 == 8: conflict-free 8-byte fragment loads
        const int st4 = row_bytes / 4;
        const int pad4 = ((8 - st4 % 32) + 32) % 32;
        a.row_stride = row_bytes + 4 * pad4;
        a.mat_stride = RT * a.row_stride;
    } else {
        a.row_stride = 8 * row_bytes + 16;  // 8-row group stride (+16: realigned reads run 2 B past a row)
        a.mat_stride = (RT / 8) * a.row_stride;
    }
    a.tiles = a.N / RT;
    a.stage_bytes = ((uint32_t)(NMAT * a.mat_stride) + 16 + 127) & ~127u;
    const size_t redb = 2 * (size_t)NMAT * WK * RT * TOKG * 4;
    // Two CTAs per SM when two stages fit in half the shared memory and the two-CTA build does
    // not spill much; else one CTA with as many stages as fit.
    bool two = GEMV_BAR_BYTES + redb + 2 * (size_t)a.stage_bytes <= GEMV_SMEM_2CTA;
    if (two) {
        static int spills = -1;
        if (spills < 0) {
            cudaFuncAttributes fa{};
            spills = cudaFuncGetAttributes(&fa, gemv_kernel<WT, GATEUP, WK, 2>) != cudaSuccess || fa.localSizeBytes > 32;
        }
        two = !spills;
    }
    const uint32_t budget = two ? GEMV_SMEM_2CTA : GEMV_SMEM_1CTA;
    int ns = (int)((budget - GEMV_BAR_BYTES - redb) / a.stage_bytes);
    if (ns > GEMV_MAX_STAGES) ns = GEMV_MAX_STAGES;
    if (ns < 2) return cudaErrorInvalidValue;
    a.n_stages = ns;
    const size_t smem = GEMV_BAR_BYTES + (size_t)ns * a.stage_bytes + redb;
    const int items = max_items * a.tiles;
    const int slots = sm_count * (two ? 2 : 1);
    const int grid = items < slots ? items : slots;
    if (grid < 1) return cudaSuccess;
    static int cache1[64] = {}, cache2[64] = {};
    cudaError_t e;
    if (two) {
        if ((e = set_smem_once(gemv_kernel<WT, GATEUP, WK, 2>, smem, cache2)) != cudaSuccess) return e;
        gemv_kernel<WT, GATEUP, WK, 2><<<grid, GEMV_THREADS, smem, st>>>(a);
    } else {
        if ((e = set_smem_once(gemv_kernel<WT, GATEUP, WK, 1>, smem, cache1)) != cudaSuccess) return e;
        gemv_kernel<WT, GATEUP, WK, 1><<<grid, GEMV_THREADS, smem, st>>>(a);
    }
    return cudaGetLastError();
}

int gemv_rows_per_item(int wt, int K, int N) {
    return wt == TMOE_WT_Q4K ? rows_per_item<TMOE_WT_Q4K>(K, N) : rows_per_item<TMOE_WT_Q6K>(K, N);
}

template <int WT, bool GATEUP>
static cudaError_t launch_wk(const GemvArgs &a, int max_items, int sm_count, cudaStream_t st) {
    switch (choose_wk<WT>(a.K, a.N)) {
    case 8: return launch_one<WT, GATEUP, 8>(a, max_items, sm_count, st);
    case 4: return launch_one<WT, GATEUP, 4>(a, max_items, sm_count, st);
    case 2: return launch_one<WT, GATEUP, 2>(a, max_items, sm_count, st);
    case 1: return launch_one<WT, GATEUP, 1>(a, max_items, sm_count, st);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemv(int wt, bool gateup, const GemvArgs &a, int max_items, int sm_count, cudaStream_t st) {
    if (a.K % TMOE_QK != 0 || a.K <= 0 || a.K > 8192) return cudaErrorInvalidValue;
    if (gemv_rows_per_item(wt, a.K, a.N) == 0) return cudaErrorInvalidValue;
    if (wt == TMOE_WT_Q4K)
        return gateup ? launch_wk<TMOE_WT_Q4K, true>(a, max_items, sm_count, st)
                      : launch_wk<TMOE_WT_Q4K, false>(a, max_items, sm_count, st);
    return gateup ? launch_wk<TMOE_WT_Q6K, true>(a, max_items, sm_count, st)
                  : launch_wk<TMOE_WT_Q6K, false>(a, max_items, sm_count, st);
}

}  // namespace tmoe
