// Expert products for the decode regime (few tokens per expert): HBM-bound dequant-GEMV over
// Q4_K / Q6_K rows with Q8_K activations, the arithmetic of ggml's CPU mul_mat_id path
// (vec_dot_q4_K_q8_K / vec_dot_q6_K_q8_K): per sub-block an exact integer dot times the
// sub-block's integer scale, summed per super-block, then scaled by d*dx (and for Q4_K minus
// dmin*dx * sum_s m_s * B_s, B_s the activation's sub-block sum).
//
// The sub-block dots run on the tensor cores as warp-level integer MMAs, 16 weight rows x 8
// tokens per instruction: m16n8k32 (s8 x s8) for Q4_K's 32-element sub-blocks and m16n8k16
// (u8 x s8) for Q6_K's 16-element ones; Q6_K feeds the raw 6-bit values and subtracts
// 32 * B_s afterwards (B_s from the Q8_K block sums) instead of re-biasing every byte.  The int32
// fragments come back to registers after every sub-block, which is what the per-sub-block scales
// need (an accumulator that stays in TMEM across K cannot take them); the scaling is a few integer
// multiply-adds per fragment.
//
// Work: items = (active expert, tile of RT rows), expert-major, a contiguous range per CTA.  One
// producer thread streams each item's rows into a ring of shared-memory stages with 1D bulk TMA
// copies (cp.async.bulk ... mbarrier::complete_tx): Q4_K one copy per row into rows padded for
// conflict-free fragment loads, Q6_K one copy per 8 rows (a 630-byte row is not a multiple of
// 16 bytes).  Eight consumer warps stage the expert's Q8_K activations in shared memory (once per
// expert), then warp (wr, wk) multiplies row tile wr over the wk-th slice of K; the WK slices are
// summed in a fixed order through shared memory.  gate/up: both matrices share the stage and the
// activation loads, and the result is silu(g) * u (swiglu_split).
#include "common.cuh"
#include "kernels.cuh"
#include "q8k.cuh"

namespace tmoe {

constexpr int GEMV_NW = 8;  // consumer warps
constexpr int GEMV_THREADS = 32 * (GEMV_NW + 1);
constexpr int GEMV_MAX_STAGES = 12;
constexpr int GEMV_BAR_BYTES = 256;  // mbarriers live in the first 256 B of shared memory
constexpr int TOKG = 8;              // tokens per MMA (the n of m16n8)
constexpr uint32_t NIB = 0x0f0f0f0fu;

template <int WT>
struct Fmt;
template <>
struct Fmt<TMOE_WT_Q4K> {
    static constexpr int block_bytes = TMOE_Q4K_BYTES;
    static constexpr int sub = 32;        // elements per sub-block (= MMA k)
    static constexpr int tile_rows = 16;  // rows of one warp tile
    static constexpr int xpad = 32;       // token row padding in shared memory (bank spread)
};
template <>
struct Fmt<TMOE_WT_Q6K> {
    static constexpr int block_bytes = TMOE_Q6K_BYTES;
    static constexpr int sub = 16;
    static constexpr int tile_rows = 32;  // an even-row and an odd-row MMA
    static constexpr int xpad = 16;
};

__device__ __forceinline__ void mma_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ void mma_k16_u8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}

// Scale and min of Q4_K sub-block s (a constant after unrolling) from the block header words
// h.y (scale bytes 0-3), h.z (4-7), h.w (8-11) (ggml get_scale_min_k4).
__device__ __forceinline__ void q4_sm(const uint4 &h, int s, int &sc, int &mn) {
    if (s < 4) {
        sc = (h.y >> (8 * s)) & 63;
        mn = (h.z >> (8 * s)) & 63;
    } else {
        const int i = 8 * (s - 4);
        sc = ((h.w >> i) & 15) | (((h.y >> (i + 6)) & 3) << 4);
        mn = ((h.w >> (i + 4)) & 15) | (((h.z >> (i + 6)) & 3) << 4);
    }
}

// Staged activations of up to TOKCAP tokens: qs [tok][K + xpad], d [K/256][TOKCAP],
// bs [K/sub][TOKCAP]: the Q8_K sums over each sub-block (32 elements for Q4_K, 16 for Q6_K).
struct XS {
    const int8_t *qs;
    const float *d;
    const int16_t *bs;
    int stride;  // K + xpad
    int tokcap;
};

// Fragment i of an m16n8 tile: MMA row g (i < 2) or g + 8 (i >= 2), token 2*t4 + (i & 1) of
// the 8-token group (g = lane / 4, t4 = lane % 4).
//
// Q4_K: 16 rows at m0 / m1 (row stride rs), tokens [tg, tg+8), super-blocks [b0, b1).  Inside a
// sub-block the k order is permuted identically for both operands (thread t4 holds elements
// 8*t4 .. 8*t4+7 of the 32), so each operand is one 8-byte load, and one load of the nibble bytes
// serves the low (2j) and high (2j+1) sub-blocks.
template <int NMAT>
__device__ __forceinline__ void q4_dot(const uint8_t *m0, const uint8_t *m1, int rs, const XS &x, int tg, int b0,
                                       int b1, float (&acc)[NMAT][4]) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
    const uint8_t *ra[NMAT], *rb[NMAT];
    ra[0] = m0 + (size_t)g * rs;
    rb[0] = m0 + (size_t)(g + 8) * rs;
    if constexpr (NMAT == 2) {
        ra[1] = m1 + (size_t)g * rs;
        rb[1] = m1 + (size_t)(g + 8) * rs;
    }
    const int8_t *xa = x.qs + (size_t)(tg + g) * x.stride;
    const int16_t *xbs = x.bs + tg + 2 * t4;
    for (int b = b0; b < b1; b++) {
        uint4 ha[NMAT], hb[NMAT];
#pragma unroll
        for (int m = 0; m < NMAT; m++) {
            ha[m] = *reinterpret_cast<const uint4 *>(ra[m] + b * TMOE_Q4K_BYTES);
            hb[m] = *reinterpret_cast<const uint4 *>(rb[m] + b * TMOE_Q4K_BYTES);
        }
        int isum[NMAT][4], msum[NMAT][4];
#pragma unroll
        for (int m = 0; m < NMAT; m++)
#pragma unroll
            for (int i = 0; i < 4; i++) isum[m][i] = msum[m][i] = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint2 xl = *reinterpret_cast<const uint2 *>(xa + 256 * b + 64 * j + 8 * t4);
            const uint2 xh = *reinterpret_cast<const uint2 *>(xa + 256 * b + 64 * j + 32 + 8 * t4);
            const uint32_t bl = *reinterpret_cast<const uint32_t *>(xbs + (size_t)(8 * b + 2 * j) * x.tokcap);
            const uint32_t bh = *reinterpret_cast<const uint32_t *>(xbs + (size_t)(8 * b + 2 * j + 1) * x.tokcap);
            const int Bl0 = (int)(int16_t)(bl & 0xffffu), Bl1 = (int)(int16_t)(bl >> 16);
            const int Bh0 = (int)(int16_t)(bh & 0xffffu), Bh1 = (int)(int16_t)(bh >> 16);
#pragma unroll
            for (int m = 0; m < NMAT; m++) {
                const uint2 wa = *reinterpret_cast<const uint2 *>(ra[m] + b * TMOE_Q4K_BYTES + 16 + 32 * j + 8 * t4);
                const uint2 wb = *reinterpret_cast<const uint2 *>(rb[m] + b * TMOE_Q4K_BYTES + 16 + 32 * j + 8 * t4);
                int dl[4], dh[4];
                mma_k32(dl, wa.x & NIB, wb.x & NIB, wa.y & NIB, wb.y & NIB, xl.x, xl.y);
                mma_k32(dh, (wa.x >> 4) & NIB, (wb.x >> 4) & NIB, (wa.y >> 4) & NIB, (wb.y >> 4) & NIB, xh.x, xh.y);
                int sla, mla, sha, mha, slb, mlb, shb, mhb;
                q4_sm(ha[m], 2 * j, sla, mla);
                q4_sm(ha[m], 2 * j + 1, sha, mha);
                q4_sm(hb[m], 2 * j, slb, mlb);
                q4_sm(hb[m], 2 * j + 1, shb, mhb);
                isum[m][0] += sla * dl[0] + sha * dh[0];
                isum[m][1] += sla * dl[1] + sha * dh[1];
                isum[m][2] += slb * dl[2] + shb * dh[2];
                isum[m][3] += slb * dl[3] + shb * dh[3];
                msum[m][0] += mla * Bl0 + mha * Bh0;
                msum[m][1] += mla * Bl1 + mha * Bh1;
                msum[m][2] += mlb * Bl0 + mhb * Bh0;
                msum[m][3] += mlb * Bl1 + mhb * Bh1;
            }
        }
        const float2 dx = *reinterpret_cast<const float2 *>(x.d + (size_t)b * x.tokcap + tg + 2 * t4);
#pragma unroll
        for (int m = 0; m < NMAT; m++) {
            const float da = h2f((uint16_t)(ha[m].x & 0xffffu)), ma = h2f((uint16_t)(ha[m].x >> 16));
            const float db = h2f((uint16_t)(hb[m].x & 0xffffu)), mb = h2f((uint16_t)(hb[m].x >> 16));
            acc[m][0] += __fmul_rn(da * dx.x, (float)isum[m][0]) - __fmul_rn(ma * dx.x, (float)msum[m][0]);
            acc[m][1] += __fmul_rn(da * dx.y, (float)isum[m][1]) - __fmul_rn(ma * dx.y, (float)msum[m][1]);
            acc[m][2] += __fmul_rn(db * dx.x, (float)isum[m][2]) - __fmul_rn(mb * dx.x, (float)msum[m][2]);
            acc[m][3] += __fmul_rn(db * dx.y, (float)isum[m][3]) - __fmul_rn(mb * dx.y, (float)msum[m][3]);
        }
    }
}

// Q6_K rows sit in 8-row groups (row_bytes = 210 * nb apart, group stride gs, a multiple of 4).
// A warp tile is 32 rows: the even rows form one MMA, the odd rows another, so that word
// alignment is uniform across each MMA's rows: a block starts 2 bytes off a word boundary iff
// row * nb + block is odd, and those words are realigned with a funnel shift.  Thread t4 holds
// elements 4*t4 .. 4*t4+3 of a 16-element sub-block.  Per half block and row, four nibble words
// (each serving the low and the high nibble sub-block) and two high-bit words (each serving four
// sub-blocks) cover the eight sub-blocks.
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

// Unsigned 6-bit values (0..63) of sub-block sl8 (0..7, a constant after unrolling) of the half.
__device__ __forceinline__ uint32_t q6_vals(const Q6Half &q, int sl8) {
    const uint32_t lo = (q.ql[sl8 & 3] >> (sl8 >= 4 ? 4 : 0)) & NIB;
    const uint32_t hi = ((q.qh[sl8 & 1] >> (2 * (sl8 >> 1))) & 0x03030303u) << 4;
    return lo | hi;
}

__device__ __forceinline__ int q6_scale(const Q6Half &q, int sl8) {
    return (int)(int8_t)((q.sc[sl8 >> 2] >> (8 * (sl8 & 3))) & 0xffu);
}

template <int NMAT>
__device__ __forceinline__ void q6_dot(const uint8_t *m0, const uint8_t *m1, int gs, int row_bytes, int nb, int rbase,
                                       const XS &x, int tg, int s0, int s1, float (&acc_e)[NMAT][4],
                                       float (&acc_o)[NMAT][4]) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
    const uint8_t *mats[2] = {m0, m1};
    // rows: even MMA 2g, 2g+16; odd MMA 2g+1, 2g+17 (tile-relative, + rbase)
    const uint8_t *rows[NMAT][4];
#pragma unroll
    for (int m = 0; m < NMAT; m++) {
        const int rr[4] = {rbase + 2 * g, rbase + 2 * g + 16, rbase + 2 * g + 1, rbase + 2 * g + 17};
#pragma unroll
        for (int k = 0; k < 4; k++) rows[m][k] = mats[m] + (size_t)(rr[k] >> 3) * gs + (size_t)(rr[k] & 7) * row_bytes;
    }
    const int8_t *xa = x.qs + (size_t)(tg + g) * x.stride;
    const int16_t *xbs = x.bs + tg + 2 * t4;
    for (int b = s0 >> 4; b * 16 < s1; b++) {
        const bool mis_e = (b & 1) != 0, mis_o = ((nb & 1) != 0) != ((b & 1) != 0);
        int isum[NMAT][2][4], corr[NMAT][2][4];
#pragma unroll
        for (int m = 0; m < NMAT; m++)
#pragma unroll
            for (int p = 0; p < 2; p++)
#pragma unroll
                for (int i = 0; i < 4; i++) isum[m][p][i] = corr[m][p][i] = 0;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int base = 16 * b + 8 * h;
            const int lo = max(s0 - base, 0), hi = min(s1 - base, 8);
            if (lo >= hi) continue;
            Q6Half q[NMAT][4];
#pragma unroll
            for (int m = 0; m < NMAT; m++)
#pragma unroll
                for (int k = 0; k < 4; k++)
                    q6_load_half(rows[m][k] + b * TMOE_Q6K_BYTES, h, t4, k < 2 ? mis_e : mis_o, q[m][k]);
#pragma unroll
            for (int sl8 = 0; sl8 < 8; sl8++) {
                if (sl8 < lo || sl8 >= hi) continue;
                const int s = base + sl8;
                const uint32_t xw = *reinterpret_cast<const uint32_t *>(xa + 16 * s + 4 * t4);
                const uint32_t bw = *reinterpret_cast<const uint32_t *>(xbs + (size_t)s * x.tokcap);
                const int B0 = (int)(int16_t)(bw & 0xffffu), B1 = (int)(int16_t)(bw >> 16);
#pragma unroll
                for (int m = 0; m < NMAT; m++) {
#pragma unroll
                    for (int p = 0; p < 2; p++) {  // p = 0 even rows, 1 odd rows
                        int d[4];
                        mma_k16_u8(d, q6_vals(q[m][2 * p], sl8), q6_vals(q[m][2 * p + 1], sl8), xw);
                        const int sca = q6_scale(q[m][2 * p], sl8), scb = q6_scale(q[m][2 * p + 1], sl8);
                        isum[m][p][0] += sca * d[0];
                        isum[m][p][1] += sca * d[1];
                        isum[m][p][2] += scb * d[2];
                        isum[m][p][3] += scb * d[3];
                        corr[m][p][0] += sca * B0;
                        corr[m][p][1] += sca * B1;
                        corr[m][p][2] += scb * B0;
                        corr[m][p][3] += scb * B1;
                    }
                }
            }
        }
        const float2 dx = *reinterpret_cast<const float2 *>(x.d + (size_t)b * x.tokcap + tg + 2 * t4);
#pragma unroll
        for (int m = 0; m < NMAT; m++) {
#pragma unroll
            for (int p = 0; p < 2; p++) {
                const float da = h2f(*reinterpret_cast<const uint16_t *>(rows[m][2 * p] + b * TMOE_Q6K_BYTES + 208));
                const float db = h2f(*reinterpret_cast<const uint16_t *>(rows[m][2 * p + 1] + b * TMOE_Q6K_BYTES + 208));
                float(&acc)[NMAT][4] = p == 0 ? acc_e : acc_o;
                acc[m][0] += __fmul_rn(da * dx.x, (float)(isum[m][p][0] - 32 * corr[m][p][0]));
                acc[m][1] += __fmul_rn(da * dx.y, (float)(isum[m][p][1] - 32 * corr[m][p][1]));
                acc[m][2] += __fmul_rn(db * dx.x, (float)(isum[m][p][2] - 32 * corr[m][p][2]));
                acc[m][3] += __fmul_rn(db * dx.y, (float)(isum[m][p][3] - 32 * corr[m][p][3]));
            }
        }
    }
}

__device__ __forceinline__ float silu_mul(float g, float u) { return (g / (1.0f + expf(-g))) * u; }

// Named barrier 1 over the consumer warps.  Each warp reconverges first (__syncwarp): lanes can
// leave a polling loop or a strided loop on different iterations, and the barrier must not see a
// diverged warp.  The non-.aligned barrier forms are used as well, which tolerate divergence.
// consumers_all: the AND of `ok` over all consumer threads.
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
__device__ __forceinline__ void consumers_sync() {
    __syncwarp();
    asm volatile("barrier.sync 1, %0;" ::"n"(GEMV_NW * 32) : "memory");
}

template <int WT, bool GATEUP, int WK, int MINB>
__global__ void __launch_bounds__(GEMV_THREADS, MINB) gemv_kernel(const GemvArgs a) {
    constexpr int WR = GEMV_NW / WK;
    constexpr int TR = Fmt<WT>::tile_rows;
    constexpr int RT = WR * TR;
    constexpr int NMAT = GATEUP ? 2 : 1;
    constexpr int SUB = Fmt<WT>::sub;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + GEMV_MAX_STAGES;
    uint8_t *stage0 = smem + GEMV_BAR_BYTES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NS = a.n_stages, K = a.K, TOKCAP = a.tokcap;
    const int row_bytes = Fmt<WT>::block_bytes * (K / TMOE_QK);
    const int rstride = a.row_stride;  // Q4_K: padded row stride; Q6_K: 8-row group stride
    const int mat_bytes = a.mat_stride;
    const int XST = K + Fmt<WT>::xpad;
    // after the stages: activations, then the cross-warp reduction buffer
    uint8_t *xbase = stage0 + (size_t)NS * a.stage_bytes;
    int8_t *xqs = reinterpret_cast<int8_t *>(xbase);
    float *xd = reinterpret_cast<float *>(xqs + (size_t)TOKCAP * XST);
    int16_t *xsb = reinterpret_cast<int16_t *>(xd + (size_t)(K / TMOE_QK) * TOKCAP);
    int *xp = reinterpret_cast<int *>(xsb + (size_t)(K / SUB) * TOKCAP);
    float *red = reinterpret_cast<float *>(xp + TOKCAP);  // [NMAT][WK][RT][TOKG]
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], GEMV_NW);
        }
        fence_barrier_init();
    }
    __syncthreads();
    // The dispatch data are checked before they become addresses: an active count above the
    // grid's sizing or an expert outside [0, n_slots) latches TMOE_DEV_ERR_BADID and the item is
    // skipped (its stage still completes and is released, so the pipeline stays in step).
    int na = a.n_active[0];
    if (na > a.max_active || na < 0) {
        if (threadIdx.x == 0 && blockIdx.x == 0) latch_error(a.err, TMOE_DEV_ERR_BADID);
        na = na < 0 ? 0 : a.max_active;
    }
    const int n_items = na * a.tiles;
    const int i0 = (int)(((int64_t)blockIdx.x * n_items) / gridDim.x);
    const int i1 = (int)(((int64_t)(blockIdx.x + 1) * n_items) / gridDim.x);

    if (warp == GEMV_NW) {  // producer
        if (lane == 0) {
            int it = 0;
            for (int item = i0; item < i1; ++item, ++it) {
                const int s = it % NS;
                if (it >= NS && !mbar_wait_bounded(&empty[s], ((it / NS) - 1) & 1)) {
                    latch_error(a.err, TMOE_DEV_ERR_TIMEOUT);
                    break;
                }
                const int e = a.active[item / a.tiles];
                const int r0 = (item % a.tiles) * RT;
                uint8_t *dst = stage0 + (size_t)s * a.stage_bytes;
                if (e < 0 || e >= a.n_slots) {  // nothing to load: complete the phase empty
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
    const int n_sub = K / SUB;
    const int ks0 = (n_sub * wk) / WK, ks1 = (n_sub * (wk + 1)) / WK;  // sub-block slice
    const int ctid = threadIdx.x;
    const XS xs{xqs, xd, xsb, XST, TOKCAP};
    const int g = lane >> 2, t4 = lane & 3;
    int staged_e = -1, staged_beg = -1;
    int it = 0;
    for (int item = i0; item < i1; ++item, ++it) {
        const int s = it % NS;
        const bool ok = mbar_wait_bounded(&full[s], (it / NS) & 1);
        if (!consumers_all(ok)) {
            if (lane == 0) latch_error(a.err, TMOE_DEV_ERR_TIMEOUT);
            break;
        }
        const int e = a.active[item / a.tiles];
        const int r0 = (item % a.tiles) * RT;
        const uint8_t *st = stage0 + (size_t)s * a.stage_bytes;
        const bool e_ok = e >= 0 && e < a.n_slots;
        int beg = e_ok ? a.offsets[e] : 0, end = e_ok ? a.offsets[e + 1] : 0;
        if (beg < 0 || end > a.n_pairs || end < beg) beg = end = 0;
        if (beg == end) {  // nothing to compute: release the stage
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            continue;
        }
        for (int cb = beg; cb < end; cb += TOKCAP) {
            const int n = min(TOKCAP, end - cb);
            if (!(staged_e == e && staged_beg == cb)) {
                consumers_sync();  // everyone is done with the previous activations
                for (int q = ctid; q < n; q += 32 * GEMV_NW) {
                    const int p = a.perm[cb + q];
                    xp[q] = (p >= 0 && p < a.n_pairs) ? p : 0;
                }
                consumers_sync();
                if (a.xf) {
                    // f32 rows: Q8_K here, one warp per (token, 256-block) (the activation of the
                    // down projection, quantised where it is consumed)
                    const int nb = K / TMOE_QK;
                    for (int u = warp; u < n * nb; u += GEMV_NW) {
                        const int q = u / nb, b = u % nb;
                        const int64_t xr = xp[q] / a.x_div;
                        const float4 *src = reinterpret_cast<const float4 *>(a.xf + xr * K + b * TMOE_QK) + 2 * lane;
                        const float4 f0 = __ldg(src), f1 = __ldg(src + 1);
                        const float v[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
                        uint2 qv;
                        float dd;
                        int s16;
                        q8k_block_warp(v, qv, dd, s16);
                        *reinterpret_cast<uint2 *>(xqs + (size_t)q * XST + b * TMOE_QK + 8 * lane) = qv;
                        if (lane == 0) xd[b * TOKCAP + q] = dd;
                        if constexpr (SUB == 16) {
                            if ((lane & 1) == 0) xsb[(16 * b + lane / 2) * TOKCAP + q] = (int16_t)s16;
                        } else {
                            const int s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 2);
                            if ((lane & 3) == 0) xsb[(8 * b + lane / 4) * TOKCAP + q] = (int16_t)s32;
                        }
                    }
                } else {
                    const int v16 = K / 16;
                    for (int idx = ctid; idx < n * v16; idx += 32 * GEMV_NW) {
                        const int q = idx / v16, c = idx % v16;
                        const int64_t xr = xp[q] / a.x_div;
                        reinterpret_cast<uint4 *>(xqs + (size_t)q * XST)[c] =
                            __ldg(reinterpret_cast<const uint4 *>(a.xq + xr * K) + c);
                    }
                    for (int idx = ctid; idx < n * (K / TMOE_QK); idx += 32 * GEMV_NW) {
                        const int q = idx / (K / TMOE_QK), b = idx % (K / TMOE_QK);
                        const int64_t xr = xp[q] / a.x_div;
                        xd[b * TOKCAP + q] = __ldg(a.xd + xr * (K / TMOE_QK) + b);
                    }
                    for (int idx = ctid; idx < n * n_sub; idx += 32 * GEMV_NW) {
                        const int q = idx / n_sub, sb = idx % n_sub;
                        const int64_t xr = xp[q] / a.x_div;
                        if constexpr (SUB == 32) {  // Q4_K: sum of the two 16-element block sums
                            const uint32_t two = __ldg(reinterpret_cast<const uint32_t *>(a.xb + xr * (K / 16)) + sb);
                            xsb[sb * TOKCAP + q] = (int16_t)((int)(int16_t)(two & 0xffffu) + (int)(int16_t)(two >> 16));
                        } else {
                            xsb[sb * TOKCAP + q] = __ldg(a.xb + xr * (K / 16) + sb);
                        }
                    }
                }
                consumers_sync();
                staged_e = e;
                staged_beg = cb;
            }
            for (int tg = 0; tg < n; tg += TOKG) {
                if constexpr (WT == TMOE_WT_Q4K) {
                    float acc[NMAT][4];
#pragma unroll
                    for (int m = 0; m < NMAT; m++) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.0f;
                    q4_dot<NMAT>(st + (size_t)(wr * TR) * rstride, st + mat_bytes + (size_t)(wr * TR) * rstride,
                                 rstride, xs, tg, ks0 / 8, ks1 / 8, acc);
#pragma unroll
                    for (int m = 0; m < NMAT; m++) {
                        float *rd = red + ((size_t)(m * WK + wk) * RT) * TOKG;
                        const int rA = wr * TR + g, rB = rA + 8;
                        *reinterpret_cast<float2 *>(rd + (size_t)rA * TOKG + 2 * t4) = make_float2(acc[m][0], acc[m][1]);
                        *reinterpret_cast<float2 *>(rd + (size_t)rB * TOKG + 2 * t4) = make_float2(acc[m][2], acc[m][3]);
                    }
                } else {
                    float acc_e[NMAT][4], acc_o[NMAT][4];
#pragma unroll
                    for (int m = 0; m < NMAT; m++)
#pragma unroll
                        for (int i = 0; i < 4; i++) acc_e[m][i] = acc_o[m][i] = 0.0f;
                    q6_dot<NMAT>(st, st + mat_bytes, rstride, row_bytes, K / TMOE_QK, wr * TR, xs, tg, ks0, ks1,
                                 acc_e, acc_o);
                    // MMA row g -> tile row 2g, row g+8 -> 2g+16; the odd MMA one row below
#pragma unroll
                    for (int m = 0; m < NMAT; m++) {
                        float *rd = red + ((size_t)(m * WK + wk) * RT) * TOKG;
                        const int rA = wr * TR + 2 * g, rB = rA + 16;
                        *reinterpret_cast<float2 *>(rd + (size_t)rA * TOKG + 2 * t4) = make_float2(acc_e[m][0], acc_e[m][1]);
                        *reinterpret_cast<float2 *>(rd + (size_t)rB * TOKG + 2 * t4) = make_float2(acc_e[m][2], acc_e[m][3]);
                        *reinterpret_cast<float2 *>(rd + (size_t)(rA + 1) * TOKG + 2 * t4) =
                            make_float2(acc_o[m][0], acc_o[m][1]);
                        *reinterpret_cast<float2 *>(rd + (size_t)(rB + 1) * TOKG + 2 * t4) =
                            make_float2(acc_o[m][2], acc_o[m][3]);
                    }
                }
                if (tg + TOKG >= n && cb + TOKCAP >= end) {  // last read of the stage
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[s]);
                }
                consumers_sync();
                // sum the WK slices in order and write the (row, token) outputs
                const int ntok = min(TOKG, n - tg);
                for (int o = ctid; o < RT * TOKG; o += 32 * GEMV_NW) {
                    const int row = o / TOKG, tk = o % TOKG;
                    if (tk >= ntok) continue;
                    float v0 = 0.0f, v1 = 0.0f;
#pragma unroll
                    for (int k = 0; k < WK; k++) {
                        v0 += red[((size_t)k * RT + row) * TOKG + tk];
                        if constexpr (GATEUP) v1 += red[((size_t)(WK + k) * RT + row) * TOKG + tk];
                    }
                    const int p = xp[tg + tk];
                    a.out[(int64_t)p * a.N + r0 + row] = GATEUP ? silu_mul(v0, v1) : v0;
                }
                consumers_sync();  // the reduction buffer is free again
            }
        }
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

struct Plan {
    int tokcap, n_stages;
    size_t smem;
};

// Shared memory per CTA for a given activation capacity; false if two stages do not fit `budget`.
template <int WT, bool GATEUP, int WK>
static bool plan_smem(const GemvArgs &a, int tokcap, uint32_t budget, Plan &p) {
    constexpr int RT = (GEMV_NW / WK) * Fmt<WT>::tile_rows;
    constexpr int NMAT = GATEUP ? 2 : 1;
    const int XST = a.K + Fmt<WT>::xpad;
    const size_t xb = (size_t)tokcap * XST + (size_t)(a.K / TMOE_QK) * tokcap * 4 +
                      (size_t)(a.K / Fmt<WT>::sub) * tokcap * 2 + (size_t)tokcap * 4 + 16;
    const size_t redb = (size_t)NMAT * WK * RT * TOKG * 4 + 16;
    if (GEMV_BAR_BYTES + xb + redb + 2 * (size_t)a.stage_bytes > budget) return false;
    int ns = (int)((budget - GEMV_BAR_BYTES - xb - redb) / a.stage_bytes);
    if (ns > GEMV_MAX_STAGES) ns = GEMV_MAX_STAGES;
    p.tokcap = tokcap;
    p.n_stages = ns;
    p.smem = GEMV_BAR_BYTES + (size_t)ns * a.stage_bytes + xb + redb;
    return true;
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
    // Two CTAs per SM when two stages and the activations of 16 (else 8) tokens fit in half the
    // shared memory and the two-CTA build does not spill; else one CTA with 16 (else 8) tokens.
    Plan p{};
    bool two = plan_smem<WT, GATEUP, WK>(a, 16, GEMV_SMEM_2CTA, p) || plan_smem<WT, GATEUP, WK>(a, 8, GEMV_SMEM_2CTA, p);
    if (two) {
        static int spills = -1;
        if (spills < 0) {
            cudaFuncAttributes fa{};
            spills = cudaFuncGetAttributes(&fa, gemv_kernel<WT, GATEUP, WK, 2>) != cudaSuccess || fa.localSizeBytes > 32;
        }
        two = !spills;
    }
    if (!two && !plan_smem<WT, GATEUP, WK>(a, 16, GEMV_SMEM_1CTA, p) &&
        !plan_smem<WT, GATEUP, WK>(a, 8, GEMV_SMEM_1CTA, p))
        return cudaErrorInvalidValue;
    a.tokcap = p.tokcap;
    a.n_stages = p.n_stages;
    const int items = max_items * a.tiles;
    const int slots = sm_count * (two ? 2 : 1);
    const int grid = items < slots ? items : slots;
    if (grid < 1) return cudaSuccess;
    static int cache1[64] = {}, cache2[64] = {};
    cudaError_t e;
    if (two) {
        if ((e = set_smem_once(gemv_kernel<WT, GATEUP, WK, 2>, p.smem, cache2)) != cudaSuccess) return e;
        gemv_kernel<WT, GATEUP, WK, 2><<<grid, GEMV_THREADS, p.smem, st>>>(a);
    } else {
        if ((e = set_smem_once(gemv_kernel<WT, GATEUP, WK, 1>, p.smem, cache1)) != cudaSuccess) return e;
        gemv_kernel<WT, GATEUP, WK, 1><<<grid, GEMV_THREADS, p.smem, st>>>(a);
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
