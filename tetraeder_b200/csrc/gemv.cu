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
// Work: items = (active expert, 16-row tile), expert-major.  An item covers all of K, so a warp
// owns its rows' sums and nothing is reduced across warps.  Each warp runs its own pipeline: it
// takes items from a global counter (dynamic balancing: items differ in token count) and
// streams their rows through its own ring of shared-memory slots with TMA, refilling a slot as
// soon as it has read it.  A fill is the item's 16 rows over a span of K:
//  - Q4_K: a chunk of super-blocks, one 3D tiled TMA copy per matrix (tensor map over
//    [expert][row][row bytes as u32]);
//  - Q6_K: all of K, one 1D bulk copy per matrix (16 consecutive rows are contiguous and a
//    multiple of 16 bytes; a chunk of one row is not even 4-byte aligned);
//  - Q6_K in 8-row fragment order (tmoe_prepack): all of K, one 1D bulk copy per 8-row group, read
//    with aligned vector loads free of bank conflicts (C2 T = 64: down 50.4 us against 54.3).
// gate/up items take rows r..r+7 of gate as MMA rows 0-7 and the same rows of up as MMA rows
// 8-15, so silu(g) * u (swiglu_split) is formed in the thread that holds both.
// Tokens: up to 16 per pass (two 8-token MMA groups); an expert with more tokens runs more
// passes over the same rows (L2-resident the second time).
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.cuh"

namespace tmoe {

constexpr int GEMV_NW = 8;  // warps per CTA, each an independent pipeline
constexpr int GEMV_THREADS = 32 * GEMV_NW;
constexpr int GEMV_MAXD = 6;    // slots per warp
constexpr int GEMV_HDR = 2048;  // mbarriers and slot records
constexpr int TOKG = 8;         // tokens per MMA (the n of m16n8)
constexpr int ITEM_ROWS = 16;   // rows per item (gate/up: 8 of each)
constexpr int Q4_CHUNK_U32 = TMOE_Q4K_BYTES / 4;  // tensor-map elements per Q4_K super-block
constexpr uint32_t NIB = 0x0f0f0f0fu;
constexpr unsigned FULL = 0xffffffffu;

// What a fill holds, written by lane 0 before the arrive on the slot's barrier.  At chunk 0 of a
// pass the fill also carries the pass's pair indices (perm[beg + 16 * pass ...], a bulk copy
// rounded out to 16 bytes; poff = where the first one landed, in ints).
struct SlotRec {
    int item, tile, pass, chunk, beg, end, poff, r0;
};
static_assert(GEMV_NW * GEMV_MAXD * (8 + (int)sizeof(SlotRec)) + 8 * 8 + 4 * GEMV_NW <= GEMV_HDR, "header");
// Bytes after a slot's weights for the pass's pair indices.  Q4_K slots stay multiples of 128
// bytes: a tensor-map copy (the Q4_K fills) must land on a 128-byte boundary of shared memory.
constexpr int PERM_STAGE = 128;
static_assert(ITEM_ROWS * TMOE_Q4K_BYTES % 128 == 0 && PERM_STAGE % 128 == 0, "Q4_K slots on 128-byte boundaries");

// Tensor maps of the Q4_K matrices (unused for Q6_K).
struct GemvMaps {
    CUtensorMap m[2];
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

// Byte i of w, zero-extended / sign-extended (prmt: a selector nibble with bit 3 set replicates
// the selected byte's sign bit).
__device__ __forceinline__ int ubyte(uint32_t w, int i) { return (int)__byte_perm(w, 0u, 0x4440u | (uint32_t)i); }
__device__ __forceinline__ int sbyte(uint32_t w, int i) {
    const uint32_t s = (uint32_t)i | ((8u | i) << 4) | ((8u | i) << 8) | ((8u | i) << 12);
    uint32_t r;
    asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "r"(s));
    return (int)r;
}

// n / d for 0 <= n < 2^24 and 1 <= d <= 2^16 with m = ceil(2^40 / d): the error of m / 2^40 is
// below 2^-40, times n below 2^-16 <= 1/d, which does not carry past the next multiple of d.
__device__ __forceinline__ int fast_div(int n, uint64_t m) { return (int)(((uint64_t)(uint32_t)n * m) >> 40); }

__device__ __forceinline__ uint2 ldg64(const void *p) { return __ldg(reinterpret_cast<const uint2 *>(p)); }
__device__ __forceinline__ uint4 ldg128(const void *p) { return __ldg(reinterpret_cast<const uint4 *>(p)); }

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *m, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// The token columns of one 8-token group as a thread sees them: the activation row of column g
// (its B operand), of columns 2*t4 and 2*t4+1 (its fragments' d), and those columns' pair rows
// in the output (-1: past the group's end).
struct TokCols {
    int xg, x0, x1;
    int pp0, pp1;
};

// The same group's activation data as this thread's base pointers, set once per pass (super-block
// kb then sits at a fixed stride from each): the B-operand row of column g at the thread's k
// offset (Q6_K rows are stored in fragment order, q8_frag_pos: the thread's 64 bytes of each
// block), that row's sub-block sum words (2 per super-block for Q4_K, 4 for Q6_K, the thread's
// one), and the super-block scales of columns 2*t4 and 2*t4+1.
struct XBase {
    const int8_t *q;
    const uint32_t *bl, *bh;
    const float *d0, *d1;
};

template <int WT>
__device__ __forceinline__ XBase x_base(const GemvArgs &a, const TokCols &c, int nb) {
    const int t4 = threadIdx.x & 3;
    constexpr int NBW = WT == TMOE_WT_Q4K ? 2 : 4;
    const int64_t sw = (int64_t)c.xg * nb * NBW + (WT == TMOE_WT_Q4K ? (t4 & 1) : t4);
    XBase p;
    p.q = a.xq + (int64_t)c.xg * a.K + (WT == TMOE_WT_Q4K ? 8 : 64) * t4;
    p.bl = a.xbl + sw;
    p.bh = a.xbh + sw;
    p.d0 = a.xd + (int64_t)c.x0 * nb;
    p.d1 = a.xd + (int64_t)c.x1 * nb;
    return p;
}

// ------------------------------------------------------------------ Q4_K
// Per super-block and 8-token group: a thread's B operands.  Inside a sub-block the k order is
// permuted identically for both operands (thread t4 holds elements 8*t4 .. 8*t4+7 of the 32),
// so each weight operand is one 8-byte load, and one load of the nibble bytes serves sub-blocks
// 2j (low nibbles) and 2j+1 (high nibbles).
struct XQ4 {
    uint2 l[4], h[4];
    uint32_t bl, bh;
    float d0, d1;
};

// From the token columns directly (two-group passes: fewer live registers than kept bases).
__device__ __forceinline__ void load_xq4(const GemvArgs &a, const TokCols &c, int kb, int nb, XQ4 &o) {
    const int t4 = threadIdx.x & 3;
    const int8_t *q = a.xq + (int64_t)c.xg * a.K + TMOE_QK * kb + 8 * t4;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        o.l[j] = ldg64(q + 64 * j);
        o.h[j] = ldg64(q + 64 * j + 32);
    }
    const int64_t w = ((int64_t)c.xg * nb + kb) * 2 + (t4 & 1);
    o.bl = t4 < 2 ? __ldg(a.xbl + w) : 0u;
    o.bh = t4 < 2 ? __ldg(a.xbh + w) : 0u;
    o.d0 = __ldg(a.xd + (int64_t)c.x0 * nb + kb);
    o.d1 = __ldg(a.xd + (int64_t)c.x1 * nb + kb);
}

// From kept bases; lo: t4 < 2 (the threads whose B operand of the min MMAs holds the 8 sub-block
// sums).
__device__ __forceinline__ void load_xq4(const XBase &p, int kb, bool lo, XQ4 &o) {
    const int8_t *q = p.q + TMOE_QK * kb;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        o.l[j] = ldg64(q + 64 * j);
        o.h[j] = ldg64(q + 64 * j + 32);
    }
    o.bl = lo ? __ldg(p.bl + 2 * kb) : 0u;
    o.bh = lo ? __ldg(p.bh + 2 * kb) : 0u;
    o.d0 = __ldg(p.d0 + kb);
    o.d1 = __ldg(p.d1 + kb);
}

// One super-block of MMA rows g (at ra) and g+8 (at rb) against NGR token groups.
//  - The high nibbles go to the MMA in place (byte & 0xf0 = 16 * q, unsigned): those products
//    are 16 times too large and the super-block's sum of them is shifted right by 4, exactly.
//  - The 6-bit scales and mins are unpacked once per row into byte-packed words.
//  - The min term sum_s m_s * B_s is two small MMAs (k = 16: 8 sub-blocks and 8 zeros):
//    mins x lo bytes + 64 * (mins x hi bytes), B_s = 64 * hi + lo.
template <int NGR>
__device__ __forceinline__ void q4_block(const uint8_t *ra, const uint8_t *rb, const XQ4 (&x)[NGR],
                                         float (*acc)[4]) {
    const int t4 = threadIdx.x & 3;
    const uint4 ha = *reinterpret_cast<const uint4 *>(ra);
    const uint4 hb = *reinterpret_cast<const uint4 *>(rb);
    const uint32_t sca0 = ha.y & 0x3f3f3f3fu, sca1 = (ha.w & 0x0f0f0f0fu) | ((ha.y >> 2) & 0x30303030u);
    const uint32_t scb0 = hb.y & 0x3f3f3f3fu, scb1 = (hb.w & 0x0f0f0f0fu) | ((hb.y >> 2) & 0x30303030u);
    int il[NGR][4], ih[NGR][4];
#pragma unroll
    for (int G = 0; G < NGR; G++)
#pragma unroll
        for (int i = 0; i < 4; i++) il[G][i] = ih[G][i] = 0;
    if constexpr (NGR == 1) {  // one group: both sub-block pairs' MMAs before their scale multiply-adds
#pragma unroll
        for (int jj = 0; jj < 4; jj += 2) {
            int dl[2][4], dh[2][4];
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int j = jj + u;
                const uint2 wa = *reinterpret_cast<const uint2 *>(ra + 16 + 32 * j + 8 * t4);
                const uint2 wb = *reinterpret_cast<const uint2 *>(rb + 16 + 32 * j + 8 * t4);
                mma_k32_u8s8(dl[u], wa.x & NIB, wb.x & NIB, wa.y & NIB, wb.y & NIB, x[0].l[j].x, x[0].l[j].y);
                mma_k32_u8s8(dh[u], wa.x & ~NIB, wb.x & ~NIB, wa.y & ~NIB, wb.y & ~NIB, x[0].h[j].x, x[0].h[j].y);
            }
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int j = jj + u;
                const uint32_t sa = j < 2 ? sca0 : sca1, sb = j < 2 ? scb0 : scb1;
                const int bi = 2 * (j & 1);
                const int sla = ubyte(sa, bi), sha = ubyte(sa, bi + 1);
                const int slb = ubyte(sb, bi), shb = ubyte(sb, bi + 1);
                il[0][0] += sla * dl[u][0];
                il[0][1] += sla * dl[u][1];
                il[0][2] += slb * dl[u][2];
                il[0][3] += slb * dl[u][3];
                ih[0][0] += sha * dh[u][0];
                ih[0][1] += sha * dh[u][1];
                ih[0][2] += shb * dh[u][2];
                ih[0][3] += shb * dh[u][3];
            }
        }
    } else
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint2 wa = *reinterpret_cast<const uint2 *>(ra + 16 + 32 * j + 8 * t4);
        const uint2 wb = *reinterpret_cast<const uint2 *>(rb + 16 + 32 * j + 8 * t4);
        const uint32_t sa = j < 2 ? sca0 : sca1, sb = j < 2 ? scb0 : scb1;
        const int bi = 2 * (j & 1);
        const int sla = ubyte(sa, bi), sha = ubyte(sa, bi + 1);
        const int slb = ubyte(sb, bi), shb = ubyte(sb, bi + 1);
#pragma unroll
        for (int G = 0; G < NGR; G++) {
            int dl[4], dh[4];
            mma_k32_u8s8(dl, wa.x & NIB, wb.x & NIB, wa.y & NIB, wb.y & NIB, x[G].l[j].x, x[G].l[j].y);
            mma_k32_u8s8(dh, wa.x & ~NIB, wb.x & ~NIB, wa.y & ~NIB, wb.y & ~NIB, x[G].h[j].x, x[G].h[j].y);
            il[G][0] += sla * dl[0];
            il[G][1] += sla * dl[1];
            il[G][2] += slb * dl[2];
            il[G][3] += slb * dl[3];
            ih[G][0] += sha * dh[0];
            ih[G][1] += sha * dh[1];
            ih[G][2] += shb * dh[2];
            ih[G][3] += shb * dh[3];
        }
    }
    const uint32_t mna0 = ha.z & 0x3f3f3f3fu, mna1 = ((ha.w >> 4) & 0x0f0f0f0fu) | ((ha.z >> 2) & 0x30303030u);
    const uint32_t mnb0 = hb.z & 0x3f3f3f3fu, mnb1 = ((hb.w >> 4) & 0x0f0f0f0fu) | ((hb.z >> 2) & 0x30303030u);
    const uint32_t a0 = t4 == 0 ? mna0 : (t4 == 1 ? mna1 : 0u);
    const uint32_t a1 = t4 == 0 ? mnb0 : (t4 == 1 ? mnb1 : 0u);
    const float da = h2f((uint16_t)(ha.x & 0xffffu)), ma = h2f((uint16_t)(ha.x >> 16));
    const float db = h2f((uint16_t)(hb.x & 0xffffu)), mb = h2f((uint16_t)(hb.x >> 16));
#pragma unroll
    for (int G = 0; G < NGR; G++) {
        int ml[4], mh[4];
        mma_k16_u8u8(ml, a0, a1, x[G].bl);
        mma_k16_u8s8(mh, a0, a1, x[G].bh);
        // fragment i: row a (i < 2) or b, token column i & 1: acc += dx * (d * isum - dmin * msum)
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int isum = il[G][i] + (ih[G][i] >> 4), msum = ml[i] + 64 * mh[i];
            const float dr = i < 2 ? da : db, mr = i < 2 ? ma : mb;
            const float t = __fmaf_rn(-mr, (float)msum, __fmul_rn(dr, (float)isum));
            acc[G][i] = __fmaf_rn((i & 1) ? x[G].d1 : x[G].d0, t, acc[G][i]);
        }
    }
}

// ------------------------------------------------------------------ Q6_K
// Thread t4 holds elements 4*t4 .. 4*t4+3 of a 16-element sub-block.  Super-block b of row r
// starts 2 bytes off a word boundary iff r * nb + b is odd (210-byte blocks; fills start at a
// row that is a multiple of 8), and such words are read as two aligned words and a funnel shift.
// Down items put the even rows on MMA rows g and the odd rows on g+8, so that each operand's
// alignment is the same across the warp (MA, MB: 0 aligned, 1 off by two); gate/up pairs rows of
// both parities in one MMA, and there each thread shifts by its own row's offset (2).
// Per half block (8 sub-blocks) and row: 4 nibble words (each serving a low and a high nibble
// sub-block), 2 high-bit words (each serving four sub-blocks) and 2 scale words.  The raw 6-bit
// values go to the MMA unsigned; the -32 bias is applied as -32 * sum_s sc_s * B_s, and that sum
// is two small MMAs (k = 16 = the block's sub-blocks).
struct XQ6 {
    uint32_t w[16];
    uint32_t bl, bh;
    float d0, d1;
};

__device__ __forceinline__ void load_xq6(const GemvArgs &a, const TokCols &c, int kb, int nb, XQ6 &o) {
    const int t4 = threadIdx.x & 3;
    const int8_t *q = a.xq + (int64_t)c.xg * a.K + TMOE_QK * kb + 64 * t4;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint4 v = ldg128(q + 16 * i);
        o.w[4 * i] = v.x, o.w[4 * i + 1] = v.y, o.w[4 * i + 2] = v.z, o.w[4 * i + 3] = v.w;
    }
    const int64_t w = ((int64_t)c.xg * nb + kb) * 4 + t4;
    o.bl = __ldg(a.xbl + w);
    o.bh = __ldg(a.xbh + w);
    o.d0 = __ldg(a.xd + (int64_t)c.x0 * nb + kb);
    o.d1 = __ldg(a.xd + (int64_t)c.x1 * nb + kb);
}

__device__ __forceinline__ void load_xq6(const XBase &p, int kb, XQ6 &o) {
    const int8_t *q = p.q + TMOE_QK * kb;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint4 v = ldg128(q + 16 * i);
        o.w[4 * i] = v.x, o.w[4 * i + 1] = v.y, o.w[4 * i + 2] = v.z, o.w[4 * i + 3] = v.w;
    }
    o.bl = __ldg(p.bl + 4 * kb);
    o.bh = __ldg(p.bh + 4 * kb);
    o.d0 = __ldg(p.d0 + kb);
    o.d1 = __ldg(p.d1 + kb);
}

// 32-bit word at p (2-byte aligned); MIS 0: p is word aligned, 1: p is 2 bytes off, 2: either.
template <int MIS>
__device__ __forceinline__ uint32_t ld32(const uint8_t *p) {
    if constexpr (MIS == 0) {
        return *reinterpret_cast<const uint32_t *>(p);
    } else if constexpr (MIS == 1) {
        const uint32_t *w = reinterpret_cast<const uint32_t *>(p - 2);
        return __funnelshift_r(w[0], w[1], 16);
    } else {
        const uintptr_t u = reinterpret_cast<uintptr_t>(p);
        const uint32_t *w = reinterpret_cast<const uint32_t *>(u & ~(uintptr_t)3);
        return __funnelshift_r(w[0], w[1], (uint32_t)(u & 3u) * 8u);
    }
}

struct Q6Half {
    uint32_t ql[4], qh[2], sc[2];
};

template <int MIS>
__device__ __forceinline__ void q6_load_half(const uint8_t *blk, int h, int t4, Q6Half &q) {
#pragma unroll
    for (int i = 0; i < 4; i++) q.ql[i] = ld32<MIS>(blk + 64 * h + 16 * i + 4 * t4);
#pragma unroll
    for (int i = 0; i < 2; i++) q.qh[i] = ld32<MIS>(blk + 128 + 32 * h + 16 * i + 4 * t4);
    q.sc[0] = ld32<MIS>(blk + 192 + 8 * h);
    q.sc[1] = ld32<MIS>(blk + 196 + 8 * h);
}

// Unsigned 6-bit values of sub-block sl8 (0..7 within the half, a constant after unrolling).
__device__ __forceinline__ uint32_t q6_vals(const Q6Half &q, int sl8) {
    const uint32_t lo = (q.ql[sl8 & 3] >> (sl8 >= 4 ? 4 : 0)) & NIB;
    const uint32_t hi = ((q.qh[sl8 & 1] >> (2 * (sl8 >> 1))) & 0x03030303u) << 4;
    return lo | hi;
}

template <int NGR, int MA, int MB>
__device__ __forceinline__ void q6_block(const uint8_t *ba, const uint8_t *bb, const XQ6 (&x)[NGR],
                                         float (*acc)[4]) {
    const int t4 = threadIdx.x & 3;
    int isum[NGR][4];
#pragma unroll
    for (int G = 0; G < NGR; G++)
#pragma unroll
        for (int i = 0; i < 4; i++) isum[G][i] = 0;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        Q6Half qa, qb;
        q6_load_half<MA>(ba, h, t4, qa);
        q6_load_half<MB>(bb, h, t4, qb);
#pragma unroll
        for (int sl8 = 0; sl8 < 8; sl8++) {
            const uint32_t va = q6_vals(qa, sl8), vb = q6_vals(qb, sl8);
            const int ca = sbyte(qa.sc[sl8 >> 2], sl8 & 3), cb = sbyte(qb.sc[sl8 >> 2], sl8 & 3);
#pragma unroll
            for (int G = 0; G < NGR; G++) {
                int d[4];
                mma_k16_u8s8(d, va, vb, x[G].w[8 * h + sl8]);
                isum[G][0] += ca * d[0];
                isum[G][1] += ca * d[1];
                isum[G][2] += cb * d[2];
                isum[G][3] += cb * d[3];
            }
        }
    }
    // scale word t4 of each row: the scales of sub-blocks 4*t4 .. 4*t4+3
    const uint32_t wa = ld32<MA>(ba + 192 + 4 * t4), wb = ld32<MB>(bb + 192 + 4 * t4);
    const float fa = h2f(*reinterpret_cast<const uint16_t *>(ba + 208));
    const float fb = h2f(*reinterpret_cast<const uint16_t *>(bb + 208));
#pragma unroll
    for (int G = 0; G < NGR; G++) {
        int cl[4], ch[4];
        mma_k16_s8u8(cl, wa, wb, x[G].bl);
        mma_k16_s8s8(ch, wa, wb, x[G].bh);
        const float dd[4] = {fa * x[G].d0, fa * x[G].d1, fb * x[G].d0, fb * x[G].d1};
#pragma unroll
        for (int i = 0; i < 4; i++) acc[G][i] += __fmul_rn(dd[i], (float)(isum[G][i] - 32 * (cl[i] + 64 * ch[i])));
    }
}

// The same super-block product from two 8-row units of the fragment-ordered layout (TMOE_Q6R_UNIT):
// MMA rows g from unit ua, g+8 from unit ub.  Every word is aligned and each load is one vector
// access over consecutive lanes (no bank conflicts): per half and unit a 128-bit ql load, a 64-bit
// qh load and a 64-bit load of the half's 8 scales (the same address across a quad).
__device__ __forceinline__ void q6r_load_half(const uint8_t *u, int h, int lane, Q6Half &q) {
    const uint4 l = *reinterpret_cast<const uint4 *>(u + 768 * h + 16 * lane);
    const uint2 hb = *reinterpret_cast<const uint2 *>(u + 768 * h + 512 + 8 * lane);
    const uint2 sc = *reinterpret_cast<const uint2 *>(u + 1536 + 16 * (lane >> 2) + 8 * h);
    q.ql[0] = l.x, q.ql[1] = l.y, q.ql[2] = l.z, q.ql[3] = l.w;
    q.qh[0] = hb.x, q.qh[1] = hb.y;
    q.sc[0] = sc.x, q.sc[1] = sc.y;
}

template <int NGR>
__device__ __forceinline__ void q6r_block(const uint8_t *ua, const uint8_t *ub, const XQ6 (&x)[NGR],
                                          float (*acc)[4]) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
    int isum[NGR][4];
#pragma unroll
    for (int G = 0; G < NGR; G++)
#pragma unroll
        for (int i = 0; i < 4; i++) isum[G][i] = 0;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        Q6Half qa, qb;
        q6r_load_half(ua, h, lane, qa);
        q6r_load_half(ub, h, lane, qb);
#pragma unroll
        for (int sl8 = 0; sl8 < 8; sl8++) {
            const uint32_t va = q6_vals(qa, sl8), vb = q6_vals(qb, sl8);
            const int ca = sbyte(qa.sc[sl8 >> 2], sl8 & 3), cb = sbyte(qb.sc[sl8 >> 2], sl8 & 3);
#pragma unroll
            for (int G = 0; G < NGR; G++) {
                int d[4];
                mma_k16_u8s8(d, va, vb, x[G].w[8 * h + sl8]);
                isum[G][0] += ca * d[0];
                isum[G][1] += ca * d[1];
                isum[G][2] += cb * d[2];
                isum[G][3] += cb * d[3];
            }
        }
    }
    // scale word t4 of each row: the scales of sub-blocks 4*t4 .. 4*t4+3
    const uint32_t wa = *reinterpret_cast<const uint32_t *>(ua + 1536 + 16 * g + 4 * t4);
    const uint32_t wb = *reinterpret_cast<const uint32_t *>(ub + 1536 + 16 * g + 4 * t4);
    const float fa = h2f(*reinterpret_cast<const uint16_t *>(ua + 1664 + 2 * g));
    const float fb = h2f(*reinterpret_cast<const uint16_t *>(ub + 1664 + 2 * g));
#pragma unroll
    for (int G = 0; G < NGR; G++) {
        int cl[4], ch[4];
        mma_k16_s8u8(cl, wa, wb, x[G].bl);
        mma_k16_s8s8(ch, wa, wb, x[G].bh);
        const float dd[4] = {fa * x[G].d0, fa * x[G].d1, fb * x[G].d0, fb * x[G].d1};
#pragma unroll
        for (int i = 0; i < 4; i++) acc[G][i] += __fmul_rn(dd[i], (float)(isum[G][i] - 32 * (cl[i] + 64 * ch[i])));
    }
}

__device__ __forceinline__ float silu_mul(float g, float u) { return (g / (1.0f + expf(-g))) * u; }

// ------------------------------------------------------------------ the warp's feed (warp-uniform state)
// Items are handed out in groups of GEMV_NW consecutive items, one per warp of a CTA: warp w takes
// item 8 * gid + w of each group gid its CTA draws.  A CTA's warps thus work on neighbouring
// rows of the same expert at about the same time and share its tokens' activation rows in L1.
// The CTA's group index i maps to gid = i * gridDim.x + blockIdx.x for i < n_static (about 4/5
// of the groups, no atomics), and the rest come dynamically from a global counter (items differ
// in token count): the first warp that needs dynamic index d claims ring entry d (once every
// warp has read index d - GQ_RING from it), draws the id and publishes it; the others wait
// (bounded) for it.
constexpr int GQ_RING = 8;
constexpr int GQ_CLAIM = -0x7fffffff;

struct GroupQueue {
    unsigned long long *ring;  // {tag = dynamic index d, gid} per entry, as one 64-bit word
    int *prog;                 // per warp: the last dynamic index it read (INT_MAX when done)
    int n_static;              // static group indices per CTA
};

__device__ __forceinline__ int gq_tag(unsigned long long v) { return (int)(uint32_t)(v & 0xffffffffull); }
__device__ __forceinline__ int gq_gid(unsigned long long v) { return (int)(uint32_t)(v >> 32); }

// The CTA's group id for index i (lane 0 only); -1 on a timeout (latched by the caller).
__device__ int gq_get(const GemvArgs &a, const GroupQueue &q, int i) {
    if (i < q.n_static) return i * (int)gridDim.x + (int)blockIdx.x;
    const int d = i - q.n_static;
    volatile unsigned long long *e = q.ring + (d % GQ_RING);
    uint64_t t0 = 0;
    for (int spin = 0;; ++spin) {
        const unsigned long long v = *e;
        if (gq_tag(v) == d) return gq_gid(v);
        if (gq_tag(v) == d - GQ_RING) {
            bool free = true;  // every warp has read index d - GQ_RING
            for (int w = 0; w < GEMV_NW; w++)
                if (((volatile int *)q.prog)[w] < d - GQ_RING) free = false;
            if (free && atomicCAS(reinterpret_cast<int *>(const_cast<unsigned long long *>(e)), d - GQ_RING,
                                  GQ_CLAIM) == d - GQ_RING) {
                const int gid = q.n_static * (int)gridDim.x + atomicAdd(a.work, 1);
                *e = ((unsigned long long)(uint32_t)gid << 32) | (uint32_t)d;
                return gid;
            }
        }
        if (spin == 64) t0 = globaltimer_ns();
        if (spin > 64 && globaltimer_ns() - t0 > TMOE_WAIT_LIMIT_NS) return -1;
    }
}

struct Feed {
    int gi;             // the CTA group index of the next draw
    int n_item, n_a;    // the next item and its active index (n_item < 0: none)
    int4 n_info;        // its record, loading
    bool n_ready;       // n_item is drawn (else the next fill draws it, after issuing its copies)
    bool ended;         // a draw found no more groups
    int item, tile, beg, end, e, pass, npass, chunk;  // the next fill (item < 0: none left)
};

// Spread dealing (a.spread: at most one item per warp of the full grid): draw 0 of warp w in CTA c
// is item 2 * ((w / 2) * gridDim.x + c) + w % 2, so pairs of neighbouring row tiles go to
// consecutive CTAs and every SM gets about the same number of items; later draws (none while the
// items fit the warps) come from the work counter, one item at a time.
__device__ __forceinline__ int spread_item0(int warp) {
    return 2 * ((warp >> 1) * (int)gridDim.x + (int)blockIdx.x) + (warp & 1);
}

__device__ __forceinline__ int grab_item(const GemvArgs &a, Feed &f, const GroupQueue &q, int n_items) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (a.spread) {
        int item = 0;
        const int dealt = GEMV_NW * (int)gridDim.x;  // items of draw 0
        if (lane == 0)
            item = f.gi == 0 ? spread_item0(warp) : dealt < n_items ? dealt + atomicAdd(a.work, 1) : n_items;
        item = __shfl_sync(FULL, item, 0);
        f.gi++;
        return item < n_items ? item : -1;
    }
    const int n_groups = (n_items + GEMV_NW - 1) / GEMV_NW;
    for (;;) {
        int gid = 0;
        if (lane == 0) {
            gid = gq_get(a, q, f.gi);
            if (gid < 0) latch_error(a.err, TMOE_DEV_ERR_TIMEOUT);
            const bool done = gid < 0 || gid >= n_groups;
            if (done || f.gi >= q.n_static) ((volatile int *)q.prog)[warp] = done ? 0x7fffffff : f.gi - q.n_static;
        }
        gid = __shfl_sync(FULL, gid, 0);
        f.gi++;
        if (gid < 0 || gid >= n_groups) return -1;
        const int item = gid * GEMV_NW + warp;
        if (item < n_items) return item;
    }
}

__device__ __forceinline__ void fetch_next(const GemvArgs &a, Feed &f, const GroupQueue &q, int n_items) {
    f.n_item = f.ended ? -1 : grab_item(a, f, q, n_items);
    f.ended = f.n_item < 0;
    f.n_ready = true;
    if (f.n_item >= 0) {
        f.n_a = fast_div(f.n_item, a.tiles_m);
        f.n_info = __ldcg(a.active + f.n_a);
    }
}

// Takes the drawn item as the next fill's (drawing it first if need be); the one after it is drawn
// by a later fill, after that fill's copies are on their way.
template <int NG>
__device__ __forceinline__ void next_item(const GemvArgs &a, Feed &f, const GroupQueue &q, int n_items) {
    const int lane = threadIdx.x & 31;
    for (;;) {
        if (!f.n_ready) fetch_next(a, f, q, n_items);
        const int item = f.n_item, ai = f.n_a;
        if (item < 0) {
            f.item = -1;
            return;
        }
        const int4 info = f.n_info;
        f.n_ready = false;
        const int e = info.x, beg = info.y, end = info.z;
        if (e < 0 || e >= a.n_slots || beg < 0 || end > a.n_pairs || end < beg) {
            if (lane == 0) latch_error(a.err, TMOE_DEV_ERR_BADID);
            continue;
        }
        if (end == beg) continue;
        f.item = item;
        f.tile = item - ai * a.tiles;
        f.e = e;
        f.beg = beg;
        f.end = end;
        f.pass = 0;
        f.npass = (end - beg + NG * TOKG - 1) / (NG * TOKG);
        f.chunk = 0;
        return;
    }
}

// Issues the next fill into `slot` (record, expect_tx, the copies) from lane 0 and advances the
// feed.  With no items left the fill is an end marker (no copies).  A pass covers NG token groups.
template <int WT, bool GATEUP, int NG>
__device__ __forceinline__ void fill(const GemvArgs &a, const GemvMaps &tm, Feed &f, uint64_t *bar, SlotRec *rec,
                                     uint8_t *slot, const GroupQueue &q, int n_items) {
    const int lane = threadIdx.x & 31;
    if (lane == 0) {
        if (f.item < 0) {
            rec->item = -1;
            mbar_arrive_expect_tx(bar, 0u);
        } else {
            const int nb = a.K / TMOE_QK, kb0 = f.chunk * a.chunk_blocks;
            const uint32_t r_bytes = (uint32_t)min(a.chunk_blocks, nb - kb0) * TMOE_Q6R_UNIT;  // Q6KR: per 8-row group
            uint32_t tx = WT == TMOE_WT_Q4K    ? 16u * (uint32_t)a.chunk_blocks * TMOE_Q4K_BYTES
                          : WT == TMOE_WT_Q6KR ? 2u * r_bytes
                                               : 16u * (uint32_t)a.nb1_0;
            uintptr_t ps = 0;
            uint32_t pbytes = 0;
            int poff = 0;
            if (f.chunk == 0) {  // the pass's pair indices, rounded out to 16 bytes
                const int t0 = f.beg + f.pass * NG * TOKG, nt = min(NG * TOKG, f.end - t0);
                const uintptr_t src = reinterpret_cast<uintptr_t>(a.perm + t0);
                ps = src & ~(uintptr_t)15;
                pbytes = (uint32_t)(((src + 4u * (uint32_t)nt + 15) & ~(uintptr_t)15) - ps);
                poff = (int)((src - ps) >> 2);
                tx += pbytes;
            }
            *reinterpret_cast<int4 *>(rec) = make_int4(f.item, f.tile, f.pass, f.chunk);
            *reinterpret_cast<int4 *>(&rec->beg) = make_int4(f.beg, f.end, poff, 0);
            mbar_arrive_expect_tx(bar, tx);
            if constexpr (WT == TMOE_WT_Q4K) {
                const int x = f.chunk * a.chunk_blocks * Q4_CHUNK_U32;
                if constexpr (GATEUP) {
                    tma_load_3d(slot, &tm.m[0], x, f.tile * 8, f.e, bar);
                    tma_load_3d(slot + 8 * a.chunk_blocks * TMOE_Q4K_BYTES, &tm.m[1], x, f.tile * 8, f.e, bar);
                } else {
                    tma_load_3d(slot, &tm.m[0], x, f.tile * 16, f.e, bar);
                }
            } else if constexpr (WT == TMOE_WT_Q6KR) {
                // gate/up: 8-row group `tile` of each matrix; down: groups 2 tile and 2 tile + 1.  The
                // second copy lands a full chunk after the first (compute indexes by chunk_blocks).
                const size_t gs = (size_t)nb * TMOE_Q6R_UNIT, k0 = (size_t)kb0 * TMOE_Q6R_UNIT;
                uint8_t *slot_b = slot + (size_t)a.chunk_blocks * TMOE_Q6R_UNIT;
                if constexpr (GATEUP) {
                    bulk_g2s(slot, a.w0 + (size_t)f.e * a.nb2_0 + (size_t)f.tile * gs + k0, r_bytes, bar);
                    bulk_g2s(slot_b, a.w1 + (size_t)f.e * a.nb2_1 + (size_t)f.tile * gs + k0, r_bytes, bar);
                } else {
                    const uint8_t *src = a.w0 + (size_t)f.e * a.nb2_0 + (size_t)(2 * f.tile) * gs + k0;
                    bulk_g2s(slot, src, r_bytes, bar);
                    bulk_g2s(slot_b, src + gs, r_bytes, bar);
                }
            } else {
                const uint32_t rb = (uint32_t)a.nb1_0;
                if constexpr (GATEUP) {
                    bulk_g2s(slot, a.w0 + (size_t)f.e * a.nb2_0 + (size_t)f.tile * 8 * rb, 8u * rb, bar);
                    bulk_g2s(slot + 8 * rb, a.w1 + (size_t)f.e * a.nb2_1 + (size_t)f.tile * 8 * rb, 8u * rb, bar);
                } else {
                    bulk_g2s(slot, a.w0 + (size_t)f.e * a.nb2_0 + (size_t)f.tile * 16 * rb, 16u * rb, bar);
                }
            }
            if (pbytes) bulk_g2s(slot + a.wbytes, reinterpret_cast<const void *>(ps), pbytes, bar);
        }
    }
    __syncwarp();
    if (f.item < 0) return;
    if (++f.chunk == a.n_chunks) {
        f.chunk = 0;
        if (++f.pass == f.npass) next_item<NG>(a, f, q, n_items);
    }
    // the item after this one is drawn once the fill about to be issued is this item's last
    if (!f.n_ready && f.item >= 0 && f.chunk == a.n_chunks - 1 && f.pass == f.npass - 1)
        fetch_next(a, f, q, n_items);
}

// ------------------------------------------------------------------ kernel
// NG: token groups per pass (1: decode batches of a few tokens per expert, where the second
// group's registers would only cost occupancy of the scheduler; 2: larger batches).
template <int WT, bool GATEUP, int MINB, int NG>
__global__ void __launch_bounds__(GEMV_THREADS, MINB)
    gemv_kernel(const GemvArgs a, const __grid_constant__ GemvMaps tm) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const int D = a.d_slots, nb = a.K / TMOE_QK;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * GEMV_MAXD;
    SlotRec *recs = reinterpret_cast<SlotRec *>(smem + GEMV_NW * GEMV_MAXD * 8) + warp * GEMV_MAXD;
    uint8_t *slots = smem + GEMV_HDR + (size_t)warp * D * a.slot_bytes;
    if (lane == 0) {
        if constexpr (WT == TMOE_WT_Q4K) {  // the tensor maps' descriptors, fetched while the prologue runs
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm.m[0])) : "memory");
            if constexpr (GATEUP)
                asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm.m[1])) : "memory");
        }
        for (int s = 0; s < D; s++) mbar_init(&bars[s], 1);
        fence_barrier_init();
    }
    __syncwarp();
    // Programmatic launch: gate/up reads what the routing kernel (its predecessor) wrote, so it
    // waits here.  The layer's down GEMV (a.early) has a predecessor that only writes its
    // activations: the dispatch data and the weights are two and more launches back, so it issues
    // its first fills before it waits.  Any other launch waits here.
    const bool early = !GATEUP && a.early;
    if (!early) {
        pdl_wait();
        pdl_trigger();
    }

    // The warp's first item is in the CTA's first (static) group: its record is loaded alongside
    // the active count, not after it (an index past the count reads a stale record, never used).
    const int item0 = a.spread ? spread_item0(warp) : (int)blockIdx.x * GEMV_NW + warp;
    const int a0 = fast_div(item0, a.tiles_m);
    const int4 info0 = __ldcg(a.active + min(a0, a.max_active - 1));
    // Dispatch data are checked before they become addresses: an active count above the grid's
    // sizing latches TMOE_DEV_ERR_BADID and is clamped; bad experts or offsets are skipped.
    int na = __ldcg(a.n_active);
    if (na > a.max_active || na < 0) {
        if (threadIdx.x == 0 && blockIdx.x == 0) latch_error(a.err, TMOE_DEV_ERR_BADID);
        na = na < 0 ? 0 : a.max_active;
    }
    const int n_items = na * a.tiles;
    GroupQueue q;
    q.ring = reinterpret_cast<unsigned long long *>(smem + GEMV_NW * GEMV_MAXD * (8 + (int)sizeof(SlotRec)));
    q.prog = reinterpret_cast<int *>(q.ring + GQ_RING);
    q.n_static = max(1, (((n_items + GEMV_NW - 1) / GEMV_NW) * 4 / 5) / (int)gridDim.x);
    if (threadIdx.x < GQ_RING) q.ring[threadIdx.x] = (uint32_t)((int)threadIdx.x - GQ_RING);  // "index d - ring read"
    if (threadIdx.x < GEMV_NW) q.prog[threadIdx.x] = -1;
    __syncthreads();
    Feed f;
    f.ended = false;
    if (item0 < n_items) {  // static group 0 = this CTA's index
        f.gi = 1;
        f.n_item = item0;
        f.n_a = a0;
        f.n_info = info0;
        f.n_ready = true;
    } else {
        f.gi = 0;
        f.n_ready = false;
    }
    next_item<NG>(a, f, q, n_items);
    for (int s = 0; s < D; s++)
        fill<WT, GATEUP, NG>(a, tm, f, &bars[s], &recs[s], slots + (size_t)s * a.slot_bytes, q, n_items);
    if (early) {
        pdl_wait();
        pdl_trigger();
    }

    TokCols tc[NG];
    XBase xb0;  // NG == 1: the group's bases, kept for the pass (two-group passes address from tc)
    int ng = 1;
    float acc[NG][4];
    int s = 0;
    uint32_t ph = 0;
    for (;;) {
        // every lane takes the same path (a completion right at the limit could split them)
        if (!__all_sync(FULL, mbar_wait_bounded(&bars[s], ph))) {
            // The copies of this fill never landed: report, and wait (bounded) for the other
            // slots' copies so that none is in flight when the CTA's shared memory goes away.
            if (lane == 0) latch_error(a.err, TMOE_DEV_ERR_TIMEOUT);
            for (int k = 1; k < D; k++) {
                int s2 = s + k, p2 = ph;
                if (s2 >= D) s2 -= D, p2 ^= 1;
                mbar_wait_bounded(&bars[s2], p2);
            }
            return;
        }
        const int4 rv = *reinterpret_cast<const int4 *>(&recs[s]);
        const int item = rv.x;
        if (item < 0) return;  // every later fill is an end marker too: nothing in flight
        const int tile = rv.y, pass = rv.z, chunk = rv.w;
        const int b0 = chunk * a.chunk_blocks;
        const int nblk = min(a.chunk_blocks, nb - b0);
        const uint8_t *sl = slots + (size_t)s * a.slot_bytes;
        if (chunk == 0) {  // a new pass: the token columns of its (up to) two groups
            const int4 bv = *reinterpret_cast<const int4 *>(&recs[s].beg);
            const int t0 = bv.x + pass * NG * TOKG;
            const int nt = min(NG * TOKG, bv.y - t0);
            const int *pp = reinterpret_cast<const int *>(sl + a.wbytes) + bv.z;  // the pass's pairs
            ng = nt > TOKG ? 2 : 1;
#pragma unroll
            for (int G = 0; G < NG; G++) {
                const int ntok = min(TOKG, nt - G * TOKG);
                // past the group's end the group's first token stands in (never written)
                int pg = ntok > 0 ? pp[G * TOKG + (g < ntok ? g : 0)] : 0;
                int p0 = ntok > 0 ? pp[G * TOKG + (2 * t4 < ntok ? 2 * t4 : 0)] : 0;
                int p1 = ntok > 0 ? pp[G * TOKG + (2 * t4 + 1 < ntok ? 2 * t4 + 1 : 0)] : 0;
                pg = (pg >= 0 && pg < a.n_pairs) ? pg : 0;
                const bool v0 = 2 * t4 < ntok && p0 >= 0 && p0 < a.n_pairs;
                const bool v1 = 2 * t4 + 1 < ntok && p1 >= 0 && p1 < a.n_pairs;
                p0 = (p0 >= 0 && p0 < a.n_pairs) ? p0 : 0;
                p1 = (p1 >= 0 && p1 < a.n_pairs) ? p1 : 0;
                tc[G].xg = fast_div(pg, a.xdiv_m);
                tc[G].x0 = fast_div(p0, a.xdiv_m);
                tc[G].x1 = fast_div(p1, a.xdiv_m);
                tc[G].pp0 = v0 ? p0 : -1;
                tc[G].pp1 = v1 ? p1 : -1;
            }
            if constexpr (NG == 1) xb0 = x_base<WT>(a, tc[0], nb);
#pragma unroll
            for (int G = 0; G < NG; G++) acc[G][0] = acc[G][1] = acc[G][2] = acc[G][3] = 0.0f;
        }
        const int S = a.row_stride;
        if constexpr (WT == TMOE_WT_Q6KR) {  // MMA rows g: unit a's row g, g+8: unit b's row g
            const uint8_t *ua = sl, *ub = sl + (size_t)a.chunk_blocks * TMOE_Q6R_UNIT;
            for (int bi = 0; bi < nblk; bi++) {
                const int kb = b0 + bi;
                if constexpr (NG == 1) {
                    XQ6 x[1];
                    load_xq6(xb0, kb, x[0]);
                    q6r_block<1>(ua + bi * TMOE_Q6R_UNIT, ub + bi * TMOE_Q6R_UNIT, x, acc);
                } else if (ng == 1) {
                    XQ6 x[1];
                    load_xq6(a, tc[0], kb, nb, x[0]);
                    q6r_block<1>(ua + bi * TMOE_Q6R_UNIT, ub + bi * TMOE_Q6R_UNIT, x, acc);
                } else {
                    XQ6 x[2];
                    load_xq6(a, tc[0], kb, nb, x[0]);
                    load_xq6(a, tc[NG - 1], kb, nb, x[1]);
                    q6r_block<2>(ua + bi * TMOE_Q6R_UNIT, ub + bi * TMOE_Q6R_UNIT, x, acc);
                }
            }
        } else if constexpr (NG == 1) {
            if constexpr (WT == TMOE_WT_Q4K) {
                const uint8_t *ra = sl + (size_t)g * S, *rb = sl + (size_t)(g + 8) * S;
                const bool lo = t4 < 2;
                if (nblk == 2) {  // both super-blocks' activations in flight before the MMAs
                    XQ4 x0[1], x1[1];
                    load_xq4(xb0, b0, lo, x0[0]);
                    load_xq4(xb0, b0 + 1, lo, x1[0]);
                    q4_block<1>(ra, rb, x0, acc);
                    q4_block<1>(ra + TMOE_Q4K_BYTES, rb + TMOE_Q4K_BYTES, x1, acc);
                } else {
                    for (int bi = 0; bi < nblk; bi++) {
                        XQ4 x[1];
                        load_xq4(xb0, b0 + bi, lo, x[0]);
                        q4_block<1>(ra + bi * TMOE_Q4K_BYTES, rb + bi * TMOE_Q4K_BYTES, x, acc);
                    }
                }
            } else if constexpr (GATEUP) {
                const uint8_t *ra = sl + (size_t)g * S, *rb = sl + (size_t)(g + 8) * S;
                for (int kb = 0; kb < nb; kb++) {
                    XQ6 x[1];
                    load_xq6(xb0, kb, x[0]);
                    q6_block<1, 2, 2>(ra + kb * TMOE_Q6K_BYTES, rb + kb * TMOE_Q6K_BYTES, x, acc);
                }
            } else {
                const uint8_t *ra = sl + (size_t)(2 * g) * S, *rb = sl + (size_t)(2 * g + 1) * S;
                for (int kb = 0; kb < nb; kb++) {
                    const int ma = kb & 1, mb = (nb + kb) & 1;
                    const uint8_t *pa = ra + kb * TMOE_Q6K_BYTES, *pb = rb + kb * TMOE_Q6K_BYTES;
                    XQ6 x[1];
                    load_xq6(xb0, kb, x[0]);
                    if (ma == 0 && mb == 0) q6_block<1, 0, 0>(pa, pb, x, acc);
                    else if (ma == 0) q6_block<1, 0, 1>(pa, pb, x, acc);
                    else if (mb == 0) q6_block<1, 1, 0>(pa, pb, x, acc);
                    else q6_block<1, 1, 1>(pa, pb, x, acc);
                }
            }
        } else if constexpr (WT == TMOE_WT_Q4K) {
            const uint8_t *ra = sl + (size_t)g * S, *rb = sl + (size_t)(g + 8) * S;
            for (int bi = 0; bi < nblk; bi++) {
                const int kb = b0 + bi;
                if (ng == 1) {
                    XQ4 x[1];
                    load_xq4(a, tc[0], kb, nb, x[0]);
                    q4_block<1>(ra + bi * TMOE_Q4K_BYTES, rb + bi * TMOE_Q4K_BYTES, x, acc);
                } else {
                    XQ4 x[2];
                    load_xq4(a, tc[0], kb, nb, x[0]);
                    load_xq4(a, tc[NG - 1], kb, nb, x[1]);
                    q4_block<2>(ra + bi * TMOE_Q4K_BYTES, rb + bi * TMOE_Q4K_BYTES, x, acc);
                }
            }
        } else if constexpr (GATEUP) {  // MMA rows g: gate row g, g+8: up row g
            const uint8_t *ra = sl + (size_t)g * S, *rb = sl + (size_t)(g + 8) * S;
            for (int kb = 0; kb < nb; kb++) {
                if (ng == 1) {
                    XQ6 x[1];
                    load_xq6(a, tc[0], kb, nb, x[0]);
                    q6_block<1, 2, 2>(ra + kb * TMOE_Q6K_BYTES, rb + kb * TMOE_Q6K_BYTES, x, acc);
                } else {
                    XQ6 x[2];
                    load_xq6(a, tc[0], kb, nb, x[0]);
                    load_xq6(a, tc[NG - 1], kb, nb, x[1]);
                    q6_block<2, 2, 2>(ra + kb * TMOE_Q6K_BYTES, rb + kb * TMOE_Q6K_BYTES, x, acc);
                }
            }
        } else {  // MMA rows g: row 2g (block kb off by two iff kb odd), g+8: row 2g+1 (iff nb+kb odd)
            const uint8_t *ra = sl + (size_t)(2 * g) * S, *rb = sl + (size_t)(2 * g + 1) * S;
            for (int kb = 0; kb < nb; kb++) {
                const int ma = kb & 1, mb = (nb + kb) & 1;
                const uint8_t *pa = ra + kb * TMOE_Q6K_BYTES, *pb = rb + kb * TMOE_Q6K_BYTES;
                if (ng == 1) {
                    XQ6 x[1];
                    load_xq6(a, tc[0], kb, nb, x[0]);
                    if (ma == 0 && mb == 0) q6_block<1, 0, 0>(pa, pb, x, acc);
                    else if (ma == 0) q6_block<1, 0, 1>(pa, pb, x, acc);
                    else if (mb == 0) q6_block<1, 1, 0>(pa, pb, x, acc);
                    else q6_block<1, 1, 1>(pa, pb, x, acc);
                } else {
                    XQ6 x[2];
                    load_xq6(a, tc[0], kb, nb, x[0]);
                    load_xq6(a, tc[NG - 1], kb, nb, x[1]);
                    if (ma == 0 && mb == 0) q6_block<2, 0, 0>(pa, pb, x, acc);
                    else if (ma == 0) q6_block<2, 0, 1>(pa, pb, x, acc);
                    else if (mb == 0) q6_block<2, 1, 0>(pa, pb, x, acc);
                    else q6_block<2, 1, 1>(pa, pb, x, acc);
                }
            }
        }
        __syncwarp();  // every lane's reads of the slot are done (their values are consumed)
        fill<WT, GATEUP, NG>(a, tm, f, &bars[s], &recs[s], slots + (size_t)s * a.slot_bytes, q, n_items);
        if (chunk == a.n_chunks - 1) {  // this pass's sums are complete
            // output rows of MMA rows g and g+8
            int row_a, row_b;
            if constexpr (GATEUP) {
                row_a = row_b = tile * 8 + g;
            } else if constexpr (WT != TMOE_WT_Q6K) {
                row_a = tile * 16 + g;
                row_b = row_a + 8;
            } else {
                row_a = tile * 16 + 2 * g;
                row_b = row_a + 1;
            }
#pragma unroll
            for (int G = 0; G < NG; G++) {
                if (G >= ng) break;
                const int q0 = tc[G].pp0, q1 = tc[G].pp1;
                if constexpr (GATEUP) {
                    if (q0 >= 0) a.out[(int64_t)q0 * a.N + row_a] = silu_mul(acc[G][0], acc[G][2]);
                    if (q1 >= 0) a.out[(int64_t)q1 * a.N + row_a] = silu_mul(acc[G][1], acc[G][3]);
                } else {
                    if (q0 >= 0) {
                        a.out[(int64_t)q0 * a.N + row_a] = acc[G][0];
                        a.out[(int64_t)q0 * a.N + row_b] = acc[G][2];
                    }
                    if (q1 >= 0) {
                        a.out[(int64_t)q1 * a.N + row_a] = acc[G][1];
                        a.out[(int64_t)q1 * a.N + row_b] = acc[G][3];
                    }
                }
            }
        }
        if (++s == D) s = 0, ph ^= 1;
    }
}

// ------------------------------------------------------------------ launcher
constexpr int GEMV_SMEM_1CTA = 226 * 1024;
constexpr int GEMV_SMEM_2CTA = 113 * 1024;  // two CTAs: 2 x (113 + 1 reserved) KB = 228 KB

struct GemvPlan {
    int cb, ctas_per_sm, d;
};

// Q4_K: a chunk of two super-blocks (a 288-byte row stride: the 8-byte fragment loads of rows
// g = 0..7 hit distinct banks) with two CTAs per SM and two slots per warp: a third slot fits but
// was slower (C2 decode T = 64: gate/up 61.7 us against 60.5, the layer 129.7 against 126.4 us),
// the 36 KB it takes per CTA being worth more as L1 for the activation rows.  Q6_K: all of K; two
// CTAs per SM if a slot per warp fits, else one (one CTA with two slots per warp: down 71.6 us
// against 56.7 with two CTAs of one slot).  The same for Q6_K in 8-row fragment order (fills of
// one super-block into three slots per warp were slower: C2 T = 64 down 55.6 us against 50.4).
template <int WT>
static GemvPlan plan_for(int K) {
    const int nb = K / TMOE_QK;
    const int cb = WT == TMOE_WT_Q4K ? (nb >= 2 ? 2 : 1) : nb;
    const int slot = (WT == TMOE_WT_Q4K    ? ITEM_ROWS * TMOE_Q4K_BYTES * cb
                      : WT == TMOE_WT_Q6KR ? 2 * nb * TMOE_Q6R_UNIT
                                           : ITEM_ROWS * TMOE_Q6K_BYTES * nb + 16) +
                     PERM_STAGE;
    const int d2 = (GEMV_SMEM_2CTA - GEMV_HDR) / (GEMV_NW * slot);
    if (WT == TMOE_WT_Q4K && d2 >= 2) return {cb, 2, 2};
    if (d2 >= 1) return {cb, 2, d2 < GEMV_MAXD ? d2 : GEMV_MAXD};
    const int d1 = (GEMV_SMEM_1CTA - GEMV_HDR) / (GEMV_NW * slot);
    if (d1 >= 1) return {cb, 1, d1 < GEMV_MAXD ? d1 : GEMV_MAXD};
    return {0, 0, 0};
}

static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

// [expert][row][row bytes as u32] with a box of cb super-blocks by `rows` rows of one expert.
static bool encode_rows_map(CUtensorMap *m, const uint8_t *base, int K, int N, int n_slots, size_t nb1, size_t nb2,
                            int cb, int rows) {
    const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)(K / TMOE_QK) * Q4_CHUNK_U32, (cuuint64_t)N, (cuuint64_t)n_slots};
    const cuuint64_t strides[2] = {(cuuint64_t)nb1, (cuuint64_t)nb2};
    const cuuint32_t box[3] = {(cuuint32_t)(cb * Q4_CHUNK_U32), (cuuint32_t)rows, 1u};
    const cuuint32_t es[3] = {1u, 1u, 1u};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint8_t *>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
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

template <int WT, bool GATEUP>
static cudaError_t launch_t(const GemvArgs &args_in, int max_items, int sm_count, cudaStream_t st) {
    GemvArgs a = args_in;
    const GemvPlan pl = plan_for<WT>(a.K);
    if (pl.cb == 0) return cudaErrorInvalidValue;
    const int nb = a.K / TMOE_QK;
    a.chunk_blocks = pl.cb;
    a.n_chunks = (nb + pl.cb - 1) / pl.cb;
    a.row_stride = (WT == TMOE_WT_Q4K ? TMOE_Q4K_BYTES : TMOE_Q6K_BYTES) * pl.cb;
    // (Q6_K: + one word that the realigning loads of the last row may touch)
    a.wbytes = WT == TMOE_WT_Q4K    ? ITEM_ROWS * a.row_stride
               : WT == TMOE_WT_Q6KR ? 2 * pl.cb * TMOE_Q6R_UNIT
                                    : ITEM_ROWS * a.row_stride + 16;
    a.slot_bytes = a.wbytes + PERM_STAGE;
    if (WT == TMOE_WT_Q4K && a.slot_bytes % 128 != 0) return cudaErrorInvalidValue;
    a.d_slots = pl.d;
    a.tiles = a.N / (GATEUP ? ITEM_ROWS / 2 : ITEM_ROWS);
    const uint64_t two40 = 1ull << 40;
    a.tiles_m = (two40 + (uint64_t)a.tiles - 1) / (uint64_t)a.tiles;
    a.xdiv_m = (two40 + (uint64_t)a.x_div - 1) / (uint64_t)a.x_div;
    GemvMaps tm;
    memset(&tm, 0, sizeof(tm));
    if (WT == TMOE_WT_Q4K) {
        const int rows = GATEUP ? ITEM_ROWS / 2 : ITEM_ROWS;
        if (!encode_rows_map(&tm.m[0], a.w0, a.K, a.N, a.n_slots, a.nb1_0, a.nb2_0, pl.cb, rows))
            return cudaErrorInvalidValue;
        if (GATEUP && !encode_rows_map(&tm.m[1], a.w1, a.K, a.N, a.n_slots, a.nb1_1, a.nb2_1, pl.cb, rows))
            return cudaErrorInvalidValue;
    }
    const size_t smem = GEMV_HDR + (size_t)GEMV_NW * pl.d * a.slot_bytes;
    const int items = max_items * a.tiles;
    int grid = (items + GEMV_NW - 1) / GEMV_NW;
    const int slots = sm_count * pl.ctas_per_sm;
    if (grid > slots) grid = slots;
    if (grid < 1) return cudaSuccess;
    // Few items (at most one per warp of the full grid): the whole grid, items dealt out spread, so
    // that every SM gets about as many (groups of 8 on fewer CTAs put 16 items on some SMs, 8 on others)
    a.spread = items <= GEMV_NW * slots ? 1 : 0;
    if (a.spread) grid = slots;
    // One token group per pass when the batch averages at most 4 pairs per active expert (decode):
    // an expert with more tokens then takes more passes over rows that L2 still holds.
    const bool one = (int64_t)a.n_pairs <= 4 * (int64_t)max_items;
    static int cache[4][64] = {};
    cudaError_t e;
#define TMOE_GEMV_LAUNCH(MINB, NG, CI)                                                                      \
    do {                                                                                                 \
        if ((e = set_smem_once(gemv_kernel<WT, GATEUP, MINB, NG>, smem, cache[CI])) != cudaSuccess) return e; \
        if ((e = launch_k(gemv_kernel<WT, GATEUP, MINB, NG>, grid, GEMV_THREADS, smem, st, a, tm)) != cudaSuccess) \
            return e;                                                                                    \
    } while (0)
    if (pl.ctas_per_sm == 2) {
        if (one) TMOE_GEMV_LAUNCH(2, 1, 0);
        else TMOE_GEMV_LAUNCH(2, 2, 1);
    } else {
        if (one) TMOE_GEMV_LAUNCH(1, 1, 2);
        else TMOE_GEMV_LAUNCH(1, 2, 3);
    }
#undef TMOE_GEMV_LAUNCH
    return cudaGetLastError();
}

int gemv_rows_per_item(int wt, int K, int N) {
    (void)wt;
    if (K <= 0 || K % TMOE_QK != 0) return 0;
    return N > 0 && N % ITEM_ROWS == 0 ? ITEM_ROWS : 0;
}

cudaError_t launch_gemv(int wt, bool gateup, const GemvArgs &a, int max_items, int sm_count, cudaStream_t st) {
    if (a.K % TMOE_QK != 0 || a.K <= 0 || a.K > 65536) return cudaErrorInvalidValue;
    if (gemv_rows_per_item(wt, a.K, a.N) == 0) return cudaErrorInvalidValue;
    // item and pair indices stay below 2^24 and divisors at most 2^16 (fast_div)
    if (a.n_pairs < 0 || a.n_pairs >= (1 << 24) || a.x_div < 1 || a.x_div > (1 << 16) ||
        (int64_t)max_items * (a.N / (ITEM_ROWS / 2)) >= (1 << 24))
        return cudaErrorInvalidValue;
    // Q6_K: contiguous rows (whole-row fills); Q4_K: rows at least a row apart on 16-byte strides
    // (tensor-map fills: a matrix's K slices as experts); 16-byte aligned expert strides
    // (Q6_K in 8-row fragment order: dense matrices, nb1 the ggml row size)
    const size_t rb = (size_t)(wt == TMOE_WT_Q4K ? TMOE_Q4K_BYTES : TMOE_Q6K_BYTES) * (a.K / TMOE_QK);
    auto rows_ok = [&](size_t nb1) { return wt == TMOE_WT_Q4K ? nb1 >= rb && nb1 % 16 == 0 : nb1 == rb; };
    if (!rows_ok(a.nb1_0) || (a.nb2_0 & 15u) || ((uintptr_t)a.w0 & 15u)) return cudaErrorInvalidValue;
    if (gateup && (!rows_ok(a.nb1_1) || (a.nb2_1 & 15u) || ((uintptr_t)a.w1 & 15u))) return cudaErrorInvalidValue;
    if (wt == TMOE_WT_Q4K)
        return gateup ? launch_t<TMOE_WT_Q4K, true>(a, max_items, sm_count, st)
                      : launch_t<TMOE_WT_Q4K, false>(a, max_items, sm_count, st);
    if (wt == TMOE_WT_Q6KR) {
        if ((size_t)a.N * rb > a.nb2_0 || (gateup && (size_t)a.N * rb > a.nb2_1)) return cudaErrorInvalidValue;
        return gateup ? launch_t<TMOE_WT_Q6KR, true>(a, max_items, sm_count, st)
                      : launch_t<TMOE_WT_Q6KR, false>(a, max_items, sm_count, st);
    }
    if (wt != TMOE_WT_Q6K) return cudaErrorInvalidValue;
    return gateup ? launch_t<TMOE_WT_Q6K, true>(a, max_items, sm_count, st)
                  : launch_t<TMOE_WT_Q6K, false>(a, max_items, sm_count, st);
}

}  // namespace tmoe
