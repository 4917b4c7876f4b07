// Expert products for the decode regime (few tokens per expert): HBM-bound dequant-GEMV over
// Q4_K / Q6_K rows with Q8_K activations, the arithmetic of ggml's CPU mul_mat_id path
// (vec_dot_q4_K_q8_K / vec_dot_q6_K_q8_K: integer sub-block sums, scaled per super-block).
//
// Work: items = (active expert, tile of RT rows).  Persistent CTAs walk the items; one producer
// thread streams each item's weight rows into a ring of shared-memory stages with 1D bulk TMA
// copies (cp.async.bulk ... mbarrier::complete_tx), 8 consumer warps unpack them into registers,
// release the stage, then loop over the expert's pairs: dp4a integer dots against the pair's
// Q8_K activation, a shuffle reduction over the LPR lanes of a row, and the row's result.
// gate/up (GATEUP): both matrices of the tile share the stage; the consumer writes
// silu(g) * u (swiglu_split) directly.
#include "common.cuh"
#include "kernels.cuh"

namespace tmoe {

constexpr int GEMV_NW = 8;            // consumer warps
constexpr int GEMV_THREADS = 32 * (GEMV_NW + 1);
constexpr int GEMV_MAX_STAGES = 12;
constexpr int GEMV_BAR_BYTES = 256;   // mbarriers live in the first 256 B of shared memory

// Q4_K unit = 64 elements of one super-block (32 B of nibbles: sub-blocks 2j and 2j+1).
struct Q4Unit {
    uint32_t lo[8], hi[8];
    int sc_lo, sc_hi, m_lo, m_hi;
    float d, dmin;
};

// Q6_K unit = 128 elements (half of a super-block), as signed int8 words.
struct Q6Unit {
    uint32_t q[32];
    int sc[8];
    float d;
};

// Scale and min of Q4_K sub-block s from the 12 packed bytes held in words s0 (bytes 0-3),
// s1 (4-7), s2 (8-11) (ggml get_scale_min_k4).
__device__ __forceinline__ void q4k_scale_min(uint32_t s0, uint32_t s1, uint32_t s2, int s, int &scale,
                                              int &min) {
    auto byte = [](uint32_t w, int i) { return (int)((w >> (8 * i)) & 0xffu); };
    if (s < 4) {
        scale = byte(s0, s) & 63;
        min = byte(s1, s) & 63;
    } else {
        const int i = s - 4;
        scale = (byte(s2, i) & 0x0f) | ((byte(s0, i) >> 6) << 4);
        min = (byte(s2, i) >> 4) | ((byte(s1, i) >> 6) << 4);
    }
}

__device__ __forceinline__ void load_q4_unit(const uint8_t *row, int c, Q4Unit &u) {
    const int b = c >> 2, j = c & 3;
    const uint8_t *blk = row + b * TMOE_Q4K_BYTES;
    uint4 h = *reinterpret_cast<const uint4 *>(blk);
    u.d = h2f((uint16_t)(h.x & 0xffffu));
    u.dmin = h2f((uint16_t)(h.x >> 16));
    q4k_scale_min(h.y, h.z, h.w, 2 * j, u.sc_lo, u.m_lo);
    q4k_scale_min(h.y, h.z, h.w, 2 * j + 1, u.sc_hi, u.m_hi);
    const uint4 *qp = reinterpret_cast<const uint4 *>(blk + 16 + 32 * j);
    uint4 a = qp[0], bq = qp[1];
    uint32_t w[8] = {a.x, a.y, a.z, a.w, bq.x, bq.y, bq.z, bq.w};
#pragma unroll
    for (int i = 0; i < 8; i++) {
        u.lo[i] = w[i] & 0x0f0f0f0fu;
        u.hi[i] = (w[i] >> 4) & 0x0f0f0f0fu;
    }
}

__device__ __forceinline__ void load_q6_unit(const uint8_t *row, int c, Q6Unit &u) {
    const int b = c >> 1, hh = c & 1;
    const uint8_t *blk = row + b * TMOE_Q6K_BYTES;
    uint32_t ql[16], qh[8];
#pragma unroll
    for (int i = 0; i < 16; i++) ql[i] = lds_u32_a2(blk + 64 * hh + 4 * i);
#pragma unroll
    for (int i = 0; i < 8; i++) qh[i] = lds_u32_a2(blk + 128 + 32 * hh + 4 * i);
    uint32_t s0 = lds_u32_a2(blk + 192 + 8 * hh), s1 = lds_u32_a2(blk + 196 + 8 * hh);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        u.sc[i] = (int)(int8_t)((s0 >> (8 * i)) & 0xff);
        u.sc[4 + i] = (int)(int8_t)((s1 >> (8 * i)) & 0xff);
    }
    u.d = h2f(*reinterpret_cast<const uint16_t *>(blk + 208));
#pragma unroll
    for (int i = 0; i < 8; i++) {
        u.q[i] = __vsub4((ql[i] & 0x0f0f0f0fu) | ((qh[i] << 4) & 0x30303030u), 0x20202020u);
        u.q[8 + i] = __vsub4((ql[8 + i] & 0x0f0f0f0fu) | ((qh[i] << 2) & 0x30303030u), 0x20202020u);
        u.q[16 + i] = __vsub4(((ql[i] >> 4) & 0x0f0f0f0fu) | (qh[i] & 0x30303030u), 0x20202020u);
        u.q[24 + i] = __vsub4(((ql[8 + i] >> 4) & 0x0f0f0f0fu) | ((qh[i] >> 2) & 0x30303030u), 0x20202020u);
    }
}

// One Q4_K unit against the pair's Q8_K row: (d*dx) * sum_s sc_s * S_s - (dmin*dx) * sum_s m_s * B_s.
__device__ __forceinline__ float dot_q4_unit(const Q4Unit &u, const int8_t *xq, const float *xd,
                                             const int16_t *xb, int c) {
    const int b = c >> 2, j = c & 3;
    const uint4 *xp = reinterpret_cast<const uint4 *>(xq + 256 * b + 64 * j);
    uint4 x0 = __ldg(xp), x1 = __ldg(xp + 1), x2 = __ldg(xp + 2), x3 = __ldg(xp + 3);
    uint2 bs = __ldg(reinterpret_cast<const uint2 *>(xb + 16 * b + 4 * j));
    float dx = __ldg(xd + b);
    int slo = 0, shi = 0;
    slo = __dp4a((int)u.lo[0], (int)x0.x, slo);
    slo = __dp4a((int)u.lo[1], (int)x0.y, slo);
    slo = __dp4a((int)u.lo[2], (int)x0.z, slo);
    slo = __dp4a((int)u.lo[3], (int)x0.w, slo);
    slo = __dp4a((int)u.lo[4], (int)x1.x, slo);
    slo = __dp4a((int)u.lo[5], (int)x1.y, slo);
    slo = __dp4a((int)u.lo[6], (int)x1.z, slo);
    slo = __dp4a((int)u.lo[7], (int)x1.w, slo);
    shi = __dp4a((int)u.hi[0], (int)x2.x, shi);
    shi = __dp4a((int)u.hi[1], (int)x2.y, shi);
    shi = __dp4a((int)u.hi[2], (int)x2.z, shi);
    shi = __dp4a((int)u.hi[3], (int)x2.w, shi);
    shi = __dp4a((int)u.hi[4], (int)x3.x, shi);
    shi = __dp4a((int)u.hi[5], (int)x3.y, shi);
    shi = __dp4a((int)u.hi[6], (int)x3.z, shi);
    shi = __dp4a((int)u.hi[7], (int)x3.w, shi);
    int b0 = (int)(int16_t)(bs.x & 0xffffu), b1 = (int)(int16_t)(bs.x >> 16);
    int b2 = (int)(int16_t)(bs.y & 0xffffu), b3 = (int)(int16_t)(bs.y >> 16);
    int isum = u.sc_lo * slo + u.sc_hi * shi;
    int msum = u.m_lo * (b0 + b1) + u.m_hi * (b2 + b3);
    return __fmul_rn(u.d * dx, (float)isum) - __fmul_rn(u.dmin * dx, (float)msum);
}

__device__ __forceinline__ float dot_q6_unit(const Q6Unit &u, const int8_t *xq, const float *xd, int c) {
    const int b = c >> 1, hh = c & 1;
    const uint4 *xp = reinterpret_cast<const uint4 *>(xq + 256 * b + 128 * hh);
    float dx = __ldg(xd + b);
    int isum = 0;
#pragma unroll
    for (int s2 = 0; s2 < 4; s2++) {  // two 16-element sub-blocks per 32 bytes of x
        uint4 xa = __ldg(xp + 2 * s2), xb = __ldg(xp + 2 * s2 + 1);
        int sa = 0, sb = 0;
        sa = __dp4a((int)u.q[8 * s2 + 0], (int)xa.x, sa);
        sa = __dp4a((int)u.q[8 * s2 + 1], (int)xa.y, sa);
        sa = __dp4a((int)u.q[8 * s2 + 2], (int)xa.z, sa);
        sa = __dp4a((int)u.q[8 * s2 + 3], (int)xa.w, sa);
        sb = __dp4a((int)u.q[8 * s2 + 4], (int)xb.x, sb);
        sb = __dp4a((int)u.q[8 * s2 + 5], (int)xb.y, sb);
        sb = __dp4a((int)u.q[8 * s2 + 6], (int)xb.z, sb);
        sb = __dp4a((int)u.q[8 * s2 + 7], (int)xb.w, sb);
        isum += u.sc[2 * s2] * sa + u.sc[2 * s2 + 1] * sb;
    }
    return __fmul_rn(u.d * dx, (float)isum);
}

template <int WT>
struct UnitOf;
template <>
struct UnitOf<TMOE_WT_Q4K> {
    using T = Q4Unit;
    static constexpr int elems = 64;
    static constexpr int block_bytes = TMOE_Q4K_BYTES;
};
template <>
struct UnitOf<TMOE_WT_Q6K> {
    using T = Q6Unit;
    static constexpr int elems = 128;
    static constexpr int block_bytes = TMOE_Q6K_BYTES;
};

template <int WT>
__device__ __forceinline__ void load_unit(const uint8_t *row, int c, typename UnitOf<WT>::T &u) {
    if constexpr (WT == TMOE_WT_Q4K)
        load_q4_unit(row, c, u);
    else
        load_q6_unit(row, c, u);
}

template <int WT>
__device__ __forceinline__ float dot_unit(const typename UnitOf<WT>::T &u, const int8_t *xq,
                                          const float *xd, const int16_t *xb, int c) {
    if constexpr (WT == TMOE_WT_Q4K)
        return dot_q4_unit(u, xq, xd, xb, c);
    else
        return dot_q6_unit(u, xq, xd, c);
}

__device__ __forceinline__ float silu_mul(float g, float u) { return (g / (1.0f + expf(-g))) * u; }

template <int WT, bool GATEUP, int LPR, int UPL>
__global__ void __launch_bounds__(GEMV_THREADS, 1) gemv_kernel(const GemvArgs a) {
    using Unit = typename UnitOf<WT>::T;
    constexpr int RPW = 32 / LPR;
    constexpr int RT = GEMV_NW * RPW;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + GEMV_MAX_STAGES;
    uint8_t *stage0 = smem + GEMV_BAR_BYTES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NS = a.n_stages;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], GEMV_NW);
        }
        fence_barrier_init();
    }
    __syncthreads();
    const int n_items = a.n_active[0] * a.tiles;
    const uint32_t row_bytes = (uint32_t)UnitOf<WT>::block_bytes * (uint32_t)(a.K / TMOE_QK);
    const uint32_t mat_bytes = RT * row_bytes;

    if (warp == GEMV_NW) {  // producer
        if (lane == 0) {
            int it = 0;
            for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++it) {
                const int s = it % NS;
                if (it >= NS && !mbar_wait_bounded(&empty[s], ((it / NS) - 1) & 1)) {
                    latch_error(a.err, TMOE_DEV_ERR_TIMEOUT);
                    break;
                }
                const int e = a.active[item / a.tiles];
                const int r0 = (item % a.tiles) * RT;
                uint8_t *dst = stage0 + (size_t)s * a.stage_bytes;
                mbar_arrive_expect_tx(&full[s], GATEUP ? 2 * mat_bytes : mat_bytes);
                bulk_g2s(dst, a.w0 + (size_t)e * a.nb2_0 + (size_t)r0 * a.nb1_0, mat_bytes, &full[s]);
                if constexpr (GATEUP)
                    bulk_g2s(dst + mat_bytes, a.w1 + (size_t)e * a.nb2_1 + (size_t)r0 * a.nb1_1, mat_bytes,
                             &full[s]);
            }
        }
        return;
    }

    const int units_per_row = a.K / UnitOf<WT>::elems;
    const int rl = warp * RPW + lane / LPR;  // row of the tile this lane works on
    const int li = lane % LPR;
    int it = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++it) {
        const int s = it % NS;
        if (!mbar_wait_bounded(&full[s], (it / NS) & 1)) {
            latch_error(a.err, TMOE_DEV_ERR_TIMEOUT);
            break;
        }
        const int e = a.active[item / a.tiles];
        const int r0 = (item % a.tiles) * RT;
        const uint8_t *st = stage0 + (size_t)s * a.stage_bytes;
        Unit u0[UPL];
        Unit u1[GATEUP ? UPL : 1];
#pragma unroll
        for (int k = 0; k < UPL; k++) {
            const int c = li + LPR * k;
            if (c < units_per_row) {
                load_unit<WT>(st + (size_t)rl * row_bytes, c, u0[k]);
                if constexpr (GATEUP) load_unit<WT>(st + mat_bytes + (size_t)rl * row_bytes, c, u1[k]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);

        const int beg = a.offsets[e], end = a.offsets[e + 1];
        for (int i = beg; i < end; i++) {
            const int p = a.perm[i];
            const int64_t xr = p / a.x_div;
            const int8_t *xq = a.xq + xr * a.K;
            const float *xd = a.xd + xr * (a.K / TMOE_QK);
            const int16_t *xb = a.xb + xr * (a.K / 16);
            float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll
            for (int k = 0; k < UPL; k++) {
                const int c = li + LPR * k;
                if (c < units_per_row) {
                    acc0 += dot_unit<WT>(u0[k], xq, xd, xb, c);
                    if constexpr (GATEUP) acc1 += dot_unit<WT>(u1[k], xq, xd, xb, c);
                }
            }
            acc0 = warp_sum_xor(acc0, LPR);
            if constexpr (GATEUP) acc1 = warp_sum_xor(acc1, LPR);
            if (li == 0) {
                float v = GATEUP ? silu_mul(acc0, acc1) : acc0;
                a.out[(int64_t)p * a.N + r0 + rl] = v;
            }
        }
    }
}

// ------------------------------------------------------------------ launcher
template <int WT, bool GATEUP, int LPR, int UPL>
static cudaError_t launch_one(const GemvArgs &args_in, int max_items, int sm_count, cudaStream_t st) {
    GemvArgs a = args_in;
    constexpr int RT = GEMV_NW * (32 / LPR);
    const uint32_t row_bytes = (uint32_t)UnitOf<WT>::block_bytes * (uint32_t)(a.K / TMOE_QK);
    const uint32_t mat = RT * row_bytes;
    a.tiles = a.N / RT;
    a.stage_bytes = ((GATEUP ? 2 : 1) * mat + 16 + 127) & ~127u;
    const uint32_t budget = 200 * 1024;
    int ns = (int)((budget - GEMV_BAR_BYTES) / a.stage_bytes);
    if (ns > GEMV_MAX_STAGES) ns = GEMV_MAX_STAGES;
    if (ns < 2) return cudaErrorInvalidValue;
    a.n_stages = ns;
    size_t smem = GEMV_BAR_BYTES + (size_t)ns * a.stage_bytes;
    auto kern = gemv_kernel<WT, GATEUP, LPR, UPL>;
    // The attribute is set once per device and size, so that launches after the first are plain
    // stream work (safe inside CUDA-graph capture).
    static int set_bytes[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if ((int)smem > set_bytes[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        set_bytes[dev] = (int)smem;
    }
    int items = max_items * a.tiles;
    int grid = items < sm_count ? items : sm_count;
    if (grid < 1) return cudaSuccess;
    kern<<<grid, GEMV_THREADS, smem, st>>>(a);
    return cudaGetLastError();
}

int gemv_rows_per_item(int wt, bool gateup, int K) {
    int units = K / (wt == TMOE_WT_Q4K ? 64 : 128);
    int lpr = (gateup ? units <= 16 : units <= 24) ? 8 : 32;
    return GEMV_NW * (32 / lpr);
}

cudaError_t launch_gemv(int wt, bool gateup, const GemvArgs &a, int max_items, int sm_count,
                        cudaStream_t st) {
    const int units = a.K / (wt == TMOE_WT_Q4K ? 64 : 128);
    if (a.K % TMOE_QK != 0 || units <= 0) return cudaErrorInvalidValue;
    if (a.N % gemv_rows_per_item(wt, gateup, a.K) != 0) return cudaErrorInvalidValue;
    if (wt == TMOE_WT_Q4K) {
        if (gateup) {
            if (units <= 8) return launch_one<TMOE_WT_Q4K, true, 8, 1>(a, max_items, sm_count, st);
            if (units <= 16) return launch_one<TMOE_WT_Q4K, true, 8, 2>(a, max_items, sm_count, st);
            if (units <= 32) return launch_one<TMOE_WT_Q4K, true, 32, 1>(a, max_items, sm_count, st);
            if (units <= 64) return launch_one<TMOE_WT_Q4K, true, 32, 2>(a, max_items, sm_count, st);
        } else {
            if (units <= 8) return launch_one<TMOE_WT_Q4K, false, 8, 1>(a, max_items, sm_count, st);
            if (units <= 16) return launch_one<TMOE_WT_Q4K, false, 8, 2>(a, max_items, sm_count, st);
            if (units <= 24) return launch_one<TMOE_WT_Q4K, false, 8, 3>(a, max_items, sm_count, st);
            if (units <= 32) return launch_one<TMOE_WT_Q4K, false, 32, 1>(a, max_items, sm_count, st);
            if (units <= 64) return launch_one<TMOE_WT_Q4K, false, 32, 2>(a, max_items, sm_count, st);
            if (units <= 128) return launch_one<TMOE_WT_Q4K, false, 32, 4>(a, max_items, sm_count, st);
        }
    } else {
        if (gateup) {
            if (units <= 8) return launch_one<TMOE_WT_Q6K, true, 8, 1>(a, max_items, sm_count, st);
            if (units <= 16) return launch_one<TMOE_WT_Q6K, true, 8, 2>(a, max_items, sm_count, st);
            if (units <= 32) return launch_one<TMOE_WT_Q6K, true, 32, 1>(a, max_items, sm_count, st);
        } else {
            if (units <= 8) return launch_one<TMOE_WT_Q6K, false, 8, 1>(a, max_items, sm_count, st);
            if (units <= 16) return launch_one<TMOE_WT_Q6K, false, 8, 2>(a, max_items, sm_count, st);
            if (units <= 24) return launch_one<TMOE_WT_Q6K, false, 8, 3>(a, max_items, sm_count, st);
            if (units <= 32) return launch_one<TMOE_WT_Q6K, false, 32, 1>(a, max_items, sm_count, st);
            if (units <= 64) return launch_one<TMOE_WT_Q6K, false, 32, 2>(a, max_items, sm_count, st);
        }
    }
    return cudaErrorInvalidValue;
}

}  // namespace tmoe
