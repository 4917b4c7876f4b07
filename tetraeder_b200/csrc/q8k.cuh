// Q8_K quantisation of one 256-element block by one warp (ggml quantize_row_q8_K_ref restated):
// the first element of largest magnitude maps to -127, iscale = -127 / max,
// q = min(127, round_half_even(iscale * x)), d = 1 / iscale, plus the 16-element block sums.
// Every use (the standalone kernel and the fused sites) calls this routine, so the bytes agree.
#pragma once

#include "common.cuh"
#include "kernels.cuh"

namespace tmoe {

// Lane l holds elements 8l .. 8l+7 in v.  Returns the lane's 8 quantised values packed in q
// (little-endian), the block's d, and s16 = the sum over the lane's 16-element group (lanes 2g
// and 2g+1 both hold group g's sum).
__device__ __forceinline__ void q8k_block_warp(const float (&v)[8], uint2 &q, float &d, int &s16) {
    const int lane = threadIdx.x & 31;
    float amax = 0.0f, maxv = 0.0f;
    int idx = 0x7fffffff;
#pragma unroll
    for (int c = 0; c < 8; c++) {
        const float ax = fabsf(v[c]);
        if (ax > amax) {
            amax = ax;
            maxv = v[c];
            idx = 8 * lane + c;
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, amax, off);
        const float ov = __shfl_xor_sync(0xffffffffu, maxv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
        if (oa > amax || (oa == amax && oi < idx)) {
            amax = oa;
            maxv = ov;
            idx = oi;
        }
    }
    int qi[8];
    d = 0.0f;
    if (amax == 0.0f) {
#pragma unroll
        for (int c = 0; c < 8; c++) qi[c] = 0;
    } else {
        const float iscale = __fdiv_rn(-127.0f, maxv);
#pragma unroll
        for (int c = 0; c < 8; c++) {
            const int t = __float2int_rn(__fmul_rn(iscale, v[c]));
            qi[c] = t > 127 ? 127 : t;
        }
        d = __fdiv_rn(1.0f, iscale);
    }
    int s = 0;
#pragma unroll
    for (int c = 0; c < 8; c++) s += qi[c];
    s16 = s + __shfl_xor_sync(0xffffffffu, s, 1);
    q.x = (uint32_t)(qi[0] & 0xff) | ((uint32_t)(qi[1] & 0xff) << 8) | ((uint32_t)(qi[2] & 0xff) << 16) |
          ((uint32_t)(qi[3] & 0xff) << 24);
    q.y = (uint32_t)(qi[4] & 0xff) | ((uint32_t)(qi[5] & 0xff) << 8) | ((uint32_t)(qi[6] & 0xff) << 16) |
          ((uint32_t)(qi[7] & 0xff) << 24);
}

}  // namespace tmoe

namespace tmoe {

// Stores the warp's Q8_K block b of row `row` (from q8k_block_warp) in the Q8Rows layout, with the
// sub-block sums of the consumer's weight type split into exact low / high bytes.  The 256 values
// of a block are stored in the consumer's order (q8_frag_pos): for Q6_K the fragment order, in
// which the GEMV thread of MMA column t4 reads its operand bytes of the block as 64 contiguous bytes.
__device__ __forceinline__ void q8k_store_warp(const Q8Rows &o, int64_t row, int K, int b, const uint2 &q, float d,
                                               int s16) {
    const int lane = threadIdx.x & 31;
    const int nb = K / TMOE_QK;
    int8_t *blk = o.qs + row * K + (int64_t)b * TMOE_QK;
    if (o.wt == TMOE_WT_Q4K) {
        *reinterpret_cast<uint2 *>(blk + q8_frag_pos(o.wt, 8 * lane)) = q;
    } else {
        *reinterpret_cast<uint32_t *>(blk + q8_frag_pos(o.wt, 8 * lane)) = q.x;
        *reinterpret_cast<uint32_t *>(blk + q8_frag_pos(o.wt, 8 * lane + 4)) = q.y;
    }
    if (lane == 0) o.d[row * nb + b] = d;
    uint32_t lo = 0, hi = 0;
    if (o.wt != TMOE_WT_Q4K) {  // Q6_K: 16-element sums: lane 2g holds sum g; 4 sums per word
        if ((lane & 1) == 0) {
            const int i = (lane >> 1) & 3;
            lo = (uint32_t)(s16 & 63) << (8 * i);
            hi = (uint32_t)((s16 >> 6) & 0xff) << (8 * i);
        }
        for (int off = 2; off <= 4; off <<= 1) {
            lo |= __shfl_xor_sync(0xffffffffu, lo, off);
            hi |= __shfl_xor_sync(0xffffffffu, hi, off);
        }
        if ((lane & 7) == 0) {
            const int64_t w = (row * nb + b) * 4 + (lane >> 3);
            o.bl[w] = lo;
            o.bh[w] = hi;
        }
    } else {  // 32-element sums: lanes 4g hold sum g after adding the neighbour pair
        const int s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 2);
        if ((lane & 3) == 0) {
            const int i = (lane >> 2) & 3;
            lo = (uint32_t)(s32 & 63) << (8 * i);
            hi = (uint32_t)((s32 >> 6) & 0xff) << (8 * i);
        }
        for (int off = 4; off <= 8; off <<= 1) {
            lo |= __shfl_xor_sync(0xffffffffu, lo, off);
            hi |= __shfl_xor_sync(0xffffffffu, hi, off);
        }
        if ((lane & 15) == 0) {
            const int64_t w = (row * nb + b) * 2 + (lane >> 4);
            o.bl[w] = lo;
            o.bh[w] = hi;
        }
    }
}

}  // namespace tmoe
