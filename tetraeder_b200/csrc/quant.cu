// Block (de)quantisation on the device, the drop-in for crates/ggml-sys/src/quant.rs
// (quantize :52, to_f32 :19) for Q4_K and Q6_K.
//
// The quantiser is this project's own fit of the block formats (per 32-sub-block min/max for
// Q4_K, per 16-sub-block amax/31 for Q6_K, 6-bit / int8 scales relative to the super-block
// maximum, f16 super-block scales), written with explicit round-to-nearest operations so that
// its bytes equal the CPU oracle's bit for bit.  The decoders follow ggml's dequantize_row_q4_K
// / q6_K operation order: (d*sc)*q - (dmin*m) and (d*sc)*q.
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.cuh"

namespace tmoe {

__device__ __forceinline__ uint16_t f2h_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }

// One thread per super-block.
__global__ void quantize_q4k_kernel(const float *__restrict__ x, int64_t nblocks, uint8_t *__restrict__ out) {
    int64_t bi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (bi >= nblocks) return;
    const float *xb = x + bi * 256;
    uint8_t *blk = out + bi * TMOE_Q4K_BYTES;
    float scale[8], mn[8], max_scale = 0.0f, max_min = 0.0f;
    for (int s = 0; s < 8; s++) {
        float lo = xb[32 * s], hi = lo;
        for (int l = 1; l < 32; l++) {
            float v = xb[32 * s + l];
            lo = v < lo ? v : lo;
            hi = v > hi ? v : hi;
        }
        if (lo > 0.0f) lo = 0.0f;
        scale[s] = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
        mn[s] = -lo;
        if (scale[s] > max_scale) max_scale = scale[s];
        if (mn[s] > max_min) max_min = mn[s];
    }
    uint16_t dh = f2h_bits(__fdiv_rn(max_scale, 63.0f)), mh = f2h_bits(__fdiv_rn(max_min, 63.0f));
    float d = h2f(dh), dmin = h2f(mh);
    int sc[8], m[8];
    for (int s = 0; s < 8; s++) {
        int a = d > 0.0f ? __float2int_rn(__fdiv_rn(scale[s], d)) : 0;
        int b = dmin > 0.0f ? __float2int_rn(__fdiv_rn(mn[s], dmin)) : 0;
        sc[s] = a < 0 ? 0 : (a > 63 ? 63 : a);
        m[s] = b < 0 ? 0 : (b > 63 ? 63 : b);
    }
    uint8_t hdr[16];
    hdr[0] = dh & 0xff, hdr[1] = dh >> 8, hdr[2] = mh & 0xff, hdr[3] = mh >> 8;
    for (int s = 0; s < 4; s++) {
        hdr[4 + s] = (uint8_t)(sc[s] | ((sc[s + 4] >> 4) << 6));
        hdr[8 + s] = (uint8_t)(m[s] | ((m[s + 4] >> 4) << 6));
        hdr[12 + s] = (uint8_t)((sc[s + 4] & 0x0f) | ((m[s + 4] & 0x0f) << 4));
    }
    for (int i = 0; i < 16; i++) blk[i] = hdr[i];
    for (int j = 0; j < 4; j++)
        for (int l = 0; l < 32; l++) {
            int q2[2];
            for (int hlf = 0; hlf < 2; hlf++) {
                int i = 64 * j + 32 * hlf + l, s = i / 32;
                float step = __fmul_rn(d, (float)sc[s]);
                float off = __fmul_rn(dmin, (float)m[s]);
                int q = step > 0.0f ? __float2int_rn(__fdiv_rn(__fadd_rn(xb[i], off), step)) : 0;
                q2[hlf] = q < 0 ? 0 : (q > 15 ? 15 : q);
            }
            blk[16 + 32 * j + l] = (uint8_t)(q2[0] | (q2[1] << 4));
        }
}

__global__ void quantize_q6k_kernel(const float *__restrict__ x, int64_t nblocks, uint8_t *__restrict__ out) {
    int64_t bi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (bi >= nblocks) return;
    const float *xb = x + bi * 256;
    uint8_t *blk = out + bi * TMOE_Q6K_BYTES;
    float scale[16], max_scale = 0.0f;
    for (int s = 0; s < 16; s++) {
        float a = 0.0f;
        for (int l = 0; l < 16; l++) a = fmaxf(a, fabsf(xb[16 * s + l]));
        scale[s] = __fdiv_rn(a, 31.0f);
        if (scale[s] > max_scale) max_scale = scale[s];
    }
    uint16_t dh = f2h_bits(__fdiv_rn(max_scale, 127.0f));
    float d = h2f(dh);
    int sc[16];
    for (int s = 0; s < 16; s++) {
        int a = d > 0.0f ? __float2int_rn(__fdiv_rn(scale[s], d)) : 0;
        sc[s] = a < -128 ? -128 : (a > 127 ? 127 : a);
        blk[192 + s] = (uint8_t)(int8_t)sc[s];
    }
    blk[208] = dh & 0xff, blk[209] = dh >> 8;
    for (int h = 0; h < 2; h++) {
        for (int r = 0; r < 64; r++) {  // ql byte 64h + r: low nibble element r, high nibble r + 64
            int q2[2];
            for (int hlf = 0; hlf < 2; hlf++) {
                int i = 128 * h + r + 64 * hlf;
                float step = __fmul_rn(d, (float)sc[i / 16]);
                int q = step != 0.0f ? __float2int_rn(__fdiv_rn(xb[i], step)) : 0;
                q = (q < -32 ? -32 : (q > 31 ? 31 : q)) + 32;
                q2[hlf] = q;
            }
            blk[64 * h + r] = (uint8_t)((q2[0] & 0x0f) | ((q2[1] & 0x0f) << 4));
        }
        for (int l = 0; l < 32; l++) {  // qh byte 32h + l: bits 4-5 of elements l, l+32, l+64, l+96
            uint8_t v = 0;
            for (int g = 0; g < 4; g++) {
                int i = 128 * h + 32 * g + l;
                float step = __fmul_rn(d, (float)sc[i / 16]);
                int q = step != 0.0f ? __float2int_rn(__fdiv_rn(xb[i], step)) : 0;
                q = (q < -32 ? -32 : (q > 31 ? 31 : q)) + 32;
                v |= (uint8_t)(((q >> 4) & 3) << (2 * g));
            }
            blk[128 + 32 * h + l] = v;
        }
    }
}

// Elements 32c .. 32c+31 of the super-block at `blk` (one Q4_K sub-block or two Q6_K sub-blocks).
__device__ void dequant32(int wt, const uint8_t *__restrict__ blk, int c, float *__restrict__ o) {
    if (wt == TMOE_WT_Q4K) {
        float d = h2f((uint16_t)(blk[0] | (blk[1] << 8))), dmin = h2f((uint16_t)(blk[2] | (blk[3] << 8)));
        const uint8_t *sc = blk + 4;
        int s = c, scale, mn;
        if (s < 4) {
            scale = sc[s] & 63;
            mn = sc[s + 4] & 63;
        } else {
            scale = (sc[s + 4] & 0x0f) | ((sc[s - 4] >> 6) << 4);
            mn = (sc[s + 4] >> 4) | ((sc[s] >> 6) << 4);
        }
        float d1 = __fmul_rn(d, (float)scale), m1 = __fmul_rn(dmin, (float)mn);
        const uint8_t *qs = blk + 16 + 32 * (c / 2);
        for (int l = 0; l < 32; l++) {
            int q = (c & 1) ? (qs[l] >> 4) : (qs[l] & 0x0f);
            o[l] = __fsub_rn(__fmul_rn(d1, (float)q), m1);
        }
    } else {
        const uint8_t *ql = blk, *qh = blk + 128;
        const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192);
        float d = h2f((uint16_t)(blk[208] | (blk[209] << 8)));
        for (int l = 0; l < 32; l++) {
            int i = 32 * c + l, h = i / 128, r = i % 128;
            int lo = r < 64 ? (ql[64 * h + r] & 0x0f) : (ql[64 * h + r - 64] >> 4);
            int hi = (qh[32 * h + (r % 32)] >> (2 * (r / 32))) & 3;
            o[l] = __fmul_rn(__fmul_rn(d, (float)sc[i / 16]), (float)((lo | (hi << 4)) - 32));
        }
    }
}

// One thread per 32 outputs.
__global__ void dequantize_kernel(int wt, const uint8_t *__restrict__ in, int64_t n, float *__restrict__ out) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g * 32 >= n) return;
    const int64_t b = g / 8;
    const uint8_t *blk = in + b * (wt == TMOE_WT_Q4K ? TMOE_Q4K_BYTES : TMOE_Q6K_BYTES);
    dequant32(wt, blk, (int)(g % 8), out + g * 32);
}

// get_rows: out[i][:] = row rows[i] of W (F32, F16, Q4_K or Q6_K rows of K elements, nb1 bytes
// apart).  One CTA per output row.
__global__ void get_rows_kernel(int32_t type, const uint8_t *__restrict__ W, size_t nb1, int K, int64_t n_rows_w,
                                const int32_t *__restrict__ rows, float *__restrict__ out, int *err) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = blockIdx.x;
    const int32_t r = rows[i];
    float *o = out + i * K;
    if (r < 0 || r >= n_rows_w) {  // an out-of-range row: zeros and the error flag
        for (int c = threadIdx.x; c < K; c += blockDim.x) o[c] = 0.0f;
        if (threadIdx.x == 0 && err) atomicCAS(err, 0, TMOE_DEV_ERR_BADID);
        return;
    }
    const uint8_t *row = W + (size_t)r * nb1;
    if (type == 0) {
        for (int c = threadIdx.x; c < K; c += blockDim.x) o[c] = reinterpret_cast<const float *>(row)[c];
    } else if (type == 1) {
        for (int c = threadIdx.x; c < K; c += blockDim.x) o[c] = h2f(reinterpret_cast<const uint16_t *>(row)[c]);
    } else {
        const int wt = type == 12 ? TMOE_WT_Q4K : TMOE_WT_Q6K;
        const int bb = wt == TMOE_WT_Q4K ? TMOE_Q4K_BYTES : TMOE_Q6K_BYTES;
        for (int g = threadIdx.x; g < K / 32; g += blockDim.x) dequant32(wt, row + (size_t)(g / 8) * bb, g % 8, o + g * 32);
    }
}

cudaError_t launch_quantize(int wt, const float *x, int64_t nblocks, uint8_t *out, cudaStream_t st) {
    if (nblocks <= 0) return cudaSuccess;
    unsigned grid = (unsigned)((nblocks + 127) / 128);
    if (wt == TMOE_WT_Q4K)
        quantize_q4k_kernel<<<grid, 128, 0, st>>>(x, nblocks, out);
    else
        quantize_q6k_kernel<<<grid, 128, 0, st>>>(x, nblocks, out);
    return cudaGetLastError();
}

cudaError_t launch_get_rows(int32_t type, const uint8_t *W, size_t nb1, int K, int64_t n_rows_w, const int32_t *rows,
                            int64_t n, float *out, int *err, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    if (n > 0x7fffffff) return cudaErrorInvalidValue;
    launch_k(get_rows_kernel, (unsigned)n, 128, 0, st, type, W, nb1, K, n_rows_w, rows, out, err);
    return cudaGetLastError();
}

cudaError_t launch_dequantize(int wt, const uint8_t *in, int64_t n, float *out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    int64_t chunks = n / 32;
    dequantize_kernel<<<(unsigned)((chunks + 255) / 256), 256, 0, st>>>(wt, in, n, out);
    return cudaGetLastError();
}

// One CTA per (8-row group, matrix): the group's 8 ggml rows are staged in shared memory, then
// every output unit is written in order as 16-byte words (each byte taken through q6r_offset's
// inverse: the unit's byte o holds byte off of row g, found by search over the 210 offsets once
// per CTA into a shared table).
__global__ void __launch_bounds__(256) prepack_q6k_kernel(const uint8_t *__restrict__ src, size_t nb1, size_t nb2,
                                                          int nb, uint8_t *__restrict__ dst, int64_t groups) {
    extern __shared__ __align__(16) uint8_t pk_smem[];
    uint16_t *inv = reinterpret_cast<uint16_t *>(pk_smem);  // unit byte -> g * 210 + off
    uint8_t *rows = pk_smem + 2 * TMOE_Q6R_UNIT;
    const int64_t grp = blockIdx.x, mat = blockIdx.y;
    for (int i = threadIdx.x; i < 8 * TMOE_Q6K_BYTES; i += blockDim.x) {
        const int g = i / TMOE_Q6K_BYTES, off = i - g * TMOE_Q6K_BYTES;
        inv[q6r_offset(g, off)] = (uint16_t)i;
    }
    const int rb = nb * TMOE_Q6K_BYTES;
    const uint8_t *s0 = src + (size_t)mat * nb2 + (size_t)grp * 8 * nb1;
    if (nb1 == (size_t)rb && ((uintptr_t)s0 & 15) == 0) {  // the 8 rows are one span of 8 * rb = 16 * 105 nb bytes
        for (int i = threadIdx.x; i < 8 * rb / 16; i += blockDim.x)
            reinterpret_cast<uint4 *>(rows)[i] = __ldg(reinterpret_cast<const uint4 *>(s0) + i);
    } else {
        for (int i = threadIdx.x; i < 8 * rb; i += blockDim.x) {
            const int g = i / rb, c = i - g * rb;
            rows[i] = s0[(size_t)g * nb1 + c];
        }
    }
    __syncthreads();
    uint8_t *out = dst + ((size_t)mat * groups + (size_t)grp) * (size_t)nb * TMOE_Q6R_UNIT;
    for (int w = threadIdx.x; w < nb * TMOE_Q6R_UNIT / 16; w += blockDim.x) {
        const int b = (16 * w) / TMOE_Q6R_UNIT, o0 = 16 * w - b * TMOE_Q6R_UNIT;
        __align__(16) uint8_t v[16];
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const int i = inv[o0 + j], g = i / TMOE_Q6K_BYTES, off = i - g * TMOE_Q6K_BYTES;
            v[j] = rows[g * rb + b * TMOE_Q6K_BYTES + off];
        }
        *reinterpret_cast<uint4 *>(out + 16 * (size_t)w) = *reinterpret_cast<const uint4 *>(v);
    }
}

cudaError_t launch_prepack_q6k(const uint8_t *src, size_t nb1, size_t nb2, int64_t n_rows, int K, int64_t n_mats,
                               uint8_t *dst, cudaStream_t st) {
    if (n_rows <= 0 || n_mats <= 0) return cudaSuccess;
    const int nb = K / TMOE_QK;
    const size_t smem = 2 * TMOE_Q6R_UNIT + (size_t)8 * nb * TMOE_Q6K_BYTES;
    if (K <= 0 || K % TMOE_QK || n_rows % 8 || ((uintptr_t)dst & 15) || smem > 200 * 1024 || n_mats > 65535 ||
        n_rows / 8 > 0x7fffffff)
        return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        const cudaError_t e =
            cudaFuncSetAttribute(prepack_q6k_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    const int64_t groups = n_rows / 8;
    prepack_q6k_kernel<<<dim3((unsigned)groups, (unsigned)n_mats), 256, smem, st>>>(src, nb1, nb2, nb, dst, groups);
    return cudaGetLastError();
}

}  // namespace tmoe
