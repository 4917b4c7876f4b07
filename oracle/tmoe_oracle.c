/*
 * tmoe_oracle.c -- CPU restatement of Tetraeder's Qwen3-MoE layer hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA path and the timed CPU
 * baseline.  See tmoe_oracle.h for the reference lines each part follows.
 * Build: oracle/Makefile (gcc -O3 -fopenmp -ffp-contract=off).
 */
#include "tmoe_oracle.h"

#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* half precision (IEEE binary16)                                            */
/* ------------------------------------------------------------------------ */

float tmo_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t bits;
    float f;
    if (e == 0) {
        /* zero or subnormal: m * 2^-24, exact in f32 */
        f = (float)m * (1.0f / 16777216.0f);
        return sign ? -f : f;
    }
    if (e == 31)
        bits = sign | 0x7f800000u | (m << 13);
    else
        bits = sign | ((e + 112u) << 23) | (m << 13);
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t tmo_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) /* inf / nan */
        return sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u);
    if (ax >= 0x477ff000u) /* >= 65520 rounds to inf */
        return sign | 0x7c00u;
    if (ax < 0x38800000u) { /* below 2^-14: subnormal half */
        float v;
        memcpy(&v, &ax, 4);
        float r = rintf(v * 16777216.0f); /* exact scaling, round half even */
        return sign | (uint16_t)r;
    }
    uint32_t mant = ax & 0x7fffffu;
    uint32_t h = ((((ax >> 23) - 112u)) << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return sign | (uint16_t)h;
}

/* ------------------------------------------------------------------------ */
/* block formats                                                             */
/* ------------------------------------------------------------------------ */

size_t tmo_row_size(int type, int64_t ncols) {
    switch (type) {
    case TMO_TYPE_F32: return (size_t)ncols * 4;
    case TMO_TYPE_F16: return (size_t)ncols * 2;
    case TMO_TYPE_Q4_K: return (size_t)(ncols / TMO_QK_K) * TMO_Q4K_BYTES;
    case TMO_TYPE_Q6_K: return (size_t)(ncols / TMO_QK_K) * TMO_Q6K_BYTES;
    case TMO_TYPE_Q8_K: return (size_t)(ncols / TMO_QK_K) * TMO_Q8K_BYTES;
    default: return 0;
    }
}

static inline int nearest(float v) { return (int)rintf(v); } /* round half to even */

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline void wr16(uint8_t *p, uint16_t v) {
    p[0] = (uint8_t)(v & 0xff);
    p[1] = (uint8_t)(v >> 8);
}

/* Q4_K scale/min of sub-block s (0..7) from the 12 packed bytes (ggml get_scale_min_k4). */
static inline void q4k_scale_min(const uint8_t *sc, int s, int *scale, int *min) {
    if (s < 4) {
        *scale = sc[s] & 63;
        *min = sc[s + 4] & 63;
    } else {
        *scale = (sc[s + 4] & 0x0f) | ((sc[s - 4] >> 6) << 4);
        *min = (sc[s + 4] >> 4) | ((sc[s] >> 6) << 4);
    }
}

/* Our own Q4_K fit: per 32-sub-block min/max range, then 6-bit scales relative to the
 * super-block maxima.  Element i of the super-block: i = 64*j + l (l < 32) is the low nibble
 * of qs[32*j + l], i = 64*j + 32 + l its high nibble; sub-block of i is i / 32. */
static void quantize_block_q4k(const float *x, uint8_t *blk) {
    float scale[8], mn[8];
    float max_scale = 0.f, max_min = 0.f;
    for (int s = 0; s < 8; s++) {
        float lo = x[32 * s], hi = x[32 * s];
        for (int l = 1; l < 32; l++) {
            float v = x[32 * s + l];
            if (v < lo) lo = v;
            if (v > hi) hi = v;
        }
        if (lo > 0.f) lo = 0.f;
        scale[s] = (hi - lo) / 15.f;
        mn[s] = -lo;
        if (scale[s] > max_scale) max_scale = scale[s];
        if (mn[s] > max_min) max_min = mn[s];
    }
    uint16_t dh = tmo_f32_to_f16(max_scale / 63.f);
    uint16_t mh = tmo_f32_to_f16(max_min / 63.f);
    float d = tmo_f16_to_f32(dh), dmin = tmo_f16_to_f32(mh);
    int sc[8], m[8];
    for (int s = 0; s < 8; s++) {
        int a = d > 0.f ? nearest(scale[s] / d) : 0;
        int b = dmin > 0.f ? nearest(mn[s] / dmin) : 0;
        sc[s] = a < 0 ? 0 : (a > 63 ? 63 : a);
        m[s] = b < 0 ? 0 : (b > 63 ? 63 : b);
    }
    memset(blk, 0, TMO_Q4K_BYTES);
    wr16(blk, dh);
    wr16(blk + 2, mh);
    uint8_t *scp = blk + 4;
    for (int s = 0; s < 4; s++) {
        scp[s] = (uint8_t)(sc[s] | ((sc[s + 4] >> 4) << 6));
        scp[s + 4] = (uint8_t)(m[s] | ((m[s + 4] >> 4) << 6));
        scp[s + 8] = (uint8_t)((sc[s + 4] & 0x0f) | ((m[s + 4] & 0x0f) << 4));
    }
    uint8_t *qs = blk + 16;
    for (int i = 0; i < 256; i++) {
        int s = i / 32;
        float step = d * (float)sc[s];
        float off = dmin * (float)m[s];
        int q = step > 0.f ? nearest((x[i] + off) / step) : 0;
        q = q < 0 ? 0 : (q > 15 ? 15 : q);
        int j = i / 64, l = i % 64;
        if (l < 32)
            qs[32 * j + l] |= (uint8_t)q;
        else
            qs[32 * j + (l - 32)] |= (uint8_t)(q << 4);
    }
}

/* Our own Q6_K fit: per 16-sub-block amax/31, int8 scales relative to the super-block maximum.
 * Element i = 128*h + r: low nibble in ql[64*h + r] (r < 64) or the high nibble of
 * ql[64*h + r - 64]; bits 4-5 in qh[32*h + r%32] at shift 2*(r/32); value q - 32. */
static void quantize_block_q6k(const float *x, uint8_t *blk) {
    float scale[16], max_scale = 0.f;
    for (int s = 0; s < 16; s++) {
        float a = 0.f;
        for (int l = 0; l < 16; l++) {
            float v = fabsf(x[16 * s + l]);
            if (v > a) a = v;
        }
        scale[s] = a / 31.f;
        if (scale[s] > max_scale) max_scale = scale[s];
    }
    uint16_t dh = tmo_f32_to_f16(max_scale / 127.f);
    float d = tmo_f16_to_f32(dh);
    int sc[16];
    for (int s = 0; s < 16; s++) {
        int a = d > 0.f ? nearest(scale[s] / d) : 0;
        sc[s] = a < -128 ? -128 : (a > 127 ? 127 : a);
    }
    memset(blk, 0, TMO_Q6K_BYTES);
    uint8_t *ql = blk, *qh = blk + 128;
    int8_t *scp = (int8_t *)(blk + 192);
    for (int s = 0; s < 16; s++) scp[s] = (int8_t)sc[s];
    wr16(blk + 208, dh);
    for (int i = 0; i < 256; i++) {
        float step = d * (float)sc[i / 16];
        int q = step != 0.f ? nearest(x[i] / step) : 0;
        q = q < -32 ? -32 : (q > 31 ? 31 : q);
        q += 32;
        int h = i / 128, r = i % 128;
        if (r < 64)
            ql[64 * h + r] |= (uint8_t)(q & 0x0f);
        else
            ql[64 * h + r - 64] |= (uint8_t)((q & 0x0f) << 4);
        qh[32 * h + (r % 32)] |= (uint8_t)(((q >> 4) & 3) << (2 * (r / 32)));
    }
}

void tmo_quantize_q4k(const float *x, void *out, int64_t nrows, int64_t ncols) {
    int64_t nb = ncols / TMO_QK_K;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < nrows; r++)
        for (int64_t b = 0; b < nb; b++)
            quantize_block_q4k(x + r * ncols + b * TMO_QK_K,
                               (uint8_t *)out + (r * nb + b) * TMO_Q4K_BYTES);
}

void tmo_quantize_q6k(const float *x, void *out, int64_t nrows, int64_t ncols) {
    int64_t nb = ncols / TMO_QK_K;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < nrows; r++)
        for (int64_t b = 0; b < nb; b++)
            quantize_block_q6k(x + r * ncols + b * TMO_QK_K,
                               (uint8_t *)out + (r * nb + b) * TMO_Q6K_BYTES);
}

/* Dequantisation, in the operation order of ggml dequantize_row_q4_K / q6_K and gguf-py:
 * Q4_K: (d*sc)*q - (dmin*m); Q6_K: (d*sc)*(q-32). */
static void dequant_block_q4k(const uint8_t *blk, float *y) {
    float d = tmo_f16_to_f32(rd16(blk)), dmin = tmo_f16_to_f32(rd16(blk + 2));
    const uint8_t *scp = blk + 4, *qs = blk + 16;
    for (int j = 0; j < 4; j++) {
        int sc0, m0, sc1, m1;
        q4k_scale_min(scp, 2 * j, &sc0, &m0);
        q4k_scale_min(scp, 2 * j + 1, &sc1, &m1);
        float d0 = d * (float)sc0, mm0 = dmin * (float)m0;
        float d1 = d * (float)sc1, mm1 = dmin * (float)m1;
        for (int l = 0; l < 32; l++) {
            y[64 * j + l] = d0 * (float)(qs[32 * j + l] & 0x0f) - mm0;
            y[64 * j + 32 + l] = d1 * (float)(qs[32 * j + l] >> 4) - mm1;
        }
    }
}

static void dequant_block_q6k(const uint8_t *blk, float *y) {
    const uint8_t *ql = blk, *qh = blk + 128;
    const int8_t *scp = (const int8_t *)(blk + 192);
    float d = tmo_f16_to_f32(rd16(blk + 208));
    for (int i = 0; i < 256; i++) {
        int h = i / 128, r = i % 128;
        int lo = r < 64 ? (ql[64 * h + r] & 0x0f) : (ql[64 * h + r - 64] >> 4);
        int hi = (qh[32 * h + (r % 32)] >> (2 * (r / 32))) & 3;
        int q = (lo | (hi << 4)) - 32;
        y[i] = (d * (float)scp[i / 16]) * (float)q;
    }
}

void tmo_dequantize(int type, const void *in, float *out, int64_t n) {
    const uint8_t *p = (const uint8_t *)in;
    switch (type) {
    case TMO_TYPE_F32: memcpy(out, in, (size_t)n * 4); break;
    case TMO_TYPE_F16:
        for (int64_t i = 0; i < n; i++) out[i] = tmo_f16_to_f32(rd16(p + 2 * i));
        break;
    case TMO_TYPE_Q4_K:
        for (int64_t b = 0; b < n / TMO_QK_K; b++)
            dequant_block_q4k(p + b * TMO_Q4K_BYTES, out + b * TMO_QK_K);
        break;
    case TMO_TYPE_Q6_K:
        for (int64_t b = 0; b < n / TMO_QK_K; b++)
            dequant_block_q6k(p + b * TMO_Q6K_BYTES, out + b * TMO_QK_K);
        break;
    case TMO_TYPE_Q8_K: tmo_dequantize_q8k((const tmo_block_q8k *)in, out, n); break;
    default: break;
    }
}

/* ggml quantize_row_q8_K_ref, restated: the element of largest magnitude (first one on ties)
 * maps to -127; iscale = -127/max; q = min(127, round_half_even(iscale*x)); d = 1/iscale. */
void tmo_quantize_q8k(const float *x, tmo_block_q8k *y, int64_t n) {
    for (int64_t b = 0; b < n / TMO_QK_K; b++, x += TMO_QK_K) {
        float amax = 0.f, maxv = 0.f;
        for (int j = 0; j < TMO_QK_K; j++) {
            float ax = fabsf(x[j]);
            if (ax > amax) {
                amax = ax;
                maxv = x[j];
            }
        }
        if (amax == 0.f) {
            memset(&y[b], 0, sizeof(y[b]));
            continue;
        }
        float iscale = -127.f / maxv;
        for (int j = 0; j < TMO_QK_K; j++) {
            int v = nearest(iscale * x[j]);
            y[b].qs[j] = (int8_t)(v > 127 ? 127 : v);
        }
        for (int j = 0; j < TMO_QK_K / 16; j++) {
            int s = 0;
            for (int i = 0; i < 16; i++) s += y[b].qs[16 * j + i];
            y[b].bsums[j] = (int16_t)s;
        }
        y[b].d = 1.f / iscale;
    }
}

void tmo_dequantize_q8k(const tmo_block_q8k *y, float *x, int64_t n) {
    for (int64_t b = 0; b < n / TMO_QK_K; b++)
        for (int j = 0; j < TMO_QK_K; j++) x[b * TMO_QK_K + j] = y[b].d * (float)y[b].qs[j];
}

/* vec_dot_q4_K_q8_K semantics: per super-block, the integer sums of each 32-sub-block times its
 * 6-bit scale, and the block sums times the 6-bit mins; scaled by d*dx and dmin*dx. */
float tmo_vec_dot_q4k_q8k(int64_t ncols, const void *w, const tmo_block_q8k *x) {
    const uint8_t *blk = (const uint8_t *)w;
    float acc = 0.f;
    for (int64_t b = 0; b < ncols / TMO_QK_K; b++, blk += TMO_Q4K_BYTES) {
        const int8_t *q8 = x[b].qs;
        const uint8_t *qs = blk + 16;
        int32_t isum = 0, msum = 0;
        for (int j = 0; j < 4; j++) {
            int sc0, m0, sc1, m1;
            q4k_scale_min(blk + 4, 2 * j, &sc0, &m0);
            q4k_scale_min(blk + 4, 2 * j + 1, &sc1, &m1);
            int32_t s0 = 0, s1 = 0;
            for (int l = 0; l < 32; l++) {
                s0 += (int32_t)(qs[32 * j + l] & 0x0f) * q8[64 * j + l];
                s1 += (int32_t)(qs[32 * j + l] >> 4) * q8[64 * j + 32 + l];
            }
            isum += sc0 * s0 + sc1 * s1;
            msum += m0 * (x[b].bsums[4 * j] + x[b].bsums[4 * j + 1]) +
                    m1 * (x[b].bsums[4 * j + 2] + x[b].bsums[4 * j + 3]);
        }
        float d = tmo_f16_to_f32(rd16(blk)) * x[b].d;
        float dmin = tmo_f16_to_f32(rd16(blk + 2)) * x[b].d;
        acc += d * (float)isum;
        acc -= dmin * (float)msum;
    }
    return acc;
}

/* vec_dot_q6_K_q8_K semantics: per 16-sub-block integer sums of (q-32)*qx times the int8 scale,
 * scaled by d*dx. */
float tmo_vec_dot_q6k_q8k(int64_t ncols, const void *w, const tmo_block_q8k *x) {
    const uint8_t *blk = (const uint8_t *)w;
    float acc = 0.f;
    for (int64_t b = 0; b < ncols / TMO_QK_K; b++, blk += TMO_Q6K_BYTES) {
        const uint8_t *ql = blk, *qh = blk + 128;
        const int8_t *scp = (const int8_t *)(blk + 192);
        const int8_t *q8 = x[b].qs;
        int32_t isum = 0;
        for (int s = 0; s < 16; s++) {
            int32_t ss = 0;
            for (int l = 0; l < 16; l++) {
                int i = 16 * s + l, h = i / 128, r = i % 128;
                int lo = r < 64 ? (ql[64 * h + r] & 0x0f) : (ql[64 * h + r - 64] >> 4);
                int hi = (qh[32 * h + (r % 32)] >> (2 * (r / 32))) & 3;
                ss += ((lo | (hi << 4)) - 32) * q8[i];
            }
            isum += scp[s] * ss;
        }
        float d = tmo_f16_to_f32(rd16(blk + 208)) * x[b].d;
        acc += d * (float)isum;
    }
    return acc;
}

/* ------------------------------------------------------------------------ */
/* SIMD forms of the two dots (AVX2); mul_mat_id / experts use the
 * multi-column form (tmo_dot_cols) */
/* ------------------------------------------------------------------------ */
/* ggml's CPU path computes the same integer sub-block sums with byte multiply-adds (maddubs:
 * unsigned weight bytes times signed activation bytes, pairs summed to 16 bits, then to 32).  These
 * restate that method on the same blocks: the integer sums are exact, and the float scaling is the
 * scalar functions' statement for statement, so the results equal tmo_vec_dot_q4k_q8k /
 * tmo_vec_dot_q6k_q8k bit for bit (tests/test_oracle.py checks it).  They make the timed CPU
 * baseline a vectorised CPU path, as the reference's is. */
#if defined(__AVX2__)
#include <immintrin.h>

/* Sum of the 8 int32 lanes, and of the 4 lanes of each 128-bit half. */
static inline int32_t hsum8(__m256i v) {
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4e));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xb1));
    return _mm_cvtsi128_si32(s);
}
static inline int32_t hsum4(__m128i s) {
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4e));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xb1));
    return _mm_cvtsi128_si32(s);
}

/* 32 unsigned bytes (at most 63) times 32 signed bytes -> 8 int32 partial sums (exact). */
static inline __m256i dot32(__m256i u, __m256i s) {
    return _mm256_madd_epi16(_mm256_maddubs_epi16(u, s), _mm256_set1_epi16(1));
}

float tmo_vec_dot_q4k_q8k_simd(int64_t ncols, const void *w, const tmo_block_q8k *x) {
    const uint8_t *blk = (const uint8_t *)w;
    const __m256i low = _mm256_set1_epi8(0x0f);
    float acc = 0.f;
    for (int64_t b = 0; b < ncols / TMO_QK_K; b++, blk += TMO_Q4K_BYTES) {
        const int8_t *q8 = x[b].qs;
        const uint8_t *qs = blk + 16;
        int32_t isum = 0, msum = 0;
        for (int j = 0; j < 4; j++) {
            int sc0, m0, sc1, m1;
            q4k_scale_min(blk + 4, 2 * j, &sc0, &m0);
            q4k_scale_min(blk + 4, 2 * j + 1, &sc1, &m1);
            const __m256i qv = _mm256_loadu_si256((const __m256i *)(qs + 32 * j));
            const __m256i lo = _mm256_and_si256(qv, low), hi = _mm256_and_si256(_mm256_srli_epi16(qv, 4), low);
            const int32_t s0 = hsum8(dot32(lo, _mm256_loadu_si256((const __m256i *)(q8 + 64 * j))));
            const int32_t s1 = hsum8(dot32(hi, _mm256_loadu_si256((const __m256i *)(q8 + 64 * j + 32))));
            isum += sc0 * s0 + sc1 * s1;
            msum += m0 * (x[b].bsums[4 * j] + x[b].bsums[4 * j + 1]) +
                    m1 * (x[b].bsums[4 * j + 2] + x[b].bsums[4 * j + 3]);
        }
        float d = tmo_f16_to_f32(rd16(blk)) * x[b].d;
        float dmin = tmo_f16_to_f32(rd16(blk + 2)) * x[b].d;
        acc += d * (float)isum;
        acc -= dmin * (float)msum;
    }
    return acc;
}

/* Q6_K: per 128-element half h, element r of the half is the low nibble of ql[64h + r] (r < 64) or
 * the high nibble of ql[64h + r - 64], with bits 4-5 from qh[32h + r % 32] >> 2 (r / 32); the 6-bit
 * value goes in unsigned and the -32 is -32 times the activation's 16-element block sum. */
float tmo_vec_dot_q6k_q8k_simd(int64_t ncols, const void *w, const tmo_block_q8k *x) {
    const uint8_t *blk = (const uint8_t *)w;
    const __m256i low = _mm256_set1_epi8(0x0f), two = _mm256_set1_epi8(0x03);
    float acc = 0.f;
    for (int64_t b = 0; b < ncols / TMO_QK_K; b++, blk += TMO_Q6K_BYTES) {
        const uint8_t *ql = blk, *qh = blk + 128;
        const int8_t *scp = (const int8_t *)(blk + 192);
        const int8_t *q8 = x[b].qs;
        int32_t isum = 0;
        for (int h = 0; h < 2; h++) {
            const __m256i l0 = _mm256_loadu_si256((const __m256i *)(ql + 64 * h));
            const __m256i l1 = _mm256_loadu_si256((const __m256i *)(ql + 64 * h + 32));
            const __m256i hb = _mm256_loadu_si256((const __m256i *)(qh + 32 * h));
            __m256i q[4];
            q[0] = _mm256_or_si256(_mm256_and_si256(l0, low), _mm256_slli_epi16(_mm256_and_si256(hb, two), 4));
            q[1] = _mm256_or_si256(_mm256_and_si256(l1, low),
                                   _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(hb, 2), two), 4));
            q[2] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(l0, 4), low),
                                   _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(hb, 4), two), 4));
            q[3] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(l1, 4), low),
                                   _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(hb, 6), two), 4));
            for (int v = 0; v < 4; v++) {
                const int base = 128 * h + 32 * v; /* elements base .. base+31: sub-blocks s, s+1 */
                const __m256i p = dot32(q[v], _mm256_loadu_si256((const __m256i *)(q8 + base)));
                const int s = base / 16;
                const int32_t ss0 = hsum4(_mm256_castsi256_si128(p)) - 32 * x[b].bsums[s];
                const int32_t ss1 = hsum4(_mm256_extracti128_si256(p, 1)) - 32 * x[b].bsums[s + 1];
                isum += scp[s] * ss0 + scp[s + 1] * ss1;
            }
        }
        float d = tmo_f16_to_f32(rd16(blk + 208)) * x[b].d;
        acc += d * (float)isum;
    }
    return acc;
}

/* One weight row against up to TMO_COLS (8) activation rows, the organisation of ggml's CPU mat-mul
 * kernels: the row's quants are unpacked once per super-block and serve every column, and the
 * sub-block scales multiply the 16-bit pair sums in vector registers (madd), so a super-block takes
 * one horizontal sum per column instead of one per sub-block.  The integer sums are the same
 * integers in another order (no lane can overflow: a Q4_K pair sum is at most 2 * 15 * 127, a Q6_K
 * one 2 * 63 * 127, times a scale below 2^7), and the float scaling is the scalar statement's, so
 * out[c] equals tmo_vec_dot_q4k_q8k / tmo_vec_dot_q6k_q8k of column c bit for bit. */
static void dot_cols_q4k(int64_t ncols, const uint8_t *blk, const tmo_block_q8k *const *xs, int nc, float *out) {
    const __m256i low = _mm256_set1_epi8(0x0f);
    float acc[TMO_COLS] = {0.f};
    for (int64_t b = 0; b < ncols / TMO_QK_K; b++, blk += TMO_Q4K_BYTES) {
        /* the 6-bit scales and mins of q4k_scale_min, four at a time as bytes of 32-bit words */
        uint32_t w0, w1, w2;
        memcpy(&w0, blk + 4, 4);
        memcpy(&w1, blk + 8, 4);
        memcpy(&w2, blk + 12, 4);
        const uint64_t sc8 = (uint64_t)(w0 & 0x3f3f3f3fu) |
                             ((uint64_t)((w2 & 0x0f0f0f0fu) | ((w0 >> 2) & 0x30303030u)) << 32);
        const uint64_t mn8 = (uint64_t)(w1 & 0x3f3f3f3fu) |
                             ((uint64_t)(((w2 >> 4) & 0x0f0f0f0fu) | ((w1 >> 2) & 0x30303030u)) << 32);
        const __m128i sc16 = _mm_cvtepu8_epi16(_mm_cvtsi64_si128((long long)sc8)); /* lanes: scale 0..7 */
        const __m128i mn16 = _mm_cvtepu8_epi16(_mm_cvtsi64_si128((long long)mn8));
        const __m256i scb = _mm256_broadcastsi128_si256(sc16);
        __m256i q[8], scv[8];
        for (int j = 0; j < 4; j++) {
            const __m256i qv = _mm256_loadu_si256((const __m256i *)(blk + 16 + 32 * j));
            q[2 * j] = _mm256_and_si256(qv, low);
            q[2 * j + 1] = _mm256_and_si256(_mm256_srli_epi16(qv, 4), low);
        }
        for (int s = 0; s < 8; s++) /* every 16-bit lane: scale s (bytes 2s, 2s+1 of each half) */
            scv[s] = _mm256_shuffle_epi8(scb, _mm256_set1_epi16((short)(0x0100 * (2 * s + 1) + 2 * s)));
        /* 16-bit lane i: the min of sub-block i / 2 (bsums i is a 16-element half of it) */
        const __m256i mnv = _mm256_set_m128i(_mm_unpackhi_epi16(mn16, mn16), _mm_unpacklo_epi16(mn16, mn16));
        const float dw = tmo_f16_to_f32(rd16(blk)), mw = tmo_f16_to_f32(rd16(blk + 2));
        for (int c = 0; c < nc; c++) {
            const tmo_block_q8k *x = xs[c] + b;
            __m256i a = _mm256_setzero_si256();
            for (int s = 0; s < 8; s++)
                a = _mm256_add_epi32(a, _mm256_madd_epi16(_mm256_maddubs_epi16(q[s], _mm256_loadu_si256(
                                                              (const __m256i *)(x->qs + 32 * s))), scv[s]));
            const __m256i m = _mm256_madd_epi16(_mm256_loadu_si256((const __m256i *)x->bsums), mnv);
            /* both horizontal sums at once: [a01 a23 m01 m23 | a45 a67 m45 m67] -> [isum, msum, ..] */
            const __m256i h = _mm256_hadd_epi32(a, m);
            __m128i hs = _mm_add_epi32(_mm256_castsi256_si128(h), _mm256_extracti128_si256(h, 1));
            hs = _mm_hadd_epi32(hs, hs);
            const int32_t isum = _mm_cvtsi128_si32(hs), msum = _mm_extract_epi32(hs, 1);
            const float d = dw * x->d, dmin = mw * x->d;
            acc[c] += d * (float)isum;
            acc[c] -= dmin * (float)msum;
        }
    }
    for (int c = 0; c < nc; c++) out[c] = acc[c];
}

static void dot_cols_q6k(int64_t ncols, const uint8_t *blk, const tmo_block_q8k *const *xs, int nc, float *out) {
    const __m256i low = _mm256_set1_epi8(0x0f), two = _mm256_set1_epi8(0x03);
    float acc[TMO_COLS] = {0.f};
    for (int64_t b = 0; b < ncols / TMO_QK_K; b++, blk += TMO_Q6K_BYTES) {
        const uint8_t *ql = blk, *qh = blk + 128;
        const int8_t *scp = (const int8_t *)(blk + 192);
        __m256i q[8], scv[8];
        for (int h = 0; h < 2; h++) {
            const __m256i l0 = _mm256_loadu_si256((const __m256i *)(ql + 64 * h));
            const __m256i l1 = _mm256_loadu_si256((const __m256i *)(ql + 64 * h + 32));
            const __m256i hb = _mm256_loadu_si256((const __m256i *)(qh + 32 * h));
            q[4 * h] = _mm256_or_si256(_mm256_and_si256(l0, low), _mm256_slli_epi16(_mm256_and_si256(hb, two), 4));
            q[4 * h + 1] = _mm256_or_si256(_mm256_and_si256(l1, low),
                                           _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(hb, 2), two), 4));
            q[4 * h + 2] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(l0, 4), low),
                                           _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(hb, 4), two), 4));
            q[4 * h + 3] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(l1, 4), low),
                                           _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(hb, 6), two), 4));
        }
        /* the 16 scales as 16-bit lanes: the -32 bias is -32 * sum_s sc_s * bsums_s */
        const __m256i sc16 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i *)scp));
        /* register v holds elements 32 v .. 32 v + 31: sub-blocks 2 v (low half, every lane scale 2 v)
         * and 2 v + 1 (high half); scales 0-7 sit in sc16's low 128 bits, 8-15 in its high ones */
        const __m256i slo = _mm256_permute2x128_si256(sc16, sc16, 0x00), shi = _mm256_permute2x128_si256(sc16, sc16, 0x11);
        for (int v = 0; v < 8; v++) {
            const int w = 2 * (v & 3); /* the pair's first scale within its 8 */
            const __m256i m = _mm256_set_m128i(_mm_set1_epi16((short)(0x0100 * (2 * w + 3) + 2 * w + 2)),
                                               _mm_set1_epi16((short)(0x0100 * (2 * w + 1) + 2 * w)));
            scv[v] = _mm256_shuffle_epi8(v < 4 ? slo : shi, m);
        }
        const float dw = tmo_f16_to_f32(rd16(blk + 208));
        for (int c = 0; c < nc; c++) {
            const tmo_block_q8k *x = xs[c] + b;
            __m256i a = _mm256_setzero_si256();
            for (int v = 0; v < 8; v++)
                a = _mm256_add_epi32(a, _mm256_madd_epi16(_mm256_maddubs_epi16(q[v], _mm256_loadu_si256(
                                                              (const __m256i *)(x->qs + 32 * v))), scv[v]));
            const __m256i bias = _mm256_madd_epi16(_mm256_loadu_si256((const __m256i *)x->bsums), sc16);
            const int32_t isum = hsum8(_mm256_sub_epi32(a, _mm256_slli_epi32(bias, 5)));
            const float d = dw * x->d;
            acc[c] += d * (float)isum;
        }
    }
    for (int c = 0; c < nc; c++) out[c] = acc[c];
}

#endif

void tmo_dot_cols(int type, int64_t ncols, const void *w, const tmo_block_q8k *const *xs, int nc, float *out) {
    if (nc < 1 || nc > TMO_COLS) return;
#if defined(__AVX2__)
    if (type == TMO_TYPE_Q4_K) return dot_cols_q4k(ncols, (const uint8_t *)w, xs, nc, out);
    if (type == TMO_TYPE_Q6_K) return dot_cols_q6k(ncols, (const uint8_t *)w, xs, nc, out);
#else
    for (int c = 0; c < nc; c++)
        out[c] = type == TMO_TYPE_Q4_K ? tmo_vec_dot_q4k_q8k(ncols, w, xs[c]) : tmo_vec_dot_q6k_q8k(ncols, w, xs[c]);
#endif
}

#if !defined(__AVX2__)
float tmo_vec_dot_q4k_q8k_simd(int64_t ncols, const void *w, const tmo_block_q8k *x) {
    return tmo_vec_dot_q4k_q8k(ncols, w, x);
}
float tmo_vec_dot_q6k_q8k_simd(int64_t ncols, const void *w, const tmo_block_q8k *x) {
    return tmo_vec_dot_q6k_q8k(ncols, w, x);
}
#endif

/* ------------------------------------------------------------------------ */
/* canonical router arithmetic                                               */
/* ------------------------------------------------------------------------ */

float tmo_exp_canon(float x) {
    if (x != x) return x;
    if (x < -87.0f) return 0.0f;
    if (x > 88.0f) return INFINITY;
    float kf = rintf(x * 1.44269504088896341f);
    float r = fmaf(kf, -0.693145751953125f, x);
    r = fmaf(kf, -1.42860682030941723212e-6f, r);
    float p = 1.98412698412698412698e-4f;
    p = fmaf(p, r, 1.38888888888888888889e-3f);
    p = fmaf(p, r, 8.33333333333333333333e-3f);
    p = fmaf(p, r, 4.16666666666666666667e-2f);
    p = fmaf(p, r, 1.66666666666666666667e-1f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ki = (int)kf;
    uint32_t sb = (uint32_t)(ki + 127) << 23;
    float scale;
    memcpy(&scale, &sb, 4);
    return p * scale;
}

static float butterfly32(float *p) {
    float q[32];
    for (int off = 16; off >= 1; off >>= 1) {
        for (int l = 0; l < 32; l++) q[l] = p[l] + p[l ^ off];
        memcpy(p, q, sizeof(q));
    }
    return p[0];
}

static double butterfly32d(double *p) {
    double q[32];
    for (int off = 16; off >= 1; off >>= 1) {
        for (int l = 0; l < 32; l++) q[l] = p[l] + p[l ^ off];
        memcpy(p, q, sizeof(q));
    }
    return p[0];
}

float tmo_router_dot(const float *w, const float *x, int64_t n) {
    float part[32];
    for (int l = 0; l < 32; l++) {
        float acc = 0.f;
        for (int64_t m = 0; m * 128 < n; m++)
            for (int c = 0; c < 4; c++) {
                int64_t i = 128 * m + 4 * l + c;
                if (i < n) acc = fmaf(w[i], x[i], acc);
            }
        part[l] = acc;
    }
    return butterfly32(part);
}

void tmo_rms_norm(const float *x, const float *norm_w, float eps, float *out, int64_t n) {
    double part[32];
    for (int l = 0; l < 32; l++) {
        double acc = 0.0;
        for (int64_t m = 0; m * 128 < n; m++)
            for (int c = 0; c < 4; c++) {
                int64_t i = 128 * m + 4 * l + c;
                if (i < n) acc += (double)(x[i] * x[i]);
            }
        part[l] = acc;
    }
    double sum = butterfly32d(part);
    float mean = (float)(sum / (double)n);
    float scale = 1.0f / sqrtf(mean + eps);
    for (int64_t i = 0; i < n; i++) {
        float v = x[i] * scale;
        out[i] = norm_w ? v * norm_w[i] : v;
    }
}

void tmo_softmax_topk(const float *logits, int E, int k, float *probs_out, int32_t *ids, float *w) {
    float mx = -INFINITY;
    for (int e = 0; e < E; e++)
        if (logits[e] > mx) mx = logits[e];
    float *ex = (float *)malloc(sizeof(float) * (size_t)E);
    float part[32];
    for (int e = 0; e < E; e++) ex[e] = tmo_exp_canon(logits[e] - mx);
    for (int l = 0; l < 32; l++) {
        float acc = 0.f;
        for (int e = l; e < E; e += 32) acc += ex[e];
        part[l] = acc;
    }
    float sum = butterfly32(part);
    for (int e = 0; e < E; e++) ex[e] = ex[e] / sum;
    if (probs_out) memcpy(probs_out, ex, sizeof(float) * (size_t)E);
    /* top-k: descending probability, ties to the lower index */
    unsigned char *taken = (unsigned char *)calloc((size_t)E, 1);
    for (int j = 0; j < k; j++) {
        int best = -1;
        for (int e = 0; e < E; e++) {
            if (taken[e]) continue;
            if (best < 0 || ex[e] > ex[best]) best = e;
        }
        taken[best] = 1;
        ids[j] = best;
    }
    float s = 0.f;
    for (int j = 0; j < k; j++) s += ex[ids[j]];
    if (!(s >= 6.103515625e-5f)) s = 6.103515625e-5f; /* clamp(min, inf) of qwen3moe.rs:2887 */
    for (int j = 0; j < k; j++) w[j] = ex[ids[j]] / s;
    free(taken);
    free(ex);
}

void tmo_router_logits(const float *xn, const float *router_w, int64_t T, int64_t H, int64_t E,
                       float *logits) {
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; t++)
        for (int64_t e = 0; e < E; e++)
            logits[t * E + e] = tmo_router_dot(router_w + e * H, xn + t * H, H);
}

/* The same dots with the 32 lanes in vector registers.  A row of n (a multiple of 128) is first
 * stored lane-major: element 128 m + 4 l + c at 128 m + 32 c + l, so that step (m, c) of every
 * lane is one contiguous 32-float run; each lane then takes the same fused multiply-adds in the same
 * order as tmo_router_dot, and the same butterfly, so the logits are the same bits. */
static void lane_major(const float *src, float *dst, int64_t n) {
    for (int64_t m = 0; m < n / 128; m++)
        for (int c = 0; c < 4; c++)
            for (int l = 0; l < 32; l++) dst[128 * m + 32 * c + l] = src[128 * m + 4 * l + c];
}
#if defined(__AVX2__) && defined(__FMA__)
static float router_dot_lanes(const float *wp, const float *xp, int64_t n) {
    __m256 a[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps()};
    for (int64_t i = 0; i < n; i += 32)
        for (int v = 0; v < 4; v++)
            a[v] = _mm256_fmadd_ps(_mm256_loadu_ps(wp + i + 8 * v), _mm256_loadu_ps(xp + i + 8 * v), a[v]);
    float part[32];
    for (int v = 0; v < 4; v++) _mm256_storeu_ps(part + 8 * v, a[v]);
    return butterfly32(part);
}
#define TMO_ROUTER_LANES 1
#else
#define TMO_ROUTER_LANES 0
#endif

void tmo_route(const float *x, int64_t T, int64_t H, int64_t E, int k, int use_norm,
               const float *norm_w, float eps, const float *router_w, const float *logits_in,
               float *xn_out, float *logits_out, int32_t *ids, float *w) {
    const int lanes = TMO_ROUTER_LANES && router_w && H % 128 == 0;
    float *wp = lanes ? (float *)malloc(sizeof(float) * (size_t)(E * H)) : NULL;
    if (wp) {
#pragma omp parallel for schedule(static)
        for (int64_t e = 0; e < E; e++) lane_major(router_w + e * H, wp + e * H, H);
    }
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; t++) {
        float *xn = (float *)malloc(sizeof(float) * (size_t)H);
        float *lg = (float *)malloc(sizeof(float) * (size_t)E);
        float *xp = wp ? (float *)malloc(sizeof(float) * (size_t)H) : NULL;
        if (use_norm)
            tmo_rms_norm(x + t * H, norm_w, eps, xn, H);
        else
            memcpy(xn, x + t * H, sizeof(float) * (size_t)H);
        if (xn_out) memcpy(xn_out + t * H, xn, sizeof(float) * (size_t)H);
        if (xp) lane_major(xn, xp, H);
        for (int64_t e = 0; e < E; e++) {
#if TMO_ROUTER_LANES
            if (xp) {
                lg[e] = router_dot_lanes(wp + e * H, xp, H);
                continue;
            }
#endif
            lg[e] = router_w ? tmo_router_dot(router_w + e * H, xn, H) : logits_in[t * E + e];
        }
        free(xp);
        if (logits_out) memcpy(logits_out + t * E, lg, sizeof(float) * (size_t)E);
        tmo_softmax_topk(lg, (int)E, k, NULL, ids + t * k, w + t * k);
        free(lg);
        free(xn);
    }
    free(wp);
}

void tmo_map_ids(const int32_t *ids, int64_t n, const int32_t *table, int64_t E, int32_t *out) {
    for (int64_t i = 0; i < n; i++)
        out[i] = (ids[i] >= 0 && ids[i] < E) ? table[ids[i]] : -1;
}

int64_t tmo_sort_pairs(const int32_t *ids, int64_t T, int k, int64_t E, int32_t *counts,
                       int32_t *offsets, int32_t *perm) {
    memset(counts, 0, sizeof(int32_t) * (size_t)E);
    for (int64_t p = 0; p < T * k; p++)
        if (ids[p] >= 0 && ids[p] < E) counts[ids[p]]++;
    offsets[0] = 0;
    for (int64_t e = 0; e < E; e++) offsets[e + 1] = offsets[e] + counts[e];
    int32_t *fill = (int32_t *)calloc((size_t)E, sizeof(int32_t));
    for (int64_t p = 0; p < T * k; p++) {
        int32_t e = ids[p];
        if (e >= 0 && e < E) perm[offsets[e] + fill[e]++] = (int32_t)p;
    }
    free(fill);
    return offsets[E];
}

/* ------------------------------------------------------------------------ */
/* expert products                                                           */
/* ------------------------------------------------------------------------ */

static int type_ok(int type) {
    return type == TMO_TYPE_Q4_K || type == TMO_TYPE_Q6_K || type == TMO_TYPE_F16 ||
           type == TMO_TYPE_F32;
}

/* The activation row as the weight type's dot expects it: Q8_K blocks for the K-quants, or the
 * f32 values rounded through the type (f16) for the float types; `deq` gets the f32 view of it. */
static void prep_act(int type, const float *x, int64_t K, tmo_block_q8k *q, float *deq) {
    if (type == TMO_TYPE_Q4_K || type == TMO_TYPE_Q6_K) {
        tmo_quantize_q8k(x, q, K);
        if (deq) tmo_dequantize_q8k(q, deq, K);
    } else if (type == TMO_TYPE_F16) {
        for (int64_t i = 0; i < K; i++) deq[i] = tmo_f16_to_f32(tmo_f32_to_f16(x[i]));
    } else {
        memcpy(deq, x, sizeof(float) * (size_t)K);
    }
}

static float row_dot(int type, int mode, const uint8_t *wrow, int64_t K, const tmo_block_q8k *q,
                     const float *deq, float *scratch) {
    if (mode == TMO_MODE_Q8K && type == TMO_TYPE_Q4_K) return tmo_vec_dot_q4k_q8k_simd(K, wrow, q);
    if (mode == TMO_MODE_Q8K && type == TMO_TYPE_Q6_K) return tmo_vec_dot_q6k_q8k_simd(K, wrow, q);
    tmo_dequantize(type, wrow, scratch, K);
    double s = 0.0;
    for (int64_t i = 0; i < K; i++) s += (double)scratch[i] * (double)deq[i];
    return (float)s;
}

int tmo_mul_mat_id(int type, const void *W, size_t nb1, size_t nb2, int64_t K, int64_t N, int64_t E,
                   const float *b, int64_t b1, int64_t T, const int32_t *ids, int n_used, float *out,
                   int mode, int nthreads) {
    if (!type_ok(type) || K <= 0 || N <= 0 || (b1 != 1 && b1 != n_used)) return -1;
    if ((type == TMO_TYPE_Q4_K || type == TMO_TYPE_Q6_K) && K % TMO_QK_K) return -1;
    if (nthreads <= 0) nthreads = omp_get_max_threads();
    int64_t nb = (K + TMO_QK_K - 1) / TMO_QK_K;
    int64_t ncol = T * b1;
    tmo_block_q8k *q = (tmo_block_q8k *)malloc(sizeof(tmo_block_q8k) * (size_t)(ncol * nb));
    float *deq = (float *)malloc(sizeof(float) * (size_t)(ncol * K));
    /* the f32 view of the activations is read only by the f64 mode and the float types */
    const int need_deq = !(mode == TMO_MODE_Q8K && (type == TMO_TYPE_Q4_K || type == TMO_TYPE_Q6_K));
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t c = 0; c < ncol; c++) prep_act(type, b + c * K, K, q + c * nb, need_deq ? deq + c * K : NULL);
    int32_t *counts = (int32_t *)malloc(sizeof(int32_t) * (size_t)E);
    int32_t *offs = (int32_t *)malloc(sizeof(int32_t) * (size_t)(E + 1));
    int32_t *perm = (int32_t *)malloc(sizeof(int32_t) * (size_t)(T * n_used + 1));
    tmo_sort_pairs(ids, T, n_used, E, counts, offs, perm);
    for (int64_t p = 0; p < T * n_used; p++)
        if (ids[p] < 0 || ids[p] >= E) memset(out + p * N, 0, sizeof(float) * (size_t)N);
    const int64_t RB = 16;
    int64_t nrb = (N + RB - 1) / RB;
#pragma omp parallel num_threads(nthreads)
    {
        float *scratch = (float *)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(dynamic)
        for (int64_t item = 0; item < E * nrb; item++) {
            int64_t e = item / nrb, r0 = (item % nrb) * RB;
            if (!counts[e]) continue;
            for (int64_t r = r0; r < r0 + RB && r < N; r++) {
                const uint8_t *wrow = (const uint8_t *)W + e * nb2 + r * nb1;
                if (mode == TMO_MODE_Q8K && (type == TMO_TYPE_Q4_K || type == TMO_TYPE_Q6_K)) {
                    for (int32_t i = offs[e]; i < offs[e + 1]; i += TMO_COLS) {
                        const int nc = offs[e + 1] - i < TMO_COLS ? offs[e + 1] - i : TMO_COLS;
                        const tmo_block_q8k *xs[TMO_COLS];
                        float res[TMO_COLS];
                        for (int c = 0; c < nc; c++) {
                            int64_t p = perm[i + c], t = p / n_used, j = p % n_used;
                            xs[c] = q + (t * b1 + (b1 == 1 ? 0 : j)) * nb;
                        }
                        tmo_dot_cols(type, K, wrow, xs, nc, res);
                        for (int c = 0; c < nc; c++) out[(int64_t)perm[i + c] * N + r] = res[c];
                    }
                    continue;
                }
                for (int32_t i = offs[e]; i < offs[e + 1]; i++) {
                    int64_t p = perm[i], t = p / n_used, j = p % n_used;
                    int64_t c = t * b1 + (b1 == 1 ? 0 : j);
                    out[p * N + r] = row_dot(type, mode, wrow, K, q + c * nb, deq + c * K, scratch);
                }
            }
        }
        free(scratch);
    }
    free(perm);
    free(offs);
    free(counts);
    free(deq);
    free(q);
    return 0;
}

int tmo_experts(const float *x, int64_t T, int64_t H, int64_t I, int64_t E, int k,
                const int32_t *ids, const float *w, int gate_type, const void *gate, size_t gate_nb1,
                size_t gate_nb2, int up_type, const void *up, size_t up_nb1, size_t up_nb2,
                int down_type, const void *down, size_t down_nb1, size_t down_nb2, float *out,
                float *act_out, int mode, int nthreads) {
    if (nthreads <= 0) nthreads = omp_get_max_threads();
    float *u = (float *)malloc(sizeof(float) * (size_t)(T * k * I));
    float *g = (float *)malloc(sizeof(float) * (size_t)(T * k * I));
    float *dn = (float *)malloc(sizeof(float) * (size_t)(T * k * H));
    int rc = 0;
    rc |= tmo_mul_mat_id(up_type, up, up_nb1, up_nb2, H, I, E, x, 1, T, ids, k, u, mode, nthreads);
    rc |= tmo_mul_mat_id(gate_type, gate, gate_nb1, gate_nb2, H, I, E, x, 1, T, ids, k, g, mode,
                         nthreads);
    if (rc) goto done;
    /* swiglu_split: silu(gate) * up, silu(v) = v / (1 + e^-v) (ggml_silu_f32) */
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t i = 0; i < T * k * I; i++) g[i] = (g[i] / (1.0f + expf(-g[i]))) * u[i];
    if (act_out) memcpy(act_out, g, sizeof(float) * (size_t)(T * k * I));
    rc |= tmo_mul_mat_id(down_type, down, down_nb1, down_nb2, I, H, E, g, k, T, ids, k, dn, mode,
                         nthreads);
    if (rc) goto done;
    /* ctx.mul(experts, w), then the fold of adds in choice order (sum_experts) */
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t t = 0; t < T; t++)
        for (int64_t h = 0; h < H; h++) {
            float acc = dn[(t * k + 0) * H + h] * w[t * k + 0];
            for (int j = 1; j < k; j++) acc = acc + dn[(t * k + j) * H + h] * w[t * k + j];
            out[t * H + h] = acc;
        }
done:
    free(dn);
    free(g);
    free(u);
    return rc;
}
