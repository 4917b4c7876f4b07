// Canonical router arithmetic shared by the router kernels (route.cu) and the fused
// top-k + dispatch kernel (dispatch.cu).  Every floating-point step that feeds the top-k is
// written with explicit round-to-nearest intrinsics in one fixed order, so that the selected ids
// are bit-identical with the CPU oracle:
//   exp:      Cody-Waite reduction by ln 2 and a degree-7 Taylor polynomial (own code);
//   softmax:  lane l sums e^(x-max) over experts l, l+32, ... then a butterfly over lane
//             distances 16, 8, 4, 2, 1; p = e / sum (IEEE division);
//   top-k:    k rounds of a warp argmax under the total order (p descending, index ascending)
//             (warp reductions on the probabilities' bit patterns);
//   weights:  w_j = sel_j / max(sel_0 + sel_1 + ..., 6.1035156e-5) (qwen3moe.rs:2886-2888).
#pragma once

#include "common.cuh"

namespace tmoe {

__device__ __forceinline__ float exp_canon(float x) {
    // k = rint(x log2 e) through the 1.5 * 2^23 shift (exact rounding to an integer, ties to even,
    // for |x log2 e| < 2^22), and no branches, so that a thread's several exps overlap
    const float y = __fmul_rn(x, 1.44269504088896341f);
    const float sh = __fadd_rn(y, 12582912.0f);
    const float kf = __fsub_rn(sh, 12582912.0f);
    float r = __fmaf_rn(kf, -0.693145751953125f, x);
    r = __fmaf_rn(kf, -1.42860682030941723212e-6f, r);
    float p = 1.98412698412698412698e-4f;
    p = __fmaf_rn(p, r, 1.38888888888888888889e-3f);
    p = __fmaf_rn(p, r, 8.33333333333333333333e-3f);
    p = __fmaf_rn(p, r, 4.16666666666666666667e-2f);
    p = __fmaf_rn(p, r, 1.66666666666666666667e-1f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const unsigned ki = (unsigned)__float_as_int(sh) - 0x4B400000u;
    const float v = __fmul_rn(p, __uint_as_float((ki + 127u) << 23));
    return x != x ? x : (x < -87.0f ? 0.0f : (x > 88.0f ? __int_as_float(0x7f800000) : v));
}

__device__ __forceinline__ float butterfly_f32(float v) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

__device__ __forceinline__ double butterfly_f64(double v) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

// One warp, one token: softmax over the E logits at lg, top-k, renormalised weights.
// Lane j < k ends with choice j: *id = expert, *wt = weight.  probs may be NULL.
template <int MAXPER>
__device__ __forceinline__ void topk_token(const float *__restrict__ lg, int E, int k, float *__restrict__ probs,
                                           int &id, float &wt) {
    const int lane = threadIdx.x & 31;
    float v[MAXPER];
    float mx = __int_as_float(0xff800000);
#pragma unroll
    for (int i = 0; i < MAXPER; i++) {
        const int e = lane + 32 * i;
        v[i] = e < E ? lg[e] : __int_as_float(0xff800000);
        if (e < E && v[i] > mx) mx = v[i];
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float part = 0.0f;
#pragma unroll
    for (int i = 0; i < MAXPER; i++) {
        const int e = lane + 32 * i;
        if (e < E) {
            v[i] = exp_canon(__fsub_rn(v[i], mx));
            part = __fadd_rn(part, v[i]);
        } else {
            v[i] = -1.0f;  // below every probability: never selected
        }
    }
    const float sum = butterfly_f32(part);
#pragma unroll
    for (int i = 0; i < MAXPER; i++) {
        const int e = lane + 32 * i;
        if (e < E) {
            v[i] = __fdiv_rn(v[i], sum);
            if (probs) probs[e] = v[i];
        }
    }
    // k rounds of a warp argmax under (p descending, index ascending): probabilities are in
    // [0, 1], so their bit patterns order like the values; key = bits + 1 for a candidate, 0 for
    // a removed (or absent, or NaN) one.  Two warp reductions per round: the largest key, then
    // the smallest index holding it.
    // The keys are computed once; taking a candidate sets its key to 0.
    uint32_t key[MAXPER];
#pragma unroll
    for (int i = 0; i < MAXPER; i++) {
        const int e = lane + 32 * i;
        key[i] = (e < E && v[i] >= 0.0f) ? __float_as_uint(v[i]) + 1u : 0u;
    }
    float sel_mine = 0.0f;
    int id_mine = -1;
    for (int j = 0; j < k; j++) {
        uint32_t bk = 0u;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < MAXPER; i++) {
            if (key[i] > bk) {  // e increases with i: an equal key keeps the lower index
                bk = key[i];
                bi = lane + 32 * i;
            }
        }
        const uint32_t mk = __reduce_max_sync(0xffffffffu, bk);
        const int mi = (int)__reduce_min_sync(0xffffffffu, bk == mk ? (uint32_t)bi : 0xffffffffu);
        if ((mi & 31) == lane) {
#pragma unroll
            for (int i = 0; i < MAXPER; i++)
                if (lane + 32 * i == mi) key[i] = 0u;
        }
        if (lane == j) {
            sel_mine = __uint_as_float(mk - 1u);
            id_mine = mi;
        }
    }
    float s = 0.0f;
    for (int j = 0; j < k; j++) s = __fadd_rn(s, __shfl_sync(0xffffffffu, sel_mine, j));
    if (!(s >= 6.103515625e-5f)) s = 6.103515625e-5f;
    id = id_mine;
    wt = __fdiv_rn(sel_mine, s);
}

}  // namespace tmoe
