// Router (qwen3moe.rs:2871-2890): rms_norm * ffn_norm, logits = gate_inp . xn, softmax,
// top-k (descending, ties to the lower index), weights = sel / clamp(sum sel, 6.1035156e-5).
//
// Every floating-point step that feeds the top-k is written with explicit round-to-nearest
// intrinsics in one fixed order, so that the selected ids are bit-identical with the CPU oracle:
//   router dot: lane l accumulates elements i with (i/4)%32 == l in increasing i (fma), then a
//               butterfly over lane distances 16, 8, 4, 2, 1;
//   exp:        Cody-Waite reduction by ln 2 and a degree-7 Taylor polynomial (own code);
//   softmax:    lane l sums e^(x-max) over experts l, l+32, ... then the same butterfly;
//               p = e / sum (IEEE division).
#include "common.cuh"
#include "kernels.cuh"

namespace tmoe {

__device__ __forceinline__ float exp_canon(float x) {
    if (x != x) return x;
    if (x < -87.0f) return 0.0f;
    if (x > 88.0f) return __int_as_float(0x7f800000);
    float kf = rintf(__fmul_rn(x, 1.44269504088896341f));
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
    int ki = static_cast<int>(kf);
    return __fmul_rn(p, __int_as_float((ki + 127) << 23));
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

// One warp per token: ggml rms_norm (f64 sum of f32 squares) times the optional norm weight.
__global__ void rms_norm_kernel(const float *__restrict__ x, const float *__restrict__ norm_w,
                                float eps, int64_t T, int H, float *__restrict__ out) {
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    const float *xr = x + (int64_t)warp * H;
    double acc = 0.0;
    for (int m = 0; m * 128 < H; m++)
        for (int c = 0; c < 4; c++) {
            int i = 128 * m + 4 * lane + c;
            if (i < H) acc = __dadd_rn(acc, (double)__fmul_rn(xr[i], xr[i]));
        }
    double sum = butterfly_f64(acc);
    float mean = __double2float_rn(__ddiv_rn(sum, (double)H));
    float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    float *o = out + (int64_t)warp * H;
    for (int i = lane; i < H; i += 32) {
        float v = __fmul_rn(xr[i], scale);
        o[i] = norm_w ? __fmul_rn(v, norm_w[i]) : v;
    }
}

// logits[t][e] = canonical dot(router_w[e], xn[t]).  One warp per expert row e, TT tokens per
// warp (m outer, tokens inner keeps each token's per-lane order sequential in i).
template <int TT>
__global__ void router_logits_kernel(const float *__restrict__ xn, const float *__restrict__ rw,
                                     int64_t T, int H, int E, float *__restrict__ logits) {
    int e = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    int lane = threadIdx.x & 31;
    int64_t t0 = (int64_t)blockIdx.y * TT;
    if (e >= E) return;
    float acc[TT];
#pragma unroll
    for (int j = 0; j < TT; j++) acc[j] = 0.0f;
    const float *wr = rw + (int64_t)e * H;
    const bool vec = (H % 4) == 0;
    for (int m = 0; m * 128 < H; m++) {
        int i0 = 128 * m + 4 * lane;
        float w4[4];
        if (vec && i0 + 3 < H) {
            float4 v = __ldg(reinterpret_cast<const float4 *>(wr + i0));
            w4[0] = v.x, w4[1] = v.y, w4[2] = v.z, w4[3] = v.w;
        } else {
            for (int c = 0; c < 4; c++) w4[c] = (i0 + c < H) ? wr[i0 + c] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < TT; j++) {
            int64_t t = t0 + j;
            if (t >= T) break;
            const float *xr = xn + t * H;
            float x4[4];
            if (vec && i0 + 3 < H) {
                float4 v = __ldg(reinterpret_cast<const float4 *>(xr + i0));
                x4[0] = v.x, x4[1] = v.y, x4[2] = v.z, x4[3] = v.w;
            } else {
                for (int c = 0; c < 4; c++) x4[c] = (i0 + c < H) ? xr[i0 + c] : 0.0f;
            }
#pragma unroll
            for (int c = 0; c < 4; c++)
                if (i0 + c < H) acc[j] = __fmaf_rn(w4[c], x4[c], acc[j]);
        }
    }
#pragma unroll
    for (int j = 0; j < TT; j++) {
        float s = butterfly_f32(acc[j]);
        int64_t t = t0 + j;
        if (lane == 0 && t < T) logits[t * E + e] = s;
    }
}

// One warp per token: canonical softmax, top-k, renormalised weights.  E <= 32*MAXPER, k <= 32.
template <int MAXPER>
__global__ void softmax_topk_kernel(const float *__restrict__ logits, int64_t T, int E, int k,
                                    int32_t *__restrict__ ids, float *__restrict__ w,
                                    float *__restrict__ probs_out) {
    int64_t t = (int64_t)(blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5));
    int lane = threadIdx.x & 31;
    if (t >= T) return;
    const float *lg = logits + t * E;
    float v[MAXPER];
    float mx = __int_as_float(0xff800000);
#pragma unroll
    for (int i = 0; i < MAXPER; i++) {
        int e = lane + 32 * i;
        v[i] = e < E ? lg[e] : __int_as_float(0xff800000);
        if (e < E && v[i] > mx) mx = v[i];
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float part = 0.0f;
#pragma unroll
    for (int i = 0; i < MAXPER; i++) {
        int e = lane + 32 * i;
        if (e < E) {
            v[i] = exp_canon(__fsub_rn(v[i], mx));
            part = __fadd_rn(part, v[i]);
        } else {
            v[i] = -1.0f;  // below every probability: never selected
        }
    }
    float sum = butterfly_f32(part);
#pragma unroll
    for (int i = 0; i < MAXPER; i++) {
        int e = lane + 32 * i;
        if (e < E) {
            v[i] = __fdiv_rn(v[i], sum);
            if (probs_out) probs_out[t * E + e] = v[i];
        }
    }
    // k rounds of a warp argmax with the total order (p desc, index asc).
    float sel_mine = 0.0f;  // lane j keeps the probability of choice j
    int id_mine = -1;
    for (int j = 0; j < k; j++) {
        float bp = -2.0f;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < MAXPER; i++) {
            int e = lane + 32 * i;
            if (e < E && v[i] >= 0.0f && (v[i] > bp || (v[i] == bp && e < bi))) {
                bp = v[i];
                bi = e;
            }
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            float op = __shfl_xor_sync(0xffffffffu, bp, off);
            int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (op > bp || (op == bp && oi < bi)) {
                bp = op;
                bi = oi;
            }
        }
        if ((bi & 31) == lane) {
#pragma unroll
            for (int i = 0; i < MAXPER; i++)
                if (lane + 32 * i == bi) v[i] = -1.0f;
        }
        if (lane == j) {
            sel_mine = bp;
            id_mine = bi;
        }
    }
    // s = sel_0 + sel_1 + ... in choice order (sequential, as the oracle).
    float s = 0.0f;
    for (int j = 0; j < k; j++) s = __fadd_rn(s, __shfl_sync(0xffffffffu, sel_mine, j));
    if (!(s >= 6.103515625e-5f)) s = 6.103515625e-5f;
    if (lane < k) {
        ids[t * k + lane] = id_mine;
        w[t * k + lane] = __fdiv_rn(sel_mine, s);
    }
}

// Q8_K of rows of K f32 (ggml quantize_row_q8_K_ref restated): one warp per 256-block, lane l
// holds elements 8l..8l+7.  Output SoA: qs int8 [rows][K], d f32 [rows][K/256], bsums int16
// [rows][K/16].  Rows whose `valid` entry is negative are skipped (valid may be NULL).
__global__ void quantize_q8k_kernel(const float *__restrict__ x, int64_t rows, int K,
                                    const int32_t *__restrict__ valid, int8_t *__restrict__ qs,
                                    float *__restrict__ d, int16_t *__restrict__ bsums) {
    int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    int nb = K / TMOE_QK;
    int64_t row = gw / nb;
    int b = (int)(gw % nb);
    if (row >= rows) return;
    if (valid && valid[row] < 0) return;
    const float *xr = x + row * K + (int64_t)b * TMOE_QK + 8 * lane;
    float4 a0 = *reinterpret_cast<const float4 *>(xr);
    float4 a1 = *reinterpret_cast<const float4 *>(xr + 4);
    float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    float amax = 0.0f, maxv = 0.0f;
    int idx = 0x7fffffff;
#pragma unroll
    for (int c = 0; c < 8; c++) {
        float ax = fabsf(v[c]);
        if (ax > amax) {
            amax = ax;
            maxv = v[c];
            idx = 8 * lane + c;
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        float oa = __shfl_xor_sync(0xffffffffu, amax, off);
        float ov = __shfl_xor_sync(0xffffffffu, maxv, off);
        int oi = __shfl_xor_sync(0xffffffffu, idx, off);
        if (oa > amax || (oa == amax && oi < idx)) {
            amax = oa;
            maxv = ov;
            idx = oi;
        }
    }
    int8_t q[8];
    float dd = 0.0f;
    if (amax == 0.0f) {
#pragma unroll
        for (int c = 0; c < 8; c++) q[c] = 0;
    } else {
        float iscale = __fdiv_rn(-127.0f, maxv);
#pragma unroll
        for (int c = 0; c < 8; c++) {
            int qi = __float2int_rn(__fmul_rn(iscale, v[c]));
            q[c] = (int8_t)(qi > 127 ? 127 : qi);
        }
        dd = __fdiv_rn(1.0f, iscale);
    }
    int s = 0;
#pragma unroll
    for (int c = 0; c < 8; c++) s += q[c];
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    uint32_t lo = (uint8_t)q[0] | ((uint32_t)(uint8_t)q[1] << 8) | ((uint32_t)(uint8_t)q[2] << 16) |
                  ((uint32_t)(uint8_t)q[3] << 24);
    uint32_t hi = (uint8_t)q[4] | ((uint32_t)(uint8_t)q[5] << 8) | ((uint32_t)(uint8_t)q[6] << 16) |
                  ((uint32_t)(uint8_t)q[7] << 24);
    *reinterpret_cast<uint2 *>(qs + row * K + (int64_t)b * TMOE_QK + 8 * lane) = make_uint2(lo, hi);
    if ((lane & 1) == 0) bsums[row * (K / 16) + (int64_t)b * 16 + lane / 2] = (int16_t)s;
    if (lane == 0) d[row * nb + b] = dd;
}

// ------------------------------------------------------------------ launchers
cudaError_t launch_rms_norm(const float *x, const float *norm_w, float eps, int64_t T, int H,
                            float *out, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    int warps = 8;
    unsigned grid = (unsigned)((T + warps - 1) / warps);
    rms_norm_kernel<<<grid, warps * 32, 0, st>>>(x, norm_w, eps, T, H, out);
    return cudaGetLastError();
}

cudaError_t launch_router_logits(const float *xn, const float *rw, int64_t T, int H, int E,
                                 float *logits, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    constexpr int TT = 8;
    int warps = 4;
    dim3 grid((E + warps - 1) / warps, (unsigned)((T + TT - 1) / TT));
    router_logits_kernel<TT><<<grid, warps * 32, 0, st>>>(xn, rw, T, H, E, logits);
    return cudaGetLastError();
}

cudaError_t launch_softmax_topk(const float *logits, int64_t T, int E, int k, int32_t *ids,
                                float *w, float *probs, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    int warps = 8;
    unsigned grid = (unsigned)((T + warps - 1) / warps);
    if (E <= 32)
        softmax_topk_kernel<1><<<grid, warps * 32, 0, st>>>(logits, T, E, k, ids, w, probs);
    else if (E <= 64)
        softmax_topk_kernel<2><<<grid, warps * 32, 0, st>>>(logits, T, E, k, ids, w, probs);
    else if (E <= 128)
        softmax_topk_kernel<4><<<grid, warps * 32, 0, st>>>(logits, T, E, k, ids, w, probs);
    else if (E <= 256)
        softmax_topk_kernel<8><<<grid, warps * 32, 0, st>>>(logits, T, E, k, ids, w, probs);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

cudaError_t launch_quantize_q8k(const float *x, int64_t rows, int K, const int32_t *valid,
                                int8_t *qs, float *d, int16_t *bsums, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    int64_t warps = rows * (K / TMOE_QK);
    int per_block = 8;
    unsigned grid = (unsigned)((warps + per_block - 1) / per_block);
    quantize_q8k_kernel<<<grid, per_block * 32, 0, st>>>(x, rows, K, valid, qs, d, bsums);
    return cudaGetLastError();
}

}  // namespace tmoe
