// The decode step around the MoE layer (config 3: the full Qwen3-MoE model), per the reference's
// attention() (crates/model/src/attn.rs:246-405) and build_step (crates/model/src/qwen3moe.rs:2777-2870):
//   rope_neox_kernel      ggml rope_ext, NeoX mode (attn.rs:225-236: freq_scale 1, ext_factor 0,
//                         attn_factor 1): pairs (i, i + n_rot/2), theta = pos * base^(-2i/n_rot)
//   kv_store_kernel       set_rows of the new K and V rows into the F16 cache (attn.rs:339-350)
//   attn_decode_kernel    flash_attn_ext for one new token per sequence (attn.rs:352-377): the
//                         causal window is the sequence's positions 0..pos; GQA, the query heads
//                         of one KV head share its K/V reads.  Split over the context, each split
//                         keeping an online softmax (max, sum, weighted V); attn_merge_kernel joins
//                         the splits
//   add_kernel, argmax_kernel   the residual adds and greedy sampling
// The projections are the GEMV of gemv.cu (tmoe_mul_mat_id with one expert), the norms
// rms_norm_kernel (route.cu), the token embedding get_rows_kernel (quant.cu).
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.cuh"

namespace tmoe {

// x [n_tok][n_head][head_dim] in place, token t at position pos[t].
__global__ void rope_neox_kernel(float *__restrict__ x, const int32_t *__restrict__ pos, int64_t n_tok, int n_head,
                                 int head_dim, int n_rot, float freq_base) {
    const int64_t row = blockIdx.x;  // token * n_head + head
    const int64_t t = row / n_head;
    if (t >= n_tok) return;
    const float p = (float)pos[t];
    float *v = x + row * head_dim;
    const int half = n_rot / 2;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const float theta = p * powf(freq_base, -2.0f * (float)i / (float)n_rot);
        float s, c;
        sincosf(theta, &s, &c);
        const float x0 = v[i], x1 = v[i + half];
        v[i] = x0 * c - x1 * s;
        v[i + half] = x0 * s + x1 * c;
    }
}

// cache[b][pos[b]][:] = rows[b][:] (n_kv * head_dim values, as F16) for K and V.
__global__ void kv_store_kernel(const float *__restrict__ k, const float *__restrict__ v, __half *__restrict__ kc,
                                __half *__restrict__ vc, const int32_t *__restrict__ pos, int n_ctx, int width,
                                int *err) {
    const int b = blockIdx.x;
    const int p = pos[b];
    if (p < 0 || p >= n_ctx) {
        if (threadIdx.x == 0 && err) atomicCAS(err, 0, TMOE_DEV_ERR_BADID);
        return;
    }
    const size_t dst = ((size_t)b * n_ctx + p) * width;
    for (int i = threadIdx.x; i < width; i += blockDim.x) {
        kc[dst + i] = __float2half_rn(k[(size_t)b * width + i]);
        vc[dst + i] = __float2half_rn(v[(size_t)b * width + i]);
    }
}

// One CTA per (split, KV head, sequence), 128 threads.  G query heads share the KV head.  Tiles of
// AT_TILE positions: K and V staged in shared memory (K rows padded by one word so that the 32
// positions of a warp hit distinct banks); warp w scores heads w, w+4, ... (lane = position);
// the online softmax per head lives in its warp; thread t accumulates output dimensions t (and
// t + 128 for larger heads) of every head.
constexpr int AT_TILE = 32;
constexpr int AT_THREADS = 128;
constexpr int AT_MAX_G = 8;

template <int HD>
__global__ void __launch_bounds__(AT_THREADS) attn_decode_kernel(const float *__restrict__ q,
                                                                 const __half *__restrict__ kc,
                                                                 const __half *__restrict__ vc,
                                                                 const int32_t *__restrict__ pos, int n_head,
                                                                 int n_kv, int n_ctx, float scale,
                                                                 float *__restrict__ part) {
    constexpr int KW = HD / 2 + 1;  // words per staged K row (half2 + one pad word)
    __shared__ float qs[AT_MAX_G][HD];
    __shared__ uint32_t ks[AT_TILE][KW];
    __shared__ __align__(16) __half vs[AT_TILE][HD];
    __shared__ float ps[AT_MAX_G][AT_TILE];
    __shared__ float alpha_s[AT_MAX_G];
    const int s = blockIdx.x, g = blockIdx.y, b = blockIdx.z, S = gridDim.x;
    const int G = n_head / n_kv;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int len = min(pos[b] + 1, n_ctx);
    const int per = ((len + S - 1) / S + AT_TILE - 1) / AT_TILE * AT_TILE;
    const int p0 = s * per, p1 = min(len, p0 + per);
    for (int i = tid; i < G * HD; i += AT_THREADS)
        qs[i / HD][i % HD] = q[((size_t)b * n_head + (size_t)g * G + i / HD) * HD + i % HD] * scale;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};  // per head of this warp (w, w + 4)
    constexpr int DPT = HD >= AT_THREADS ? HD / AT_THREADS : 1;  // output dims per thread
    float acc[AT_MAX_G][DPT];
#pragma unroll
    for (int h = 0; h < AT_MAX_G; h++)
#pragma unroll
        for (int j = 0; j < DPT; j++) acc[h][j] = 0.0f;
    const size_t row_stride = (size_t)n_kv * HD;
    const __half *kb = kc + (size_t)b * n_ctx * row_stride + (size_t)g * HD;
    const __half *vb = vc + (size_t)b * n_ctx * row_stride + (size_t)g * HD;
    __syncthreads();
    for (int t0 = p0; t0 < p1; t0 += AT_TILE) {
        const int nt = min(AT_TILE, p1 - t0);
        // stage K and V of the tile (16-byte loads: HD / 8 per row)
        for (int i = tid; i < AT_TILE * (HD / 8); i += AT_THREADS) {
            const int r = i / (HD / 8), c = i % (HD / 8);
            uint4 kv4 = make_uint4(0, 0, 0, 0), vv4 = make_uint4(0, 0, 0, 0);
            if (r < nt) {
                kv4 = *reinterpret_cast<const uint4 *>(kb + (size_t)(t0 + r) * row_stride + 8 * c);
                vv4 = *reinterpret_cast<const uint4 *>(vb + (size_t)(t0 + r) * row_stride + 8 * c);
            }
            ks[r][4 * c] = kv4.x, ks[r][4 * c + 1] = kv4.y, ks[r][4 * c + 2] = kv4.z, ks[r][4 * c + 3] = kv4.w;
            *reinterpret_cast<uint4 *>(&vs[r][8 * c]) = vv4;
        }
        __syncthreads();
        // scores and the online softmax of heads warp, warp + 4
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
            const int h = warp + 4 * hh;
            if (h >= G) break;
            float sc = -INFINITY;
            if (lane < nt) {
                float d = 0.0f;
#pragma unroll 8
                for (int j = 0; j < HD / 2; j++) {
                    const float2 kf = __half22float2(*reinterpret_cast<const __half2 *>(&ks[lane][j]));
                    d = fmaf(qs[h][2 * j], kf.x, d);
                    d = fmaf(qs[h][2 * j + 1], kf.y, d);
                }
                sc = d;
            }
            float mx = sc;
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float m_new = fmaxf(m[hh], mx);
            const float pe = lane < nt ? __expf(sc - m_new) : 0.0f;
            float sum = pe;
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            const float a = m[hh] == -INFINITY ? 0.0f : __expf(m[hh] - m_new);
            l[hh] = l[hh] * a + sum;
            m[hh] = m_new;
            ps[h][lane] = pe;
            if (lane == 0) alpha_s[h] = a;
        }
        __syncthreads();
        // P . V
#pragma unroll
        for (int j = 0; j < DPT; j++) {
            const int d = tid + j * AT_THREADS;
            if (d >= HD) break;
#pragma unroll
            for (int h = 0; h < AT_MAX_G; h++)
                if (h < G) acc[h][j] *= alpha_s[h];
            for (int r = 0; r < nt; r++) {
                const float vv = __half2float(vs[r][d]);
#pragma unroll
                for (int h = 0; h < AT_MAX_G; h++)
                    if (h < G) acc[h][j] = fmaf(ps[h][r], vv, acc[h][j]);
            }
        }
        __syncthreads();
    }
    // partials: [b][head][s] = {m, l, acc[HD]}
    const size_t pstride = (size_t)HD + 2;
#pragma unroll
    for (int hh = 0; hh < 2; hh++) {
        const int h = warp + 4 * hh;
        if (h < G && lane == 0) {
            float *pp = part + (((size_t)b * n_head + (size_t)g * G + h) * S + s) * pstride;
            pp[0] = m[hh], pp[1] = l[hh];
        }
    }
#pragma unroll
    for (int j = 0; j < DPT; j++) {
        const int d = tid + j * AT_THREADS;
        if (d >= HD) break;
#pragma unroll
        for (int h = 0; h < AT_MAX_G; h++)
            if (h < G) part[(((size_t)b * n_head + (size_t)g * G + h) * S + s) * pstride + 2 + d] = acc[h][j];
    }
}

// out[b][head][:] from the S partials of (b, head): one CTA per (b, head).
__global__ void attn_merge_kernel(const float *__restrict__ part, int S, int HD, float *__restrict__ out) {
    const size_t bh = blockIdx.x;
    const float *pp = part + bh * S * ((size_t)HD + 2);
    float M = -INFINITY;
    for (int s = 0; s < S; s++) M = fmaxf(M, pp[s * (HD + 2)]);
    float L = 0.0f;
    for (int s = 0; s < S; s++) {
        const float ms = pp[s * (HD + 2)];
        if (ms != -INFINITY) L += __expf(ms - M) * pp[s * (HD + 2) + 1];
    }
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
    for (int d = threadIdx.x; d < HD; d += blockDim.x) {
        float o = 0.0f;
        for (int s = 0; s < S; s++) {
            const float ms = pp[s * (HD + 2)];
            if (ms != -INFINITY) o += __expf(ms - M) * pp[s * (HD + 2) + 2 + d];
        }
        out[bh * HD + d] = o * inv;
    }
}

__global__ void add_kernel(const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ out,
                           int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = a[i] + b[i];
}

// out[r] = the first index of the largest value of row r.  One CTA per row.
__global__ void argmax_kernel(const float *__restrict__ x, int64_t n, int32_t *__restrict__ out) {
    const float *row = x + (int64_t)blockIdx.x * n;
    float best = -INFINITY;
    int64_t bi = 0x7fffffff;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = row[i];
        if (v > best || (v == best && i < bi)) best = v, bi = i;
    }
    __shared__ float sv[32];
    __shared__ int64_t si[32];
    for (int o = 16; o >= 1; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) best = ov, bi = oi;
    }
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) sv[w] = best, si[w] = bi;
    __syncthreads();
    if (w == 0) {
        const int nw = blockDim.x >> 5;
        best = lane < nw ? sv[lane] : -INFINITY;
        bi = lane < nw ? si[lane] : 0x7fffffff;
        for (int o = 16; o >= 1; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > best || (ov == best && oi < bi)) best = ov, bi = oi;
        }
        if (lane == 0) out[blockIdx.x] = (int32_t)bi;
    }
}

// The dispatch of a dense product (one matrix, every row of x): active = {0, 0, T}, one active
// expert, pairs in order, the GEMV's work counters zeroed.
__global__ void dense_prep_kernel(int T, int4 *__restrict__ active, int32_t *__restrict__ n_active,
                                  int32_t *__restrict__ perm, int *__restrict__ counters, int n_counters) {
    for (int i = threadIdx.x; i < T; i += blockDim.x) perm[i] = i;
    if (threadIdx.x < n_counters) counters[threadIdx.x] = 0;
    if (threadIdx.x == 0) active[0] = make_int4(0, 0, T, 0), n_active[0] = 1;
}

// ------------------------------------------------------------------ launchers
cudaError_t launch_dense_prep(int T, int4 *active, int32_t *n_active, int32_t *perm, int *counters, int n_counters,
                              cudaStream_t st) {
    if (n_counters > 256) return cudaErrorInvalidValue;
    dense_prep_kernel<<<1, 256, 0, st>>>(T, active, n_active, perm, counters, n_counters);
    return cudaGetLastError();
}

cudaError_t launch_rope_neox(float *x, const int32_t *pos, int64_t n_tok, int n_head, int head_dim, int n_rot,
                             float freq_base, cudaStream_t st) {
    if (n_tok <= 0) return cudaSuccess;
    if (n_rot <= 0 || n_rot > head_dim || n_rot % 2 || n_tok * n_head > 0x7fffffff) return cudaErrorInvalidValue;
    rope_neox_kernel<<<(unsigned)(n_tok * n_head), 64, 0, st>>>(x, pos, n_tok, n_head, head_dim, n_rot, freq_base);
    return cudaGetLastError();
}

int attn_splits(int B, int n_kv, int n_ctx, int sm_count) {
    const int want = (4 * sm_count + B * n_kv - 1) / (B * n_kv);
    const int most = (n_ctx + AT_TILE - 1) / AT_TILE;
    return want < 1 ? 1 : (want > 64 ? 64 : (want > most ? most : want));
}

size_t attn_scratch_floats(int B, int n_head, int head_dim, int n_kv, int n_ctx, int sm_count) {
    return (size_t)B * n_head * attn_splits(B, n_kv, n_ctx, sm_count) * ((size_t)head_dim + 2);
}

cudaError_t launch_attn_decode(const float *q, const float *k, const float *v, __half *kc, __half *vc,
                               const int32_t *pos, int B, int n_head, int n_kv, int head_dim, int n_ctx, float scale,
                               float *part, float *out, int sm_count, int *err, cudaStream_t st) {
    if (B <= 0) return cudaSuccess;
    if (n_kv <= 0 || n_head % n_kv || n_head / n_kv > AT_MAX_G || (head_dim != 64 && head_dim != 128) ||
        n_ctx <= 0 || B > 65535 || n_kv > 65535)
        return cudaErrorInvalidValue;
    const int width = n_kv * head_dim;
    kv_store_kernel<<<B, 128, 0, st>>>(k, v, kc, vc, pos, n_ctx, width, err);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int S = attn_splits(B, n_kv, n_ctx, sm_count);
    const dim3 grid(S, n_kv, B);
    if (head_dim == 128)
        attn_decode_kernel<128><<<grid, AT_THREADS, 0, st>>>(q, kc, vc, pos, n_head, n_kv, n_ctx, scale, part);
    else
        attn_decode_kernel<64><<<grid, AT_THREADS, 0, st>>>(q, kc, vc, pos, n_head, n_kv, n_ctx, scale, part);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    attn_merge_kernel<<<B * n_head, 128, 0, st>>>(part, S, head_dim, out);
    return cudaGetLastError();
}

cudaError_t launch_add(const float *a, const float *b, float *out, int64_t n, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    add_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(a, b, out, n);
    return cudaGetLastError();
}

cudaError_t launch_argmax(const float *x, int64_t rows, int64_t n, int32_t *out, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    if (rows > 0x7fffffff || n <= 0) return cudaErrorInvalidValue;
    argmax_kernel<<<(unsigned)rows, 256, 0, st>>>(x, n, out);
    return cudaGetLastError();
}

}  // namespace tmoe
