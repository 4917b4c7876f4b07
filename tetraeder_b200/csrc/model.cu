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
//   qk_norm_rope_kernel   the per-head norms of Q and K and their RoPE in one launch (attn.rs:320-325)
//   add_kernel, argmax_kernel   the residual adds and greedy sampling
// The projections are the GEMV of gemv.cu (tmoe_mul_mat: dense_prep_kernel's dispatch of one
// matrix), the norms rms_norm_kernel (route.cu), the token embedding get_rows_kernel (quant.cu).
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.cuh"

namespace tmoe {

// x [n_tok][n_head][head_dim] in place, token t at position pos[t].
__global__ void rope_neox_kernel(float *__restrict__ x, const int32_t *__restrict__ pos, int64_t n_tok, int n_head,
                                 int head_dim, int n_rot, float freq_base) {
    pdl_wait();
    pdl_trigger();
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

// The per-head RMS norms of Q and K times q_norm / k_norm, then NeoX RoPE, in one launch: a CTA per
// row (token, head) of q [T][n_head][d] and k [T][n_kv][d], one thread per element (d <= 128).  The
// mean square is summed in f64, as rms_norm_kernel does.
__global__ void qk_norm_rope_kernel(float *__restrict__ q, float *__restrict__ k, const float *__restrict__ qw,
                                    const float *__restrict__ kw, const int32_t *__restrict__ pos, int n_head,
                                    int n_kv, int d, int n_rot, float freq_base, float eps) {
    pdl_wait();
    pdl_trigger();
    __shared__ float row[128];
    __shared__ double part[4];
    const int r = blockIdx.x, per_tok = n_head + n_kv;
    const int t = r / per_tok, hh = r % per_tok;
    float *x = hh < n_head ? q + ((size_t)t * n_head + hh) * d : k + ((size_t)t * n_kv + (hh - n_head)) * d;
    const float *w = hh < n_head ? qw : kw;
    const int i = threadIdx.x;
    const float v = i < d ? x[i] : 0.0f;
    double sq = (double)__fmul_rn(v, v);
    for (int o = 16; o >= 1; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if ((i & 31) == 0) part[i >> 5] = sq;
    __syncthreads();
    double sum = 0.0;
    for (int j = 0; j < (int)(blockDim.x >> 5); j++) sum += part[j];
    const float mean = __double2float_rn(__ddiv_rn(sum, (double)d));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    const float nv = i < d ? __fmul_rn(__fmul_rn(v, scale), w[i]) : 0.0f;
    if (i < d) row[i] = nv;
    __syncthreads();
    const int half = n_rot / 2;
    if (i < half) {
        const float theta = (float)pos[t] * powf(freq_base, -2.0f * (float)i / (float)n_rot);
        float sn, cs;
        sincosf(theta, &sn, &cs);
        const float x0 = row[i], x1 = row[i + half];
        x[i] = x0 * cs - x1 * sn;
        x[i + half] = x0 * sn + x1 * cs;
    } else if (i >= n_rot && i < d) {
        x[i] = nv;
    }
}

// cache[b][pos[b]][:] = rows[b][:] (n_kv * head_dim values, as F16) for K and V.
__global__ void kv_store_kernel(const float *__restrict__ k, const float *__restrict__ v, __half *__restrict__ kc,
                                __half *__restrict__ vc, const int32_t *__restrict__ pos, int n_ctx, int width,
                                int *err) {
    pdl_wait();
    pdl_trigger();
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

// One CTA per (split, KV head, sequence), 4 warps, on the tensor cores (mma.sync m16n8k16, f16
// operands, f32 accumulators).  The G <= 8 query heads of the KV head are the 16-row A operand
// (rows past G zero); each warp takes tiles of AT_TILE = 16 positions of the CTA's split (warp w:
// tiles w, w + 4, ...), staged by cp.async into its own two padded shared-memory stages (rows past
// the split's end zero-filled and masked to -inf):
//   S = Q K^T   (2 position blocks x HD/16 dim blocks; K rows through ldmatrix: a K row is a
//               column of the col-major B operand);
//   online softmax of each head (row) over the tile, in the S fragments (a quad of lanes shares a
//               row);
//   O += P V    (the S fragments, as f16, are P's A fragments; V through ldmatrix.trans).
// At the end the four warps' (max, sum, O) are merged in shared memory and written as the split's
// partial for attn_merge_kernel.
constexpr int AT_TILE = 16;
constexpr int AT_WARPS = 4;
constexpr int AT_THREADS = 32 * AT_WARPS;
constexpr int AT_MAX_G = 8;

template <int HD>
struct AttnSmem {
    static constexpr int ROW = HD + 8;  // halfs per staged row: 16 bytes of padding, conflict-free ldmatrix
    static constexpr int STAGE = 2 * AT_TILE * ROW;  // K then V
    static constexpr size_t BYTES = (size_t)AT_WARPS * 2 * STAGE * 2;
};

__device__ __forceinline__ void at_cp16(uint32_t dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void at_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void at_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}

template <int HD>
__global__ void __launch_bounds__(AT_THREADS) attn_decode_kernel(const float *__restrict__ q,
                                                                 const __half *__restrict__ kc,
                                                                 const __half *__restrict__ vc,
                                                                 const int32_t *__restrict__ pos, int n_head,
                                                                 int n_kv, int n_ctx, float scale,
                                                                 float *__restrict__ part) {
    pdl_wait();
    pdl_trigger();
    using SM = AttnSmem<HD>;
    constexpr int KB = HD / 16;  // dim blocks of the QK^T product
    constexpr int NB = HD / 8;   // dim blocks of the output
    extern __shared__ __align__(16) __half at_smem[];
    const int s = blockIdx.x, g = blockIdx.y, b = blockIdx.z, S = gridDim.x;
    const int G = n_head / n_kv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gr = lane >> 2, t4 = lane & 3;
    const int len = min(pos[b] + 1, n_ctx);
    const int per = ((len + S - 1) / S + AT_TILE - 1) / AT_TILE * AT_TILE;
    const int p0 = min(len, s * per), p1 = min(len, p0 + per);
    const size_t row_stride = (size_t)n_kv * HD;
    const __half *kb = kc + (size_t)b * n_ctx * row_stride + (size_t)g * HD;
    const __half *vb = vc + (size_t)b * n_ctx * row_stride + (size_t)g * HD;
    __half *stage0 = at_smem + (size_t)warp * 2 * SM::STAGE;

    // Q fragments (rows = heads of this KV head), f16; the scale goes on the f32 scores, as ggml's
    // flash attention over an F16 cache converts Q to F16 and scales the Q.K dot
    uint32_t qa[KB][4];
    {
        const float *qb = q + ((size_t)b * n_head + (size_t)g * G) * HD;
#pragma unroll
        for (int k = 0; k < KB; k++) {
            const int c0 = 16 * k + 2 * t4;
            float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            if (gr < G) {
                v[0] = qb[gr * HD + c0], v[1] = qb[gr * HD + c0 + 1];
                v[4] = qb[gr * HD + c0 + 8], v[5] = qb[gr * HD + c0 + 9];
            }
            qa[k][0] = pack_h2(v[0], v[1]);
            qa[k][1] = 0u;  // rows 8..15: no head
            qa[k][2] = pack_h2(v[4], v[5]);
            qa[k][3] = 0u;
        }
    }
    float o[NB][4];
#pragma unroll
    for (int n = 0; n < NB; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m_run = -INFINITY, l_run = 0.0f;  // of row gr (the rows gr + 8 hold no head)

    const int n_tiles = (p1 - p0 + AT_TILE - 1) / AT_TILE;
    auto issue = [&](int i, int st) {  // tile i of this warp into stage st
        const int t0 = p0 + (warp + i * AT_WARPS) * AT_TILE;
        __half *ks = stage0 + st * SM::STAGE, *vs = ks + AT_TILE * SM::ROW;
        constexpr int CH = HD / 8;  // 16-byte chunks per row
        for (int c = lane; c < AT_TILE * CH; c += 32) {
            const int r = c / CH, col = 8 * (c % CH);
            const bool ok = t0 + r < p1;
            const size_t off = (size_t)(ok ? t0 + r : p0) * row_stride + col;
            at_cp16(smem_u32(ks + r * SM::ROW + col), kb + off, ok);
            at_cp16(smem_u32(vs + r * SM::ROW + col), vb + off, ok);
        }
        at_commit();
    };
    const int mine = n_tiles > warp ? (n_tiles - warp + AT_WARPS - 1) / AT_WARPS : 0;
    if (mine > 0) issue(0, 0);
    for (int i = 0; i < mine; i++) {
        if (i + 1 < mine) {
            issue(i + 1, (i + 1) & 1);
            at_wait<1>();
        } else {
            at_wait<0>();
        }
        __syncwarp();
        const __half *ks = stage0 + (i & 1) * SM::STAGE, *vs = ks + AT_TILE * SM::ROW;
        const int t0 = p0 + (warp + i * AT_WARPS) * AT_TILE;
        // S = Q K^T: 16 heads x 16 positions
        float sc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
        for (int nb = 0; nb < 2; nb++)
#pragma unroll
            for (int k = 0; k < KB; k += 2) {
                // matrices: positions 8nb + 0..7 x dims 16k + {0, 8}, 16(k+1) + {0, 8}
                const int r = 8 * nb + (lane & 7), cblk = 16 * k + 8 * (lane >> 3);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(smem_u32(ks + r * SM::ROW + cblk), b0, b1, b2, b3);
                mma_f16(sc[nb], qa[k][0], qa[k][1], qa[k][2], qa[k][3], b0, b1);
                if (k + 1 < KB) mma_f16(sc[nb], qa[k + 1][0], qa[k + 1][1], qa[k + 1][2], qa[k + 1][3], b2, b3);
            }
        // scale; mask positions past the split; then the online softmax of row gr
#pragma unroll
        for (int nb = 0; nb < 2; nb++)
#pragma unroll
            for (int j = 0; j < 2; j++)
                sc[nb][j] = t0 + 8 * nb + 2 * t4 + j >= p1 ? -INFINITY : sc[nb][j] * scale;
        float mx = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run, mx);  // finite: every tile holds at least one position
        const float alpha = m_run == -INFINITY ? 0.0f : __expf(m_run - m_new);
        float pr[2][2];
        float sum = 0.0f;
#pragma unroll
        for (int nb = 0; nb < 2; nb++)
#pragma unroll
            for (int j = 0; j < 2; j++) {
                pr[nb][j] = __expf(sc[nb][j] - m_new);
                sum += pr[nb][j];
            }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        l_run = l_run * alpha + sum;
        m_run = m_new;
        // P as the A operand (k = the 16 positions): rows gr (heads), rows gr + 8 zero
        const uint32_t pa0 = pack_h2(pr[0][0], pr[0][1]), pa2 = pack_h2(pr[1][0], pr[1][1]);
#pragma unroll
        for (int n = 0; n < NB; n++) o[n][0] *= alpha, o[n][1] *= alpha;
#pragma unroll
        for (int n = 0; n < NB; n += 2) {
            // matrices: positions 0..7 / 8..15 x dims 8n + 0..7, then 8(n+1) + 0..7, transposed
            const int r = (lane & 7) + 8 * ((lane >> 3) & 1), cblk = 8 * n + 8 * (lane >> 4);
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(smem_u32(vs + r * SM::ROW + cblk), b0, b1, b2, b3);
            mma_f16(o[n], pa0, 0u, pa2, 0u, b0, b1);
            mma_f16(o[n + 1], pa0, 0u, pa2, 0u, b2, b3);
        }
        __syncwarp();  // every lane's ldmatrix of this stage is done before it is refilled
    }
    at_wait<0>();
    __syncthreads();
    // merge the warps: row gr of each warp -> shared memory, then the CTA combines them
    float *red = reinterpret_cast<float *>(at_smem);  // [warp][8 rows][2 + HD]
    constexpr int RW = 2 + HD;
    if (gr < AT_MAX_G) {
        float *rr = red + ((size_t)warp * AT_MAX_G + gr) * RW;
        if (t4 == 0) rr[0] = m_run, rr[1] = l_run;
#pragma unroll
        for (int n = 0; n < NB; n++) rr[2 + 8 * n + 2 * t4] = o[n][0], rr[2 + 8 * n + 2 * t4 + 1] = o[n][1];
    }
    __syncthreads();
    const size_t pstride = (size_t)HD + 2;
    for (int i = threadIdx.x; i < G * HD; i += AT_THREADS) {
        const int h = i / HD, d = i % HD;
        float M = -INFINITY;
        for (int w = 0; w < AT_WARPS; w++) M = fmaxf(M, red[((size_t)w * AT_MAX_G + h) * RW]);
        float L = 0.0f, acc = 0.0f;
        for (int w = 0; w < AT_WARPS; w++) {
            const float *rr = red + ((size_t)w * AT_MAX_G + h) * RW;
            if (rr[0] == -INFINITY) continue;
            const float f = __expf(rr[0] - M);
            L += f * rr[1];
            acc += f * rr[2 + d];
        }
        float *pp = part + (((size_t)b * n_head + (size_t)g * G + h) * S + s) * pstride;
        if (d == 0) pp[0] = M, pp[1] = L;
        pp[2 + d] = acc;
    }
}

// out[b][head][:] from the S partials of (b, head): one CTA per (b, head).
__global__ void attn_merge_kernel(const float *__restrict__ part, int S, int HD, float *__restrict__ out) {
    pdl_wait();
    pdl_trigger();
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

// ------------------------------------------------------------------ prefill attention
// cache[seq][pos0 + i][:] = rows[i][:] (n_kv * head_dim values as F16) for K and V, i < S: the
// set_rows of a multi-token step's new K/V rows.
__global__ void kv_store_rows_kernel(const float *__restrict__ k, const float *__restrict__ v, __half *__restrict__ kc,
                                     __half *__restrict__ vc, int seq, int pos0, int n_ctx, int width) {
    const size_t i = blockIdx.x;
    const size_t dst = ((size_t)seq * n_ctx + pos0 + i) * width;
    const float4 *k4 = reinterpret_cast<const float4 *>(k + i * width);
    const float4 *v4 = reinterpret_cast<const float4 *>(v + i * width);
    for (int c = threadIdx.x; c < width / 4; c += blockDim.x) {
        const float4 a = k4[c], b = v4[c];
        reinterpret_cast<__half2 *>(kc + dst)[2 * c] = __floats2half2_rn(a.x, a.y);
        reinterpret_cast<__half2 *>(kc + dst)[2 * c + 1] = __floats2half2_rn(a.z, a.w);
        reinterpret_cast<__half2 *>(vc + dst)[2 * c] = __floats2half2_rn(b.x, b.y);
        reinterpret_cast<__half2 *>(vc + dst)[2 * c + 1] = __floats2half2_rn(b.z, b.w);
    }
}

// Causal attention of S new queries of one sequence (query i at position pos0 + i attends to the
// cache's positions 0 .. pos0 + i), the masked flash attention of a prefill step.  One CTA per
// (64-query block, query head), 4 warps of 16 query rows each; the query head's KV head (GQA:
// head / (n_head / n_kv)) is read from the F16 cache in 64-position tiles, staged by cp.async into
// two shared stages that all four warps read.  Per tile and warp, on the tensor cores (mma.sync
// m16n8k16, f16 operands, f32 accumulators), as in the decode kernel:
//   S = Q K^T (16 x 64: K rows through ldmatrix), scaled in f32, masked above the diagonal;
//   online softmax of each row in the S fragments (a quad of lanes shares a row);
//   O += P V  (the S fragments, as f16, are P's A fragments; V through ldmatrix.trans).
// The longest query blocks (the last ones) are launched first.
constexpr int AP_Q = 64;  // query rows per CTA
constexpr int AP_K = 64;  // positions per staged tile
constexpr int AP_WARPS = 4;
constexpr int AP_THREADS = 32 * AP_WARPS;

template <int HD>
struct PrefillSmem {
    static constexpr int ROW = HD + 8;                 // halfs per staged row (conflict-free ldmatrix)
    static constexpr int STAGE = 2 * AP_K * ROW;       // K then V
    static constexpr size_t BYTES = (size_t)2 * STAGE * 2;
};

template <int HD>
__global__ void __launch_bounds__(AP_THREADS) attn_prefill_kernel(const float *__restrict__ q,
                                                                  const __half *__restrict__ kc,
                                                                  const __half *__restrict__ vc, int seq, int pos0,
                                                                  int S, int n_head, int n_kv, int n_ctx, float scale,
                                                                  float *__restrict__ out) {
    using SM = PrefillSmem<HD>;
    constexpr int KB = HD / 16, NB = HD / 8, CH = HD / 8;  // CH: 16-byte chunks per row
    extern __shared__ __align__(16) __half ap_smem[];
    const int qb = gridDim.x - 1 - blockIdx.x, h = blockIdx.y;
    const int kvh = h / (n_head / n_kv);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gr = lane >> 2, t4 = lane & 3;
    const int r0 = qb * AP_Q + warp * 16;  // this warp's first query row
    const int rA = r0 + gr, rB = r0 + gr + 8;
    const int qpA = pos0 + rA, qpB = pos0 + rB;
    const int warp_last = pos0 + min(r0 + 15, S - 1);  // the warp's last query position
    const int kv_end = pos0 + min(S, (qb + 1) * AP_Q);  // keys 0 .. kv_end - 1 serve this CTA
    const size_t row_stride = (size_t)n_kv * HD;
    const __half *kb = kc + (size_t)seq * n_ctx * row_stride + (size_t)kvh * HD;
    const __half *vb = vc + (size_t)seq * n_ctx * row_stride + (size_t)kvh * HD;

    // Q fragments of rows rA and rB (f16, unscaled; rows past S read as zero and are not written)
    uint32_t qa[KB][4];
    {
        const size_t qs = (size_t)n_head * HD;
        const float *qa_row = q + (size_t)min(rA, S - 1) * qs + (size_t)h * HD;
        const float *qb_row = q + (size_t)min(rB, S - 1) * qs + (size_t)h * HD;
        const bool va = rA < S, vb_ = rB < S;
#pragma unroll
        for (int k = 0; k < KB; k++) {
            const int c0 = 16 * k + 2 * t4;
            const float2 a0 = va ? *reinterpret_cast<const float2 *>(qa_row + c0) : make_float2(0.f, 0.f);
            const float2 a1 = va ? *reinterpret_cast<const float2 *>(qa_row + c0 + 8) : make_float2(0.f, 0.f);
            const float2 b0 = vb_ ? *reinterpret_cast<const float2 *>(qb_row + c0) : make_float2(0.f, 0.f);
            const float2 b1 = vb_ ? *reinterpret_cast<const float2 *>(qb_row + c0 + 8) : make_float2(0.f, 0.f);
            qa[k][0] = pack_h2(a0.x, a0.y);
            qa[k][1] = pack_h2(b0.x, b0.y);
            qa[k][2] = pack_h2(a1.x, a1.y);
            qa[k][3] = pack_h2(b1.x, b1.y);
        }
    }
    float o[NB][4];
#pragma unroll
    for (int n = 0; n < NB; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float mA = -INFINITY, mB = -INFINITY, lA = 0.0f, lB = 0.0f;

    const int n_tiles = (kv_end + AP_K - 1) / AP_K;
    auto issue = [&](int t, int st) {  // tile t into stage st, all threads; rows past kv_end zero
        __half *ks = ap_smem + st * SM::STAGE, *vs = ks + AP_K * SM::ROW;
        const int p0 = t * AP_K;
        for (int c = threadIdx.x; c < AP_K * CH; c += AP_THREADS) {
            const int r = c / CH, col = 8 * (c % CH);
            const bool ok = p0 + r < kv_end;
            const size_t off = (size_t)(ok ? p0 + r : 0) * row_stride + col;
            at_cp16(smem_u32(ks + r * SM::ROW + col), kb + off, ok);
            at_cp16(smem_u32(vs + r * SM::ROW + col), vb + off, ok);
        }
        at_commit();
    };
    issue(0, 0);
    for (int t = 0; t < n_tiles; t++) {
        if (t + 1 < n_tiles) {
            issue(t + 1, (t + 1) & 1);
            at_wait<1>();
        } else {
            at_wait<0>();
        }
        __syncthreads();
        const int p0 = t * AP_K;
        if (p0 <= warp_last) {  // else every position of the tile is after this warp's queries
            const __half *ks = ap_smem + (t & 1) * SM::STAGE, *vs = ks + AP_K * SM::ROW;
            float sc[8][4];
#pragma unroll
            for (int nb = 0; nb < 8; nb++) sc[nb][0] = sc[nb][1] = sc[nb][2] = sc[nb][3] = 0.0f;
#pragma unroll
            for (int nb = 0; nb < 8; nb++)
#pragma unroll
                for (int k = 0; k < KB; k += 2) {
                    const int r = 8 * nb + (lane & 7), cblk = 16 * k + 8 * (lane >> 3);
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(smem_u32(ks + r * SM::ROW + cblk), b0, b1, b2, b3);
                    mma_f16(sc[nb], qa[k][0], qa[k][1], qa[k][2], qa[k][3], b0, b1);
                    mma_f16(sc[nb], qa[k + 1][0], qa[k + 1][1], qa[k + 1][2], qa[k + 1][3], b2, b3);
                }
            // scale, the causal mask (and positions past kv_end), the row maxima
            float xA = -INFINITY, xB = -INFINITY;
#pragma unroll
            for (int nb = 0; nb < 8; nb++)
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const int kp = p0 + 8 * nb + 2 * t4 + j;
                    sc[nb][j] = kp > qpA || kp >= kv_end ? -INFINITY : sc[nb][j] * scale;
                    sc[nb][2 + j] = kp > qpB || kp >= kv_end ? -INFINITY : sc[nb][2 + j] * scale;
                    xA = fmaxf(xA, sc[nb][j]);
                    xB = fmaxf(xB, sc[nb][2 + j]);
                }
            xA = fmaxf(xA, __shfl_xor_sync(0xffffffffu, xA, 1));
            xA = fmaxf(xA, __shfl_xor_sync(0xffffffffu, xA, 2));
            xB = fmaxf(xB, __shfl_xor_sync(0xffffffffu, xB, 1));
            xB = fmaxf(xB, __shfl_xor_sync(0xffffffffu, xB, 2));
            // position 0 is in tile 0 for every row, so the running maxima are finite from there on
            const float nA = fmaxf(mA, xA), nB = fmaxf(mB, xB);
            const float aA = mA == -INFINITY ? 0.0f : __expf(mA - nA), aB = mB == -INFINITY ? 0.0f : __expf(mB - nB);
            float sA = 0.0f, sB = 0.0f;
#pragma unroll
            for (int nb = 0; nb < 8; nb++)
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    sc[nb][j] = __expf(sc[nb][j] - nA);
                    sc[nb][2 + j] = __expf(sc[nb][2 + j] - nB);
                    sA += sc[nb][j];
                    sB += sc[nb][2 + j];
                }
            sA += __shfl_xor_sync(0xffffffffu, sA, 1);
            sA += __shfl_xor_sync(0xffffffffu, sA, 2);
            sB += __shfl_xor_sync(0xffffffffu, sB, 1);
            sB += __shfl_xor_sync(0xffffffffu, sB, 2);
            lA = lA * aA + sA, lB = lB * aB + sB;
            mA = nA, mB = nB;
#pragma unroll
            for (int n = 0; n < NB; n++) o[n][0] *= aA, o[n][1] *= aA, o[n][2] *= aB, o[n][3] *= aB;
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {  // P V over the tile's 4 k16 position blocks
                const uint32_t pa0 = pack_h2(sc[2 * kk][0], sc[2 * kk][1]);
                const uint32_t pa1 = pack_h2(sc[2 * kk][2], sc[2 * kk][3]);
                const uint32_t pa2 = pack_h2(sc[2 * kk + 1][0], sc[2 * kk + 1][1]);
                const uint32_t pa3 = pack_h2(sc[2 * kk + 1][2], sc[2 * kk + 1][3]);
#pragma unroll
                for (int n = 0; n < NB; n += 2) {
                    const int r = 16 * kk + (lane & 7) + 8 * ((lane >> 3) & 1), cblk = 8 * n + 8 * (lane >> 4);
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(smem_u32(vs + r * SM::ROW + cblk), b0, b1, b2, b3);
                    mma_f16(o[n], pa0, pa1, pa2, pa3, b0, b1);
                    mma_f16(o[n + 1], pa0, pa1, pa2, pa3, b2, b3);
                }
            }
        }
        __syncthreads();  // every warp is done with this stage before it is refilled
    }
    const size_t os = (size_t)n_head * HD;
    const float iA = lA > 0.0f ? 1.0f / lA : 0.0f, iB = lB > 0.0f ? 1.0f / lB : 0.0f;
#pragma unroll
    for (int n = 0; n < NB; n++) {
        const int c = 8 * n + 2 * t4;
        if (rA < S)
            *reinterpret_cast<float2 *>(out + (size_t)rA * os + (size_t)h * HD + c) = make_float2(o[n][0] * iA, o[n][1] * iA);
        if (rB < S)
            *reinterpret_cast<float2 *>(out + (size_t)rB * os + (size_t)h * HD + c) = make_float2(o[n][2] * iB, o[n][3] * iB);
    }
}

__global__ void add_kernel(const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ out,
                           int64_t n) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = a[i] + b[i];
}

// out[r] = the first index of the largest value of row r.  One CTA per row.
__global__ void __launch_bounds__(1024) argmax_kernel(const float *__restrict__ x, int64_t n, bool vec4,
                                                      int32_t *__restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const float *row = x + (int64_t)blockIdx.x * n;
    float best = -INFINITY;
    int64_t bi = 0x7fffffff;
    if (vec4) {  // n % 4 == 0 and the rows 16-byte aligned: four elements a load, two loads in flight
        const float4 *r4 = reinterpret_cast<const float4 *>(row);
        const int64_t n4 = n / 4, step = blockDim.x;
        for (int64_t j = threadIdx.x; j < n4; j += 2 * step) {
            const float4 a = __ldcs(r4 + j);
            const float4 b = j + step < n4 ? __ldcs(r4 + j + step) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
            const float va[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int c = 0; c < 8; c++) {
                const int64_t i = (c < 4 ? j : j + step) * 4 + (c & 3);
                if (va[c] > best || (va[c] == best && i < bi)) best = va[c], bi = i;
            }
        }
    } else {
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
            const float v = row[i];
            if (v > best || (v == best && i < bi)) best = v, bi = i;
        }
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

// The dispatch of a dense product (one matrix, every row of x): the T rows in groups of `group`
// tokens, each group an active entry of the same matrix, so that the GEMV spreads the matrix's row
// tiles times the groups over the SMs (a group's second read of the rows comes from L2); the GEMV's
// work counters zeroed.  With ks > 1 the product is split along K into ks slices, slice s being
// "expert" s of the GEMV (the matrix's columns s*K/ks.., an expert stride of one slice's bytes) and
// token t's slice s its pair t*ks + s: the Q8_K rows of x [T][K] read as [T*ks][K/ks], the partial
// outputs as [T][ks][N].  Entry j = s * ng + g holds slice s of group g; perm[s*T + t] = t*ks + s.
__global__ void dense_prep_kernel(int T, int group, int ks, int4 *__restrict__ active, int32_t *__restrict__ n_active,
                                  int32_t *__restrict__ perm, int *__restrict__ counters, int n_counters) {
    pdl_wait();
    pdl_trigger();
    const int ng = (T + group - 1) / group;
    for (int i = threadIdx.x; i < T * ks; i += blockDim.x) perm[i] = (i % T) * ks + i / T;
    for (int j = threadIdx.x; j < ng * ks; j += blockDim.x) {
        const int s = j / ng, g = j % ng;
        active[j] = make_int4(s, s * T + g * group, s * T + min(T, (g + 1) * group), 0);
    }
    if (threadIdx.x < n_counters) counters[threadIdx.x] = 0;
    if (threadIdx.x == 0) n_active[0] = ng * ks;
}

// out[t][n] = sum over s of part[t][s][n], the slices added in order (the same sums every call).
__global__ void splitk_sum_kernel(const float *__restrict__ part, int64_t T, int N, int ks, float *__restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // a group of 4 outputs
    const int64_t n4 = (int64_t)N / 4;
    if (i >= T * n4) return;
    const int64_t t = i / n4, c = i % n4;
    const float4 *p = reinterpret_cast<const float4 *>(part + t * ks * (int64_t)N) + c;
    float4 a = __ldcs(p);
    for (int s = 1; s < ks; s++) {
        const float4 b = __ldcs(p + s * n4);
        a.x += b.x, a.y += b.y, a.z += b.z, a.w += b.w;
    }
    reinterpret_cast<float4 *>(out + t * (int64_t)N)[c] = a;
}

// ------------------------------------------------------------------ launchers
cudaError_t launch_dense_prep(int T, int group, int ks, int4 *active, int32_t *n_active, int32_t *perm, int *counters,
                              int n_counters, cudaStream_t st) {
    if (n_counters > 256 || group < 1 || ks < 1 || (int64_t)T * ks >= (1 << 24)) return cudaErrorInvalidValue;
    launch_k(dense_prep_kernel, 1, 256, 0, st, T, group, ks, active, n_active, perm, counters, n_counters);
    return cudaGetLastError();
}

cudaError_t launch_splitk_sum(const float *part, int64_t T, int N, int ks, float *out, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (N % 4 || ks < 1 || ((uintptr_t)part & 15) || ((uintptr_t)out & 15)) return cudaErrorInvalidValue;
    const int64_t n = T * (N / 4);
    launch_k(splitk_sum_kernel, (unsigned)((n + 255) / 256), 256, 0, st, part, T, N, ks, out);
    return cudaGetLastError();
}

cudaError_t launch_qk_norm_rope(float *q, float *k, const float *qw, const float *kw, const int32_t *pos, int64_t T,
                                int n_head, int n_kv, int d, int n_rot, float freq_base, float eps, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (d <= 0 || d > 128 || d % 32 || n_rot <= 0 || n_rot > d || n_rot % 2 || T * (n_head + n_kv) > 0x7fffffff)
        return cudaErrorInvalidValue;
    launch_k(qk_norm_rope_kernel, (unsigned)(T * (n_head + n_kv)), d, 0, st, q, k, qw, kw, pos, n_head, n_kv, d, n_rot,
             freq_base, eps);
    return cudaGetLastError();
}

cudaError_t launch_rope_neox(float *x, const int32_t *pos, int64_t n_tok, int n_head, int head_dim, int n_rot,
                             float freq_base, cudaStream_t st) {
    if (n_tok <= 0) return cudaSuccess;
    if (n_rot <= 0 || n_rot > head_dim || n_rot % 2 || n_tok * n_head > 0x7fffffff) return cudaErrorInvalidValue;
    launch_k(rope_neox_kernel, (unsigned)(n_tok * n_head), 64, 0, st, x, pos, n_tok, n_head, head_dim, n_rot, freq_base);
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
    launch_k(kv_store_kernel, B, 128, 0, st, k, v, kc, vc, pos, n_ctx, width, err);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int S = attn_splits(B, n_kv, n_ctx, sm_count);
    const dim3 grid(S, n_kv, B);
    static int set128[64] = {}, set64[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (head_dim == 128) {
        constexpr size_t smem = AttnSmem<128>::BYTES;
        if (!set128[dev] &&
            (e = cudaFuncSetAttribute(attn_decode_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem)) != cudaSuccess)
            return e;
        set128[dev] = 1;
        launch_k(attn_decode_kernel<128>, grid, AT_THREADS, smem, st, q, kc, vc, pos, n_head, n_kv, n_ctx, scale, part);
    } else {
        constexpr size_t smem = AttnSmem<64>::BYTES;
        if (!set64[dev] &&
            (e = cudaFuncSetAttribute(attn_decode_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem)) != cudaSuccess)
            return e;
        set64[dev] = 1;
        launch_k(attn_decode_kernel<64>, grid, AT_THREADS, smem, st, q, kc, vc, pos, n_head, n_kv, n_ctx, scale, part);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    launch_k(attn_merge_kernel, B * n_head, 128, 0, st, part, S, head_dim, out);
    return cudaGetLastError();
}

cudaError_t launch_attn_prefill(const float *q, const float *k, const float *v, __half *kc, __half *vc, int seq,
                                int pos0, int S, int n_head, int n_kv, int head_dim, int n_ctx, float scale, float *out,
                                cudaStream_t st) {
    if (S <= 0) return cudaSuccess;
    if (n_kv <= 0 || n_head % n_kv || (head_dim != 64 && head_dim != 128) || n_head > 65535 || seq < 0 ||
        pos0 < 0 || (int64_t)pos0 + S > n_ctx)
        return cudaErrorInvalidValue;
    const int width = n_kv * head_dim;
    kv_store_rows_kernel<<<S, 128, 0, st>>>(k, v, kc, vc, seq, pos0, n_ctx, width);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const dim3 grid((S + AP_Q - 1) / AP_Q, n_head);
    static int set128[64] = {}, set64[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (head_dim == 128) {
        constexpr size_t smem = PrefillSmem<128>::BYTES;
        if (!set128[dev] &&
            (e = cudaFuncSetAttribute(attn_prefill_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem)) != cudaSuccess)
            return e;
        set128[dev] = 1;
        attn_prefill_kernel<128><<<grid, AP_THREADS, smem, st>>>(q, kc, vc, seq, pos0, S, n_head, n_kv, n_ctx, scale,
                                                                 out);
    } else {
        constexpr size_t smem = PrefillSmem<64>::BYTES;
        if (!set64[dev] &&
            (e = cudaFuncSetAttribute(attn_prefill_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem)) != cudaSuccess)
            return e;
        set64[dev] = 1;
        attn_prefill_kernel<64><<<grid, AP_THREADS, smem, st>>>(q, kc, vc, seq, pos0, S, n_head, n_kv, n_ctx, scale,
                                                                out);
    }
    return cudaGetLastError();
}

cudaError_t launch_add(const float *a, const float *b, float *out, int64_t n, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    launch_k(add_kernel, (unsigned)((n + 255) / 256), 256, 0, st, a, b, out, n);
    return cudaGetLastError();
}

cudaError_t launch_argmax(const float *x, int64_t rows, int64_t n, int32_t *out, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    if (rows > 0x7fffffff || n <= 0) return cudaErrorInvalidValue;
    const bool vec4 = n % 4 == 0 && ((uintptr_t)x & 15) == 0;
    launch_k(argmax_kernel, (unsigned)rows, 1024, 0, st, x, n, vec4, out);
    return cudaGetLastError();
}

}  // namespace tmoe
