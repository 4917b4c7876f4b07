// Router (qwen3moe.rs:2871-2890): rms_norm * ffn_norm, logits = gate_inp . xn, softmax,
// top-k (descending, ties to the lower index), weights = sel / clamp(sum sel, 6.1035156e-5);
// and the Q8_K quantisation of activation rows (ggml's vec_dot_type for the K-quants).
//
// The router dot is canonical so that the logits are bit-identical with the CPU oracle: lane l
// of a warp accumulates the elements i with (i/4) % 32 == l in increasing i with fma, then a
// butterfly over lane distances 16, 8, 4, 2, 1.  The rest of the canonical order is in route.cuh.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "q8k.cuh"
#include "route.cuh"

namespace tmoe {

// One warp per token: ggml rms_norm (f64 sum of f32 squares) times the optional norm weight.
__global__ void rms_norm_kernel(const float *__restrict__ x, const float *__restrict__ norm_w, float eps, int64_t T,
                                int H, float *__restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= T) return;
    const float *xr = x + warp * H;
    double acc = 0.0;
    for (int m = 0; m * 128 < H; m++)
        for (int c = 0; c < 4; c++) {
            const int i = 128 * m + 4 * lane + c;
            if (i < H) acc = __dadd_rn(acc, (double)__fmul_rn(xr[i], xr[i]));
        }
    const double sum = butterfly_f64(acc);
    const float mean = __double2float_rn(__ddiv_rn(sum, (double)H));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    float *o = out + warp * H;
    for (int i = lane; i < H; i += 32) {
        const float v = __fmul_rn(xr[i], scale);
        o[i] = norm_w ? __fmul_rn(v, norm_w[i]) : v;
    }
}

// The same norm with a CTA of 256 threads per row, for batches of few rows (one warp per row would
// leave most SMs idle): per-thread f64 partial sums of the f32 squares, a butterfly per warp, the
// warps' sums added in order; the same f32 mean, scale and products as rms_norm_kernel.
__global__ void __launch_bounds__(256) rms_norm_row_kernel(const float *__restrict__ x, const float *__restrict__ norm_w,
                                                          float eps, int H, float *__restrict__ out) {
    pdl_wait();
    pdl_trigger();
    __shared__ double part[8];
    const int64_t row = blockIdx.x;
    const float *xr = x + row * H;
    double acc = 0.0;
    for (int i = threadIdx.x; i < H; i += 256) acc = __dadd_rn(acc, (double)__fmul_rn(xr[i], xr[i]));
    acc = butterfly_f64(acc);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    double sum = 0.0;
    for (int w = 0; w < 8; w++) sum = __dadd_rn(sum, part[w]);
    const float mean = __double2float_rn(__ddiv_rn(sum, (double)H));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    float *o = out + row * H;
    for (int i = threadIdx.x; i < H; i += 256) {
        const float v = __fmul_rn(xr[i], scale);
        o[i] = norm_w ? __fmul_rn(v, norm_w[i]) : v;
    }
}

// Router logits, H % 512 == 0: a CTA of RL_WARPS warps (one expert each) and TT tokens.  The
// tokens' rows are staged whole in shared memory with 16-byte loads; each warp then streams its
// expert's row with all loads of an 512-element stretch in flight.  When q8 != NULL, the CTAs of
// the first expert column also write the tokens' Q8_K rows (the activation quantisation of the
// expert products), from the same staged rows.
constexpr int RL_WARPS = 8;

template <int TT>
__global__ void __launch_bounds__(RL_WARPS * 32) router_logits_kernel(const float *__restrict__ xn,
                                                                      const float *__restrict__ rw, int64_t T, int H,
                                                                      int E, float *__restrict__ logits, Q8Rows q8) {
    extern __shared__ float4 xs4[];  // [TT][H/4]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.x * RL_WARPS + warp;
    const int64_t t0 = (int64_t)blockIdx.y * TT;
    const int nt = (int)min((int64_t)TT, T - t0);
    const int H4 = H / 4;
    for (int idx = threadIdx.x; idx < TT * H4; idx += RL_WARPS * 32) {
        const int j = idx / H4;
        xs4[idx] = j < nt ? __ldg(reinterpret_cast<const float4 *>(xn + (t0 + j) * H) + (idx - j * H4))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncthreads();
    if (q8.qs && blockIdx.x == 0) {  // Q8_K of the staged rows: one warp per (token, 256-block)
        const int nb = H / TMOE_QK;
        for (int u = warp; u < nt * nb; u += RL_WARPS) {
            const int j = u / nb, b = u % nb;
            const float4 a0 = xs4[j * H4 + b * 64 + 2 * lane], a1 = xs4[j * H4 + b * 64 + 2 * lane + 1];
            const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            uint2 q;
            float d;
            int s16;
            q8k_block_warp(v, q, d, s16);
            q8k_store_warp(q8, t0 + j, H, b, q, d, s16);
        }
    }
    if (e >= E) return;
    const float4 *w4 = reinterpret_cast<const float4 *>(rw + (int64_t)e * H);
    float acc[TT];
#pragma unroll
    for (int j = 0; j < TT; j++) acc[j] = 0.0f;
    for (int m0 = 0; m0 < H / 128; m0 += 4) {  // H % 512 == 0
        float4 w[4];
#pragma unroll
        for (int u = 0; u < 4; u++) w[u] = __ldg(w4 + 32 * (m0 + u) + lane);
#pragma unroll
        for (int u = 0; u < 4; u++) {
#pragma unroll
            for (int j = 0; j < TT; j++) {
                const float4 x = xs4[j * H4 + 32 * (m0 + u) + lane];
                acc[j] = __fmaf_rn(w[u].x, x.x, acc[j]);
                acc[j] = __fmaf_rn(w[u].y, x.y, acc[j]);
                acc[j] = __fmaf_rn(w[u].z, x.z, acc[j]);
                acc[j] = __fmaf_rn(w[u].w, x.w, acc[j]);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < TT; j++) {
        const float s = butterfly_f32(acc[j]);
        if (lane == 0 && j < nt) logits[(t0 + j) * E + e] = s;
    }
}

// Router logits for many tokens (H % 128 == 0): persistent CTAs of 8 warps over tiles of 16 tokens
// x 64 experts.  K streams in chunks of 128 columns through a ring of RT_STAGES shared-memory
// stages (one bulk copy per 512-byte row chunk); the ring runs on across tiles, so the next tile's
// chunks arrive while a tile finishes.  A warp holds 8 tokens x 16 experts; lane l keeps the
// canonical partial sums of slice l for all 128 logits in registers (the same fma chain as
// router_logits_kernel), so one shared-memory load feeds 32 (w) or 64 (x) FMAs.  The 32 partials
// of a logit are then summed over the lanes in the butterfly's tree (pairs at lane distance 16, 8,
// 4, 2, 1), transposed so that 32 logits take 31 shuffles instead of 160: bit-identical to
// butterfly_f32 since each add has the same operands.
constexpr int RT_TOK = 16, RT_EXP = 64, RT_KC = 128, RT_STAGES = 4;
constexpr int RT_STAGE_FLOATS = (RT_TOK + RT_EXP) * RT_KC;
constexpr size_t RT_SMEM = (size_t)RT_STAGES * RT_STAGE_FLOATS * 4;

__device__ __forceinline__ void rt_tma_load_2d(void *dst, const CUtensorMap *m, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ float transposed_butterfly(float (&v)[32], int lane) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const bool up = (lane & off) != 0;
#pragma unroll
        for (int j = 0; j < off; j++) {
            const float send = up ? v[j] : v[j + off];
            const float keep = up ? v[j + off] : v[j];
            v[j] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, off));
        }
    }
    return v[0];  // the logit of index `lane`
}

__global__ void __launch_bounds__(256, 1) router_logits_tiled_kernel(const float *__restrict__ xn,
                                                                     const float *__restrict__ rw, int64_t T, int H,
                                                                     int E, float *__restrict__ logits, int *err,
                                                                     const __grid_constant__ CUtensorMap map_x,
                                                                     const __grid_constant__ CUtensorMap map_w) {
    extern __shared__ __align__(128) float rt_smem[];  // [RT_STAGES][16 token rows + 64 expert rows][RT_KC]
    __shared__ __align__(8) uint64_t full[RT_STAGES];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_ch = H / RT_KC;
    const int tiles_e = (E + RT_EXP - 1) / RT_EXP;
    const int64_t n_tiles = ((T + RT_TOK - 1) / RT_TOK) * tiles_e;
    // the CTA's tiles: blockIdx.x + i * gridDim.x; the expert tiles of a token tile are adjacent
    const int64_t my_tiles = n_tiles > blockIdx.x ? (n_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int64_t n_steps = my_tiles * n_ch;
    if (threadIdx.x == 0) {
        for (int s = 0; s < RT_STAGES; s++) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    // step j (tile j / n_ch, chunk j % n_ch) into stage j % RT_STAGES: one 2D tensor copy of the
    // token rows and one of the expert rows (rows past T or E are zero-filled, never stored)
    auto issue = [&](int64_t j) {
        const int64_t tile = blockIdx.x + (j / n_ch) * gridDim.x;
        const int c = (int)(j % n_ch);
        const int t0 = (int)((tile / tiles_e) * RT_TOK);
        const int e0 = (int)(tile % tiles_e) * RT_EXP;
        float *st = rt_smem + (j % RT_STAGES) * RT_STAGE_FLOATS;
        uint64_t *bar = &full[j % RT_STAGES];
        if (lane == 0) {
            mbar_arrive_expect_tx(bar, (uint32_t)RT_STAGE_FLOATS * 4);
            rt_tma_load_2d(st, &map_x, c * RT_KC, t0, bar);
            rt_tma_load_2d(st + RT_TOK * RT_KC, &map_w, c * RT_KC, e0, bar);
        }
        __syncwarp();
    };
    if (warp == 0)
        for (int64_t j = 0; j < RT_STAGES && j < n_steps; j++) issue(j);
    const int wt = warp & 1, we = warp >> 1;  // 2 token groups x 4 expert groups
    float acc[8][16];
    for (int64_t j = 0; j < n_steps; j++) {
        const int c = (int)(j % n_ch);
        if (c == 0) {
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int q = 0; q < 16; q++) acc[i][q] = 0.0f;
        }
        const int s = (int)(j % RT_STAGES);
        const bool ok = mbar_wait_bounded(&full[s], (uint32_t)(j / RT_STAGES) & 1u);
        // one block barrier per step: every thread leaves together on a timeout, and past it every
        // warp is done with step j - 1, whose stage is then refilled (RT_STAGES - 1 steps ahead)
        if (__syncthreads_or(!ok)) {
            if (threadIdx.x == 0) latch_error(err, TMOE_DEV_ERR_TIMEOUT);
            return;
        }
        if (warp == 0 && j >= 1 && j - 1 + RT_STAGES < n_steps) issue(j - 1 + RT_STAGES);
        const float4 *xs = reinterpret_cast<const float4 *>(rt_smem + s * RT_STAGE_FLOATS) + wt * 8 * (RT_KC / 4);
        const float4 *ws =
            reinterpret_cast<const float4 *>(rt_smem + s * RT_STAGE_FLOATS + RT_TOK * RT_KC) + we * 16 * (RT_KC / 4);
#pragma unroll
        for (int ms = 0; ms < RT_KC / 128; ms++) {
            float4 wv[16];
#pragma unroll
            for (int ee = 0; ee < 16; ee++) wv[ee] = ws[ee * (RT_KC / 4) + ms * 32 + lane];
#pragma unroll
            for (int tt = 0; tt < 8; tt++) {
                const float4 xv = xs[tt * (RT_KC / 4) + ms * 32 + lane];
                // element order per accumulator: .x, .y, .z, .w; consecutive FMAs are independent
#pragma unroll
                for (int ee = 0; ee < 16; ee++) acc[tt][ee] = __fmaf_rn(wv[ee].x, xv.x, acc[tt][ee]);
#pragma unroll
                for (int ee = 0; ee < 16; ee++) acc[tt][ee] = __fmaf_rn(wv[ee].y, xv.y, acc[tt][ee]);
#pragma unroll
                for (int ee = 0; ee < 16; ee++) acc[tt][ee] = __fmaf_rn(wv[ee].z, xv.z, acc[tt][ee]);
#pragma unroll
                for (int ee = 0; ee < 16; ee++) acc[tt][ee] = __fmaf_rn(wv[ee].w, xv.w, acc[tt][ee]);
            }
        }
        if (c == n_ch - 1) {  // the tile's logits
            const int64_t tile = blockIdx.x + (j / n_ch) * gridDim.x;
            const int64_t t0 = (tile / tiles_e) * RT_TOK;
            const int e0 = (int)(tile % tiles_e) * RT_EXP;
#pragma unroll
            for (int g = 0; g < 4; g++) {  // 32 logits each: 4 tokens (4 (g & 1) ..) x 8 experts (8 (g >> 1) ..)
                float v[32];
#pragma unroll
                for (int q = 0; q < 32; q++) v[q] = acc[4 * (g & 1) + q / 8][8 * (g >> 1) + q % 8];
                const float sum = transposed_butterfly(v, lane);
                const int64_t t = t0 + wt * 8 + 4 * (g & 1) + lane / 8;
                const int e = e0 + we * 16 + 8 * (g >> 1) + lane % 8;
                if (t < T && e < E) logits[t * E + e] = sum;
            }
        }
    }
}

// Router logits for any H: one warp per (expert, token), scalar loads in the canonical order.
__global__ void router_logits_generic_kernel(const float *__restrict__ xn, const float *__restrict__ rw, int64_t T,
                                             int H, int E, float *__restrict__ logits) {
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= T * E) return;
    const int64_t t = gw / E;
    const int e = (int)(gw % E);
    const float *wr = rw + (int64_t)e * H, *xr = xn + t * H;
    float acc = 0.0f;
    for (int m = 0; m * 128 < H; m++)
        for (int c = 0; c < 4; c++) {
            const int i = 128 * m + 4 * lane + c;
            if (i < H) acc = __fmaf_rn(wr[i], xr[i], acc);
        }
    const float s = butterfly_f32(acc);
    if (lane == 0) logits[t * E + e] = s;
}

// One warp per token: canonical softmax, top-k, renormalised weights.  E <= 32*MAXPER, k <= 32.
template <int MAXPER>
__global__ void softmax_topk_kernel(const float *__restrict__ logits, int64_t T, int E, int k,
                                    int32_t *__restrict__ ids, float *__restrict__ w, float *__restrict__ probs_out) {
    const int64_t t = (int64_t)(blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5));
    const int lane = threadIdx.x & 31;
    if (t >= T) return;
    int id;
    float wt;
    topk_token<MAXPER>(logits + t * E, E, k, probs_out ? probs_out + t * E : nullptr, id, wt);
    if (lane < k) {
        ids[t * k + lane] = id;
        w[t * k + lane] = wt;
    }
}

// Q8_K of rows of K f32: one warp per 256-block, stored in the Q8Rows layout of the consumer's
// weight type.  Rows whose `valid` entry is negative are skipped.
__global__ void quantize_q8k_kernel(const float *__restrict__ x, int64_t rows, int K, const int32_t *__restrict__ valid,
                                    Q8Rows out) {
    pdl_wait();
    pdl_trigger();
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int nb = K / TMOE_QK;
    const int64_t row = gw / nb;
    const int b = (int)(gw % nb);
    if (row >= rows) return;
    if (valid && valid[row] < 0) return;
    const float *xr = x + row * K + (int64_t)b * TMOE_QK + 8 * lane;
    const float4 a0 = *reinterpret_cast<const float4 *>(xr), a1 = *reinterpret_cast<const float4 *>(xr + 4);
    const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    uint2 q;
    float dd;
    int s16;
    q8k_block_warp(v, q, dd, s16);
    q8k_store_warp(out, row, K, b, q, dd, s16);
}

// bf16 -> f32: the bf16 bits are the top half of the f32's, so the widening is exact.
__global__ void widen_bf16_kernel(const uint4 *__restrict__ x, int64_t n8, float4 *__restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n8) return;
    const uint4 v = x[i];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    out[2 * i] = make_float4(__uint_as_float(w[0] << 16), __uint_as_float(w[0] & 0xffff0000u),
                             __uint_as_float(w[1] << 16), __uint_as_float(w[1] & 0xffff0000u));
    out[2 * i + 1] = make_float4(__uint_as_float(w[2] << 16), __uint_as_float(w[2] & 0xffff0000u),
                                 __uint_as_float(w[3] << 16), __uint_as_float(w[3] & 0xffff0000u));
}

// ------------------------------------------------------------------ launchers
cudaError_t launch_rms_norm(const float *x, const float *norm_w, float eps, int64_t T, int H, float *out,
                            cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (T <= 2048 && H >= 1024) {  // few long rows: a CTA per row
        launch_k(rms_norm_row_kernel, (unsigned)T, 256, 0, st, x, norm_w, eps, H, out);
        return cudaGetLastError();
    }
    const int warps = 8;
    launch_k(rms_norm_kernel, (unsigned)((T + warps - 1) / warps), warps * 32, 0, st, x, norm_w, eps, T, H, out);
    return cudaGetLastError();
}

static bool router_tiled(int64_t T, int H) { return T >= 1024 && T < (1ll << 31) && H % RT_KC == 0; }

// f32 [rows][H] with a box of RT_KC columns x box_rows rows, no swizzle (rows 512 bytes apart).
static bool encode_f32_rows(CUtensorMap *m, const float *base, int64_t rows, int H, int box_rows) {
    static PFN_cuTensorMapEncodeTiled_v12000 enc = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)H, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)H * 4};
    const cuuint32_t box[2] = {(cuuint32_t)RT_KC, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1u, 1u};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_router_logits(const float *xn, const float *rw, int64_t T, int H, int E, float *logits,
                                 const Q8Rows *q8, int *err, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    CUtensorMap map_x, map_w;
    if (!q8 && router_tiled(T, H) && E >= RT_EXP && ((uintptr_t)xn & 15) == 0 && ((uintptr_t)rw & 15) == 0 &&
        encode_f32_rows(&map_x, xn, T, H, RT_TOK) && encode_f32_rows(&map_w, rw, E, H, RT_EXP)) {
        static int set_tiled[64] = {};
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
        if (!set_tiled[dev]) {
            cudaError_t e = cudaFuncSetAttribute(router_logits_tiled_kernel,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)RT_SMEM);
            if (e != cudaSuccess) return e;
            set_tiled[dev] = 1;
        }
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const int64_t tiles = ((T + RT_TOK - 1) / RT_TOK) * ((E + RT_EXP - 1) / RT_EXP);
        const unsigned grid = (unsigned)std::min<int64_t>(tiles, sms > 0 ? sms : 148);
        router_logits_tiled_kernel<<<grid, 256, RT_SMEM, st>>>(xn, rw, T, H, E, logits, err, map_x, map_w);
        return cudaGetLastError();
    }
    constexpr int TT = 8;
    const size_t smem = (size_t)TT * H * 4;
    if (H % 512 == 0 && smem <= 200 * 1024) {
        static int set_bytes[64] = {};
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
        if (smem > 48 * 1024 && (int)smem > set_bytes[dev]) {
            cudaError_t e =
                cudaFuncSetAttribute(router_logits_kernel<TT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            set_bytes[dev] = (int)smem;
        }
        dim3 grid((E + RL_WARPS - 1) / RL_WARPS, (unsigned)((T + TT - 1) / TT));
        const Q8Rows none{nullptr, nullptr, nullptr, nullptr, 0};
        router_logits_kernel<TT><<<grid, RL_WARPS * 32, smem, st>>>(xn, rw, T, H, E, logits, q8 ? *q8 : none);
        return cudaGetLastError();
    }
    if (q8) return cudaErrorInvalidValue;  // the caller quantises separately for such H
    const int64_t warps = T * E;
    router_logits_generic_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(xn, rw, T, H, E, logits);
    return cudaGetLastError();
}

bool router_fuses_q8(int H, int64_t T) {
    return !router_tiled(T, H) && H % 512 == 0 && (size_t)8 * H * 4 <= 200 * 1024;
}

cudaError_t launch_softmax_topk(const float *logits, int64_t T, int E, int k, int32_t *ids, float *w, float *probs,
                                cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    const int warps = 8;
    const unsigned grid = (unsigned)((T + warps - 1) / warps);
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

cudaError_t launch_quantize_q8k(const float *x, int64_t rows, int K, const int32_t *valid, const Q8Rows &out,
                                cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    const int64_t warps = rows * (K / TMOE_QK);
    const int per_block = 8;
    const cudaError_t e = launch_k(quantize_q8k_kernel, (unsigned)((warps + per_block - 1) / per_block),
                                   per_block * 32, 0, st, x, rows, K, valid, out);
    return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_widen_bf16(const uint16_t *x, int64_t n, float *out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    if (n % 8 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
        return cudaErrorInvalidValue;
    const int64_t n8 = n / 8;
    widen_bf16_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, st>>>(reinterpret_cast<const uint4 *>(x), n8,
                                                                   reinterpret_cast<float4 *>(out));
    return cudaGetLastError();
}

}  // namespace tmoe
