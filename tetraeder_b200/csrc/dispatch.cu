// Token-to-expert dispatch: per-expert counts, offsets and the stable permutation of pairs
// (token-major, choice-minor within each expert: qwen3moe.rs:2126-2150 group_pairs, the order
// ggml's mul_mat_id row mapping visits), the EP id map, and the weighted combine in choice order
// (qwen3moe.rs:2912-2923).
#include "common.cuh"
#include "kernels.cuh"

namespace tmoe {

constexpr int SORT_WARPS = 32;

// One CTA of 1024 threads.  Warp w owns the contiguous pair segment [w*seg, (w+1)*seg):
//   1. per-warp histograms in shared memory;
//   2. per expert, an exclusive scan over the warps plus the expert offset gives each warp its
//      first slot for that expert;
//   3. each warp walks its segment in order, 32 pairs at a time; __match_any_sync ranks the lanes
//      of equal expert, so the scatter is stable.
// ids outside [0, n_slots) are not dispatched; ids >= n_slots also latch TMOE_DEV_ERR_BADID.
// Also writes the increasing list of experts with pairs (`active`, `n_active[0]`).
__global__ void __launch_bounds__(1024) sort_pairs_kernel(
    const int32_t *__restrict__ ids, int n_pairs, int n_slots, int32_t *__restrict__ counts,
    int32_t *__restrict__ offsets, int32_t *__restrict__ perm, int32_t *__restrict__ active,
    int32_t *__restrict__ n_active, int *err) {
    extern __shared__ int32_t sh[];
    int32_t *hist = sh;                          // [SORT_WARPS][n_slots]
    int32_t *offs = sh + SORT_WARPS * n_slots;   // [n_slots + 1]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < SORT_WARPS * n_slots; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    int seg = (n_pairs + SORT_WARPS - 1) / SORT_WARPS;
    seg = (seg + 31) & ~31;
    const int p0 = warp * seg, p1 = min(n_pairs, p0 + seg);
    bool bad = false;
    for (int p = p0 + lane; p < p1; p += 32) {
        int e = ids[p];
        if (e >= n_slots) bad = true;
        if (e >= 0 && e < n_slots) atomicAdd(&hist[warp * n_slots + e], 1);
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) latch_error(err, TMOE_DEV_ERR_BADID);
    __syncthreads();
    for (int e = threadIdx.x; e < n_slots; e += blockDim.x) {
        int run = 0;
        for (int w = 0; w < SORT_WARPS; w++) {
            int c = hist[w * n_slots + e];
            hist[w * n_slots + e] = run;
            run += c;
        }
        counts[e] = run;
        offs[e] = run;
    }
    __syncthreads();
    if (warp == 0) {  // exclusive scan of the counts, 32 experts per step
        int carry = 0;
        for (int base = 0; base < n_slots; base += 32) {
            int e = base + lane;
            int c = e < n_slots ? offs[e] : 0;
            int inc = c;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                int o = __shfl_up_sync(0xffffffffu, inc, off);
                if (lane >= off) inc += o;
            }
            if (e < n_slots) offs[e] = carry + inc - c;
            carry += __shfl_sync(0xffffffffu, inc, 31);
        }
        if (lane == 0) offs[n_slots] = carry;
    }
    __syncthreads();
    for (int e = threadIdx.x; e <= n_slots; e += blockDim.x) offsets[e] = offs[e];
    if (warp == 0) {
        int na = 0;
        for (int base = 0; base < n_slots; base += 32) {
            int e = base + lane;
            bool has = e < n_slots && (offs[e + 1] - offs[e]) > 0;
            unsigned m = __ballot_sync(0xffffffffu, has);
            if (has) active[na + __popc(m & ((1u << lane) - 1u))] = e;
            na += __popc(m);
        }
        if (lane == 0) n_active[0] = na;
    }
    for (int e = threadIdx.x; e < n_slots; e += blockDim.x)
        for (int w = 0; w < SORT_WARPS; w++) hist[w * n_slots + e] += offs[e];
    __syncthreads();
    const unsigned lt = (1u << lane) - 1u;
    for (int base = p0; base < p1; base += 32) {
        int p = base + lane;
        int e = p < p1 ? ids[p] : -1;
        bool ok = e >= 0 && e < n_slots;
        int key = ok ? e : -1;
        unsigned peers = __match_any_sync(0xffffffffu, key);
        if (ok) {
            int rank = __popc(peers & lt);
            perm[hist[warp * n_slots + e] + rank] = p;
        }
        __syncwarp();
        if (ok && (peers & lt) == 0) hist[warp * n_slots + e] += __popc(peers);
        __syncwarp();
    }
}

__global__ void map_ids_kernel(const int32_t *__restrict__ ids, int64_t n,
                               const int32_t *__restrict__ table, int64_t n_table,
                               int32_t *__restrict__ out) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    int e = ids[i];
    out[i] = (e >= 0 && e < n_table) ? table[e] : -1;
}

// Zero the output rows of pairs with no expert (id < 0 or >= n_slots).
__global__ void zero_invalid_rows_kernel(const int32_t *__restrict__ ids, int64_t n_pairs,
                                         int n_slots, int N, float *__restrict__ out) {
    int64_t p = blockIdx.x;
    if (p >= n_pairs) return;
    int e = ids[p];
    if (e >= 0 && e < n_slots) return;
    float *o = out + p * N;
    for (int i = threadIdx.x; i < N; i += blockDim.x) o[i] = 0.0f;
}

// out[t][h] = ((m_0 + m_1) + m_2) + ...  with m_j = d[t*k+j][h] * w[t][j], d = 0 for no expert
// (ctx.mul(experts, w) then the fold of sum_experts).
__global__ void combine_kernel(const float *__restrict__ dout, const int32_t *__restrict__ ids,
                               const float *__restrict__ w, int64_t T, int k, int H, int n_slots,
                               float *__restrict__ out) {
    int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i >= T * H) return;
    int64_t t = i / H;
    int h = (int)(i % H);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < k; j++) {
        int e = ids[t * k + j];
        float wj = w[t * k + j];
        float4 d = make_float4(0.f, 0.f, 0.f, 0.f);
        if (e >= 0 && e < n_slots) d = *reinterpret_cast<const float4 *>(dout + (t * k + j) * H + h);
        float4 m = make_float4(__fmul_rn(d.x, wj), __fmul_rn(d.y, wj), __fmul_rn(d.z, wj),
                               __fmul_rn(d.w, wj));
        if (j == 0)
            acc = m;
        else
            acc = make_float4(__fadd_rn(acc.x, m.x), __fadd_rn(acc.y, m.y), __fadd_rn(acc.z, m.z),
                              __fadd_rn(acc.w, m.w));
    }
    *reinterpret_cast<float4 *>(out + i) = acc;
}

// ------------------------------------------------------------------ launchers
size_t sort_pairs_smem(int n_slots) { return sizeof(int32_t) * ((size_t)SORT_WARPS * n_slots + n_slots + 1); }

cudaError_t launch_sort_pairs(const int32_t *ids, int n_pairs, int n_slots, int32_t *counts,
                              int32_t *offsets, int32_t *perm, int32_t *active, int32_t *n_active,
                              int *err, cudaStream_t st) {
    size_t smem = sort_pairs_smem(n_slots);
    static int set_bytes[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (smem > 48 * 1024 && (int)smem > set_bytes[dev]) {
        cudaError_t e = cudaFuncSetAttribute(sort_pairs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
        set_bytes[dev] = (int)smem;
    }
    sort_pairs_kernel<<<1, 1024, smem, st>>>(ids, n_pairs, n_slots, counts, offsets, perm, active,
                                             n_active, err);
    return cudaGetLastError();
}

cudaError_t launch_map_ids(const int32_t *ids, int64_t n, const int32_t *table, int64_t n_table,
                           int32_t *out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    map_ids_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(ids, n, table, n_table, out);
    return cudaGetLastError();
}

cudaError_t launch_zero_invalid_rows(const int32_t *ids, int64_t n_pairs, int n_slots, int N,
                                     float *out, cudaStream_t st) {
    if (n_pairs <= 0) return cudaSuccess;
    zero_invalid_rows_kernel<<<(unsigned)n_pairs, 128, 0, st>>>(ids, n_pairs, n_slots, N, out);
    return cudaGetLastError();
}

cudaError_t launch_combine(const float *dout, const int32_t *ids, const float *w, int64_t T, int k,
                           int H, int n_slots, float *out, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    int64_t n4 = T * H / 4;
    combine_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(dout, ids, w, T, k, H, n_slots, out);
    return cudaGetLastError();
}

}  // namespace tmoe
