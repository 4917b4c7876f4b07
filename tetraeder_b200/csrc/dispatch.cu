// Token-to-expert dispatch: per-expert counts, offsets and the stable permutation of pairs
// (token-major, choice-minor within each expert: qwen3moe.rs:2126-2150 group_pairs, the order
// ggml's mul_mat_id row mapping visits), the EP id map (qwen3moe_shard.rs:1043-1050), the fused
// top-k + map + dispatch kernel of the decode regime, and the weighted combine in choice order
// (qwen3moe.rs:2912-2923).
#include "common.cuh"
#include "kernels.cuh"
#include "route.cuh"

namespace tmoe {

constexpr int SORT_WARPS = 32;

// The dispatch of n_pairs ids (ids may live in shared memory) by one CTA of 1024 threads.  Warp w
// owns the contiguous pair segment [w*seg, (w+1)*seg):
//   1. per-warp histograms in shared memory;
//   2. per expert, an exclusive scan over the warps plus the expert offset gives each warp its
//      first slot for that expert;
//   3. each warp walks its segment in order, 32 pairs at a time; __match_any_sync ranks the lanes
//      of equal expert, so the scatter is stable.
// ids outside [0, n_slots) are not dispatched; ids >= n_slots also latch TMOE_DEV_ERR_BADID.
// Also writes the increasing list of experts with pairs (n_active[0] of them) with their pair
// ranges: active[i] = {e, offsets[e], offsets[e + 1], 0}.
// sh: SORT_WARPS * n_slots + n_slots + 1 ints of shared memory.
__device__ void sort_pairs_cta(const int32_t *ids, int n_pairs, int n_slots, int32_t *__restrict__ counts,
                               int32_t *__restrict__ offsets, int32_t *__restrict__ perm,
                               int4 *__restrict__ active, int32_t *__restrict__ n_active, int *counters,
                               int n_counters, int *err, int32_t *sh) {
    int32_t *hist = sh;                         // [SORT_WARPS][n_slots]
    int32_t *offs = sh + SORT_WARPS * n_slots;  // [n_slots + 1]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (counters && (int)threadIdx.x < n_counters) counters[threadIdx.x] = 0;  // work counters of the GEMVs
    for (int i = threadIdx.x; i < SORT_WARPS * n_slots; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    int seg = (n_pairs + SORT_WARPS - 1) / SORT_WARPS;
    seg = (seg + 31) & ~31;
    const int p0 = warp * seg, p1 = min(n_pairs, p0 + seg);
    bool bad = false;
    for (int p = p0 + lane; p < p1; p += 32) {
        const int e = ids[p];
        if (e >= n_slots) bad = true;
        if (e >= 0 && e < n_slots) atomicAdd(&hist[warp * n_slots + e], 1);
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) latch_error(err, TMOE_DEV_ERR_BADID);
    __syncthreads();
    for (int e = threadIdx.x; e < n_slots; e += blockDim.x) {
        int run = 0;
        for (int w = 0; w < SORT_WARPS; w++) {
            const int c = hist[w * n_slots + e];
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
            const int e = base + lane;
            const int c = e < n_slots ? offs[e] : 0;
            int inc = c;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int o = __shfl_up_sync(0xffffffffu, inc, off);
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
            const int e = base + lane;
            const bool has = e < n_slots && (offs[e + 1] - offs[e]) > 0;
            const unsigned m = __ballot_sync(0xffffffffu, has);
            if (has) active[na + __popc(m & ((1u << lane) - 1u))] = make_int4(e, offs[e], offs[e + 1], 0);
            na += __popc(m);
        }
        if (lane == 0) n_active[0] = na;
    }
    for (int e = threadIdx.x; e < n_slots; e += blockDim.x)
        for (int w = 0; w < SORT_WARPS; w++) hist[w * n_slots + e] += offs[e];
    __syncthreads();
    const unsigned lt = (1u << lane) - 1u;
    for (int base = p0; base < p1; base += 32) {
        const int p = base + lane;
        const int e = p < p1 ? ids[p] : -1;
        const bool ok = e >= 0 && e < n_slots;
        const unsigned peers = __match_any_sync(0xffffffffu, ok ? e : -1);
        if (ok) perm[hist[warp * n_slots + e] + __popc(peers & lt)] = p;
        __syncwarp();
        if (ok && (peers & lt) == 0) hist[warp * n_slots + e] += __popc(peers);
        __syncwarp();
    }
}

__global__ void __launch_bounds__(1024) sort_pairs_kernel(const int32_t *__restrict__ ids, int n_pairs, int n_slots,
                                                          int32_t *__restrict__ counts, int32_t *__restrict__ offsets,
                                                          int32_t *__restrict__ perm, int4 *__restrict__ active,
                                                          int32_t *__restrict__ n_active, int *counters, int n_counters,
                                                          int *err) {
    extern __shared__ int32_t sh[];
    sort_pairs_cta(ids, n_pairs, n_slots, counts, offsets, perm, active, n_active, counters, n_counters, err, sh);
}

// Decode regime (T*k <= ROUTE_FUSED_MAX_PAIRS): softmax/top-k of every token, the optional EP
// map, and the dispatch of the (mapped) ids, in one CTA of 1024 threads.  ids_out / w_out get the
// router's choices; mapped gets the ids the experts see (= ids_out without a table).
template <int MAXPER>
__global__ void __launch_bounds__(1024) route_dispatch_kernel(const float *__restrict__ logits, int T, int E, int k,
                                                              const int32_t *__restrict__ table, int n_table,
                                                              int32_t *__restrict__ ids_out, float *__restrict__ w_out,
                                                              int32_t *__restrict__ mapped, int n_slots,
                                                              int32_t *__restrict__ counts, int32_t *__restrict__ offsets,
                                                              int32_t *__restrict__ perm, int4 *__restrict__ active,
                                                              int32_t *__restrict__ n_active, int *counters,
                                                              int n_counters, int *err) {
    extern __shared__ int32_t sh[];
    int32_t *sid = sh;  // [T*k] mapped ids
    int32_t *sort_sh = sh + ((T * k + 3) & ~3);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int t = warp; t < T; t += 32) {
        int id;
        float wt;
        topk_token<MAXPER>(logits + (int64_t)t * E, E, k, nullptr, id, wt);
        if (lane < k) {
            const int m = table ? ((id >= 0 && id < n_table) ? table[id] : -1) : id;
            ids_out[t * k + lane] = id;
            w_out[t * k + lane] = wt;
            mapped[t * k + lane] = m;
            sid[t * k + lane] = m;
        }
    }
    __syncthreads();
    sort_pairs_cta(sid, T * k, n_slots, counts, offsets, perm, active, n_active, counters, n_counters, err, sort_sh);
}

__global__ void map_ids_kernel(const int32_t *__restrict__ ids, int64_t n, const int32_t *__restrict__ table,
                               int64_t n_table, int32_t *__restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int e = ids[i];
    out[i] = (e >= 0 && e < n_table) ? table[e] : -1;
}

// Zero the output rows of pairs with no expert (id < 0 or >= n_slots).
__global__ void zero_invalid_rows_kernel(const int32_t *__restrict__ ids, int64_t n_pairs, int n_slots, int N,
                                         float *__restrict__ out) {
    const int64_t p = blockIdx.x;
    if (p >= n_pairs) return;
    const int e = ids[p];
    if (e >= 0 && e < n_slots) return;
    float *o = out + p * N;
    for (int i = threadIdx.x; i < N; i += blockDim.x) o[i] = 0.0f;
}

// out[t][h] = ((m_0 + m_1) + m_2) + ...  with m_j = d[t*k+j][h] * w[t][j], d = 0 for no expert
// (ctx.mul(experts, w) then the fold of sum_experts).  One thread per 4 outputs; all of the token's
// ids, weights and rows are loaded before the fold.
template <int KMAX>
__global__ void combine_kernel(const float *__restrict__ dout, const int32_t *__restrict__ ids,
                               const float *__restrict__ w, int64_t T, int k, int H, int n_slots,
                               float *__restrict__ out) {
    const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i >= T * H) return;
    const int64_t t = i / H;
    const int h = (int)(i % H);
    int e[KMAX];
    float wj[KMAX];
    float4 d[KMAX];
#pragma unroll
    for (int j = 0; j < KMAX; j++) {
        if (j < k) {
            e[j] = __ldg(ids + t * k + j);
            wj[j] = __ldg(w + t * k + j);
        }
    }
#pragma unroll
    for (int j = 0; j < KMAX; j++) {
        d[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j < k && e[j] >= 0 && e[j] < n_slots) d[j] = __ldg(reinterpret_cast<const float4 *>(dout + (t * k + j) * H + h));
    }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < KMAX; j++) {
        if (j >= k) break;
        const float4 m = make_float4(__fmul_rn(d[j].x, wj[j]), __fmul_rn(d[j].y, wj[j]), __fmul_rn(d[j].z, wj[j]),
                                     __fmul_rn(d[j].w, wj[j]));
        acc = j == 0 ? m
                     : make_float4(__fadd_rn(acc.x, m.x), __fadd_rn(acc.y, m.y), __fadd_rn(acc.z, m.z),
                                   __fadd_rn(acc.w, m.w));
    }
    *reinterpret_cast<float4 *>(out + i) = acc;
}

// ------------------------------------------------------------------ launchers
size_t sort_pairs_smem(int n_slots) { return sizeof(int32_t) * ((size_t)SORT_WARPS * n_slots + n_slots + 1); }

template <typename KernT>
static cudaError_t set_smem_once(KernT kern, size_t smem, int *cache) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (smem > 48 * 1024 && (int)smem > cache[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        cache[dev] = (int)smem;
    }
    return cudaSuccess;
}

cudaError_t launch_sort_pairs(const int32_t *ids, int n_pairs, int n_slots, int32_t *counts, int32_t *offsets,
                              int32_t *perm, int4 *active, int32_t *n_active, int *counters, int n_counters,
                              int *err, cudaStream_t st) {
    const size_t smem = sort_pairs_smem(n_slots);
    static int cache[64] = {};
    cudaError_t e = set_smem_once(sort_pairs_kernel, smem, cache);
    if (e != cudaSuccess) return e;
    sort_pairs_kernel<<<1, 1024, smem, st>>>(ids, n_pairs, n_slots, counts, offsets, perm, active, n_active, counters,
                                             n_counters, err);
    return cudaGetLastError();
}

bool route_dispatch_fits(int64_t T, int k, int E, int n_slots) {
    return T * k <= ROUTE_FUSED_MAX_PAIRS && E <= 256 && n_slots <= 256;
}

cudaError_t launch_route_dispatch(const float *logits, int T, int E, int k, const int32_t *table, int n_table,
                                  int32_t *ids_out, float *w_out, int32_t *mapped, int n_slots, int32_t *counts,
                                  int32_t *offsets, int32_t *perm, int4 *active, int32_t *n_active,
                                  int *counters, int n_counters, int *err, cudaStream_t st) {
    const size_t smem = sizeof(int32_t) * ((size_t)((T * k + 3) & ~3)) + sort_pairs_smem(n_slots);
    static int cache[4][64] = {};
#define TMOE_RD(MP, CI)                                                                                        \
    do {                                                                                                       \
        cudaError_t e = set_smem_once(route_dispatch_kernel<MP>, smem, cache[CI]);                             \
        if (e != cudaSuccess) return e;                                                                        \
        route_dispatch_kernel<MP><<<1, 1024, smem, st>>>(logits, T, E, k, table, n_table, ids_out, w_out,      \
                                                         mapped, n_slots, counts, offsets, perm, active,      \
                                                         n_active, counters, n_counters, err);                 \
    } while (0)
    if (E <= 32)
        TMOE_RD(1, 0);
    else if (E <= 64)
        TMOE_RD(2, 1);
    else if (E <= 128)
        TMOE_RD(4, 2);
    else if (E <= 256)
        TMOE_RD(8, 3);
    else
        return cudaErrorInvalidValue;
#undef TMOE_RD
    return cudaGetLastError();
}

cudaError_t launch_map_ids(const int32_t *ids, int64_t n, const int32_t *table, int64_t n_table, int32_t *out,
                           cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    map_ids_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(ids, n, table, n_table, out);
    return cudaGetLastError();
}

cudaError_t launch_zero_invalid_rows(const int32_t *ids, int64_t n_pairs, int n_slots, int N, float *out,
                                     cudaStream_t st) {
    if (n_pairs <= 0) return cudaSuccess;
    zero_invalid_rows_kernel<<<(unsigned)n_pairs, 128, 0, st>>>(ids, n_pairs, n_slots, N, out);
    return cudaGetLastError();
}

cudaError_t launch_combine(const float *dout, const int32_t *ids, const float *w, int64_t T, int k, int H,
                           int n_slots, float *out, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    const int64_t n4 = T * H / 4;
    const unsigned grid = (unsigned)((n4 + 127) / 128);
    if (k <= 8)
        combine_kernel<8><<<grid, 128, 0, st>>>(dout, ids, w, T, k, H, n_slots, out);
    else if (k <= 16)
        combine_kernel<16><<<grid, 128, 0, st>>>(dout, ids, w, T, k, H, n_slots, out);
    else
        combine_kernel<32><<<grid, 128, 0, st>>>(dout, ids, w, T, k, H, n_slots, out);
    return cudaGetLastError();
}

}  // namespace tmoe
