// Expert parallelism with token dispatch/combine over an all-to-all (the mode beside the reference's
// all-reduce): each rank holds its own tokens and a contiguous share of the experts (the reference's
// partition rule, qwen3moe_shard.rs:617-626). A token is sent once to every rank that holds at least one of
// its k experts, with its k choices mapped to that rank's local expert ids (-1 for the others) and its k
// weights; the receiving rank runs the layer's expert products and its choice-ordered combine over the
// received rows -- exactly the partial sum of the reference's EP mode for that rank
// (qwen3moe_shard.rs:1043-1056) -- and sends the partial row back; the source rank adds the partials of its
// tokens in rank order. Messages have a fixed capacity (`cap` rows per peer, the handle's token capacity per
// rank), so their sizes are known to the host without a readback and the step stays stream-ordered; rows past
// a peer's count carry -1 ids and cost no expert work.
#include "common.cuh"
#include "kernels.cuh"

namespace tmoe {

// One CTA per destination rank d: the tokens with a choice on d, in token order, get rows
// 0, 1, ... of d's message.  row_of[t * g + d] = the row or -1; the message carries the token's
// local ids and weights, and tok[d][row] = t for the row gather.  Rows past the count get -1 ids.
// The message to this rank itself (d == self) is written straight into the receive buffers.
__global__ void __launch_bounds__(1024) ep_pack_kernel(const int32_t *__restrict__ ids, const float *__restrict__ w,
                                                       int T, int k, int per, int g, int cap, int self,
                                                       int32_t *__restrict__ row_of, int32_t *__restrict__ s_ids_,
                                                       float *__restrict__ s_w_, int32_t *__restrict__ r_ids,
                                                       float *__restrict__ r_w, int32_t *__restrict__ s_tok,
                                                       int32_t *__restrict__ counts) {
    __shared__ int warp_sum[32];
    __shared__ int base;
    const int d = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int32_t *s_ids = d == self ? r_ids : s_ids_;
    float *s_w = d == self ? r_w : s_w_;
    const int lo = d * per, hi = lo + per;
    if (tid == 0) base = 0;
    __syncthreads();
    for (int t0 = 0; t0 < T; t0 += blockDim.x) {
        const int t = t0 + tid;
        bool has = false;
        if (t < T)
            for (int j = 0; j < k; j++) {
                const int e = ids[(int64_t)t * k + j];
                has |= e >= lo && e < hi;
            }
        const unsigned b = __ballot_sync(0xffffffffu, has);
        if (lane == 0) warp_sum[warp] = __popc(b);
        __syncthreads();
        int before = 0, total = 0;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) {
            before += i < warp ? warp_sum[i] : 0;
            total += warp_sum[i];
        }
        const int row = base + before + __popc(b & ((1u << lane) - 1));
        if (t < T) {
            row_of[(int64_t)t * g + d] = has ? row : -1;
            if (has && row < cap) {
                for (int j = 0; j < k; j++) {
                    const int e = ids[(int64_t)t * k + j];
                    s_ids[((int64_t)d * cap + row) * k + j] = e >= lo && e < hi ? e - lo : -1;
                    s_w[((int64_t)d * cap + row) * k + j] = w[(int64_t)t * k + j];
                }
                s_tok[(int64_t)d * cap + row] = t;
            }
        }
        __syncthreads();
        if (tid == 0) base += total;
        __syncthreads();
    }
    const int n = min(base, cap);
    if (tid == 0) counts[d] = n;
    for (int i = n * k + tid; i < cap * k; i += blockDim.x) s_ids[(int64_t)d * cap * k + i] = -1;
}

// The rows of every message: s_x[d][row] = x[tok[d][row]] for row < counts[d] (one warp per row);
// this rank's own rows go straight into the receive buffer r_x.
__global__ void ep_gather_rows_kernel(const float *__restrict__ x, int H, int g, int cap, int self,
                                      const int32_t *__restrict__ s_tok, const int32_t *__restrict__ counts,
                                      float *__restrict__ s_x, float *__restrict__ r_x) {
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= (int64_t)g * cap) return;
    const int d = (int)(gw / cap), row = (int)(gw % cap);
    if (row >= counts[d]) return;
    const float4 *src = reinterpret_cast<const float4 *>(x + (int64_t)s_tok[gw] * H);
    float4 *dst = reinterpret_cast<float4 *>((d == self ? r_x : s_x) + gw * H);
    for (int i = lane; i < H / 4; i += 32) dst[i] = src[i];
}

// out[t] = the partial rows of token t from the ranks that computed some of its choices, added
// in rank order (one thread per 4 outputs; this rank's own partials are read where it computed
// them, `part`).  A token none of whose choices is held anywhere (all ids outside the experts)
// gets zeros.
__global__ void ep_combine_kernel(const float *__restrict__ ret, const float *__restrict__ part, int self,
                                  const int32_t *__restrict__ row_of, int T, int H, int g, int cap,
                                  float *__restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // float4 of out
    const int H4 = H / 4;
    if (i >= (int64_t)T * H4) return;
    const int64_t t = i / H4;
    const int c = (int)(i % H4);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    bool first = true;
    for (int d = 0; d < g; d++) {
        const int r = __ldg(row_of + t * g + d);
        if (r < 0 || r >= cap) continue;
        const float *src = (d == self ? part : ret) + ((int64_t)d * cap + r) * H;
        const float4 v = reinterpret_cast<const float4 *>(src)[c];
        if (first) {
            acc = v;
            first = false;
        } else {
            acc.x = __fadd_rn(acc.x, v.x), acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z), acc.w = __fadd_rn(acc.w, v.w);
        }
    }
    reinterpret_cast<float4 *>(out)[i] = acc;
}

// ------------------------------------------------------------------ the exchange over peer memory
// The same messages as the NCCL exchange, but written by the sending rank straight into the
// receiving rank's buffers through NVLink: block `self` of rank d's r_ids / r_w / r_x for the
// dispatch, block `self` of rank d's ret for the return.  The buffers of every rank are mapped
// into this process once (CUDA IPC).  After the last CTA of a writing kernel has seen every CTA's
// writes fenced at system scope, it bumps this rank's count of messages sent in that direction
// and stores the count (release, system scope) into each peer's counter for this rank; a
// receiver waits (bounded) for every peer's counter to pass its own count of messages consumed.
// Counts only grow, so a captured graph replays the same kernels without any reset.  A rank
// writes a peer's buffers only after that peer has consumed the previous message there: the
// dispatch of call n + 1 follows this rank's combine of call n, which waited for the peers'
// returns of call n, which each peer sends after its expert products of call n.
__device__ __forceinline__ void st_release_sys(int *p, int v) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_sys(const int *p) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Called by every thread of every CTA once its writes are issued: the last CTA signals the peers.
__device__ void ep_signal_last(int dir, int g, int self, const EpPeers &P, int *ctl) {
    __shared__ int last, count;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        last = atomicAdd(&ctl[2 + dir], 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    if (threadIdx.x == 0) {
        __threadfence_system();
        count = ctl[dir] + 1;
        ctl[dir] = count;
        ctl[2 + dir] = 0;  // the tally of the next call
    }
    __syncthreads();
    const int p = threadIdx.x;
    if (p < g && p != self) st_release_sys(P.flags[p] + dir * g + self, count);
}

// ep_pack_kernel with each destination's block in that rank's receive buffers.
__global__ void __launch_bounds__(1024) ep_pack_p2p_kernel(const int32_t *__restrict__ ids,
                                                           const float *__restrict__ w, int T, int k, int per,
                                                           int g, int cap, int self, const EpPeers P,
                                                           int32_t *__restrict__ row_of, int32_t *__restrict__ s_tok,
                                                           int32_t *__restrict__ counts) {
    pdl_wait();
    pdl_trigger();
    __shared__ int warp_sum[32];
    __shared__ int base;
    const int d = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int32_t *d_ids = P.r_ids[d] + (int64_t)self * cap * k;
    float *d_w = P.r_w[d] + (int64_t)self * cap * k;
    const int lo = d * per, hi = lo + per;
    if (tid == 0) base = 0;
    __syncthreads();
    for (int t0 = 0; t0 < T; t0 += blockDim.x) {
        const int t = t0 + tid;
        bool has = false;
        if (t < T)
            for (int j = 0; j < k; j++) {
                const int e = ids[(int64_t)t * k + j];
                has |= e >= lo && e < hi;
            }
        const unsigned b = __ballot_sync(0xffffffffu, has);
        if (lane == 0) warp_sum[warp] = __popc(b);
        __syncthreads();
        int before = 0, total = 0;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) {
            before += i < warp ? warp_sum[i] : 0;
            total += warp_sum[i];
        }
        const int row = base + before + __popc(b & ((1u << lane) - 1));
        if (t < T) {
            row_of[(int64_t)t * g + d] = has ? row : -1;
            if (has && row < cap) {
                for (int j = 0; j < k; j++) {
                    const int e = ids[(int64_t)t * k + j];
                    d_ids[(int64_t)row * k + j] = e >= lo && e < hi ? e - lo : -1;
                    d_w[(int64_t)row * k + j] = w[(int64_t)t * k + j];
                }
                s_tok[(int64_t)d * cap + row] = t;
            }
        }
        __syncthreads();
        if (tid == 0) base += total;
        __syncthreads();
    }
    const int n = min(base, cap);
    if (tid == 0) counts[d] = n;
    for (int i = n * k + tid; i < cap * k; i += blockDim.x) d_ids[i] = -1;
    __threadfence_system();
}

// The message rows into each destination's r_x, one warp per row; then the dispatch signal.
__global__ void ep_gather_p2p_kernel(const float *__restrict__ x, int H, int g, int cap, int self, const EpPeers P,
                                     const int32_t *__restrict__ s_tok, const int32_t *__restrict__ counts,
                                     int *ctl) {
    pdl_wait();
    pdl_trigger();
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw < (int64_t)g * cap) {
        const int d = (int)(gw / cap), row = (int)(gw % cap);
        if (row < counts[d]) {
            const float4 *src = reinterpret_cast<const float4 *>(x + (int64_t)s_tok[gw] * H);
            float4 *dst = reinterpret_cast<float4 *>(P.r_x[d] + ((int64_t)self * cap + row) * H);
            for (int i = lane; i < H / 4; i += 32) dst[i] = src[i];
        }
    }
    ep_signal_last(0, g, self, P, ctl);
}

// The partial rows back to their tokens' ranks: row r of block d (received from rank d) goes to
// row r of block `self` of rank d's ret, when the row has an expert here (one warp per row).
__global__ void ep_return_p2p_kernel(const float *__restrict__ part, const int32_t *__restrict__ r_ids, int k, int H,
                                     int g, int cap, int self, const EpPeers P, int *ctl) {
    pdl_wait();
    pdl_trigger();
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw < (int64_t)g * cap) {
        const int d = (int)(gw / cap), row = (int)(gw % cap);
        const bool has = __any_sync(0xffffffffu, lane < k && __ldg(r_ids + gw * k + lane) >= 0);
        if (d != self && has) {
            const float4 *src = reinterpret_cast<const float4 *>(part + gw * H);
            float4 *dst = reinterpret_cast<float4 *>(P.ret[d] + ((int64_t)self * cap + row) * H);
            for (int i = lane; i < H / 4; i += 32) dst[i] = src[i];
        }
    }
    ep_signal_last(1, g, self, P, ctl);
}

__global__ void ep_wait_kernel(int dir, int g, int self, const int *flags, int *ctl, int *err) {
    pdl_wait();
    pdl_trigger();
    const int p = threadIdx.x;
    if (p >= g || p == self) return;
    int *seen = ctl + 4 + dir * g + p;
    const int want = *seen + 1;
    const uint64_t t0 = globaltimer_ns();
    uint32_t nap = 32;
    while (ld_acquire_sys(flags + dir * g + p) - want < 0) {
        if (globaltimer_ns() - t0 > TMOE_WAIT_LIMIT_NS) {
            latch_error(err, TMOE_DEV_ERR_TIMEOUT);
            break;
        }
        __nanosleep(nap);
        if (nap < 1024) nap *= 2;
    }
    *seen = want;
    __threadfence_system();
}

cudaError_t launch_ep_dispatch_p2p(const int32_t *ids, const float *w, const float *x, int T, int k, int H, int per,
                                   int g, int cap, int self, const EpPeers &P, int32_t *row_of, int32_t *s_tok,
                                   int32_t *counts, int *ctl, cudaStream_t st) {
    if (g <= 0 || g > EP_MAX_PEERS || cap <= 0 || self < 0 || self >= g || k > 32 || H % 4) return cudaErrorInvalidValue;
    cudaError_t e = launch_k(ep_pack_p2p_kernel, g, 1024, 0, st, ids, w, T, k, per, g, cap, self, P, row_of, s_tok,
                             counts);
    if (e != cudaSuccess) return e;
    const int64_t warps = (int64_t)g * cap;
    e = launch_k(ep_gather_p2p_kernel, (unsigned)((warps + 7) / 8), 256, 0, st, x, H, g, cap, self, P, s_tok, counts,
                 ctl);
    return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_ep_return_p2p(const float *part, const int32_t *r_ids, int k, int H, int g, int cap, int self,
                                 const EpPeers &P, int *ctl, cudaStream_t st) {
    if (g <= 0 || g > EP_MAX_PEERS || cap <= 0 || self < 0 || self >= g || k > 32 || H % 4) return cudaErrorInvalidValue;
    const int64_t warps = (int64_t)g * cap;
    const cudaError_t e = launch_k(ep_return_p2p_kernel, (unsigned)((warps + 7) / 8), 256, 0, st, part, r_ids, k, H,
                                   g, cap, self, P, ctl);
    return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_ep_wait(int dir, int g, int self, const int *flags, int *ctl, int *err, cudaStream_t st) {
    if (g <= 0 || g > 32 || self < 0 || self >= g) return cudaErrorInvalidValue;
    const cudaError_t e = launch_k(ep_wait_kernel, 1, 32, 0, st, dir, g, self, flags, ctl, err);
    return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_ep_pack(const int32_t *ids, const float *w, const float *x, int T, int k, int H, int per, int g,
                           int cap, int self, int32_t *row_of, int32_t *s_ids, float *s_w, int32_t *r_ids,
                           float *r_w, int32_t *s_tok, int32_t *counts, float *s_x, float *r_x, cudaStream_t st) {
    if (g <= 0 || cap <= 0 || self < 0 || self >= g) return cudaErrorInvalidValue;
    ep_pack_kernel<<<g, 1024, 0, st>>>(ids, w, T, k, per, g, cap, self, row_of, s_ids, s_w, r_ids, r_w, s_tok, counts);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int64_t warps = (int64_t)g * cap;
    ep_gather_rows_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(x, H, g, cap, self, s_tok, counts, s_x, r_x);
    return cudaGetLastError();
}

cudaError_t launch_ep_combine(const float *ret, const float *part, int self, const int32_t *row_of, int T, int H,
                              int g, int cap, float *out, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    if (H % 4 || self < 0 || self >= g) return cudaErrorInvalidValue;
    const int64_t n4 = (int64_t)T * H / 4;
    const cudaError_t e = launch_k(ep_combine_kernel, (unsigned)((n4 + 255) / 256), 256, 0, st, ret, part, self, row_of,
                                   T, H, g, cap, out);
    return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace tmoe
