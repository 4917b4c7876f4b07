// Expert parallelism with token dispatch/combine over an all-to-all (the survey's mode B): each
// rank holds its own tokens and a contiguous share of the experts (the reference's partition rule,
// qwen3moe_shard.rs:617-626).  A token is sent once to every rank that holds at least one of its k
// experts, with its k choices mapped to that rank's local expert ids (-1 for the others) and its
// k weights; the receiving rank runs the layer's expert products and its choice-ordered combine
// over the received rows -- exactly the partial sum of the reference's EP mode for that rank
// (qwen3moe_shard.rs:1043-1056) -- and sends the partial row back; the source rank adds the
// partials of its tokens in rank order.
//
// Messages have a fixed capacity (`cap` rows per peer, the handle's token capacity per rank), so
// their sizes are known to the host without a readback and the step stays stream-ordered; rows
// past a peer's count carry -1 ids and cost no expert work.
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
    ep_combine_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(ret, part, self, row_of, T, H, g, cap, out);
    return cudaGetLastError();
}

}  // namespace tmoe
