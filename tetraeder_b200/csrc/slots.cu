// The expert-slot cache of one MoE layer on the device: the reference's host-side LayerSlots
// (crates/memory/src/slots.rs:131-177), Streamer::plan (crates/model/src/experts.rs:624-662) and
// make_resident (experts.rs:1507-1543), run by one CTA on the router's ids, so that a streamed layer
// step needs no device->host readback of the ids (qwen3moe.rs:1829) and no host planning: the
// step stays stream-ordered and can be captured in a CUDA graph.  Misses are paged in by a copy
// kernel that reads the pinned host expert store through its mapped device address.
//
// Per step the planner writes, for chunk c < n_chunks: map[c][e] = the slot of expert e if e is in
// chunk c, else -1; loads[c][0..n_loads[c]) = (expert, slot) of the chunk's misses.  Chunks past
// n_chunks keep all -1 maps and no loads, so the host can issue a fixed number of chunk passes.
#include "common.cuh"
#include "kernels.cuh"

namespace tmoe {

constexpr int SP_THREADS = 1024;
constexpr int SP_MAX_E = 1024;
constexpr int SP_MAX_SLOTS = 1024;

// LRU candidate order: the smaller stamp, then the lower slot (the reference's min_by_key keeps the
// first of equal keys).
__device__ __forceinline__ void lru_better(unsigned long long &bs, int &bi, unsigned long long s, int i) {
    if (i >= 0 && (bi < 0 || s < bs || (s == bs && i < bi))) bs = s, bi = i;
}

__global__ void __launch_bounds__(SP_THREADS) slot_plan_kernel(const int32_t *__restrict__ ids, int n_pairs,
                                                               SlotsDev s, int *err) {
    __shared__ int first[SP_MAX_E], cnt[SP_MAX_E], order[SP_MAX_E], seq[SP_MAX_E];
    __shared__ int slot_of[SP_MAX_E];
    __shared__ unsigned char pinned[SP_MAX_E];
    __shared__ int owner[SP_MAX_SLOTS];
    __shared__ unsigned long long stamp[SP_MAX_SLOTS];
    __shared__ int n_distinct, bad;
    const int E = s.n_expert, tid = threadIdx.x, lane = tid & 31;
    const int active = min(s.active[0], s.max_slots);
    for (int e = tid; e < E; e += blockDim.x) {
        first[e] = INT32_MAX, cnt[e] = 0;
        slot_of[e] = s.slot_of[e], pinned[e] = s.pinned[e];
    }
    for (int i = tid; i < s.max_slots; i += blockDim.x) owner[i] = s.owner[i], stamp[i] = s.stamp[i];
    for (int i = tid; i < s.max_chunks * E; i += blockDim.x) s.map[i] = -1;
    for (int i = tid; i < s.max_chunks; i += blockDim.x) s.n_loads[i] = 0;
    if (tid == 0) n_distinct = 0, bad = 0;
    __syncthreads();
    // first appearance and pair counts; lanes routed to the same expert are merged first
    for (int base = 0; base < n_pairs; base += blockDim.x) {
        const int p = base + tid;
        int e = p < n_pairs ? ids[p] : -1;
        if (p < n_pairs && (e < 0 || e >= E)) {
            bad = 1;
            e = -1;
        }
        const unsigned m = __match_any_sync(0xffffffffu, e);
        if (e >= 0 && lane == __ffs(m) - 1) {
            atomicMin(&first[e], p);  // the lowest lane holds the group's first pair
            atomicAdd(&cnt[e], __popc(m));
        }
    }
    __syncthreads();
    if (bad) {  // the reference: "router chose expert {e}, out of range"
        if (tid == 0) {
            latch_error(err, TMOE_DEV_ERR_BADID);
            s.n_chunks[0] = 0;
        }
        return;
    }
    for (int e = tid; e < E; e += blockDim.x) {
        if (cnt[e]) {
            s.counts[e] += (unsigned long long)cnt[e];
            int r = 0;
            for (int f = 0; f < E; f++) r += first[f] < first[e];
            order[r] = e;
            atomicAdd(&n_distinct, 1);
        }
    }
    __syncthreads();
    if (tid >= 32) return;
    // warp 0: residents first, then misses, each in order of first appearance
    const int nd = n_distinct;
    int w = 0;
    for (int pass = 0; pass < 2; pass++)
        for (int i0 = 0; i0 < nd; i0 += 32) {
            const int i = i0 + lane;
            const bool take = i < nd && ((slot_of[order[i]] >= 0) == (pass == 0));
            const unsigned b = __ballot_sync(0xffffffffu, take);
            if (take) seq[w + __popc(b & ((1u << lane) - 1))] = order[i];
            w += __popc(b);
        }
    __syncwarp();
    const int n = max(active, 1);
    const int n_chunks = (nd + n - 1) / n;
    if (n_chunks > s.max_chunks) {
        if (lane == 0) latch_error(err, TMOE_DEV_ERR_NOSLOT), s.n_chunks[0] = 0;
        return;
    }
    unsigned long long clock = s.meta[0], hits = 0, misses = 0;
    int failed = 0;
    for (int q = 0; q < nd && !failed; q++) {  // make_resident of each chunk, in order
        const int c = q / n, e = seq[q];
        clock++;
        int sl = slot_of[e];
        if (sl >= 0) {
            if (lane == 0) stamp[sl] = clock;
            hits++;
        } else {
            int fr = -1;  // the first free slot below `active`
            for (int i0 = 0; i0 < active && fr < 0; i0 += 32) {
                const unsigned b = __ballot_sync(0xffffffffu, i0 + lane < active && owner[i0 + lane] < 0);
                if (b) fr = i0 + __ffs(b) - 1;
            }
            sl = fr;
            if (sl < 0) {  // the least recently used unpinned slot
                unsigned long long bs = 0;
                int bi = -1;
                for (int i = lane; i < active; i += 32) {
                    const int o = owner[i];
                    if (o >= 0 && !pinned[o]) lru_better(bs, bi, stamp[i], i);
                }
#pragma unroll
                for (int off = 16; off >= 1; off >>= 1) {
                    const unsigned long long os = __shfl_xor_sync(0xffffffffu, bs, off);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
                    lru_better(bs, bi, os, oi);
                }
                sl = bi;
            }
            if (sl < 0) {  // every slot pinned: the reference's "no free expert slot (all pinned)"
                failed = 1;
                break;
            }
            if (lane == 0) {
                const int ev = owner[sl];
                if (ev >= 0) slot_of[ev] = -1;
                owner[sl] = e, slot_of[e] = sl, stamp[sl] = clock;
                const int li = s.n_loads[c];
                s.loads[c * s.max_slots + li] = make_int2(e, sl);
                s.n_loads[c] = li + 1;
            }
            misses++;
        }
        if (lane == 0) s.map[c * E + e] = sl;
        __syncwarp();
    }
    if (lane == 0) {
        s.meta[0] = clock, s.meta[1] += hits, s.meta[2] += misses;
        if (failed) s.meta[3] += 1, latch_error(err, TMOE_DEV_ERR_NOSLOT);
        s.n_chunks[0] = failed ? 0 : n_chunks;
    }
    __syncwarp();
    for (int e = lane; e < E; e += 32) s.slot_of[e] = slot_of[e];
    for (int i = lane; i < s.max_slots; i += 32) s.owner[i] = owner[i], s.stamp[i] = stamp[i];
}

// Copies the experts of chunk c's loads from the host store into their slots: blockIdx.y = load,
// blockIdx.z = matrix (gate, up, down), blockIdx.x strides over the matrix's 16-byte units with
// four loads in flight per thread (the source is host memory across the PCIe link).
__global__ void __launch_bounds__(256) slot_page_kernel(SlotsDev s, int c, SlotCopy cp) {
    const int li = blockIdx.y;
    if (li >= s.n_loads[c]) return;
    const int2 ld = s.loads[c * s.max_slots + li];
    const int m = blockIdx.z;  // constant indices only: the parameter struct stays in constant memory
    const uint8_t *sb = m == 0 ? cp.src[0] : m == 1 ? cp.src[1] : cp.src[2];
    uint8_t *db = m == 0 ? cp.dst[0] : m == 1 ? cp.dst[1] : cp.dst[2];
    const size_t snb = m == 0 ? cp.src_nb2[0] : m == 1 ? cp.src_nb2[1] : cp.src_nb2[2];
    const size_t dnb = m == 0 ? cp.dst_nb2[0] : m == 1 ? cp.dst_nb2[1] : cp.dst_nb2[2];
    const size_t nbytes = m == 0 ? cp.bytes[0] : m == 1 ? cp.bytes[1] : cp.bytes[2];
    const uint4 *src = reinterpret_cast<const uint4 *>(sb + (size_t)ld.x * snb);
    uint4 *dst = reinterpret_cast<uint4 *>(db + (size_t)ld.y * dnb);
    const size_t n16 = nbytes >> 4;
    const size_t step = (size_t)gridDim.x * blockDim.x;
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + 3 * step < n16; i += 4 * step) {
        const uint4 a = src[i], b = src[i + step], c2 = src[i + 2 * step], d = src[i + 3 * step];
        dst[i] = a, dst[i + step] = b, dst[i + 2 * step] = c2, dst[i + 3 * step] = d;
    }
    for (; i < n16; i += step) dst[i] = src[i];
}

// Residency from a host list (make_resident / a hot set): the same lookups as a planned step, one
// chunk, the list's order.
__global__ void slot_lookup_list_kernel(const int32_t *__restrict__ list, int n, SlotsDev s, int *err) {
    __shared__ int owner[SP_MAX_SLOTS];
    __shared__ unsigned long long stamp[SP_MAX_SLOTS];
    __shared__ int slot_of[SP_MAX_E];
    __shared__ unsigned char pinned[SP_MAX_E];
    const int E = s.n_expert, lane = threadIdx.x;
    const int active = min(s.active[0], s.max_slots);
    for (int e = lane; e < E; e += 32) slot_of[e] = s.slot_of[e], pinned[e] = s.pinned[e];
    for (int i = lane; i < s.max_slots; i += 32) owner[i] = s.owner[i], stamp[i] = s.stamp[i];
    if (lane == 0) s.n_loads[0] = 0, s.n_chunks[0] = 1;
    __syncwarp();
    unsigned long long clock = s.meta[0], hits = 0, misses = 0;
    int failed = 0;
    for (int q = 0; q < n; q++) {
        const int e = list[q];
        if (e < 0 || e >= E) {  // out of range: a bypass in the reference's lookup
            if (lane == 0) s.meta[3] += 1;
            continue;
        }
        clock++;
        int sl = slot_of[e];
        if (sl >= 0) {
            if (lane == 0) stamp[sl] = clock;
            hits++;
            __syncwarp();
            continue;
        }
        int fr = -1;
        for (int i0 = 0; i0 < active && fr < 0; i0 += 32) {
            const unsigned b = __ballot_sync(0xffffffffu, i0 + lane < active && owner[i0 + lane] < 0);
            if (b) fr = i0 + __ffs(b) - 1;
        }
        sl = fr;
        if (sl < 0) {
            unsigned long long bs = 0;
            int bi = -1;
            for (int i = lane; i < active; i += 32) {
                const int o = owner[i];
                if (o >= 0 && !pinned[o]) lru_better(bs, bi, stamp[i], i);
            }
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) {
                const unsigned long long os = __shfl_xor_sync(0xffffffffu, bs, off);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
                lru_better(bs, bi, os, oi);
            }
            sl = bi;
        }
        if (sl < 0) {
            failed = 1;
            break;
        }
        if (lane == 0) {
            const int ev = owner[sl];
            if (ev >= 0) slot_of[ev] = -1;
            owner[sl] = e, slot_of[e] = sl, stamp[sl] = clock;
            const int li = s.n_loads[0];
            s.loads[li] = make_int2(e, sl);
            s.n_loads[0] = li + 1;
        }
        misses++;
        __syncwarp();
    }
    if (lane == 0) {
        s.meta[0] = clock, s.meta[1] += hits, s.meta[2] += misses;
        if (failed) s.meta[3] += 1, latch_error(err, TMOE_DEV_ERR_NOSLOT);
    }
    __syncwarp();
    for (int e = lane; e < E; e += 32) s.slot_of[e] = slot_of[e];
    for (int i = lane; i < s.max_slots; i += 32) s.owner[i] = owner[i], s.stamp[i] = stamp[i];
}

bool slots_fit(int n_expert, int max_slots) {
    return n_expert >= 1 && n_expert <= SP_MAX_E && max_slots >= 1 && max_slots <= SP_MAX_SLOTS &&
           max_slots <= 65535;
}

cudaError_t launch_slot_plan(const int32_t *ids, int n_pairs, const SlotsDev &s, int *err, cudaStream_t st) {
    slot_plan_kernel<<<1, SP_THREADS, 0, st>>>(ids, n_pairs, s, err);
    return cudaGetLastError();
}

cudaError_t launch_slot_lookup_list(const int32_t *list, int n, const SlotsDev &s, int *err, cudaStream_t st) {
    slot_lookup_list_kernel<<<1, 32, 0, st>>>(list, n, s, err);
    return cudaGetLastError();
}

cudaError_t launch_slot_page(const SlotsDev &s, int chunk, const SlotCopy &cp, int sm_count, cudaStream_t st) {
    // about two CTAs per SM over the largest possible load list
    const int per_load = 3 * s.max_slots;
    const int gx = max(1, min(64, (2 * sm_count + per_load - 1) / per_load));
    slot_page_kernel<<<dim3(gx, s.max_slots, 3), 256, 0, st>>>(s, chunk, cp);
    return cudaGetLastError();
}

}  // namespace tmoe
