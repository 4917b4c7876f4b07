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

// One chunk's lookups by one warp, in order (LayerSlots::lookup, slots.rs:138-177): the general
// path, used when a chunk's misses could run out of other victims (pinned residents outside the
// chunk) and must then evict entries of the chunk itself exactly as the serial lookups do.
// Returns the index of the lookup that found no slot, or -1.
__device__ int chunk_serial(int c, int qa, int qb, const int *seq, int *slot_of, const unsigned char *pinned,
                            int *owner, unsigned long long *stamp, int active, unsigned long long clock0,
                            int *n_loads, unsigned long long &hits, unsigned long long &misses, const SlotsDev &s) {
    const int lane = threadIdx.x & 31, E = s.n_expert;
    for (int q = qa; q < qb; q++) {
        const int e = seq[q];
        const unsigned long long clock = clock0 + q + 1;
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
            if (sl < 0) return q;  // every slot pinned: "no free expert slot (all pinned)"
            if (lane == 0) {
                const int ev = owner[sl];
                if (ev >= 0) slot_of[ev] = -1;
                owner[sl] = e, slot_of[e] = sl, stamp[sl] = clock;
                s.loads[c * s.max_slots + n_loads[c]] = make_int2(e, sl);
                n_loads[c]++;
            }
            misses++;
        }
        if (lane == 0) s.map[c * E + e] = sl;
        __syncwarp();
    }
    return -1;
}

// The plan of a layer step (Streamer::plan + make_resident per chunk), one CTA:
//  1. first appearance and pair count per expert, in per-group private tables (no atomics
//     across groups), merged;
//  2. the distinct experts ranked by first appearance, residents first;
//  3. per chunk: the hits refresh their stamps; then, since the plan puts residents first, every
//     chunk's hits precede its misses, so its misses take -- in order -- the free slots
//     (ascending), then the unpinned residents outside the chunk by ascending stamp (ties: the
//     lower slot), which is exactly what successive LRU lookups pick: one rank-by-count sort per
//     chunk instead of one argmin per miss.  A chunk whose misses could outnumber those candidates
//     (only possible with pinned residents outside it) makes the serial lookups instead.
constexpr int SP_GROUP_WORDS = 8192;  // first + count tables of all groups: at most 32 KB

__global__ void __launch_bounds__(SP_THREADS) slot_plan_kernel(const int32_t *__restrict__ ids, int n_pairs,
                                                               SlotsDev s, int n_groups, int *err) {
    extern __shared__ int sp_dyn[];  // [n_groups][E] first, then [n_groups][E] counts
    __shared__ int first[SP_MAX_E], order[SP_MAX_E], seq[SP_MAX_E], slot_of[SP_MAX_E];
    __shared__ unsigned char pinned[SP_MAX_E], in_chunk[SP_MAX_E];
    __shared__ int owner[SP_MAX_SLOTS], cand[SP_MAX_SLOTS];
    __shared__ unsigned long long stamp[SP_MAX_SLOTS];
    __shared__ int n_loads[SP_MAX_E];
    __shared__ int n_distinct, bad, n_free, n_cand, failed_at;
    const int E = s.n_expert, S = s.max_slots, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int active = min(s.active[0], S);
    int *gfirst = sp_dyn, *gcnt = sp_dyn + n_groups * E;
    for (int i = tid; i < n_groups * E; i += blockDim.x) gfirst[i] = INT32_MAX, gcnt[i] = 0;
    for (int e = tid; e < E; e += blockDim.x) slot_of[e] = s.slot_of[e], pinned[e] = s.pinned[e], in_chunk[e] = 0;
    for (int i = tid; i < S; i += blockDim.x) owner[i] = s.owner[i], stamp[i] = s.stamp[i];
    for (int i = tid; i < s.max_chunks * E; i += blockDim.x) s.map[i] = -1;
    for (int i = tid; i < s.max_chunks; i += blockDim.x) n_loads[i] = 0;
    if (tid == 0) n_distinct = 0, bad = 0, failed_at = -1;
    __syncthreads();
    {  // 1. group g of warps takes pairs [g * span, (g + 1) * span), 32 at a time per warp
        const int nw = blockDim.x >> 5, wpg = nw / n_groups, g = warp / wpg, wi = warp % wpg;
        const int span = (n_pairs + n_groups - 1) / n_groups;
        const int p0 = g * span, p1 = min(n_pairs, p0 + span);
        int *fg = gfirst + g * E, *cg = gcnt + g * E;
        for (int base = p0 + 32 * wi; base < p1; base += 32 * wpg) {
            const int p = base + lane;
            if (p < p1) {
                const int e = __ldg(ids + p);
                if (e < 0 || e >= E) {
                    bad = 1;
                } else {
                    atomicMin(&fg[e], p);
                    atomicAdd(&cg[e], 1);
                }
            }
        }
    }
    __syncthreads();
    if (bad) {  // the reference: "router chose expert {e}, out of range"
        for (int i = tid; i < s.max_chunks; i += blockDim.x) s.n_loads[i] = 0;
        if (tid == 0) latch_error(err, TMOE_DEV_ERR_BADID), s.n_chunks[0] = 0;
        return;
    }
    for (int e = tid; e < E; e += blockDim.x) {
        int f = INT32_MAX, n = 0;
        for (int g = 0; g < n_groups; g++) f = min(f, gfirst[g * E + e]), n += gcnt[g * E + e];
        first[e] = n ? f : INT32_MAX;
        if (n) s.counts[e] += (unsigned long long)n;
    }
    __syncthreads();
    // 2. rank by first appearance (first appearances are distinct pair indices)
    for (int e = tid; e < E; e += blockDim.x) {
        if (first[e] != INT32_MAX) {
            int r = 0;
            for (int f = 0; f < E; f++) r += first[f] < first[e];
            order[r] = e;
            atomicAdd(&n_distinct, 1);
        }
    }
    __syncthreads();
    const int nd = n_distinct;
    if (warp == 0) {  // residents first, then misses, each in order of first appearance
        int w = 0;
        for (int pass = 0; pass < 2; pass++)
            for (int i0 = 0; i0 < nd; i0 += 32) {
                const int i = i0 + lane;
                const bool take = i < nd && ((slot_of[order[i]] >= 0) == (pass == 0));
                const unsigned b = __ballot_sync(0xffffffffu, take);
                if (take) seq[w + __popc(b & ((1u << lane) - 1))] = order[i];
                w += __popc(b);
            }
    }
    __syncthreads();
    const int n = max(active, 1);
    const int n_chunks = (nd + n - 1) / n;
    if (n_chunks > s.max_chunks) {
        for (int i = tid; i < s.max_chunks; i += blockDim.x) s.n_loads[i] = 0;
        if (tid == 0) latch_error(err, TMOE_DEV_ERR_NOSLOT), s.n_chunks[0] = 0;
        return;
    }
    const unsigned long long clock0 = s.meta[0];
    unsigned long long hits = 0, misses = 0;  // warp 0's counts on the serial path
    int par_hits = 0, par_misses = 0;
    for (int c = 0; c < n_chunks; c++) {
        const int qa = c * n, qb = min(nd, qa + n);
        // 3a. hits (residents at the start of the chunk) refresh their stamps
        for (int q = qa + tid; q < qb; q += blockDim.x) {
            const int e = seq[q];
            in_chunk[e] = 1;
            const int sl = slot_of[e];
            if (sl >= 0) {
                stamp[sl] = clock0 + q + 1;
                s.map[c * E + e] = sl;
            }
        }
        if (tid == 0) n_free = 0, n_cand = 0;
        __syncthreads();
        int h = 0;  // the chunk's hits: a prefix of it
        for (int q = qa; q < qb && slot_of[seq[q]] >= 0; q++) h++;
        const int m = (qb - qa) - h;
        // 3b. victims: free slots (ascending), then unpinned residents outside the chunk by stamp
        for (int i = tid; i < active; i += blockDim.x) {
            const int o = owner[i];
            if (o < 0) atomicAdd(&n_free, 1);
            else if (!pinned[o] && !in_chunk[o]) atomicAdd(&n_cand, 1);
        }
        __syncthreads();
        const int nf = n_free, nc = n_cand;
        if (m > nf + nc) {  // only with pinned residents outside the chunk: the serial lookups
            if (warp == 0) {
                const int fq = chunk_serial(c, qa, qb, seq, slot_of, pinned, owner, stamp, active, clock0, n_loads,
                                            hits, misses, s);
                if (lane == 0) failed_at = fq;
                __syncwarp();
            }
            __syncthreads();
            for (int q = qa + tid; q < qb; q += blockDim.x) in_chunk[seq[q]] = 0;
            __syncthreads();
            if (failed_at >= 0) break;
            continue;
        }
        for (int i = tid; i < active; i += blockDim.x) {
            const int o = owner[i];
            int r = -1;
            if (o < 0) {  // rank among the free slots: by index
                r = 0;
                for (int j = 0; j < i; j++) r += owner[j] < 0;
            } else if (!pinned[o] && !in_chunk[o]) {  // after the free slots: by (stamp, slot)
                r = nf;
                const unsigned long long si = stamp[i];
                for (int j = 0; j < active; j++) {
                    const int oj = owner[j];
                    if (oj >= 0 && !pinned[oj] && !in_chunk[oj] && (stamp[j] < si || (stamp[j] == si && j < i))) r++;
                }
            }
            if (r >= 0 && r < m) cand[r] = i;
        }
        __syncthreads();
        // 3c. miss i takes cand[i]
        for (int i = tid; i < m; i += blockDim.x) {
            const int q = qa + h + i, e = seq[q], sl = cand[i];
            const int ev = owner[sl];
            if (ev >= 0) slot_of[ev] = -1;
            owner[sl] = e, slot_of[e] = sl, stamp[sl] = clock0 + q + 1;
            s.loads[c * S + i] = make_int2(e, sl);
            s.map[c * E + e] = sl;
        }
        if (tid == 0) n_loads[c] = m, par_hits += h, par_misses += m;
        __syncthreads();
        for (int q = qa + tid; q < qb; q += blockDim.x) in_chunk[seq[q]] = 0;
        __syncthreads();
    }
    if (tid == 0) {  // every lookup advances the clock, the failed one included (slots.rs:143)
        const bool failed = failed_at >= 0;
        s.meta[0] = clock0 + (unsigned long long)(failed ? failed_at + 1 : nd);
        s.meta[1] += hits + (unsigned long long)par_hits;
        s.meta[2] += misses + (unsigned long long)par_misses;
        if (failed) s.meta[3] += 1, latch_error(err, TMOE_DEV_ERR_NOSLOT);
        s.n_chunks[0] = failed ? 0 : n_chunks;
    }
    __syncthreads();
    for (int e = tid; e < E; e += blockDim.x) s.slot_of[e] = slot_of[e];
    for (int i = tid; i < S; i += blockDim.x) s.owner[i] = owner[i], s.stamp[i] = stamp[i];
    for (int i = tid; i < s.max_chunks; i += blockDim.x) s.n_loads[i] = n_loads[i];
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

// The overlapped miss path: the loads of chunk c >= 1 go first into a staging area (one expert
// of gate, up and down bytes back to back per load index), paged in from the host store on a side
// stream while earlier chunks compute, by a lean kernel (128 threads, few registers, few CTAs) that
// can share SMs with the compute kernels; right before chunk c computes, a device copy moves them
// into their slots (after chunk c - 1, whose slots they may replace, has finished).
__device__ __forceinline__ void copy16_x4(uint4 *dst, const uint4 *src, size_t n16, size_t i, size_t step) {
    for (; i + 3 * step < n16; i += 4 * step) {
        const uint4 a = src[i], b = src[i + step], c2 = src[i + 2 * step], d = src[i + 3 * step];
        dst[i] = a, dst[i + step] = b, dst[i + 2 * step] = c2, dst[i + 3 * step] = d;
    }
    for (; i < n16; i += step) dst[i] = src[i];
}

__global__ void __launch_bounds__(128, 16) slot_stage_kernel(SlotsDev s, int c, SlotCopy cp, uint8_t *staging,
                                                             size_t ebytes) {
    const int nl = s.n_loads[c];
    const size_t step = (size_t)gridDim.x * blockDim.x, i0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (int li = 0; li < nl; li++) {
        const int e = s.loads[c * s.max_slots + li].x;
        uint8_t *dst = staging + (size_t)li * ebytes;
#pragma unroll 1
        for (int m = 0; m < 3; m++) {
            const uint8_t *sb = m == 0 ? cp.src[0] : m == 1 ? cp.src[1] : cp.src[2];
            const size_t snb = m == 0 ? cp.src_nb2[0] : m == 1 ? cp.src_nb2[1] : cp.src_nb2[2];
            const size_t nbytes = m == 0 ? cp.bytes[0] : m == 1 ? cp.bytes[1] : cp.bytes[2];
            copy16_x4(reinterpret_cast<uint4 *>(dst), reinterpret_cast<const uint4 *>(sb + (size_t)e * snb),
                      nbytes >> 4, i0, step);
            dst += nbytes;
        }
    }
}

// blockIdx.y = load, blockIdx.z = matrix: staging -> the load's slot.
__global__ void __launch_bounds__(256) slot_unstage_kernel(SlotsDev s, int c, SlotCopy cp, const uint8_t *staging,
                                                           size_t ebytes) {
    const int li = blockIdx.y;
    if (li >= s.n_loads[c]) return;
    const int slot = s.loads[c * s.max_slots + li].y;
    const int m = blockIdx.z;
    uint8_t *db = m == 0 ? cp.dst[0] : m == 1 ? cp.dst[1] : cp.dst[2];
    const size_t dnb = m == 0 ? cp.dst_nb2[0] : m == 1 ? cp.dst_nb2[1] : cp.dst_nb2[2];
    const size_t nbytes = m == 0 ? cp.bytes[0] : m == 1 ? cp.bytes[1] : cp.bytes[2];
    const size_t off = m == 0 ? 0 : m == 1 ? cp.bytes[0] : cp.bytes[0] + cp.bytes[1];
    copy16_x4(reinterpret_cast<uint4 *>(db + (size_t)slot * dnb),
              reinterpret_cast<const uint4 *>(staging + (size_t)li * ebytes + off), nbytes >> 4,
              (size_t)blockIdx.x * blockDim.x + threadIdx.x, (size_t)gridDim.x * blockDim.x);
}

bool slots_fit(int n_expert, int max_slots) {
    return n_expert >= 1 && n_expert <= SP_MAX_E && max_slots >= 1 && max_slots <= SP_MAX_SLOTS &&
           max_slots <= 65535;
}

cudaError_t launch_slot_plan(const int32_t *ids, int n_pairs, const SlotsDev &s, int *err, cudaStream_t st) {
    int groups = 32;  // a power of two dividing the 32 warps, its tables within SP_GROUP_WORDS
    while (groups > 1 && groups * 2 * s.n_expert > SP_GROUP_WORDS) groups >>= 1;
    const size_t smem = (size_t)groups * 2 * s.n_expert * 4;
    static int set_bytes[64] = {};  // static + dynamic shared memory exceed the default 48 KB
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!set_bytes[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(slot_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   SP_GROUP_WORDS * 4);
        if (e != cudaSuccess) return e;
        set_bytes[dev] = 1;
    }
    slot_plan_kernel<<<1, SP_THREADS, smem, st>>>(ids, n_pairs, s, groups, err);
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

cudaError_t launch_slot_stage(const SlotsDev &s, int chunk, const SlotCopy &cp, uint8_t *staging, size_t ebytes,
                              cudaStream_t st) {
    slot_stage_kernel<<<32, 128, 0, st>>>(s, chunk, cp, staging, ebytes);
    return cudaGetLastError();
}

cudaError_t launch_slot_unstage(const SlotsDev &s, int chunk, const SlotCopy &cp, const uint8_t *staging,
                                size_t ebytes, int sm_count, cudaStream_t st) {
    const int per_load = 3 * s.max_slots;
    const int gx = max(1, min(64, (4 * sm_count + per_load - 1) / per_load));
    slot_unstage_kernel<<<dim3(gx, s.max_slots, 3), 256, 0, st>>>(s, chunk, cp, staging, ebytes);
    return cudaGetLastError();
}

}  // namespace tmoe
