// Shared device helpers for the MoE layer kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define TMOE_QK 256
#define TMOE_Q4K_BYTES 144
#define TMOE_Q6K_BYTES 210

// Q6_K in 8-row fragment order (made by tmoe_prepack): a matrix of N rows is N/8 row groups, each
// K/256 units of 1680 bytes, one per super-block, holding the same 8 x 210 bytes as ggml's rows
// rearranged for a warp's m16n8k16 fragments.  Row g (0..7) of the group, half h (0, 1) of the
// super-block, lane L = 4 g + t4:
//   768 h + 16 L        ql bytes 64 h + 16 i + 4 t4 .. +3 for i = 0..3 (16 bytes: one 128-bit load)
//   768 h + 512 + 8 L   qh bytes 128 + 32 h + 16 i + 4 t4 .. +3 for i = 0, 1 (8 bytes)
//   1536 + 16 g         the row's 16 scale bytes (ggml bytes 192..207)
//   1664 + 2 g          the row's d (ggml bytes 208, 209)
#define TMOE_Q6R_UNIT 1680

namespace tmoe {
// Where byte `off` (0..209) of row g's ggml super-block lands in its 8-row unit.
__host__ __device__ __forceinline__ int q6r_offset(int g, int off) {
    if (off < 128) return 768 * (off >> 6) + 16 * (4 * g + ((off >> 2) & 3)) + 4 * ((off >> 4) & 3) + (off & 3);
    if (off < 192) {
        const int o = off - 128;
        return 768 * (o >> 5) + 512 + 8 * (4 * g + ((o >> 2) & 3)) + 4 * ((o >> 4) & 1) + (o & 3);
    }
    if (off < 208) return 1536 + 16 * g + (off - 192);
    return 1664 + 2 * g + (off - 208);
}
}  // namespace tmoe

// Device error codes latched in tmoe_handle's flag word (first error wins).
#define TMOE_DEV_ERR_TIMEOUT 1
#define TMOE_DEV_ERR_BADID 2
#define TMOE_DEV_ERR_NOSLOT 3  // every expert slot is pinned: a miss has nowhere to go

// A bounded wait gives up after this many nanoseconds of %globaltimer.
#define TMOE_WAIT_LIMIT_NS 1000000000ull

namespace tmoe {

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void latch_error(int *flag, int code) {
    if (flag) atomicCAS(flag, 0, code);
}

// IEEE binary16 -> f32 without the cuda_fp16 header dependency in hot loops.
__device__ __forceinline__ float h2f(uint16_t h) {
    float f;
    asm("{ .reg .f16 t; mov.b16 t, %1; cvt.f32.f16 %0, t; }" : "=f"(f) : "h"(h));
    return f;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait that lets the thread sleep up to `hint_ns` for the phase (it wakes when the phase
// completes), so that a waiting warp issues few instructions.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Waits for the phase with `parity` to complete; false after TMOE_WAIT_LIMIT_NS.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait_sleep(bar, parity, 100000u)) {
        if (globaltimer_ns() - t0 > TMOE_WAIT_LIMIT_NS) return false;
    }
    return true;
}

// ---------------------------------------------------------------- bulk async copy (TMA, 1D)
// global -> shared, completion counted on `bar` in bytes.  dst/src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ---------------------------------------------------------------- programmatic dependent launch
// A kernel launched with programmatic stream serialization (launch_k under a PdlScope) may start
// while the kernel before it in the stream is still running.  pdl_wait() returns once that kernel
// has completed and its writes are visible (for a plain launch it returns at once); pdl_trigger()
// lets the next such kernel start.  Every kernel here triggers only after its own wait, so when a
// kernel starts, the kernel two launches back has completed: code before the wait may read what
// that one and earlier kernels wrote (through L2), and nothing of its direct predecessor.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- warp helpers
__device__ __forceinline__ float warp_sum_xor(float v, int width) {
    for (int off = width / 2; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

__device__ __forceinline__ int warp_isum_xor(int v, int width) {
    for (int off = width / 2; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// 32-bit word at a shared address that is 2-byte aligned (Q6_K rows are 630 B apart).
__device__ __forceinline__ uint32_t lds_u32_a2(const uint8_t *p) {
    uintptr_t a = reinterpret_cast<uintptr_t>(p);
    if ((a & 3u) == 0) return *reinterpret_cast<const uint32_t *>(p);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    return __funnelshift_r(w[0], w[1], 16);
}

}  // namespace tmoe
