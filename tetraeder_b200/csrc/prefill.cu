// Expert products for the prefill / large-batch regime (many tokens per expert): grouped GEMMs on
// the 5th-generation tensor cores.  tcgen05.mma (kind::f16, fp16 operands, f32 accumulators in
// TMEM) issued by one thread, operands staged in shared memory by TMA with 128-byte swizzle, a
// persistent CTA per SM walking the tiles of all active experts.
//
// Numerics.  The reference CPU path quantises the activations to Q8_K before the expert dots
// (ggml's vec_dot_type for the K-quants); here the activations go through the same Q8_K round
// trip and are then held exactly enough in fp16 (d * q, q an int8), the weights are dequantised
// to fp16 (d * scale * q - dmin * min), and the products are summed in f32.  The result differs
// from the reference's integer block sums by fp16 rounding of the dequantised values only.
//
// Dataflow of a layer (rows in the dispatch's expert-sorted pair order r, perm[r] = pair):
//   prep_rows_kernel   x rows -> Q8_K round trip -> fp16 A1[r][H]
//   dequant_f16_kernel expert weights of the active experts -> fp16 [expert][row][K]
//   gemm (SWIGLU)      act[r][I] = silu(A1 . gate^T) * (A1 . up^T)
//   prep_rows_kernel   act rows -> Q8_K round trip -> fp16 A2[r][I]
//   gemm (SCATTER)     dout[perm[r]][H] = A2 . down^T
// GEMM tile: 128 rows of one expert x 256 output columns (SWIGLU: 128 gate + the same 128 up
// features), K in steps of 64 (one 128-byte swizzle atom), 4 MMAs of K = 16 per step.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.cuh"
#include "q8k.cuh"

namespace tmoe {

constexpr int PF_BM = 128;
constexpr int PF_BN = 256;
constexpr int PF_BK = 64;
constexpr int PF_STAGES = 4;
constexpr int PF_THREADS = 192;  // warp 0: TMA, warp 1: MMA, warps 2-5: epilogue
constexpr int PF_A_BYTES = PF_BM * PF_BK * 2;
constexpr int PF_B_BYTES = PF_BN * PF_BK * 2;
constexpr int PF_STAGE_BYTES = PF_A_BYTES + PF_B_BYTES;
constexpr int PF_SMEM = PF_STAGES * PF_STAGE_BYTES + 1024 /* barriers */ + 1024 /* alignment */;
constexpr uint32_t PF_TMEM_COLS = 512;  // two accumulators of 256 f32 columns

// ------------------------------------------------------------------ tcgen05 / TMA helpers
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives on `bar` once every MMA this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 consecutive f32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *m, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile in the 128-byte swizzle layout that
// TMA writes for a box of 64 fp16 columns: rows of 128 bytes, 8-row groups 1024 bytes apart
// (stride byte offset), start address advanced by 32 bytes per K = 16 step inside the atom.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr & 0x3ffffu) >> 4);  // start address >> 4, bits [0, 14)
    d |= (uint64_t)1 << 16;                             // leading byte offset (unused for this layout)
    d |= (uint64_t)(1024 >> 4) << 32;                   // stride byte offset >> 4, bits [32, 46)
    d |= (uint64_t)1 << 46;                             // descriptor version of sm_100
    d |= (uint64_t)2 << 61;                             // layout: 128-byte swizzle
    return d;
}

// Instruction descriptor of kind::f16: fp16 A and B (K-major), f32 D, M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ float silu_mul_pf(float g, float u) { return (g / (1.0f + expf(-g))) * u; }

// ------------------------------------------------------------------ preparation kernels
// A rows of the GEMM: row r of `rows` (expert-sorted pairs; src row = perm[r] / x_div) through the
// Q8_K round trip, as fp16.  One warp per (row, 256-block); rows from n_valid[0] on (no dispatched
// pair: no tile reads them) are skipped.
__global__ void prep_rows_kernel(const float *__restrict__ src, const int32_t *__restrict__ perm, int n_rows,
                                 const int32_t *__restrict__ n_valid, int x_div, int K, __half *__restrict__ dst) {
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int nb = K / TMOE_QK;
    const int64_t r = gw / nb;
    const int b = (int)(gw % nb);
    if (r >= n_rows || (n_valid && r >= n_valid[0])) return;
    int p = perm ? perm[r] : (int)r;
    if (p < 0) p = 0;
    const float *xr = src + (int64_t)(p / x_div) * K + b * TMOE_QK + 8 * lane;
    const float4 a0 = *reinterpret_cast<const float4 *>(xr), a1 = *reinterpret_cast<const float4 *>(xr + 4);
    const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    uint2 q;
    float d;
    int s16;
    q8k_block_warp(v, q, d, s16);
    __align__(16) __half h[8];
#pragma unroll
    for (int c = 0; c < 8; c++) {
        const int qi = (int)(int8_t)(((c < 4 ? q.x : q.y) >> (8 * (c & 3))) & 0xff);
        h[c] = __float2half_rn(__fmul_rn(d, (float)qi));
    }
    *reinterpret_cast<uint4 *>(dst + r * K + b * TMOE_QK + 8 * lane) = *reinterpret_cast<const uint4 *>(h);
}

// fp16 copies of the active experts' rows: dst[e][row][K] for the experts of `active` (others are
// left alone).  A CTA takes DQ_ROWS consecutive rows of one active expert: the rows' bytes (contiguous
// in the ggml layout) are staged in shared memory with 16-byte loads, then each warp dequantises one
// super-block at a time, lane t the 8 consecutive elements 8t..8t+7 (one 16-byte store), whose Q4_K
// quants are 8 consecutive bytes of one 32-byte run and whose Q6_K low/high quants are 8 consecutive
// bytes of ql and of qh.  Values: Q4_K fp16((d*sc)*q - dmin*m), Q6_K fp16((d*sc)*(q - 32)).
constexpr int DQ_ROWS = 16;

__device__ __forceinline__ uint2 lds_u64_a2(const uint8_t *p) {
    return make_uint2(lds_u32_a2(p), lds_u32_a2(p + 4));
}

template <int WT>
__global__ void __launch_bounds__(256) dequant_f16_kernel(const uint8_t *__restrict__ w, size_t nb2, int N, int K,
                                                          const int4 *__restrict__ active,
                                                          const int32_t *__restrict__ n_active, int max_active,
                                                          __half *__restrict__ dst) {
    extern __shared__ __align__(16) uint8_t dq_rows[];
    const int ai = blockIdx.y;
    if (ai >= min(n_active[0], max_active)) return;
    constexpr int BB = WT == TMOE_WT_Q4K ? TMOE_Q4K_BYTES : TMOE_Q6K_BYTES;  // per row and super-block
    const int nb = K / TMOE_QK;
    const int row_bytes = nb * BB;
    const int e = active[ai].x;
    const int row0 = blockIdx.x * DQ_ROWS, nr = min(DQ_ROWS, N - row0);
    const uint4 *src = reinterpret_cast<const uint4 *>(w + (size_t)e * nb2 + (size_t)row0 * row_bytes);
    const int n16 = (nr * row_bytes) >> 4;  // nr * row_bytes % 16 == 0 (checked by the launcher)
    for (int i = threadIdx.x; i < n16; i += blockDim.x)
        reinterpret_cast<uint4 *>(dq_rows)[i] = __ldg(src + i);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int u = warp; u < nr * nb; u += blockDim.x >> 5) {
        const int r = u / nb, b = u - r * nb;
        // ggml layout: the row's block; 8-row fragment order: the block's unit, row r % 8 of it
        const uint8_t *blk = WT == TMOE_WT_Q6KR ? dq_rows + (r >> 3) * (nb * TMOE_Q6R_UNIT) + b * TMOE_Q6R_UNIT
                                                : dq_rows + r * row_bytes + b * BB;
        __align__(16) __half h[8];
        // Two elements per step: their quant bytes become the fp16 pair (1024 + q) by exponent magic
        // (one byte permute), an exact half2 subtraction leaves the integers, and the value is
        // formed in f32 and rounded to fp16 once, as (float)q would give it.
        if constexpr (WT == TMOE_WT_Q4K) {
            const int c = lane >> 2;  // sub-block of 32
            const float d = h2f(*reinterpret_cast<const uint16_t *>(blk)),
                        dmin = h2f(*reinterpret_cast<const uint16_t *>(blk + 2));
            const uint8_t *sc = blk + 4;
            int scale, mn;
            if (c < 4) {
                scale = sc[c] & 63;
                mn = sc[c + 4] & 63;
            } else {
                scale = (sc[c + 4] & 0x0f) | ((sc[c - 4] >> 6) << 4);
                mn = (sc[c + 4] >> 4) | ((sc[c] >> 6) << 4);
            }
            const float d1 = __fmul_rn(d, (float)scale), m1 = __fmul_rn(dmin, (float)mn);
            const uint2 q = *reinterpret_cast<const uint2 *>(blk + 16 + 32 * (c >> 1) + 8 * (lane & 3));
            const int sh = (c & 1) * 4;
            const uint32_t qw[2] = {(q.x >> sh) & 0x0f0f0f0fu, (q.y >> sh) & 0x0f0f0f0fu};
            const __half2 base = __float2half2_rn(1024.0f);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t bits = __byte_perm(qw[i >> 1], 0x64u, (i & 1) ? 0x4342u : 0x4140u);
                __half2 v;
                memcpy(&v, &bits, 4);
                const float2 f = __half22float2(__hsub2(v, base));
                const __half2 r2 =
                    __floats2half2_rn(__fsub_rn(__fmul_rn(d1, f.x), m1), __fsub_rn(__fmul_rn(d1, f.y), m1));
                memcpy(&h[2 * i], &r2, 4);
            }
        } else {
            const int hh = lane >> 4, rr = 8 * (lane & 15);  // element k = 128 hh + rr + i
            // byte `off` of the row's ggml block (words: off % 4 == 0)
            const int g8 = r & 7;
            auto at = [&](int off) { return WT == TMOE_WT_Q6KR ? blk + q6r_offset(g8, off) : blk + off; };
            auto u64 = [&](int off) {
                return WT == TMOE_WT_Q6KR ? make_uint2(*reinterpret_cast<const uint32_t *>(at(off)),
                                                       *reinterpret_cast<const uint32_t *>(at(off + 4)))
                                          : lds_u64_a2(blk + off);
            };
            const uint2 lo = u64(64 * hh + (rr & 63));
            const uint2 hi = u64(128 + 32 * hh + (rr & 31));
            const int lsh = rr < 64 ? 0 : 4, hsh = 2 * (rr >> 5);
            const float d = h2f((uint16_t)(*at(208) | (*at(209) << 8)));
            const float ds = __fmul_rn(d, (float)*reinterpret_cast<const int8_t *>(at(192 + ((128 * hh + rr) >> 4))));
            // the 6-bit quants of elements 0-3 and 4-7, one per byte
            const uint32_t qw[2] = {((lo.x >> lsh) & 0x0f0f0f0fu) | (((hi.x >> hsh) & 0x03030303u) << 4),
                                    ((lo.y >> lsh) & 0x0f0f0f0fu) | (((hi.y >> hsh) & 0x03030303u) << 4)};
            const __half2 base = __float2half2_rn(1056.0f);  // 1024 + the Q6_K bias 32
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t bits = __byte_perm(qw[i >> 1], 0x64u, (i & 1) ? 0x4342u : 0x4140u);
                __half2 v;
                memcpy(&v, &bits, 4);
                const float2 f = __half22float2(__hsub2(v, base));  // q - 32, exact
                const __half2 r2 = __floats2half2_rn(__fmul_rn(ds, f.x), __fmul_rn(ds, f.y));
                memcpy(&h[2 * i], &r2, 4);
            }
        }
        *reinterpret_cast<uint4 *>(dst + ((int64_t)e * N + row0 + r) * K + b * TMOE_QK + 8 * lane) =
            *reinterpret_cast<const uint4 *>(h);
    }
}

// tile_start[a] = sum over the active experts before a of ceil(rows / 128) * n_tiles_n;
// tile_start[n_active] = all tiles.  One CTA.
__global__ void tiles_kernel(const int4 *__restrict__ active, const int32_t *__restrict__ n_active, int max_active,
                             int n_tiles_n, int *__restrict__ tile_start) {
    __shared__ int sums[1024];
    const int na = min(n_active[0], max_active);
    int run = 0;
    for (int base = 0; base < na; base += blockDim.x) {
        const int a = base + threadIdx.x;
        const int m = a < na ? ((active[a].z - active[a].y + PF_BM - 1) / PF_BM) * n_tiles_n : 0;
        sums[threadIdx.x] = m;
        __syncthreads();
        for (int off = 1; off < (int)blockDim.x; off <<= 1) {  // inclusive scan (Hillis-Steele)
            const int v = threadIdx.x >= (unsigned)off ? sums[threadIdx.x - off] : 0;
            __syncthreads();
            sums[threadIdx.x] += v;
            __syncthreads();
        }
        if (a < na) tile_start[a] = run + sums[threadIdx.x] - m;
        run += sums[blockDim.x - 1];
        __syncthreads();
    }
    if (threadIdx.x == 0) tile_start[na] = run;
}

// ------------------------------------------------------------------ the grouped GEMM
struct PfMaps {
    CUtensorMap a;   // A rows: fp16 [rows][K], box 64 x 128
    CUtensorMap b0;  // gate (SWIGLU, box 64 x 128) or down (SCATTER, box 64 x 256): fp16 [E * N][K]
    CUtensorMap b1;  // up (SWIGLU)
};

struct PfArgs {
    int K;          // reduction length (multiple of 64)
    int N;          // rows of one expert's matrix (I for gate/up, H for down)
    int n_tiles_n;  // output column tiles per expert
    const int4 *active;
    const int32_t *n_active;
    int max_active;
    const int *tile_start;
    const int32_t *perm;
    int n_rows;     // rows of A (pairs)
    float *out;     // SWIGLU: act [rows][N]; SCATTER: dout [pairs][N]
    int *err;
};

enum { PF_SWIGLU = 0, PF_SCATTER = 1 };

// Which expert (active index), row tile and column tile a tile is.
__device__ __forceinline__ void pf_decode(const PfArgs &a, int na, int tile, int &ai, int &m, int &n) {
    int lo = 0, hi = na - 1;  // the last active index with tile_start <= tile
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(a.tile_start + mid) <= tile) lo = mid;
        else hi = mid - 1;
    }
    ai = lo;
    const int4 info = __ldg(a.active + ai);
    const int m_tiles = (info.z - info.y + PF_BM - 1) / PF_BM;
    const int local = tile - __ldg(a.tile_start + ai);
    n = local / m_tiles;  // consecutive tiles share a weight tile
    m = local % m_tiles;
}

template <int EPI>
__global__ void __launch_bounds__(PF_THREADS, 1) prefill_gemm_kernel(const __grid_constant__ PfMaps maps, const PfArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *stages = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + PF_STAGES * PF_STAGE_BYTES);
    uint64_t *empty = full + PF_STAGES;
    uint64_t *tfull = empty + PF_STAGES;
    uint64_t *tempty = tfull + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < PF_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, PF_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    int na = a.n_active[0];
    if (na > a.max_active || na < 0) na = na < 0 ? 0 : a.max_active;
    const int n_tiles = na > 0 ? __ldg(a.tile_start + na) : 0;
    const int kb_n = a.K / PF_BK;

    if (warp == 0) {
        if (lane == 0) {  // TMA producer
            int it = 0;
            for (int tile = blockIdx.x; tile < n_tiles && !*abort_flag; tile += gridDim.x) {
                int ai, m, n;
                pf_decode(a, na, tile, ai, m, n);
                const int4 info = __ldg(a.active + ai);
                const int row0 = info.y + m * PF_BM;
                for (int kb = 0; kb < kb_n; kb++, it++) {
                    const int s = it % PF_STAGES;
                    if (it >= PF_STAGES && !mbar_wait_bounded(&empty[s], ((it / PF_STAGES) - 1) & 1)) {
                        latch_error(a.err, TMOE_DEV_ERR_TIMEOUT);
                        *abort_flag = 1;
                        break;
                    }
                    uint8_t *sa = stages + (size_t)s * PF_STAGE_BYTES, *sb = sa + PF_A_BYTES;
                    mbar_arrive_expect_tx(&full[s], (uint32_t)PF_STAGE_BYTES);
                    tma_load_2d(sa, &maps.a, kb * PF_BK, row0, &full[s]);
                    if (EPI == PF_SWIGLU) {
                        const int brow = info.x * a.N + n * (PF_BN / 2);
                        tma_load_2d(sb, &maps.b0, kb * PF_BK, brow, &full[s]);
                        tma_load_2d(sb + PF_B_BYTES / 2, &maps.b1, kb * PF_BK, brow, &full[s]);
                    } else {
                        tma_load_2d(sb, &maps.b0, kb * PF_BK, info.x * a.N + n * PF_BN, &full[s]);
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            constexpr uint32_t idesc = idesc_f16(PF_BM, PF_BN);
            int it = 0, tcount = 0;
            for (int tile = blockIdx.x; tile < n_tiles && !*abort_flag; tile += gridDim.x, tcount++) {
                const int buf = tcount & 1;
                if (tcount >= 2 && !mbar_wait_bounded(&tempty[buf], ((tcount >> 1) - 1) & 1)) {
                    latch_error(a.err, TMOE_DEV_ERR_TIMEOUT);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(buf * PF_BN);
                bool ok = true;
                for (int kb = 0; kb < kb_n; kb++, it++) {
                    const int s = it % PF_STAGES;
                    if (!mbar_wait_bounded(&full[s], (it / PF_STAGES) & 1)) {
                        latch_error(a.err, TMOE_DEV_ERR_TIMEOUT);
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(stages + (size_t)s * PF_STAGE_BYTES), sb = sa + PF_A_BYTES;
#pragma unroll
                    for (int k = 0; k < PF_BK / 16; k++)
                        umma_f16(d, sw128_desc(sa + 32 * k), sw128_desc(sb + 32 * k), idesc, (kb | k) != 0);
                    umma_commit(&empty[s]);  // the stage is free once these MMAs are done
                }
                if (!ok) break;
                umma_commit(&tfull[buf]);  // the accumulator is complete
            }
        }
    } else {  // epilogue: warps 2-5, TMEM lane quarter warp % 4
        const int q = warp & 3;
        int tcount = 0;
        for (int tile = blockIdx.x; tile < n_tiles && !*abort_flag; tile += gridDim.x, tcount++) {
            const int buf = tcount & 1;
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&tfull[buf], (tcount >> 1) & 1))) {
                if (lane == 0) latch_error(a.err, TMOE_DEV_ERR_TIMEOUT);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            int ai, m, n;
            pf_decode(a, na, tile, ai, m, n);
            const int4 info = __ldg(a.active + ai);
            const int r = info.y + m * PF_BM + q * 32 + lane;
            const bool valid = r < info.z && r < a.n_rows;
            const uint32_t taddr = tmem_base + (uint32_t)(buf * PF_BN) + ((uint32_t)(q * 32) << 16);
            if (EPI == PF_SWIGLU) {
                float *orow = a.out + (int64_t)r * a.N + n * (PF_BN / 2);
#pragma unroll 1
                for (int c0 = 0; c0 < PF_BN / 2; c0 += 32) {
                    float g[32], u[32];
                    tmem_ld32(taddr + c0, g);
                    tmem_ld32(taddr + PF_BN / 2 + c0, u);
                    tmem_wait_ld();
                    if (valid) {
#pragma unroll
                        for (int i = 0; i < 32; i += 4)
                            *reinterpret_cast<float4 *>(orow + c0 + i) =
                                make_float4(silu_mul_pf(g[i], u[i]), silu_mul_pf(g[i + 1], u[i + 1]),
                                            silu_mul_pf(g[i + 2], u[i + 2]), silu_mul_pf(g[i + 3], u[i + 3]));
                    }
                }
            } else {
                const int p = valid ? (a.perm ? __ldg(a.perm + r) : r) : 0;  // no perm: rows in place (dense)
                float *orow = a.out + (int64_t)p * a.N + n * PF_BN;
#pragma unroll 1
                for (int c0 = 0; c0 < PF_BN; c0 += 32) {
                    float v[32];
                    tmem_ld32(taddr + c0, v);
                    tmem_wait_ld();
                    if (valid) {
#pragma unroll
                        for (int i = 0; i < 32; i += 4)
                            *reinterpret_cast<float4 *>(orow + c0 + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem_base, PF_TMEM_COLS);
    }
}

// ------------------------------------------------------------------ exact gate/up (Q4_K)
// The gate/up products of the large-batch regime, exact like the reference's integer block sums
// and still on tcgen05: both operands are integers that fp16 holds exactly, and f32 sums them
// exactly (below 2^24), so each super-block b of K gives exact integer dots.
//   main_b[t][n] = sum_{k in b} q_x[t][k] * (sc[n][s(k)] * q[n][k])   (q_x int8, sc*q <= 945)
//   min_b[t][n]  = sum_s  B[t][b][s] * m[n][b][s]                       (B = 64 * hi + lo: K = 16)
//   out[t][n]   += d_x[t][b] * (d[n][b] * main_b - dmin[n][b] * min_b)   (the ggml Q4_K x Q8_K dot)
// The min term shares the block's accumulator: acc = main_b - (dmin / d) * min_b, with the block
// sums as [64 hi, lo] (exact) against c = -(dmin / d) * m as a high and a low fp16 part (two K = 16
// MMAs; about 22 bits of c), and the epilogue folds out += d_x * d * acc: one TMEM value per output
// and block instead of two.
// The per-block accumulators live in TMEM (double-buffered: 2 x 128 columns) and
// the epilogue warps fold them into per-thread running sums while the next block's MMAs run.  A
// tile is 128 token rows x 64 features of gate and the same 64 of up (128 MMA columns); the
// SwiGLU happens once per tile.  Warps: 0 TMA (q_x rows, block sums), 1 MMA, 2-5 dequantise the
// weights into the swizzled fp16 layout (sc * q, the mins, d/dmin), 6-13 epilogue (lane quarter
// warp % 4; features 32h .. 32h+31 of gate and of up, h = (warp - 6) / 4).
constexpr int GU_S = 4;            // A / B stage ring
constexpr int GU_THREADS = 448;  // 14 warps
constexpr int GU_AP_BYTES = 128 * 16 * 2;  // min operand of one block: 128 rows x K 16 fp16
constexpr int GU_RAW_BYTES = 128 * TMOE_Q4K_BYTES;  // one super-block of the tile's 128 weight rows
constexpr int GU_RAWN = 3;  // raw prefetch buffers: two blocks ahead
// shared memory: the rings, the scales, 512 bytes of barriers, then the tile tables; plus 1024 bytes
// of alignment slack
constexpr int GU_FIXED = GU_S * (2 * PF_A_BYTES) + 6 * GU_AP_BYTES + GU_RAWN * GU_RAW_BYTES + 2 * 128 * 8 + 512;
constexpr uint32_t GU_TMEM_COLS = 256;  // two accumulators of 128 columns (64 gate + 64 up features)
static_assert((GU_S * 4 + 12) * 8 + 16 <= 512, "barrier room");

// K-major, no swizzle: 8-row x 16-byte core matrices, rows 16 bytes apart, 8-row groups 128 bytes
// apart (stride byte offset), the two K halves of a K = 16 tile 2048 bytes apart (leading byte
// offset).
__device__ __forceinline__ uint64_t kmajor_plain_desc(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr & 0x3ffffu) >> 4);
    d |= (uint64_t)(2048 >> 4) << 16;
    d |= (uint64_t)(128 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    return d;  // layout type 0: no swizzle
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) {
    uint32_t u;
    memcpy(&u, &h, 4);
    return u;
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait2() { asm volatile("cp.async.wait_group 2;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// A rows of the exact gate/up GEMM from the tokens' Q8_K: q_x as fp16 [rows][K], d [rows][K/256],
// and per super-block the 8 sub-block sums of 32 split as {hi, lo} with B = 64 * hi + lo, as fp16
// [rows][K/256][16].  One warp per (row, 256-block).
__global__ void prep_gateup_a_kernel(const float *__restrict__ x, const int32_t *__restrict__ perm, int n_rows,
                                     int x_div, int K, __half *__restrict__ aq, float *__restrict__ ad,
                                     __half *__restrict__ ab) {
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int nb = K / TMOE_QK;
    const int64_t r = gw / nb;
    const int b = (int)(gw % nb);
    if (r >= n_rows) return;
    int p = perm ? perm[r] : (int)r;
    if (p < 0) p = 0;
    const float *xr = x + (int64_t)(p / x_div) * K + b * TMOE_QK + 8 * lane;
    const float4 a0 = *reinterpret_cast<const float4 *>(xr), a1 = *reinterpret_cast<const float4 *>(xr + 4);
    const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    uint2 q;
    float d;
    int s16;
    q8k_block_warp(v, q, d, s16);
    __align__(16) __half h[8];
#pragma unroll
    for (int c = 0; c < 8; c++)
        h[c] = __int2half_rn((int)(int8_t)(((c < 4 ? q.x : q.y) >> (8 * (c & 3))) & 0xff));
    *reinterpret_cast<uint4 *>(aq + r * K + b * TMOE_QK + 8 * lane) = *reinterpret_cast<const uint4 *>(h);
    const int s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 2);  // lanes 4s hold sub-block s's sum
    if ((lane & 3) == 0) {
        const int sb = lane >> 2, hi = s32 >> 6, lo = s32 - 64 * hi;  // 64 hi in [-4096, 4032]: exact
        __half2 pr = __halves2half2(__int2half_rn(64 * hi), __int2half_rn(lo));
        *reinterpret_cast<__half2 *>(ab + (r * nb + b) * 16 + 2 * sb) = pr;
    }
    if (lane == 0) ad[r * nb + b] = d;
}

// Row r of the expert-sorted A operands = row perm[r] / x_div of the per-token ones: fp16 q_x
// [K], d [K/256], block sums [K/256][16].  One warp per row, 16-byte copies.
__global__ void gather_gateup_a_kernel(const __half *__restrict__ aq_t, const float *__restrict__ ad_t,
                                       const __half *__restrict__ ab_t, const int32_t *__restrict__ perm,
                                       int n_rows, const int32_t *__restrict__ n_valid, int x_div, int K,
                                       __half *__restrict__ aq, float *__restrict__ ad, __half *__restrict__ ab) {
    const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= n_rows || (n_valid && r >= n_valid[0])) return;  // past the dispatched pairs: no tile reads them
    int p = perm[r];
    if (p < 0) p = 0;
    const int64_t t = p / x_div;
    const int nb = K / TMOE_QK;
    const uint4 *sq = reinterpret_cast<const uint4 *>(aq_t + t * K);
    uint4 *dq = reinterpret_cast<uint4 *>(aq + r * K);
    for (int i = lane; i < K / 8; i += 32) dq[i] = __ldg(sq + i);
    const uint4 *sb = reinterpret_cast<const uint4 *>(ab_t + t * nb * 16);
    uint4 *db = reinterpret_cast<uint4 *>(ab + r * nb * 16);
    for (int i = lane; i < nb * 2; i += 32) db[i] = __ldg(sb + i);
    for (int i = lane; i < nb; i += 32) ad[r * nb + i] = __ldg(ad_t + t * nb + i);
}

// pf_decode over tables staged in shared memory (tile_start [na + 1], active [na]).
__device__ __forceinline__ void gu_decode(const int *ts, const int4 *act, int na, int tile, int &ai, int &m, int &n) {
    int lo = 0, hi = na - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (ts[mid] <= tile) lo = mid;
        else hi = mid - 1;
    }
    ai = lo;
    const int4 info = act[ai];
    const int m_tiles = (info.z - info.y + PF_BM - 1) / PF_BM;
    const int local = tile - ts[ai];
    n = local / m_tiles;
    m = local % m_tiles;
}

struct GuArgs {
    const uint8_t *gate, *up;
    size_t nb1, nb2_gate, nb2_up;
    int K, I;  // H, n_ff
    const int4 *active;
    const int32_t *n_active;
    int max_active;
    const int *tile_start;
    const float *ad;  // d of the rows' Q8_K blocks
    int n_rows;
    float *act;       // [rows][I], expert-sorted rows
    int *err;
};
struct GuMaps {
    CUtensorMap aq;  // fp16 [rows][K], box 64 x 128, 128-byte swizzle
    CUtensorMap ab;  // fp16 [rows][K/256 * 16], box 8 x 128, no swizzle
};

// Bounded waits of the roles; a timeout latches the error and stops the role (and the CTA).
#define GU_WAIT(bar, ph)                                                                                   \
    if (!mbar_wait_bounded(bar, ph)) {                                                                     \
        latch_error(a.err, TMOE_DEV_ERR_TIMEOUT);                                                          \
        *abort_flag = 1;                                                                                   \
        goto done;                                                                                         \
    }
#define GU_WAIT_WARP(bar, ph)                                                                              \
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(bar, ph))) {                                            \
        if (lane == 0) latch_error(a.err, TMOE_DEV_ERR_TIMEOUT);                                           \
        *abort_flag = 1;                                                                                   \
        goto done;                                                                                         \
    }

__global__ void __launch_bounds__(GU_THREADS, 1) prefill_gateup_kernel(const __grid_constant__ GuMaps maps,
                                                                        const GuArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *sA = smem;                                  // [GU_S][128 x 64 fp16, sw128]
    uint8_t *sB = sA + GU_S * PF_A_BYTES;                // [GU_S][128 x 64 fp16, sw128]
    uint8_t *sAp = sB + GU_S * PF_A_BYTES;               // [2][min operand A]
    uint8_t *sBp = sAp + 2 * GU_AP_BYTES;                // [2][hi, lo][min operand B]
    uint8_t *sRaw = sBp + 4 * GU_AP_BYTES;               // [GU_RAWN][128 rows x 144 B], the dequant prefetch
    float2 *scl = reinterpret_cast<float2 *>(sRaw + GU_RAWN * GU_RAW_BYTES);  // [2][128] {fold scale, 0}
    uint64_t *bars = reinterpret_cast<uint64_t *>(scl + 2 * 128);
    uint64_t *fa = bars, *ea = fa + GU_S, *fb = ea + GU_S, *eb = fb + GU_S;
    uint64_t *fap = eb + GU_S, *eap = fap + 2, *fbp = eap + 2, *ebp = fbp + 2, *fsc = ebp + 2, *esc = fsc + 2;
    uint64_t *tf = esc + 2, *te = tf + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(te + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *s_ts = reinterpret_cast<int *>(smem + GU_FIXED);  // tile tables: tile_start [na + 1], active [na]
    int4 *s_act = reinterpret_cast<int4 *>(s_ts + ((a.max_active + 4) & ~3));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int na = a.n_active[0];
    if (na > a.max_active || na < 0) na = na < 0 ? 0 : a.max_active;
    for (int i = threadIdx.x; i <= na; i += blockDim.x) s_ts[i] = na > 0 ? __ldg(a.tile_start + i) : 0;
    for (int i = threadIdx.x; i < na; i += blockDim.x) s_act[i] = __ldg(a.active + i);

    if (threadIdx.x == 0) {
        for (int s = 0; s < GU_S; s++) {
            mbar_init(&fa[s], 1);
            mbar_init(&ea[s], 1);
            mbar_init(&fb[s], 4);
            mbar_init(&eb[s], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&fap[i], 1);
            mbar_init(&eap[i], 1);
            mbar_init(&fbp[i], 4);
            mbar_init(&ebp[i], 1);
            mbar_init(&fsc[i], 4);
            mbar_init(&esc[i], 8);
            mbar_init(&tf[i], 1);
            mbar_init(&te[i], 8);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, GU_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int n_tiles = na > 0 ? s_ts[na] : 0;
    const int nb = a.K / TMOE_QK;

    if (warp == 0) {
        if (lane == 0) {  // TMA: q_x stages and the blocks' sums
            int it_s = 0, it_b = 0;
            for (int tile = blockIdx.x; tile < n_tiles && !*abort_flag; tile += gridDim.x) {
                int ai, m, n;
                gu_decode(s_ts, s_act, na, tile, ai, m, n);
                const int row0 = s_act[ai].y + m * PF_BM;
                for (int b = 0; b < nb; b++, it_b++) {
                    const int i = it_b & 1;
                    if (it_b >= 2) GU_WAIT(&eap[i], ((it_b >> 1) - 1) & 1);
                    mbar_arrive_expect_tx(&fap[i], (uint32_t)GU_AP_BYTES);
                    tma_load_2d(sAp + i * GU_AP_BYTES, &maps.ab, 16 * b, row0, &fap[i]);
                    tma_load_2d(sAp + i * GU_AP_BYTES + GU_AP_BYTES / 2, &maps.ab, 16 * b + 8, row0, &fap[i]);
                    for (int st = 0; st < 4; st++, it_s++) {
                        const int s = it_s % GU_S;
                        if (it_s >= GU_S) GU_WAIT(&ea[s], ((it_s / GU_S) - 1) & 1);
                        mbar_arrive_expect_tx(&fa[s], (uint32_t)PF_A_BYTES);
                        tma_load_2d(sA + s * PF_A_BYTES, &maps.aq, TMOE_QK * b + 64 * st, row0, &fa[s]);
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA
            constexpr uint32_t idesc = idesc_f16(PF_BM, 128);
            int it_s = 0, it_b = 0;
            for (int tile = blockIdx.x; tile < n_tiles && !*abort_flag; tile += gridDim.x) {
                for (int b = 0; b < nb; b++, it_b++) {
                    const int buf = it_b & 1;
                    if (it_b >= 2) GU_WAIT(&te[buf], ((it_b >> 1) - 1) & 1);
                    tc_fence_after();
                    const uint32_t dmain = tmem_base + (uint32_t)(buf * 128);
                    for (int st = 0; st < 4; st++, it_s++) {
                        const int s = it_s % GU_S;
                        GU_WAIT(&fa[s], (it_s / GU_S) & 1);
                        GU_WAIT(&fb[s], (it_s / GU_S) & 1);
                        tc_fence_after();
                        const uint32_t sa = smem_u32(sA + s * PF_A_BYTES), sb = smem_u32(sB + s * PF_A_BYTES);
#pragma unroll
                        for (int k = 0; k < 4; k++)
                            umma_f16(dmain, sw128_desc(sa + 32 * k), sw128_desc(sb + 32 * k), idesc, (st | k) != 0);
                        umma_commit(&ea[s]);
                        umma_commit(&eb[s]);
                    }
                    GU_WAIT(&fap[buf], (it_b >> 1) & 1);
                    GU_WAIT(&fbp[buf], (it_b >> 1) & 1);
                    tc_fence_after();
                    // the min term joins the block's accumulator: A' = [64 hi, lo] x B' = c split
                    // exactly into two fp16 parts (c_hi, then c_lo), c = -(dmin / s) * m
                    const uint64_t ap = kmajor_plain_desc(smem_u32(sAp + buf * GU_AP_BYTES));
                    umma_f16(dmain, ap, kmajor_plain_desc(smem_u32(sBp + buf * 2 * GU_AP_BYTES)), idesc, 1u);
                    umma_f16(dmain, ap, kmajor_plain_desc(smem_u32(sBp + buf * 2 * GU_AP_BYTES + GU_AP_BYTES)), idesc,
                             1u);
                    umma_commit(&eap[buf]);
                    umma_commit(&ebp[buf]);
                    umma_commit(&tf[buf]);
                }
            }
        }
    } else if (warp < 6) {  // dequantise: thread n = weight row n of the tile (0-63 gate, 64-127 up)
        const int n = threadIdx.x - 64;
        int it_s = 0, it_b = 0;
        // the CTA's (tile, block) sequence; each block's 144 raw bytes are copied (cp.async) into one
        // of GU_RAWN buffers two steps before the block is dequantised
        auto row_of = [&](int t) {
            int ai, m, nt;
            gu_decode(s_ts, s_act, na, t, ai, m, nt);
            const int e = s_act[ai].x;
            const int f = nt * 64 + (n & 63);
            return n < 64 ? a.gate + (size_t)e * a.nb2_gate + (size_t)f * a.nb1
                          : a.up + (size_t)e * a.nb2_up + (size_t)f * a.nb1;
        };
        uint8_t *my_raw = sRaw + n * TMOE_Q4K_BYTES;  // + buffer * GU_RAW_BYTES
        int tile = blockIdx.x, b = 0;                   // the block being dequantised
        int pt = blockIdx.x, pb = 0;                    // the next block to prefetch
        const uint8_t *prow = pt < n_tiles ? row_of(pt) : nullptr;
        int rb = 0, pbuf = 0;
        auto prefetch = [&]() {
            if (pt < n_tiles) {
                uint8_t *dst = my_raw + pbuf * GU_RAW_BYTES;
                const uint8_t *src = prow + (size_t)pb * TMOE_Q4K_BYTES;
#pragma unroll
                for (int i = 0; i < 9; i++) cp_async16(dst + 16 * i, src + 16 * i);
                if (++pb == nb) {
                    pb = 0;
                    pt += gridDim.x;
                    if (pt < n_tiles) prow = row_of(pt);
                }
            }
            cp_async_commit();
            pbuf = pbuf + 1 == GU_RAWN ? 0 : pbuf + 1;
        };
        prefetch();
        prefetch();
        const uint32_t EXP2 = 0x64006400u;  // fp16 1024 in both halves
        float fn = 1.0f;                    // the current block's main-value factor (see below)
        while (tile < n_tiles && !*abort_flag) {
            const uint8_t *cur = my_raw + rb * GU_RAW_BYTES;
            prefetch();        // two blocks ahead
            cp_async_wait2();  // this block's copies are done
            uint4 raw[9];
#pragma unroll
            for (int i = 0; i < 9; i++) raw[i] = reinterpret_cast<const uint4 *>(cur)[i];
            rb = rb + 1 == GU_RAWN ? 0 : rb + 1;
            if (++b == nb) {
                b = 0;
                tile += gridDim.x;
            }
            const uint32_t w0 = raw[0].x, sc0 = raw[0].y, sc1 = raw[0].z, sc2 = raw[0].w;
            const float d = h2f((uint16_t)(w0 & 0xffffu)), dmin = h2f((uint16_t)(w0 >> 16));
            // 6-bit scales / mins of the 8 sub-blocks, byte-packed
            const uint32_t s_lo = sc0 & 0x3f3f3f3fu, s_hi = (sc2 & 0x0f0f0f0fu) | ((sc0 >> 2) & 0x30303030u);
            const uint32_t m_lo = sc1 & 0x3f3f3f3fu, m_hi = ((sc2 >> 4) & 0x0f0f0f0fu) | ((sc1 >> 2) & 0x30303030u);
            const int i2 = it_b & 1;
            if (it_b >= 2) {
                GU_WAIT_WARP(&esc[i2], ((it_b >> 1) - 1) & 1);
                GU_WAIT_WARP(&ebp[i2], ((it_b >> 1) - 1) & 1);
            }
            // The block's fold scale sn and the factor fn of its main values: normally sn = d and fn = 1
            // (the main values sc * q stay exact integers).  Rows whose min scale dwarfs d (|dmin| >
            // 1024 |d|, or d = 0) fold with sn = |dmin| / 1024 instead, so that c below stays within
            // fp16; their main values, a tiny share of the dot there, are then rounded to fp16.
            const bool normal = d != 0.0f && fabsf(dmin) <= 1024.0f * fabsf(d);
            const float sn = normal ? d : (dmin != 0.0f ? fabsf(dmin) * (1.0f / 1024.0f) : 1.0f);
            fn = normal ? 1.0f : __fdiv_rn(d, sn);
            const float rm = -__fdiv_rn(dmin, sn);
            scl[i2 * 128 + n] = make_float2(sn, 0.0f);
            {  // min operand row n: c_s = rm * m_s at K 2s and 2s+1 (against 64 hi_s and lo_s), as
               // c_hi (first operand) + c_lo (second), each fp16
                uint32_t wh[8], wl[8];
#pragma unroll
                for (int sb = 0; sb < 8; sb++) {
                    const int mv = (int)((sb < 4 ? m_lo : m_hi) >> (8 * (sb & 3))) & 0xff;
                    const float c = __fmul_rn(rm, (float)mv);
                    const __half ch = __float2half_rn(c);
                    const __half cl = __float2half_rn(__fsub_rn(c, __half2float(ch)));
                    wh[sb] = h2_bits(__halves2half2(ch, ch));
                    wl[sb] = h2_bits(__halves2half2(cl, cl));
                }
                uint8_t *bp = sBp + i2 * 2 * GU_AP_BYTES + n * 16;
                *reinterpret_cast<uint4 *>(bp) = make_uint4(wh[0], wh[1], wh[2], wh[3]);
                *reinterpret_cast<uint4 *>(bp + 2048) = make_uint4(wh[4], wh[5], wh[6], wh[7]);
                *reinterpret_cast<uint4 *>(bp + GU_AP_BYTES) = make_uint4(wl[0], wl[1], wl[2], wl[3]);
                *reinterpret_cast<uint4 *>(bp + GU_AP_BYTES + 2048) = make_uint4(wl[4], wl[5], wl[6], wl[7]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&fsc[i2]);
                mbar_arrive(&fbp[i2]);
            }
#pragma unroll
            for (int st = 0; st < 4; st++) {
                const int s = (it_s + st) % GU_S;
                if (it_s + st >= GU_S) GU_WAIT_WARP(&eb[s], (((it_s + st) / GU_S) - 1) & 1);
                // K [64 st, 64 st + 64): low nibbles of qs[32 st ..] (sub-block 2 st), then high nibbles
                // (sub-block 2 st + 1).  fp16 of a nibble pair by exponent magic: (1024 + q) * sc -
                // 1024 * sc = q * sc; for the high nibble in place (1024 + 16 q) * sc/16 - 64 sc.  All
                // values and products stay integers below 2^11 x 2^5: exact.
                const uint4 qa = raw[1 + 2 * st], qb = raw[2 + 2 * st];
                const int scl_l = (int)((st < 2 ? s_lo : s_hi) >> (16 * (st & 1))) & 0xff;
                const int scl_h = (int)((st < 2 ? s_lo : s_hi) >> (16 * (st & 1) + 8)) & 0xff;
                // (exact for fn = 1: sc, -1024 sc, sc / 16 and -64 sc are all fp16 integers/dyadics)
                const __half ml1 = __float2half_rn(__fmul_rn(fn, (float)scl_l));
                const __half mh1 = __float2half_rn(__fmul_rn(fn, __fmul_rn((float)scl_h, 0.0625f)));
                const __half2 ml = __half2half2(ml1), al = __half2half2(__hmul(ml1, __float2half_rn(-1024.0f)));
                const __half2 mh = __half2half2(mh1), ah = __half2half2(__hmul(mh1, __float2half_rn(-1024.0f)));
                const uint32_t wq[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                uint8_t *brow = sB + s * PF_A_BYTES + n * 128;
#pragma unroll
                for (int c = 0; c < 8; c++) {  // 16-byte chunk c: elements 8c .. 8c+7
                    uint32_t hv[4];
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const int el = 8 * c + 2 * u;  // element pair el, el + 1 (same sub-block)
                        const int src = el & 31;       // byte of the 32 qs bytes
                        const uint32_t t = __byte_perm(wq[src >> 2], 0u, (src & 2) ? 0x4342u : 0x4140u);
                        __half2 v;
                        if (el < 32) {
                            const uint32_t bits = (t & 0x000f000fu) | EXP2;
                            memcpy(&v, &bits, 4);
                            v = __hfma2(v, ml, al);
                        } else {
                            const uint32_t bits = (t & 0x00f000f0u) | EXP2;
                            memcpy(&v, &bits, 4);
                            v = __hfma2(v, mh, ah);
                        }
                        hv[u] = h2_bits(v);
                    }
                    *reinterpret_cast<uint4 *>(brow + 16 * (c ^ (n & 7))) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&fb[s]);
            }
            it_s += 4;
            it_b++;
        }
    } else {  // epilogue: warps 6-13
        const int q = warp & 3, h = (warp - 6) >> 2;
        int it_b = 0;
        for (int tile = blockIdx.x; tile < n_tiles && !*abort_flag; tile += gridDim.x) {
            int ai, m, nt;
            gu_decode(s_ts, s_act, na, tile, ai, m, nt);
            const int4 info = s_act[ai];
            const int r = info.y + m * PF_BM + q * 32 + lane;
            const bool valid = r < info.z && r < a.n_rows;
            float tg[32], tu[32];
#pragma unroll
            for (int c = 0; c < 32; c++) tg[c] = tu[c] = 0.0f;
            float dx_next = valid ? __ldg(a.ad + (int64_t)r * nb) : 0.0f;
            for (int b = 0; b < nb; b++, it_b++) {
                const float dx = dx_next;  // loaded one block ahead
                if (b + 1 < nb) dx_next = valid ? __ldg(a.ad + (int64_t)r * nb + b + 1) : 0.0f;
                const int buf = it_b & 1;
                GU_WAIT_WARP(&tf[buf], (it_b >> 1) & 1);
                GU_WAIT_WARP(&fsc[buf], (it_b >> 1) & 1);
                tc_fence_after();
                const uint32_t taddr = tmem_base + (uint32_t)(buf * 128) + ((uint32_t)(q * 32) << 16);
                const float4 *sg = reinterpret_cast<const float4 *>(scl + buf * 128 + 32 * h);  // {sn, 0} x 2
                const float4 *su = sg + 32;
                float v[32];
                tmem_ld32(taddr + 32 * h, v);  // gate features 32h ..
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    const float4 s4 = sg[i >> 1];
                    tg[i] = __fmaf_rn(dx * s4.x, v[i], tg[i]);
                    tg[i + 1] = __fmaf_rn(dx * s4.z, v[i + 1], tg[i + 1]);
                }
                tmem_ld32(taddr + 64 + 32 * h, v);  // up features 32h ..
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    const float4 s4 = su[i >> 1];
                    tu[i] = __fmaf_rn(dx * s4.x, v[i], tu[i]);
                    tu[i + 1] = __fmaf_rn(dx * s4.z, v[i + 1], tu[i + 1]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&te[buf]);
                    mbar_arrive(&esc[buf]);
                }
            }
            if (valid) {
                float *orow = a.act + (int64_t)r * a.I + nt * 64 + 32 * h;
#pragma unroll
                for (int c = 0; c < 32; c += 4)
                    *reinterpret_cast<float4 *>(orow + c) =
                        make_float4(silu_mul_pf(tg[c], tu[c]), silu_mul_pf(tg[c + 1], tu[c + 1]),
                                    silu_mul_pf(tg[c + 2], tu[c + 2]), silu_mul_pf(tg[c + 3], tu[c + 3]));
            }
        }
    }
done:
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem_base, GU_TMEM_COLS);
    }
}
#undef GU_WAIT
#undef GU_WAIT_WARP

// ------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 pf_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

// fp16 [rows][K] with a box of 64 columns x box_rows rows, 128-byte swizzle.
static bool encode_f16_rows(CUtensorMap *m, const void *base, int64_t rows, int K, int box_rows) {
    const PFN_cuTensorMapEncodeTiled_v12000 enc = pf_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)PF_BK, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1u, 1u};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_prep_rows(const float *src, const int32_t *perm, int n_rows, const int32_t *n_valid, int x_div,
                             int K, __half *dst, cudaStream_t st) {
    if (n_rows <= 0) return cudaSuccess;
    const int64_t warps = (int64_t)n_rows * (K / TMOE_QK);
    prep_rows_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(src, perm, n_rows, n_valid, x_div, K, dst);
    return cudaGetLastError();
}

cudaError_t launch_dequant_f16(int wt, const uint8_t *w, size_t nb2, int N, int K, const int4 *active,
                               const int32_t *n_active, int max_active, __half *dst, cudaStream_t st) {
    if (max_active <= 0 || N <= 0) return cudaSuccess;
    const size_t row_bytes = (size_t)(K / TMOE_QK) * (wt == TMOE_WT_Q4K ? TMOE_Q4K_BYTES : TMOE_Q6K_BYTES);
    const size_t smem = DQ_ROWS * row_bytes;
    // 16-byte staging: the expert slabs and every DQ_ROWS-row run start on a 16-byte boundary
    if ((reinterpret_cast<uintptr_t>(w) & 15) || (nb2 & 15) || (smem & 15) || (N % DQ_ROWS && (row_bytes & 15)) ||
        smem > 200 * 1024 || max_active > 65535)
        return cudaErrorInvalidValue;
    const dim3 grid((unsigned)((N + DQ_ROWS - 1) / DQ_ROWS), (unsigned)max_active);
    if (wt == TMOE_WT_Q6KR && N % DQ_ROWS) return cudaErrorInvalidValue;  // whole 8-row groups per CTA
    auto kern = wt == TMOE_WT_Q4K    ? dequant_f16_kernel<TMOE_WT_Q4K>
                : wt == TMOE_WT_Q6KR ? dequant_f16_kernel<TMOE_WT_Q6KR>
                                     : dequant_f16_kernel<TMOE_WT_Q6K>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    kern<<<grid, 256, smem, st>>>(w, nb2, N, K, active, n_active, max_active, dst);
    return cudaGetLastError();
}

// The Q8_K of the T token rows (token order), then their copies in expert-sorted pair order.
cudaError_t launch_prep_gateup_a(const float *x, int T, const int32_t *perm, int n_rows, const int32_t *n_valid,
                                 int x_div, int K, __half *aq_t, float *ad_t, __half *ab_t, __half *aq, float *ad,
                                 __half *ab, bool tokens_ready, cudaStream_t st) {
    if (n_rows <= 0 || T <= 0) return cudaSuccess;
    if (!tokens_ready) {
        const int64_t warps = (int64_t)T * (K / TMOE_QK);
        prep_gateup_a_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(x, nullptr, T, 1, K, aq_t, ad_t, ab_t);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    gather_gateup_a_kernel<<<(unsigned)((n_rows + 7) / 8), 256, 0, st>>>(aq_t, ad_t, ab_t, perm, n_rows, n_valid,
                                                                         x_div, K, aq, ad, ab);
    return cudaGetLastError();
}

static bool encode_f16_plain(CUtensorMap *m, const void *base, int64_t rows, int cols, int box_cols, int box_rows) {
    const PFN_cuTensorMapEncodeTiled_v12000 enc = pf_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1u, 1u};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// act[r][I] (expert-sorted rows) = silu(x . gate^T) * (x . up^T) for Q4_K gate/up, exact block sums.
cudaError_t launch_prefill_gateup(const __half *aq, const float *ad, const __half *ab, int n_rows, int K, int I,
                                  const uint8_t *gate, const uint8_t *up, size_t nb1, size_t nb2_gate,
                                  size_t nb2_up, const int4 *active, const int32_t *n_active, int max_active,
                                  int *tile_start, float *act, int *err, int sm_count, cudaStream_t st) {
    if (n_rows <= 0) return cudaSuccess;
    if (I % 64 || K % TMOE_QK) return cudaErrorInvalidValue;
    tiles_kernel<<<1, 1024, 0, st>>>(active, n_active, max_active, I / 64, tile_start);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    GuMaps maps;
    memset(&maps, 0, sizeof maps);
    if (!encode_f16_rows(&maps.aq, aq, n_rows, K, PF_BM)) return cudaErrorInvalidValue;
    if (!encode_f16_plain(&maps.ab, ab, n_rows, (K / TMOE_QK) * 16, 8, PF_BM)) return cudaErrorInvalidValue;
    GuArgs a{gate, up, nb1, nb2_gate, nb2_up, K, I, active, n_active, max_active, tile_start, ad, n_rows, act, err};
    static int set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    const size_t tables = (size_t)((max_active + 4) & ~3) * 4 + (size_t)max_active * 16;
    const size_t smem = GU_FIXED + tables + 1024;
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    if ((int)smem > set[dev]) {
        e = cudaFuncSetAttribute(prefill_gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        set[dev] = (int)smem;
    }
    prefill_gateup_kernel<<<sm_count, GU_THREADS, smem, st>>>(maps, a);
    return cudaGetLastError();
}

bool prefill_fits(int H, int I) { return H % PF_BN == 0 && I % (PF_BN / 2) == 0 && H % PF_BK == 0 && I % PF_BK == 0; }

// gate/up (swiglu = true: act[r][I] from A1 [rows][H]) or down (dout[perm[r]][H] from A2 [rows][I]).
cudaError_t launch_prefill_gemm(bool swiglu, const __half *A, int n_rows, int K, const __half *b0, const __half *b1,
                                int n_slots, int N, const int4 *active, const int32_t *n_active, int max_active,
                                int *tile_start, const int32_t *perm, float *out, int *err, int sm_count,
                                cudaStream_t st) {
    if (n_rows <= 0) return cudaSuccess;
    const int n_tiles_n = swiglu ? N / (PF_BN / 2) : N / PF_BN;
    tiles_kernel<<<1, 1024, 0, st>>>(active, n_active, max_active, n_tiles_n, tile_start);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    PfMaps maps;
    memset(&maps, 0, sizeof maps);
    if (!encode_f16_rows(&maps.a, A, n_rows, K, PF_BM)) return cudaErrorInvalidValue;
    if (!encode_f16_rows(&maps.b0, b0, (int64_t)n_slots * N, K, swiglu ? PF_BN / 2 : PF_BN))
        return cudaErrorInvalidValue;
    if (swiglu && !encode_f16_rows(&maps.b1, b1, (int64_t)n_slots * N, K, PF_BN / 2)) return cudaErrorInvalidValue;
    PfArgs a{K, N, n_tiles_n, active, n_active, max_active, tile_start, perm, n_rows, out, err};
    static int set1[64] = {}, set2[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    int *set = swiglu ? set1 : set2;
    if (!set[dev]) {
        e = swiglu ? cudaFuncSetAttribute(prefill_gemm_kernel<PF_SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          PF_SMEM)
                   : cudaFuncSetAttribute(prefill_gemm_kernel<PF_SCATTER>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, PF_SMEM);
        if (e != cudaSuccess) return e;
        set[dev] = 1;
    }
    if (swiglu)
        prefill_gemm_kernel<PF_SWIGLU><<<sm_count, PF_THREADS, PF_SMEM, st>>>(maps, a);
    else
        prefill_gemm_kernel<PF_SCATTER><<<sm_count, PF_THREADS, PF_SMEM, st>>>(maps, a);
    return cudaGetLastError();
}

}  // namespace tmoe
