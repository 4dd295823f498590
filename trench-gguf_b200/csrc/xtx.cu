// xtx.cu - the Hessian of a layer's inputs, H += X^T X (trench-gguf tools/hessian_from_dump.py:73-79 `_xtx`: a float32
// GEMM a row chunk, accumulated in float64), on sm_100a's fifth-generation tensor cores.
//
// What is computed: for X [rows][dim] (float32, or bf16 as the activation dumps hold it) and an optional per-row scale
// s (a gated Hessian's routing weight, applied as x * s in float32 as the reference does), H[i][j] += f64(S_ij) with
// S_ij = sum_r x'_ri x'_rj float32-accurate; H float64 [dim][dim] row-major, kept exactly symmetric.
//
// How. Float32 is not a tensor-core operand, so each x' is split exactly into three bf16 parts, x' = h + m + l
// (h = bf16(x'), m = bf16(x' - h), l = bf16(x' - h - m): three 8-bit significands hold float32's 24), and
// x'_i x'_j = hh + hm + mh + mm + hl + lh + (ml + lm + ll, below 2^-24 of the product: left out) - six bf16 products
// summed in float32 in tensor memory. The tensor cores' float32 accumulation does not round to nearest (a single
// product of parts is off by up to an ulp), so the large term and the five small ones go to two accumulators: the
// small ones' own rounding then sits 2^-8 below the large sum, and the two are added in float64. A bf16 source
// without a scale is its own h: one product, one accumulator.
//  * k_xtx_planes: one pass over X writes the parts transposed into "planes" laid out as the tensor core reads its
//    shared-memory operands (K-major, no swizzle: core matrices of 8 columns of X x 16 bytes = 8 rows of X; a tile is
//    32 rows of X (the products' K) deep), so every operand tile is one contiguous 8 KB (128 columns) or 16 KB (256
//    columns) piece that a single 1-D TMA bulk copy moves.
//  * k_xtx_mma: one CTA a 128 x 256 tile of H that reaches the diagonal or above it (the lower triangle is written as
//    the upper's mirror). One thread keeps NS stages of every part's A (128 columns) and B (256 columns) tiles in
//    flight (cp.async.bulk, completion counted by mbarrier transaction bytes); one thread issues tcgen05.mma
//    (kind::f16, bf16 in, float32 accumulate, M 128, N 128, K 16) into float32 accumulators in tensor memory and
//    hands each stage back with tcgen05.commit. The work runs in units of (1,024 rows of X, one 128-column half of
//    the tile), each with its own accumulator columns, so tensor memory is double-buffered: while the tensor cores
//    compute unit u + 1, four epilogue warps read unit u out (tcgen05.ld, a row i a thread), give its columns back
//    (an mbarrier) and add the float64 sums to H[j][i] for j >= i - the lower triangle, where a warp's 32 rows i are
//    32 consecutive doubles of row j: coalesced - every element by exactly one thread, no atomics.
//  * k_xtx_mirror: the upper triangle as the lower's transpose through shared memory (coalesced both ways).
//    So each float32 (truncating) sum runs over at most 1,024 rows: float32-accurate like a float32 GEMM, and the
//    segment sums are added in float64 like the reference's chunks. Every wait is bounded: a wait that runs out sets ST_TIMEOUT in the status word,
//    the CTA lets its own copies and products finish (bounded again), frees its tensor memory and returns.
#include <cstdint>
#include <cuda_bf16.h>
#include "common.cuh"
#include "kernels.h"

namespace gq {
namespace {

constexpr int XT_K = 32;                          // rows of X (the products' K) a tile
constexpr int XT_UNIT = 8 * XT_K * 2;             // 8 columns x 32 rows of bf16: 4 core matrices of 8 x 16 bytes
constexpr int XT_BM = 128, XT_BN = 256;           // the tile of H (rows x columns)
constexpr int XT_ABYTES = XT_BM / 8 * XT_UNIT;    // 8 KB
constexpr int XT_NH = 128;                        // the columns of one product (N): half the tile
constexpr int XT_HBYTES = XT_NH / 8 * XT_UNIT;    // 8 KB: a half of the B tile
// [large | small] float32 accumulators, each two halves of 128: all of an SM's tensor memory. One CTA an SM is all
// the shared memory allows, so no other CTA of this kernel waits on the allocation; a CTA of another kernel holding
// columns (a library GEMM on another stream) only delays it until that CTA ends
constexpr int XT_TMEM_COLS = 512;
constexpr int XT_SEG = 32;                        // K tiles (1,024 rows of X) summed in float32 before float64
constexpr int XT_THREADS = 192, XT_EPI_THREADS = 128;   // warp 0 copies, warp 1 multiplies, warps 2-5 the epilogue
constexpr int XT_SMEM_BUDGET = 220 * 1024;
constexpr unsigned XT_SPIN = 1u << 24;            // try_wait rounds before a wait is declared lost

template <int NP> struct XtCfg {
    static constexpr int STAGE = NP * (XT_ABYTES + XT_HBYTES);
    static constexpr int NS = XT_SMEM_BUDGET / STAGE > 8 ? 8 : XT_SMEM_BUDGET / STAGE;   // 3 parts: 4, one part: 8
    static constexpr int SMEM = NS * STAGE;
    static constexpr int NPROD = NP == 3 ? 6 : 1;   // part products a stage
};

// the six part products (A part, B part): hh, hm, mh, mm, hl, lh
__constant__ int8_t c_pa[6] = {0, 0, 1, 1, 0, 2};
__constant__ int8_t c_pb[6] = {0, 1, 0, 1, 2, 0};

__device__ __forceinline__ uint32_t smem_addr(const void * p) { return (uint32_t) __cvta_generic_to_shared(p); }

__device__ __forceinline__ bool xt_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool xt_wait(uint32_t bar, uint32_t parity) {
    for (unsigned it = 0; it < XT_SPIN; ++it) if (xt_try(bar, parity)) return true;
    return false;
}

// shared-memory operand descriptor, K-major without swizzle: start address, the byte offset between the two core
// matrices of a K-16 step (LBO: next 8 rows of X, 128 B) and between 8-column groups (SBO: one unit, 512 B); bits
// 46-47 = 1 (the sm_100 descriptor version)
__device__ __forceinline__ uint64_t xt_desc(uint32_t saddr) {
    return (uint64_t) ((saddr >> 4) & 0x3FFFu) | ((uint64_t) (128 >> 4) << 16) | ((uint64_t) (XT_UNIT >> 4) << 32) |
           (1ull << 46);
}
// instruction descriptor of kind::f16: float32 accumulator (bits 4-5 = 1), A and B bf16 (bits 7-9, 10-12 = 1), both
// K-major (bits 15, 16 = 0), N / 8 at bits 17-22, M / 16 at bits 24-28
constexpr uint32_t XT_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t) (XT_NH >> 3) << 17) |
                              ((uint32_t) (XT_BM >> 4) << 24);

__device__ __forceinline__ void xt_mma(uint32_t tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                 ::"r"(tmem), "l"(a), "l"(b), "r"(XT_IDESC), "r"(accumulate) : "memory");
}
__device__ __forceinline__ void xt_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive float32 columns of this warp's 32 lanes (one row a thread)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
                 "%14, %15}, [%16];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                   "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                 : "r"(taddr));
}

__device__ __forceinline__ uint16_t to_bf16(float v) { return __bfloat16_as_ushort(__float2bfloat16_rn(v)); }
__device__ __forceinline__ float from_bf16(uint16_t b) { return __uint_as_float((uint32_t) b << 16); }

// parts of 8 rows of X (8 kc .. 8 kc + 7) of column i, written as one 16-byte row of a core matrix in every plane
template <int SRC, int NP>
__global__ void __launch_bounds__(256) k_xtx_planes(const void * __restrict__ x, int64_t ldx, const float * __restrict__ scale,
                                                    int64_t rows, int64_t dim, int64_t dim_pad, int64_t kc_count,
                                                    uint8_t * __restrict__ planes, int64_t plane_bytes) {
    const int64_t i = (int64_t) blockIdx.x * 256 + threadIdx.x;
    for (int64_t kc = blockIdx.y; kc < kc_count; kc += gridDim.y) {
        uint32_t w[NP][4];
#pragma unroll
        for (int p = 0; p < NP; ++p) w[p][0] = w[p][1] = w[p][2] = w[p][3] = 0;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int64_t r = kc * 8 + e;
            float v = 0.0f;
            uint16_t hb = 0;
            if (r < rows && i < dim) {
                if constexpr (SRC == SRC_BF16) {
                    hb = static_cast<const uint16_t *>(x)[r * ldx + i];
                    v = from_bf16(hb);
                } else {
                    v = static_cast<const float *>(x)[r * ldx + i];
                }
                if (scale) v = v * scale[r];
            }
            uint16_t part[NP];
            if constexpr (NP == 1) {
                part[0] = (SRC == SRC_BF16 && !scale) ? hb : to_bf16(v);
            } else {
                part[0] = to_bf16(v);
                const float r1 = v - from_bf16(part[0]);          // exact (Sterbenz)
                part[1] = to_bf16(r1);
                part[2] = to_bf16(r1 - from_bf16(part[1]));       // exact: what is left fits 8 bits
            }
#pragma unroll
            for (int p = 0; p < NP; ++p) w[p][e >> 1] |= (uint32_t) part[p] << (16 * (e & 1));
        }
        const int64_t off = ((kc / 4) * (dim_pad / 8) + i / 8) * XT_UNIT + (kc % 4) * 128 + (i % 8) * 16;
#pragma unroll
        for (int p = 0; p < NP; ++p)
            *reinterpret_cast<uint4 *>(planes + p * plane_bytes + off) = make_uint4(w[p][0], w[p][1], w[p][2], w[p][3]);
    }
}

template <int NP>
__global__ void __launch_bounds__(XT_THREADS, 1) k_xtx_mma(const uint8_t * __restrict__ planes, int64_t plane_bytes,
                                                           int64_t kt_count, int64_t dim, int64_t dim_pad, int accumulate,
                                                           double * __restrict__ H, unsigned * status) {
    using C = XtCfg<NP>;
    constexpr int NS = C::NS;
    const int a_t = blockIdx.y, b_t = blockIdx.x;
    if ((int64_t) XT_BN * (b_t + 1) - 1 < (int64_t) XT_BM * a_t) return;     // wholly below the diagonal: mirrored
    extern __shared__ __align__(1024) uint8_t xs[];
    __shared__ __align__(8) uint64_t full[NS], empty[NS], acc_full[2], acc_empty[2], done;
    __shared__ uint32_t tmem_base;
    __shared__ volatile int s_fail;
    __shared__ int64_t s_issued, s_used;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t nseg = (kt_count + XT_SEG - 1) / XT_SEG;
    // the tile's work in units u = (segment u / 2, column half u % 2): K tiles [XT_SEG seg, ..) times B's half
    // columns; unit u accumulates into the tensor-memory columns of its half, so the epilogue drains unit u while
    // the tensor cores compute unit u + 1
    const int64_t nunits = 2 * nseg;
    if (tid == 0) {
        s_fail = 0;
        s_issued = s_used = 0;
        for (int s = 0; s < NS; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&full[s])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&empty[s])) : "memory");
        }
        for (int b = 0; b < 2; ++b) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&acc_full[b])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(&acc_empty[b])), "r"(XT_EPI_THREADS) : "memory");
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&done)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_addr(&tmem_base)), "r"(XT_TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    const int64_t upk = dim_pad / 8;                      // units a K tile of a plane
    const uint8_t * a_src = planes + ((int64_t) a_t * (XT_BM / 8)) * XT_UNIT;
    const uint8_t * b_src = planes + ((int64_t) b_t * (XT_BN / 8)) * XT_UNIT;

    if (tid == 0) {                                       // producer: stage g % NS <- the g-th (unit, K tile)
        int64_t g = 0;
        for (int64_t u = 0; u < nunits && !s_fail; ++u) {
            const int64_t kt_end = (u / 2 + 1) * XT_SEG < kt_count ? (u / 2 + 1) * XT_SEG : kt_count;
            const uint8_t * bh = b_src + (u & 1) * XT_HBYTES;
            for (int64_t kt = (u / 2) * XT_SEG; kt < kt_end; ++kt, ++g) {
                const int s = (int) (g % NS);
                if (g >= NS && !xt_wait(smem_addr(&empty[s]), (uint32_t) ((g / NS - 1) & 1))) { s_fail = 1; break; }
                if (s_fail) break;
                const uint32_t bar = smem_addr(&full[s]);
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(C::STAGE) : "memory");
                uint8_t * st = xs + (size_t) s * C::STAGE;
#pragma unroll
                for (int p = 0; p < NP; ++p) {
                    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                                 ::"r"(smem_addr(st + p * XT_ABYTES)), "l"(a_src + p * plane_bytes + kt * upk * XT_UNIT),
                                   "r"(XT_ABYTES), "r"(bar) : "memory");
                    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                                 ::"r"(smem_addr(st + NP * XT_ABYTES + p * XT_HBYTES)),
                                   "l"(bh + p * plane_bytes + kt * upk * XT_UNIT), "r"(XT_HBYTES), "r"(bar) : "memory");
                }
                s_issued = g + 1;
            }
        }
    } else if (tid == 32) {                               // the MMA thread
        int64_t g = 0;
        for (int64_t u = 0; u < nunits && !s_fail; ++u) {
            const int b = (int) (u & 1);
            if (u >= 2) {                                 // unit u - 2 (same columns) has been read out
                if (!xt_wait(smem_addr(&acc_empty[b]), (uint32_t) ((u / 2 - 1) & 1))) { s_fail = 1; break; }
                tc_fence_after();
            }
            const uint32_t big = tmem + (uint32_t) (b * XT_NH), small = tmem + (uint32_t) (2 * XT_NH + b * XT_NH);
            const int64_t kt0 = (u / 2) * XT_SEG;
            const int64_t kt_end = kt0 + XT_SEG < kt_count ? kt0 + XT_SEG : kt_count;
            for (int64_t kt = kt0; kt < kt_end; ++kt, ++g) {
                const int s = (int) (g % NS);
                if (!xt_wait(smem_addr(&full[s]), (uint32_t) ((g / NS) & 1))) { s_fail = 1; break; }
                tc_fence_after();
                const uint32_t st = smem_addr(xs + (size_t) s * C::STAGE);
#pragma unroll
                for (int q = 0; q < C::NPROD; ++q) {
                    const uint32_t a0 = st + c_pa[q] * XT_ABYTES, b0 = st + NP * XT_ABYTES + c_pb[q] * XT_HBYTES;
                    const bool first = kt == kt0 && q <= 1;
#pragma unroll
                    for (int kk = 0; kk < XT_K / 16; ++kk)    // K 16 = two core matrices along K (256 bytes)
                        xt_mma(q == 0 ? big : small, xt_desc(a0 + kk * 256), xt_desc(b0 + kk * 256), !(first && kk == 0));
                }
                xt_commit(smem_addr(&empty[s]));          // the stage is free once these products are done
            }
            if (s_fail) break;
            xt_commit(smem_addr(&acc_full[b]));           // the unit's sums are ready once its products are done
        }
        s_used = g;
        xt_commit(smem_addr(&done));                      // every product issued (also after a lost wait)
    } else if (warp >= 2) {                               // epilogue: warp w reads tensor-memory lanes 32 (w % 4) ..
        const int q = warp & 3;
        const int64_t i = (int64_t) a_t * XT_BM + q * 32 + lane;        // this thread's row of the tile
        const uint32_t trow = tmem + ((uint32_t) (q * 32) << 16);
        for (int64_t u = 0; u < nunits; ++u) {
            const int b = (int) (u & 1);
            if (!xt_wait(smem_addr(&acc_full[b]), (uint32_t) ((u / 2) & 1))) { s_fail = 1; break; }
            tc_fence_after();
            const bool add = accumulate || u >= 2;
#pragma unroll 1
            for (int c0 = 0; c0 < XT_NH; c0 += 32) {
                uint32_t v[32], w[32];
                const uint32_t cb = trow + (uint32_t) (b * XT_NH + c0), cs = cb + 2 * XT_NH;
                tmem_ld16(cb, *reinterpret_cast<uint32_t (*)[16]>(v));
                tmem_ld16(cb + 16, *reinterpret_cast<uint32_t (*)[16]>(v + 16));
                if (NP == 3) {
                    tmem_ld16(cs, *reinterpret_cast<uint32_t (*)[16]>(w));
                    tmem_ld16(cs + 16, *reinterpret_cast<uint32_t (*)[16]>(w + 16));
                }
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (c0 + 32 == XT_NH) {                   // the unit's columns all read: free for unit u + 2
                    tc_fence_before();
                    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(&acc_empty[b])) : "memory");
                }
                if (i >= dim) continue;
                double t[32];                             // the unit's sums in float64 (large + small accumulator)
#pragma unroll
                for (int e = 0; e < 32; ++e)
                    t[e] = NP == 3 ? (double) __uint_as_float(v[e]) + (double) __uint_as_float(w[e])
                                   : (double) __uint_as_float(v[e]);
                // H[j][i] for j >= i - the lower triangle and the diagonal, a warp on 32 consecutive columns of row j
                // (the upper triangle is its transpose, written by k_xtx_mirror); the loads all go out first
                const int64_t j0 = (int64_t) b_t * XT_BN + b * XT_NH + c0;
                const int64_t lo = i > j0 ? i - j0 : 0, hi = dim - j0 < 32 ? dim - j0 : 32;   // e in [lo, hi) is written
                if (hi <= lo) continue;                   // (so row j0 + lo < dim: every address below is inside H)
                double * col = H + j0 * dim + i;
                if (add) {                                // every load issued before the first is used
                    double h[32];
#pragma unroll
                    for (int e = 0; e < 32; ++e) h[e] = __ldcg(col + (e >= lo && e < hi ? e : lo) * dim);
#pragma unroll
                    for (int e = 0; e < 32; ++e) t[e] += h[e];
                }
#pragma unroll
                for (int e = 0; e < 32; ++e)
                    if (e >= lo && e < hi) __stcg(col + e * dim, t[e]);
            }
            if (s_fail) break;
        }
    }
    __syncthreads();
    if (tid == 0) {                                       // products still running (a lost wait) end before the free
        if (!xt_wait(smem_addr(&done), 0)) s_fail = 1;
        if (s_fail) {                                     // report it and let this CTA's copies still in flight land
            atomicOr(status, ST_TIMEOUT);
            for (int64_t g = s_used; g < s_issued; ++g) xt_wait(smem_addr(&full[g % NS]), (uint32_t) ((g / NS) & 1));
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(XT_TMEM_COLS) : "memory");
}

// the upper triangle from the lower: H[i][j] = H[j][i] for j > i, through a 32 x 32 shared-memory tile so both the
// reads (row j of the lower block) and the writes (row i of the upper block) are coalesced
__global__ void __launch_bounds__(256) k_xtx_mirror(double * __restrict__ H, int64_t dim) {
    __shared__ double t[32][33];
    const int bi = blockIdx.y, bj = blockIdx.x;           // the upper block (rows bi, columns bj), bj >= bi
    if (bj < bi) return;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int64_t r0 = (int64_t) bj * 32, c0 = (int64_t) bi * 32;   // the lower block: rows of bj, columns of bi
#pragma unroll
    for (int k = 0; k < 32; k += 8) {
        const int64_t r = r0 + ty + k, c = c0 + tx;
        if (r < dim && c < dim) t[ty + k][tx] = H[r * dim + c];
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 32; k += 8) {
        const int64_t i = c0 + ty + k, j = r0 + tx;     // H[i][j] = lower[j][i]
        if (i < dim && j < dim && j > i) H[i * dim + j] = t[tx][ty + k];
    }
}

template <int SRC, int NP>
cudaError_t launch_planes(const void * x, int64_t ldx, const float * scale, int64_t rows, int64_t dim, int64_t dim_pad,
                          int64_t kt_count, uint8_t * planes, int64_t plane_bytes, cudaStream_t st) {
    const int64_t kc_count = kt_count * (XT_K / 8);
    const dim3 grid((unsigned) (dim_pad / 256), (unsigned) (kc_count < 8192 ? kc_count : 8192));
    k_xtx_planes<SRC, NP><<<grid, 256, 0, st>>>(x, ldx, scale, rows, dim, dim_pad, kc_count, planes, plane_bytes);
    return cudaGetLastError();
}

template <int NP>
cudaError_t launch_mma(const uint8_t * planes, int64_t plane_bytes, int64_t kt_count, int64_t dim, int64_t dim_pad,
                       int accumulate, double * H, unsigned * status, cudaStream_t st) {
    const int smem = XtCfg<NP>::SMEM;
    const cudaError_t e = cudaFuncSetAttribute(k_xtx_mma<NP>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    const dim3 grid((unsigned) (dim_pad / XT_BN), (unsigned) (dim_pad / XT_BM));
    k_xtx_mma<NP><<<grid, XT_THREADS, smem, st>>>(planes, plane_bytes, kt_count, dim, dim_pad, accumulate, H, status);
    const int64_t nb = (dim + 31) / 32;
    if (nb > 65535) return cudaErrorInvalidValue;
    k_xtx_mirror<<<dim3((unsigned) nb, (unsigned) nb), 256, 0, st>>>(H, dim);
    return cudaGetLastError();
}

}  // namespace

int xtx_parts(int src, bool scaled) { return src == SRC_BF16 && !scaled ? 1 : 3; }

size_t xtx_scratch_bytes(int src, int64_t rows, int64_t dim, bool scaled) {
    if (rows <= 0 || dim <= 0) return 0;
    const int64_t kt_count = (rows + XT_K - 1) / XT_K, dim_pad = (dim + XT_BN - 1) / XT_BN * XT_BN;
    return (size_t) xtx_parts(src, scaled) * (size_t) (kt_count * (dim_pad / 8) * XT_UNIT);
}

cudaError_t launch_xtx(int src, const void * x, int64_t ldx, const float * scale, int64_t rows, int64_t dim, double * H,
                       int accumulate, void * scratch, size_t scratch_bytes, unsigned * status, cudaStream_t st) {
    if (rows <= 0 || dim <= 0 || ldx < dim || (src != SRC_F32 && src != SRC_BF16) || !status ||
        scratch_bytes < xtx_scratch_bytes(src, rows, dim, scale != nullptr) || (reinterpret_cast<uintptr_t>(scratch) & 15))
        return cudaErrorInvalidValue;
    const int64_t kt_count = (rows + XT_K - 1) / XT_K, dim_pad = (dim + XT_BN - 1) / XT_BN * XT_BN;
    if (dim_pad / XT_BM > 65535) return cudaErrorInvalidValue;
    const int64_t plane_bytes = kt_count * (dim_pad / 8) * XT_UNIT;
    uint8_t * planes = static_cast<uint8_t *>(scratch);
    cudaError_t e;
    if (xtx_parts(src, scale != nullptr) == 1) {
        e = launch_planes<SRC_BF16, 1>(x, ldx, scale, rows, dim, dim_pad, kt_count, planes, plane_bytes, st);
        if (e == cudaSuccess) e = launch_mma<1>(planes, plane_bytes, kt_count, dim, dim_pad, accumulate, H, status, st);
    } else {
        e = src == SRC_BF16 ? launch_planes<SRC_BF16, 3>(x, ldx, scale, rows, dim, dim_pad, kt_count, planes, plane_bytes, st)
                            : launch_planes<SRC_F32, 3>(x, ldx, scale, rows, dim, dim_pad, kt_count, planes, plane_bytes, st);
        if (e == cudaSuccess) e = launch_mma<3>(planes, plane_bytes, kt_count, dim, dim_pad, accumulate, H, status, st);
    }
    return e;
}

}  // namespace gq
