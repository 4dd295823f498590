// common.cuh - shared definitions of the B200 quantizer library (libgpuq_cuda.so).
//
// Numerics contract: every kernel here reproduces ggml's float32 arithmetic bit for bit. The library is compiled
// with -fmad=false -prec-div=true -prec-sqrt=true (no FMA contraction, IEEE division and square root, no
// flush-to-zero), every expression keeps ggml's operand order, and every floating-point sum runs in ggml's index
// order inside one thread. Parallelism only ever splits independent work (trial scales, sub-blocks, candidate
// points); the choices that ggml makes sequentially are replayed sequentially.
#pragma once
#include <cstdint>
#include <cfloat>
#include <cuda_runtime.h>

namespace gq {

constexpr int QK = 256;

enum Type : int { IQ2_XXS = 16, IQ2_XS = 17, IQ3_XXS = 18, IQ1_S = 19, IQ4_NL = 20, IQ3_S = 21, IQ2_S = 22,
                  IQ4_XS = 23, IQ1_M = 29, Q8_0 = 8, Q2_K = 10, Q3_K = 11, Q4_K = 12, Q5_K = 13, Q6_K = 14,
                  Q4_0 = 2, Q5_0 = 6, Q5_1 = 7, F16 = 1 };
enum Src : int { SRC_F32 = 0, SRC_F16 = 1, SRC_Q8_0 = 8, SRC_BF16 = 30, SRC_MXFP4 = 39, SRC_NVFP4 = 40,
                 SRC_MXFP8 = 43 };

// bytes of one block of each type (ggml-common.h block_* layouts)
__host__ __device__ constexpr int block_bytes(int t) {
    return t == IQ2_XXS ? 66 : t == IQ2_XS ? 74 : t == IQ2_S ? 82 : t == IQ3_XXS ? 98 : t == IQ3_S ? 110 :
           t == IQ1_S ? 50 : t == IQ1_M ? 56 : t == IQ4_NL ? 18 : t == IQ4_XS ? 136 : t == Q2_K ? 84 :
           t == Q3_K ? 110 : t == Q4_K ? 144 : t == Q5_K ? 176 : t == Q6_K ? 210 : t == Q8_0 ? 34 :
           t == Q4_0 ? 18 : t == Q5_0 ? 22 : t == Q5_1 ? 24 : t == F16 ? 2 : 0;
}
__host__ __device__ constexpr int block_len(int t) {
    return t == F16 ? 1 : t == IQ4_NL || t == Q8_0 || t == Q4_0 || t == Q5_0 || t == Q5_1 ? 32 : QK;
}

// Source tensors. "Inline" sources are decoded by the quantize kernels themselves, in their loads (F32, F16, BF16,
// Q8_0, MXFP4); the other readable sources are "staged": one decode pass writes float32 first (NVFP4; the MXFP8 row
// layout of unsloth's type 43 - an E8M0 scale byte and 32 E4M3 bytes a block, tools/requant_table.py:8-9; and every
// 256-block k-quant and i-quant with a device to_float), after which the F32 kernels run.
// source bytes a 32-value block of an inline source, 0 for any other
__host__ __device__ constexpr int src_bytes32(int s) {
    return s == SRC_F32 ? 128 : s == SRC_F16 || s == SRC_BF16 ? 64 : s == SRC_Q8_0 ? 34 : s == SRC_MXFP4 ? 17 : 0;
}
// one value a unit (no block structure): rows of any length when nothing downstream needs 32-value blocks
__host__ __device__ constexpr bool elementwise_src(int s) { return s == SRC_F32 || s == SRC_F16 || s == SRC_BF16; }
__host__ __device__ constexpr bool is_block_src(int s) {
    return s == IQ2_XXS || s == IQ2_XS || s == IQ2_S || s == IQ3_XXS || s == IQ3_S || s == IQ1_S || s == IQ1_M ||
           s == IQ4_XS || s == Q2_K || s == Q3_K || s == Q4_K || s == Q5_K || s == Q6_K;
}
// values and bytes of one block of any readable source (0: not readable on the GPU)
__host__ __device__ constexpr int src_block_len(int s) {
    return src_bytes32(s) ? 32 : s == SRC_NVFP4 ? 64 : s == SRC_MXFP8 ? 32 : is_block_src(s) ? QK : 0;
}
__host__ __device__ constexpr int src_block_bytes(int s) {
    return src_bytes32(s) ? src_bytes32(s) : s == SRC_NVFP4 ? 36 : s == SRC_MXFP8 ? 33 : is_block_src(s) ? block_bytes(s) : 0;
}

// ---------------------------------------------------------------------------------------------- device status
// Conditions ggml would reach only through impossible states (no finite candidate in a neighbour search, a final
// code off the grid) are reported, never trapped: the kernel records the reason in the per-device status word,
// skips the block, and the host API turns the word into a 0 return.
enum Status : unsigned { ST_OK = 0, ST_NO_NEIGHBOUR = 1u, ST_OFF_GRID = 2u, ST_BAD_INPUT = 4u, ST_TIMEOUT = 8u };

// ---------------------------------------------------------------------------------------------- search tables
// Device layout of one codebook (built on the host from a gpuq_tables.bin record):
//   code3[c]  for every reachable level code c (base-3 digits for the 8-d grids, base-8 for the 4-d IQ3 grids):
//             >= 0: the grid index of the point with those levels; < 0: -(1 + (offset << 9 | count)) of the
//             code's neighbour list in `neigh` (list_off / list_cnt)
//   neigh     list = [count, entries...], entry = grid index << 16 | the point's packed levels
//             (2 bits a dimension for 8-d grids, 3 bits for 4-d); one pad word after the last list
//   glev[g]   packed levels of grid point g (same packing)
struct SearchTab {
    const int32_t * code3;
    const uint32_t * neigh;
    const uint16_t * glev;
    int ngrid;
};
constexpr int LIST_CNT_BITS = 9;   // list lengths < 512 (the longest ggml list has 292 points)
__device__ __forceinline__ int list_off(int m) { return (-m - 1) >> LIST_CNT_BITS; }
__device__ __forceinline__ int list_cnt(int m) { return (-m - 1) & ((1 << LIST_CNT_BITS) - 1); }
struct DequantTab { const uint64_t * grid; };   // ggml-common.h iq*_grid, 4-byte points zero-extended

// ---------------------------------------------------------------------------------------------- scalar helpers
__device__ __forceinline__ uint32_t f2u(float f) { return __float_as_uint(f); }
__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

// ggml's round-to-nearest-even by the 1.5*2^23 bias (ggml-quants.c nearest_int)
__device__ __forceinline__ int nearest_int(float v) {
    return (int) (f2u(v + 12582912.f) & 0x007FFFFFu) - 0x00400000;
}

// ggml's float -> IEEE half (ggml_compute_fp32_to_fp16, the bit-manipulation variant ggml-base uses)
__device__ __forceinline__ uint16_t half_bits(float f) {
    float base = (fabsf(f) * 0x1.0p+112f) * 0x1.0p-110f;
    const uint32_t w = f2u(f), shl1 = w + w, sign = w & 0x80000000u;
    uint32_t bias = shl1 & 0xFF000000u;
    if (bias < 0x71000000u) bias = 0x71000000u;
    base = u2f((bias >> 1) + 0x07800000u) + base;
    const uint32_t bits = f2u(base);
    const uint32_t nonsign = ((bits >> 13) & 0x7C00u) + (bits & 0x0FFFu);
    return (uint16_t) ((sign >> 16) | (shl1 > 0xFF000000u ? 0x7E00u : nonsign));
}

// IEEE half -> float, exact
__device__ __forceinline__ float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    if (e == 0) {
        if (m == 0) return u2f(sign);
        const int sh = __clz(m) - 21;            // bring the leading 1 to bit 10
        m = (m << sh) & 0x3FFu;
        e = 113 - sh;
        return u2f(sign | (e << 23) | (m << 13));
    }
    if (e == 31) return u2f(sign | 0x7F800000u | (m << 13));
    return u2f(sign | ((e + 112) << 23) | (m << 13));
}

// ggml_e8m0_to_fp32_half: 2^(e-128) as a float (denormal below e = 2)
__device__ __forceinline__ float e8m0_half(uint8_t e) {
    return u2f(e < 2 ? 0x00200000u << e : (uint32_t) (e - 1) << 23);
}

// the reference's MAX(a, b) / MIN(a, b) (ternaries, not fmaxf: NaN handling must match)
__device__ __forceinline__ float fmaxr(float a, float b) { return a > b ? a : b; }
__device__ __forceinline__ int imax(int a, int b) { return a > b ? a : b; }
__device__ __forceinline__ int imin(int a, int b) { return a < b ? a : b; }

}  // namespace gq
