// source.cuh - exact decoding of the source tensor's bytes (ggml's to_float of F32 / F16 / BF16 / Q8_0 / MXFP4,
// gpuq.hip:2123-2141 in trench-gguf) fused into the quantizers' loads: a super-block's 256 values go straight from
// the raw bytes in HBM to registers and shared memory, never through a float32 copy in HBM.
// Every decoded value is a small integer or a half/bfloat times a power of two or a half: exact in float32.
#pragma once
#include "common.cuh"

namespace gq {

// 8 consecutive importance weights (any 4-byte aligned pointer)
__device__ __forceinline__ void load8_f32(const float * __restrict__ p, float * out) {
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
        const float4 a = __ldg(reinterpret_cast<const float4 *>(p)), b = __ldg(reinterpret_cast<const float4 *>(p) + 1);
        out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w; out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) out[j] = __ldg(p + j);
    }
}

// a load through the read-only path (global memory) or a plain load (any address space: shared-memory tiles)
template <bool NC, typename T>
__device__ __forceinline__ T ldx(const T * p) {
    if constexpr (NC) return __ldg(p); else return *p;
}

// Values v0..v0+7 of the source tensor (v0 a multiple of 8) -> out[0..7]. NC = false: raw may point into shared memory.
template <int SRC, bool NC = true>
__device__ __forceinline__ void decode8(const uint8_t * __restrict__ raw, int64_t v0, float * out) {
    if constexpr (SRC == SRC_F32) {
        if ((reinterpret_cast<uintptr_t>(raw) & 15) == 0) {   // (128-bit loads when the caller's pointer allows)
            const float4 * p = reinterpret_cast<const float4 *>(raw) + v0 / 4;
            const float4 a = ldx<NC>(p), b = ldx<NC>(p + 1);
            out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w; out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
        } else {
            const float * p = reinterpret_cast<const float *>(raw) + v0;
#pragma unroll
            for (int j = 0; j < 8; ++j) out[j] = ldx<NC>(p + j);
        }
    } else if constexpr (SRC == SRC_F16 || SRC == SRC_BF16) {
        uint32_t w[4];
        if ((reinterpret_cast<uintptr_t>(raw) & 15) == 0) {
            const uint4 q = ldx<NC>(reinterpret_cast<const uint4 *>(raw) + v0 / 8);
            w[0] = q.x; w[1] = q.y; w[2] = q.z; w[3] = q.w;
        } else {
            const uint16_t * p = reinterpret_cast<const uint16_t *>(raw) + v0;
#pragma unroll
            for (int j = 0; j < 4; ++j) w[j] = (uint32_t) ldx<NC>(p + 2 * j) | ((uint32_t) ldx<NC>(p + 2 * j + 1) << 16);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint16_t lo = (uint16_t) (w[j] & 0xFFFFu), hi = (uint16_t) (w[j] >> 16);
            if constexpr (SRC == SRC_BF16) { out[2 * j] = u2f((uint32_t) lo << 16); out[2 * j + 1] = u2f((uint32_t) hi << 16); }
            else { out[2 * j] = half_to_float(lo); out[2 * j + 1] = half_to_float(hi); }
        }
    } else if constexpr (SRC == SRC_Q8_0) {   // block: half d, int8 qs[32]
        const uint8_t * b = raw + (v0 / 32) * 34;
        const int o = (int) (v0 % 32);
        const float d = half_to_float((uint16_t) (ldx<NC>(b) | (ldx<NC>(b + 1) << 8)));
#pragma unroll
        for (int j = 0; j < 8; ++j) out[j] = (float) (int8_t) ldx<NC>(b + 2 + o + j) * d;
    } else if constexpr (SRC == SRC_NVFP4) {   // 64 values: 4 UE4M3 scales (one a 16 values), then 4 x 8 bytes of
        const uint8_t * b = raw + (v0 / 64) * 36;   // e2m1 pairs (group j: low nibbles values 0..7, high 8..15)
        const int o = (int) (v0 % 64), j = o / 16, sh = (o & 8) ? 4 : 0;
        const uint8_t sb = ldx<NC>(b + j);
        const int ex = (sb >> 3) & 0xF, mn = sb & 7;
        // the scale is UE4M3 times 0.5 (gguf-py's ue4m3_to_fp32): mn * 2^-10 or (8 + mn) * 2^(ex - 11), exact
        const float d = (sb == 0 || sb == 0x7F) ? 0.0f : ex == 0 ? (float) mn * 0x1.0p-10f : (float) (8 + mn) * u2f((uint32_t) (ex + 116) << 23);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int c = (ldx<NC>(b + 4 + 8 * j + i) >> sh) & 15;
            const int m = c & 7;
            const int mag = m < 5 ? m : (m == 5 ? 6 : (m == 6 ? 8 : 12));
            out[i] = d * (float) (c & 8 ? -mag : mag);
        }
    } else if constexpr (SRC == SRC_MXFP8) {   // 33-byte blocks: E8M0 scale 2^(e-127) (e = 255: 0), 32 E4M3 values
        const uint8_t * b = raw + (v0 / 32) * 33;
        const int o = (int) (v0 % 32);
        const uint8_t e = ldx<NC>(b);
        const float sc = e == 255 ? 0.0f : e == 0 ? u2f(0x00400000u) : u2f((uint32_t) e << 23);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint8_t q = ldx<NC>(b + 1 + o + i);
            const int ex = (q >> 3) & 0xF, mn = q & 7;
            // E4M3 (the FN variant: no infinities; 0x7F and 0xFF the NaNs, read as +0 as the reference's table does):
            // mn * 2^-9 or (8 + mn) * 2^(ex - 10)
            float v = ex == 0 ? (float) mn * 0x1.0p-9f : (float) (8 + mn) * u2f((uint32_t) (ex + 117) << 23);
            if (q & 0x80) v = -v;
            out[i] = (ex == 15 && mn == 7) ? 0.0f * sc : v * sc;
        }
    } else {                                   // MXFP4 block: e8m0 scale, 16 bytes of two e2m1 codes
        const uint8_t * b = raw + (v0 / 32) * 17;
        const int o = (int) (v0 % 32);          // 0, 8: low nibbles of qs[o..o+7]; 16, 24: high nibbles of qs[o-16..]
        const float d = e8m0_half(ldx<NC>(b));
        const int sh = o >= 16 ? 4 : 0, q0 = o & 15;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int c = (ldx<NC>(b + 1 + q0 + j) >> sh) & 15;
            // e2m1 doubled: 0 1 2 3 4 6 8 12, bit 3 the sign
            const int m = c & 7;
            const int mag = m < 5 ? m : (m == 5 ? 6 : (m == 6 ? 8 : 12));
            out[j] = (float) (c & 8 ? -mag : mag) * d;
        }
    }
}

}  // namespace gq
