// f16.cu - the last fallback target, F16 (ggml type 1): what trench-gguf writes for rows that fit neither the asked
// type nor its 32-weight fallback (tools/requant_experts.py:187-192, `fit_type`), through ggml_quantize_chunk's F16
// path, ggml_fp32_to_fp16_row: every value converted by ggml's float -> half (ggml_compute_fp32_to_fp16, the same
// bit-level rounding as the block scales: half_bits). The reference runs it on the CPU.
//
// How: HBM bound, 8 values a thread - one decode8 of the source (any inline source, decoded in the load) and one
// 16-byte store of 8 halves; rows of F32/F16/BF16 sources may have any length, so a last partial group of 8 is
// converted value by value (the block sources' lengths are whole blocks).
#include <cstdint>
#include "common.cuh"
#include "kernels.h"
#include "source.cuh"

namespace gq {
namespace {

template <int SRC>
__device__ __forceinline__ float value_at(const uint8_t * raw, int64_t i) {
    if constexpr (SRC == SRC_F32) return reinterpret_cast<const float *>(raw)[i];
    else if constexpr (SRC == SRC_F16) return half_to_float(reinterpret_cast<const uint16_t *>(raw)[i]);
    else return __uint_as_float((uint32_t) reinterpret_cast<const uint16_t *>(raw)[i] << 16);   // BF16
}

template <int SRC>
__global__ void __launch_bounds__(256) k_to_f16(const uint8_t * __restrict__ raw, uint16_t * __restrict__ out,
                                                int64_t n, bool vec_out) {
    const int64_t i0 = ((int64_t) blockIdx.x * 256 + threadIdx.x) * 8;
    if (i0 >= n) return;
    if (i0 + 8 <= n) {
        float v[8];
        decode8<SRC>(raw, i0, v);
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) w[k] = (uint32_t) half_bits(v[2 * k]) | ((uint32_t) half_bits(v[2 * k + 1]) << 16);
        if (vec_out) {
            *reinterpret_cast<uint4 *>(out + i0) = make_uint4(w[0], w[1], w[2], w[3]);
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) out[i0 + k] = (uint16_t) (w[k >> 1] >> (16 * (k & 1)));
        }
        return;
    }
    if constexpr (SRC == SRC_F32 || SRC == SRC_F16 || SRC == SRC_BF16) {   // the ragged end of an element-wise source
        for (int64_t i = i0; i < n; ++i) out[i] = half_bits(value_at<SRC>(raw, i));
    }
}

template <int SRC>
cudaError_t launch_f16_t(const LaunchArgs & a) {
    const int64_t n = a.nblocks;                          // (F16's "block" is one value)
    const int64_t threads = (n + 7) / 8;
    const bool vec_out = (reinterpret_cast<uintptr_t>(a.out) & 15) == 0;
    k_to_f16<SRC><<<(unsigned) ((threads + 255) / 256), 256, 0, a.stream>>>(static_cast<const uint8_t *>(a.src),
                                                                          static_cast<uint16_t *>(a.out), n, vec_out);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_f16(const LaunchArgs & a) {
    if (a.nblocks <= 0 || (a.nblocks + 7) / 8 / 256 >= (int64_t) 0x7FFFFFFF) return cudaErrorInvalidValue;
    if (!elementwise_src(a.src_type) && a.nblocks % 32) return cudaErrorInvalidValue;
    switch (a.src_type) {
        case SRC_F32:   return launch_f16_t<SRC_F32>(a);
        case SRC_F16:   return launch_f16_t<SRC_F16>(a);
        case SRC_BF16:  return launch_f16_t<SRC_BF16>(a);
        case SRC_Q8_0:  return launch_f16_t<SRC_Q8_0>(a);
        case SRC_MXFP4: return launch_f16_t<SRC_MXFP4>(a);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace gq
