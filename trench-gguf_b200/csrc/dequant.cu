// dequant.cu - ggml's to_float of the i-quant types (dequantize_row_iq*, trench-gguf gpuq.hip:1850-2028), of the
// k-quants (ggml's dequantize_row_q2_K .. q6_K, which the reference leaves to ggml on the CPU) and the source decoder
// (kdq, gpuq.hip:2123-2141), HBM-bound.
//
// Layout: one warp a 256-weight super-block, lane l producing weights 8l..8l+7 (its 32-weight sub-block l/4 and
// 8-weight group l%4), stored as two 16-byte writes: a warp writes its 1 KiB of floats fully coalesced. Every
// value is computed with ggml's expression in ggml's operand order; all products are exact in float32, so the
// result equals ggml's to_float bit for bit.
#include "common.cuh"
#include "source.cuh"
#include "kernels.h"

namespace gq {
namespace {

__device__ __forceinline__ uint8_t ksigns(uint32_t k) { return (uint8_t) (k | ((__popc(k) & 1) << 7)); }
__device__ __forceinline__ float sgn(uint32_t s, int j) { return (s >> j) & 1 ? -1.f : 1.f; }
__device__ __forceinline__ uint32_t ld_u16(const uint8_t * p) { return (uint32_t) p[0] | ((uint32_t) p[1] << 8); }
__device__ __forceinline__ uint32_t ld_u32(const uint8_t * p) {
    return (uint32_t) p[0] | ((uint32_t) p[1] << 8) | ((uint32_t) p[2] << 16) | ((uint32_t) p[3] << 24);
}
__device__ __forceinline__ uint8_t gbyte(const uint64_t * grid, int gi, int j) {
    return (uint8_t) (__ldg(grid + gi) >> (8 * j));
}

__constant__ int8_t c_iq4nl[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

// ggml's 6-bit k-quant scale and min j (get_scale_min_k4): 12 bytes hold 8 pairs
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t * q, int & sc, int & m) {
    if (j < 4) { sc = q[j] & 63; m = q[j + 4] & 63; }
    else { sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4); m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4); }
}

// ggml's dequantize_row_q2_K .. q6_K (ggml-quants.c), weights v0 .. v0+7 of one super-block (v0 = 8 * lane: all
// eight share one sub-block scale). Every expression keeps ggml's operand order: the products that can round
// (q4_K/q5_K's d1 * q - m1, q6_K's (d * sc) * q) round exactly as ggml's C does.
template <int T>
__device__ __forceinline__ void dq8_kquant(const uint8_t * q, int v0, float * y) {
    if constexpr (T == Q2_K) {            // scales[16] qs[64] d dmin
        const float d = half_to_float((uint16_t) ld_u16(q + 80)), dmin = half_to_float((uint16_t) ld_u16(q + 82));
        const int h = v0 >> 7, j = (v0 >> 5) & 3, part = (v0 >> 4) & 1, l0 = v0 & 15;
        const uint8_t sc = q[8 * h + 2 * j + part];
        const float dl = d * (sc & 0xF), ml = dmin * (sc >> 4);
        const uint8_t * qs = q + 16 + 32 * h + 16 * part + l0;
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = dl * ((int8_t) ((qs[i] >> (2 * j)) & 3)) - ml;
    } else if constexpr (T == Q3_K) {     // hmask[32] qs[64] scales[12] d
        const float d_all = half_to_float((uint16_t) ld_u16(q + 108));
        const int h = v0 >> 7, j = (v0 >> 5) & 3, part = (v0 >> 4) & 1, l0 = v0 & 15;
        const int si = 8 * h + 2 * j + part;
        const uint8_t lo = q[96 + (si & 7)];
        const int sc6 = (si < 8 ? lo & 0xF : lo >> 4) | (((q[104 + (si & 3)] >> (2 * (si >> 2))) & 3) << 4);
        const float dl = d_all * ((int8_t) sc6 - 32);
        const uint8_t * qs = q + 32 + 32 * h + 16 * part + l0;
        const uint8_t * hm = q + 16 * part + l0;
        const uint8_t m = (uint8_t) (1u << (4 * h + j));
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = dl * ((int8_t) ((qs[i] >> (2 * j)) & 3) - ((hm[i] & m) ? 0 : 4));
    } else if constexpr (T == Q4_K || T == Q5_K) {   // d dmin scales[12] (qh[32]) qs[128]
        const float d = half_to_float((uint16_t) ld_u16(q)), dmin = half_to_float((uint16_t) ld_u16(q + 2));
        const int c = v0 >> 6, hi = (v0 >> 5) & 1, l0 = v0 & 31;
        int sc, m;
        scale_min_k4(2 * c + hi, q + 4, sc, m);
        const float d1 = d * sc, m1 = dmin * m;
        const uint8_t * qs = q + (T == Q4_K ? 16 : 48) + 32 * c + l0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int v = hi ? qs[i] >> 4 : qs[i] & 0xF;
            if constexpr (T == Q4_K) y[i] = d1 * v - m1;
            else y[i] = d1 * (v + ((q[16 + l0 + i] >> (2 * c + hi)) & 1 ? 16 : 0)) - m1;
        }
    } else {                              // Q6_K: ql[128] qh[64] scales[16] d
        const float d = half_to_float((uint16_t) ld_u16(q + 208));
        const int h = v0 >> 7, qq = (v0 >> 5) & 3, l0 = v0 & 31;
        const uint8_t * ql = q + 64 * h + 32 * (qq & 1) + l0;
        const uint8_t * qh = q + 128 + 32 * h + l0;
        const int8_t sc = (int8_t) q[192 + 8 * h + (l0 >> 4) + 2 * qq];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int v = ((qq < 2 ? ql[i] & 0xF : ql[i] >> 4) | (((qh[i] >> (2 * qq)) & 3) << 4)) - 32;
            y[i] = d * sc * (int8_t) v;
        }
    }
}

template <int T>
__device__ __forceinline__ void dq8(const uint8_t * q, int lane, const uint64_t * G, float * y) {
    const int ib = lane >> 2, l = lane & 3;
    if constexpr (T == Q2_K || T == Q3_K || T == Q4_K || T == Q5_K || T == Q6_K) {
        dq8_kquant<T>(q, 8 * lane, y);
    } else if constexpr (T == IQ4_XS) {
        const float d = half_to_float((uint16_t) ld_u16(q));
        const uint32_t sh = ld_u16(q + 2);
        const int ls = ((q[4 + ib / 2] >> (4 * (ib % 2))) & 0xf) | (((sh >> (2 * ib)) & 3) << 4);
        const float dl = d * (ls - 32);
        const int j0 = 8 * (l & 1), hi = l >> 1;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint8_t v = q[8 + 16 * ib + j0 + j];
            y[j] = dl * c_iq4nl[hi ? v >> 4 : v & 0xf];
        }
    } else if constexpr (T == IQ1_M) {
        const uint32_t s0 = ld_u16(q + 48), s1 = ld_u16(q + 50), s2 = ld_u16(q + 52), s3 = ld_u16(q + 54);
        const uint16_t s16 = (uint16_t) ((s0 >> 12) | ((s1 >> 8) & 0x00f0) | ((s2 >> 4) & 0x0f00) | (s3 & 0xf000));
        const float dd = half_to_float(s16);
        const uint32_t sc = ld_u16(q + 48 + 2 * (ib / 2));
        const float dl = l < 2 ? dd * (2 * ((sc >> (6 * (ib % 2))) & 0x7) + 1) : dd * (2 * ((sc >> (6 * (ib % 2) + 3)) & 0x7) + 1);
        const uint8_t * qs = q + 4 * ib, * qh = q + 32 + 2 * ib;
        const uint8_t h = qh[l / 2];
        const int gi = qs[l] | ((l % 2 ? (h << 4) : (h << 8)) & 0x700);
        const float delta = (h & (l % 2 ? 0x80 : 0x08)) ? -0.125f : 0.125f;
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] = dl * ((float) (int8_t) gbyte(G, gi, j) + delta);
    } else {
        const float d = half_to_float((uint16_t) ld_u16(q));
        if constexpr (T == IQ2_XXS) {
            const uint32_t a0 = ld_u32(q + 2 + 8 * ib), a1 = ld_u32(q + 6 + 8 * ib);
            const float db = d * (0.5f + (a1 >> 28)) * 0.25f;
            const int gi = (a0 >> (8 * l)) & 255;
            const uint8_t s = ksigns((a1 >> (7 * l)) & 127);
#pragma unroll
            for (int j = 0; j < 8; ++j) y[j] = db * gbyte(G, gi, j) * sgn(s, j);
        } else if constexpr (T == IQ2_XS) {
            const uint8_t sc = q[66 + ib];
            const float db = d * (0.5f + (l < 2 ? (sc & 0xf) : (sc >> 4))) * 0.25f;
            const uint32_t v = ld_u16(q + 2 + 2 * (4 * ib + l));
            const int gi = v & 511;
            const uint8_t s = ksigns(v >> 9);
#pragma unroll
            for (int j = 0; j < 8; ++j) y[j] = db * gbyte(G, gi, j) * sgn(s, j);
        } else if constexpr (T == IQ2_S) {
            const uint8_t sc = q[74 + ib];
            const float db = d * (0.5f + (l < 2 ? (sc & 0xf) : (sc >> 4))) * 0.25f;
            const int gi = q[2 + 4 * ib + l] | ((q[66 + ib] << (8 - 2 * l)) & 0x300);
            const uint8_t s = q[34 + 4 * ib + l];
#pragma unroll
            for (int j = 0; j < 8; ++j) y[j] = db * gbyte(G, gi, j) * sgn(s, j);
        } else if constexpr (T == IQ3_XXS) {
            const uint32_t a = ld_u32(q + 66 + 4 * ib);
            const float db = d * (0.5f + (a >> 28)) * 0.5f;
            const uint8_t s = ksigns((a >> (7 * l)) & 127);
            const int g1 = q[2 + 8 * ib + 2 * l], g2 = q[2 + 8 * ib + 2 * l + 1];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                y[j] = db * gbyte(G, g1, j) * sgn(s, j);
                y[j + 4] = db * gbyte(G, g2, j) * sgn(s, j + 4);
            }
        } else if constexpr (T == IQ3_S) {
            const uint8_t sc = q[106 + ib / 2];
            const float db = d * (1 + 2 * ((ib % 2) ? (sc >> 4) : (sc & 0xf)));
            const uint8_t hb = q[66 + ib];
            const int g1 = q[2 + 8 * ib + 2 * l] | ((hb << (8 - 2 * l)) & 256);
            const int g2 = q[2 + 8 * ib + 2 * l + 1] | ((hb << (7 - 2 * l)) & 256);
            const uint8_t s = q[74 + 4 * ib + l];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                y[j] = db * gbyte(G, g1, j) * sgn(s, j);
                y[j + 4] = db * gbyte(G, g2, j) * sgn(s, j + 4);
            }
        } else {   // IQ1_S
            const uint32_t qh = ld_u16(q + 34 + 2 * ib);
            const float dl = d * (2 * ((qh >> 12) & 7) + 1);
            const float delta = qh & 0x8000 ? -0.125f : 0.125f;
            const int gi = q[2 + 4 * ib + l] | (((qh >> (3 * l)) & 7) << 8);
#pragma unroll
            for (int j = 0; j < 8; ++j) y[j] = dl * ((float) (int8_t) gbyte(G, gi, j) + delta);
        }
    }
}

template <int T>
__global__ void __launch_bounds__(256) k_dequant(const uint8_t * __restrict__ q, float * __restrict__ out,
                                                 int64_t nblocks, const uint64_t * __restrict__ grid) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t) gridDim.x * (blockDim.x >> 5);
    for (int64_t b = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < nblocks; b += nw) {
        float y[8];
        dq8<T>(q + b * block_bytes(T), lane, grid, y);
        float4 * o = reinterpret_cast<float4 *>(out + b * QK + lane * 8);
        if ((reinterpret_cast<uintptr_t>(out) & 15) == 0) {
            o[0] = make_float4(y[0], y[1], y[2], y[3]);
            o[1] = make_float4(y[4], y[5], y[6], y[7]);
        } else {
            float * p = out + b * QK + lane * 8;
#pragma unroll
            for (int j = 0; j < 8; ++j) p[j] = y[j];
        }
    }
}

// LDLQ's block error: E = blk - to_float(q) in float32 (ggml's to_float), stored as float64 or float32
// (tools/ldlq.py:427 `E = (blk - q).to(Ud.dtype)`), one pass over the bytes and the block
template <int T, bool F64>
__global__ void __launch_bounds__(256) k_dequant_error(const uint8_t * __restrict__ q, const float * __restrict__ blk,
                                                       void * __restrict__ err, int64_t nblocks,
                                                       const uint64_t * __restrict__ grid) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t) gridDim.x * (blockDim.x >> 5);
    for (int64_t b = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < nblocks; b += nw) {
        float y[8], x[8];
        dq8<T>(q + b * block_bytes(T), lane, grid, y);
        load8_f32(blk + b * QK + lane * 8, x);
        if constexpr (F64) {
            double * e = reinterpret_cast<double *>(err) + b * QK + lane * 8;
#pragma unroll
            for (int j = 0; j < 8; ++j) e[j] = (double) (x[j] - y[j]);
        } else {
            float * e = reinterpret_cast<float *>(err) + b * QK + lane * 8;
#pragma unroll
            for (int j = 0; j < 8; ++j) e[j] = x[j] - y[j];
        }
    }
}

// 8 floats to out (16-byte stores when aligned), each times `s` when a per-matrix scale applies
__device__ __forceinline__ void store8(float * out, float * y, const float * scale, int64_t vglob, int64_t per_mat) {
    if (scale) {
        const float s = __ldg(scale + vglob / per_mat);   // (8 values never straddle two matrices: per_mat % 8 == 0)
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] = y[j] * s;
    }
    if ((reinterpret_cast<uintptr_t>(out) & 15) == 0) {
        float4 * o = reinterpret_cast<float4 *>(out);
        o[0] = make_float4(y[0], y[1], y[2], y[3]);
        o[1] = make_float4(y[4], y[5], y[6], y[7]);
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) out[j] = y[j];
    }
}

// source values -> float32, 8 a thread (the element formats); value i of the pass is value v0 + i of the tensor,
// whose matrix (v0 + i) / per_mat picks the scale
template <int SRC>
__global__ void __launch_bounds__(256) k_decode(const uint8_t * __restrict__ raw, float * __restrict__ out, int64_t n8,
                                                const float * __restrict__ scale, int64_t per_mat, int64_t v0) {
    const int64_t stride = (int64_t) gridDim.x * blockDim.x;
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += stride) {
        float y[8];
        decode8<SRC>(raw, i * 8, y);
        store8(out + i * 8, y, scale, v0 + i * 8, per_mat);
    }
}

// a k-quant / i-quant source -> float32: ggml's to_float, a warp a super-block, then the per-matrix scale
template <int T>
__global__ void __launch_bounds__(256) k_decode_blocks(const uint8_t * __restrict__ q, float * __restrict__ out,
                                                       int64_t nblocks, const uint64_t * __restrict__ grid,
                                                       const float * __restrict__ scale, int64_t per_mat, int64_t v0) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t) gridDim.x * (blockDim.x >> 5);
    for (int64_t b = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < nblocks; b += nw) {
        float y[8];
        dq8<T>(q + b * block_bytes(T), lane, grid, y);
        store8(out + b * QK + lane * 8, y, scale, v0 + b * QK + lane * 8, per_mat);
    }
}

int grid_for(int64_t units, int per_cta) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t need = (units + per_cta - 1) / per_cta;
    const int64_t cap = (int64_t) sms * 16;   // enough resident CTAs to cover HBM latency; grid-stride beyond
    return (int) (need < cap ? (need > 0 ? need : 1) : cap);
}

}  // namespace

cudaError_t launch_dequant(int type, const void * q, float * out, int64_t nblocks, DequantTab tab, cudaStream_t st) {
    const int g = grid_for(nblocks, 8);
    const uint8_t * qb = (const uint8_t *) q;
    switch (type) {
        case IQ2_XXS: k_dequant<IQ2_XXS><<<g, 256, 0, st>>>(qb, out, nblocks, tab.grid); break;
        case IQ2_XS:  k_dequant<IQ2_XS><<<g, 256, 0, st>>>(qb, out, nblocks, tab.grid); break;
        case IQ2_S:   k_dequant<IQ2_S><<<g, 256, 0, st>>>(qb, out, nblocks, tab.grid); break;
        case IQ3_XXS: k_dequant<IQ3_XXS><<<g, 256, 0, st>>>(qb, out, nblocks, tab.grid); break;
        case IQ3_S:   k_dequant<IQ3_S><<<g, 256, 0, st>>>(qb, out, nblocks, tab.grid); break;
        case IQ1_S:   k_dequant<IQ1_S><<<g, 256, 0, st>>>(qb, out, nblocks, tab.grid); break;
        case IQ1_M:   k_dequant<IQ1_M><<<g, 256, 0, st>>>(qb, out, nblocks, tab.grid); break;
        case IQ4_XS:  k_dequant<IQ4_XS><<<g, 256, 0, st>>>(qb, out, nblocks, tab.grid); break;
        case Q2_K:    k_dequant<Q2_K><<<g, 256, 0, st>>>(qb, out, nblocks, nullptr); break;
        case Q3_K:    k_dequant<Q3_K><<<g, 256, 0, st>>>(qb, out, nblocks, nullptr); break;
        case Q4_K:    k_dequant<Q4_K><<<g, 256, 0, st>>>(qb, out, nblocks, nullptr); break;
        case Q5_K:    k_dequant<Q5_K><<<g, 256, 0, st>>>(qb, out, nblocks, nullptr); break;
        case Q6_K:    k_dequant<Q6_K><<<g, 256, 0, st>>>(qb, out, nblocks, nullptr); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_dequant_error(int type, const void * q, const float * blk, void * err, bool f64, int64_t nblocks,
                                 DequantTab tab, cudaStream_t st) {
    const int g = grid_for(nblocks, 8);
    const uint8_t * qb = (const uint8_t *) q;
#define DE(T) (f64 ? (k_dequant_error<T, true><<<g, 256, 0, st>>>(qb, blk, err, nblocks, tab.grid), 0) \
                   : (k_dequant_error<T, false><<<g, 256, 0, st>>>(qb, blk, err, nblocks, tab.grid), 0))
    switch (type) {
        case IQ2_XXS: DE(IQ2_XXS); break;
        case IQ2_XS:  DE(IQ2_XS); break;
        case IQ2_S:   DE(IQ2_S); break;
        case IQ3_XXS: DE(IQ3_XXS); break;
        case IQ3_S:   DE(IQ3_S); break;
        case IQ1_S:   DE(IQ1_S); break;
        case IQ1_M:   DE(IQ1_M); break;
        case IQ4_XS:  DE(IQ4_XS); break;
        case Q2_K:    DE(Q2_K); break;
        case Q3_K:    DE(Q3_K); break;
        case Q4_K:    DE(Q4_K); break;
        case Q5_K:    DE(Q5_K); break;
        case Q6_K:    DE(Q6_K); break;
        default: return cudaErrorInvalidValue;
    }
#undef DE
    return cudaGetLastError();
}

cudaError_t launch_stage(int src, const void * raw, float * out, int64_t n, DequantTab tab, const float * scale,
                         int64_t per_mat, int64_t v0, cudaStream_t st) {
    const uint8_t * r = (const uint8_t *) raw;
    if (is_block_src(src)) {
        const int64_t nb = n / QK;
        const int g = grid_for(nb, 8);
#define KB(T) k_decode_blocks<T><<<g, 256, 0, st>>>(r, out, nb, tab.grid, scale, per_mat, v0)
        switch (src) {
            case IQ2_XXS: KB(IQ2_XXS); break;
            case IQ2_XS:  KB(IQ2_XS); break;
            case IQ2_S:   KB(IQ2_S); break;
            case IQ3_XXS: KB(IQ3_XXS); break;
            case IQ3_S:   KB(IQ3_S); break;
            case IQ1_S:   KB(IQ1_S); break;
            case IQ1_M:   KB(IQ1_M); break;
            case IQ4_XS:  KB(IQ4_XS); break;
            case Q2_K:    KB(Q2_K); break;
            case Q3_K:    KB(Q3_K); break;
            case Q4_K:    KB(Q4_K); break;
            case Q5_K:    KB(Q5_K); break;
            case Q6_K:    KB(Q6_K); break;
            default: return cudaErrorInvalidValue;
        }
#undef KB
        return cudaGetLastError();
    }
    const int64_t n8 = n / 8;
    const int g = grid_for(n8, 256);
    switch (src) {
        case SRC_F32:   k_decode<SRC_F32><<<g, 256, 0, st>>>(r, out, n8, scale, per_mat, v0); break;
        case SRC_F16:   k_decode<SRC_F16><<<g, 256, 0, st>>>(r, out, n8, scale, per_mat, v0); break;
        case SRC_BF16:  k_decode<SRC_BF16><<<g, 256, 0, st>>>(r, out, n8, scale, per_mat, v0); break;
        case SRC_Q8_0:  k_decode<SRC_Q8_0><<<g, 256, 0, st>>>(r, out, n8, scale, per_mat, v0); break;
        case SRC_MXFP4: k_decode<SRC_MXFP4><<<g, 256, 0, st>>>(r, out, n8, scale, per_mat, v0); break;
        case SRC_NVFP4: k_decode<SRC_NVFP4><<<g, 256, 0, st>>>(r, out, n8, scale, per_mat, v0); break;
        case SRC_MXFP8: k_decode<SRC_MXFP8><<<g, 256, 0, st>>>(r, out, n8, scale, per_mat, v0); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_decode(int src, const void * raw, float * out, int64_t n, DequantTab tab, cudaStream_t st) {
    return launch_stage(src, raw, out, n, tab, nullptr, 1, 0, st);
}

}  // namespace gq
