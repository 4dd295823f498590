// kquant.cu - Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, Q8_0 and IQ4_NL / IQ4_XS.
//
// What is computed: ggml's k-quant row quantizers - with an imatrix the quantize_row_*_impl searches, without one
// the *_ref searches - and IQ4_NL / IQ4_XS's quantize_row_iq4_nl_impl (trench-gguf gpuq.hip:1403-1838 and
// :1286-1398), one block at a time, byte-identical.
//
// sm_100a mapping: one warp a tile of 32 sub-blocks (4 super-blocks of Q4_K/Q5_K/IQ4_XS, 2 of Q2_K/Q3_K/Q6_K,
// 32 IQ4_NL blocks), with one LANE A SUB-BLOCK for the level searches. The searches are sequential inside a
// sub-block - an accepted affine trial moves the min that later trials use (gpuq.hip:1578-1583), the Q3_K
// coordinate descent updates its sums in place - so each lane runs its sub-block's search exactly as ggml does,
// and the 32 lanes run 32 sub-blocks side by side (the reference runs one super-block a thread). Around the
// searches the work is elementwise (weights, the final rounding against the stored fp16 scales: 8 weights a lane)
// or per super-block (sumx2 in index order, the scale codes: one lane a super-block), and the block bytes are
// assembled in parallel, one output byte a lane, and written with coalesced stores.
// Q8_0 is HBM-bound and has its own kernel: 8 weights a lane, 4 lanes a 32-weight block.
#include "common.cuh"
#include "source.cuh"
#include "kernels.h"

namespace gq {
namespace {

__constant__ int8_t c_iq4[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

template <int T> struct KT;
template <> struct KT<Q2_K>   { static constexpr int BL = 256, SB = 16; };
template <> struct KT<Q3_K>   { static constexpr int BL = 256, SB = 16; };
template <> struct KT<Q4_K>   { static constexpr int BL = 256, SB = 32; };
template <> struct KT<Q5_K>   { static constexpr int BL = 256, SB = 32; };
template <> struct KT<Q6_K>   { static constexpr int BL = 256, SB = 16; };
template <> struct KT<IQ4_XS> { static constexpr int BL = 256, SB = 32; };
template <> struct KT<IQ4_NL> { static constexpr int BL = 32, SB = 32; };

template <int T> struct alignas(16) KState {
    static constexpr int BL = KT<T>::BL, SB = KT<T>::SB, TILE = 32 * SB, NB = TILE / BL, NSUBB = BL / SB, NSUB = 32;
    // x and w hold sub-block s at s * SP. The 32-weight sub-blocks get one float of padding, so that the search
    // phase - one lane a sub-block, every lane at the same element index - reads 32 different banks (an unpadded
    // stride of 32 floats puts the whole warp on one bank: Q4_K and Q5_K with an imatrix ran 1.7x slower). The
    // 16-weight searches keep their sub-block in registers; padding them measured slightly slower.
    static constexpr int SP = SB == 32 ? SB + 1 : SB;
    __device__ static int xi(int e) {                                  // tile element e -> its slot
        if constexpr (SP == SB) return e; else return (e / SB) * SP + e % SB;
    }
    float x[32 * SP], w[32 * SP];
    uint8_t L[TILE];
    float scales[NSUB], mins[NSUB], sw[NSUB];
    float sigma2[NB];
    // per block: coded scales and the super-block scales (fp16 bits)
    uint8_t sc[NB][16], mn[NB][16];
    int8_t s6[NB][16];
    uint16_t d16[NB], dm16[NB];
    uint16_t sh[NB];
    uint8_t q3s[NB][12];
    uint8_t valid[NB];
};

// ------------------------------------------------------------------------------------------------ the searches
__device__ __forceinline__ float kw(const float * qw, const float * x, int i) { return qw ? qw[i] : x[i] * x[i]; }

// affine levels 0..nmax with a min (gpuq.hip:1513-1587; ggml make_qkx3 with an imatrix, make_qkx2 without);
// L (smem) holds the chosen levels
template <int N, bool IMAT>
__device__ float affine_levels(int nmax, const float * x, const float * wts, uint8_t * L, float * the_min,
                               float rmin, float rdelta, int nstep, bool use_mad) {
    float mn = x[0], mx = x[0];
    float sum_w = IMAT ? kw(wts, x, 0) : wts[0];
    float sum_x = sum_w * x[0];
    for (int i = 1; i < N; ++i) {
        if (x[i] < mn) mn = x[i];
        if (x[i] > mx) mx = x[i];
        const float w = IMAT ? kw(wts, x, i) : wts[i];
        sum_w += w;
        sum_x += w * x[i];
    }
    if (mn > 0) mn = 0;
    if (IMAT ? mx <= mn : mx == mn) {
        for (int i = 0; i < N; ++i) L[i] = 0;
        *the_min = -mn;
        return 0.f;
    }
    float iscale = nmax / (mx - mn);
    float scale = 1 / iscale;
    float best = 0;
    for (int i = 0; i < N; ++i) {
        L[i] = (uint8_t) imax(0, imin(nmax, nearest_int(iscale * (x[i] - mn))));
        float d = scale * L[i] + mn - x[i];
        d = use_mad ? fabsf(d) : d * d;
        best += (IMAT ? kw(wts, x, i) : wts[i]) * d;
    }
    if (nstep < 1) { *the_min = -mn; return scale; }
    for (int is = 0; is <= nstep; ++is) {
        iscale = (rmin + rdelta * is + nmax) / (mx - mn);
        float sl = 0, sl2 = 0, sxl = 0;
        uint32_t lp[N / 8];   // Laux, 4 bits a level
#pragma unroll
        for (int q = 0; q < N / 8; ++q) lp[q] = 0;
#pragma unroll
        for (int i = 0; i < N; ++i) {
            int l;
            if (IMAT) { const float v = iscale * (x[i] - mn); l = v > 0 ? nearest_int(v < nmax ? v : (float) nmax) : 0; }
            else l = imax(0, imin(nmax, nearest_int(iscale * (x[i] - mn))));
            lp[i / 8] |= (uint32_t) l << (4 * (i % 8));
            const float w = IMAT ? kw(wts, x, i) : wts[i];
            sl += w * l;
            sl2 += w * l * l;
            sxl += w * l * x[i];
        }
        const float D = sum_w * sl2 - sl * sl;
        if (!(D > 0)) continue;
        float ts = (sum_w * sxl - sum_x * sl) / D;
        float tm = (sl2 * sum_x - sl * sxl) / D;
        if (tm > 0) { tm = 0; ts = sxl / sl2; }
        float err = 0;
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const int l = (lp[i / 8] >> (4 * (i % 8))) & 15;
            float d = ts * l + tm - x[i];
            d = use_mad ? fabsf(d) : d * d;
            err += (IMAT ? kw(wts, x, i) : wts[i]) * d;
        }
        if (err < best) {
#pragma unroll
            for (int i = 0; i < N; ++i) L[i] = (uint8_t) ((lp[i / 8] >> (4 * (i % 8))) & 15);
            best = err; scale = ts; mn = tm;
        }
    }
    *the_min = -mn;
    return scale;
}

// affine levels for nmax up to 31 (Q5_K): the same search with 8-bit level storage
template <int N, bool IMAT>
__device__ float affine_levels5(int nmax, const float * x, const float * wts, uint8_t * L, float * the_min,
                                float rmin, float rdelta, int nstep) {
    float mn = x[0], mx = x[0];
    float sum_w = IMAT ? kw(wts, x, 0) : wts[0];
    float sum_x = sum_w * x[0];
    for (int i = 1; i < N; ++i) {
        if (x[i] < mn) mn = x[i];
        if (x[i] > mx) mx = x[i];
        const float w = IMAT ? kw(wts, x, i) : wts[i];
        sum_w += w;
        sum_x += w * x[i];
    }
    if (mn > 0) mn = 0;
    if (IMAT ? mx <= mn : mx == mn) {
        for (int i = 0; i < N; ++i) L[i] = 0;
        *the_min = -mn;
        return 0.f;
    }
    float iscale = nmax / (mx - mn);
    float scale = 1 / iscale;
    float best = 0;
    for (int i = 0; i < N; ++i) {
        L[i] = (uint8_t) imax(0, imin(nmax, nearest_int(iscale * (x[i] - mn))));
        const float d = scale * L[i] + mn - x[i];
        best += (IMAT ? kw(wts, x, i) : wts[i]) * (d * d);
    }
    for (int is = 0; is <= nstep; ++is) {
        iscale = (rmin + rdelta * is + nmax) / (mx - mn);
        float sl = 0, sl2 = 0, sxl = 0;
        uint32_t lp[N / 4];   // Laux, 8 bits a level
#pragma unroll
        for (int q = 0; q < N / 4; ++q) lp[q] = 0;
#pragma unroll
        for (int i = 0; i < N; ++i) {
            int l;
            if (IMAT) { const float v = iscale * (x[i] - mn); l = v > 0 ? nearest_int(v < nmax ? v : (float) nmax) : 0; }
            else l = imax(0, imin(nmax, nearest_int(iscale * (x[i] - mn))));
            lp[i / 4] |= (uint32_t) l << (8 * (i % 4));
            const float w = IMAT ? kw(wts, x, i) : wts[i];
            sl += w * l;
            sl2 += w * l * l;
            sxl += w * l * x[i];
        }
        const float D = sum_w * sl2 - sl * sl;
        if (!(D > 0)) continue;
        float ts = (sum_w * sxl - sum_x * sl) / D;
        float tm = (sl2 * sum_x - sl * sxl) / D;
        if (tm > 0) { tm = 0; ts = sxl / sl2; }
        float err = 0;
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const int l = (lp[i / 4] >> (8 * (i % 4))) & 255;
            const float d = ts * l + tm - x[i];
            err += (IMAT ? kw(wts, x, i) : wts[i]) * (d * d);
        }
        if (err < best) {
#pragma unroll
            for (int i = 0; i < N; ++i) L[i] = (uint8_t) ((lp[i / 4] >> (8 * (i % 4))) & 255);
            best = err; scale = ts; mn = tm;
        }
    }
    *the_min = -mn;
    return scale;
}

// signed levels -nmax..nmax-1 over 19 trial scales (gpuq.hip:1428-1466); L[i] = level + nmax
template <int N>
__device__ float sym_levels(int nmax, const float * x, uint8_t * L, const float * qw) {
    float amax = 0, mx = 0;
    for (int i = 0; i < N; ++i) { const float a = fabsf(x[i]); if (a > amax) { amax = a; mx = x[i]; } }
    if (amax < 1e-15f) { for (int i = 0; i < N; ++i) L[i] = 0; return 0.f; }
    float iscale = -nmax / mx;
    float slx = 0, sl2 = 0;
    for (int i = 0; i < N; ++i) {
        const int l = imax(-nmax, imin(nmax - 1, nearest_int(iscale * x[i])));
        L[i] = (uint8_t) (l + nmax);
        const float w = kw(qw, x, i);
        slx += w * x[i] * l;
        sl2 += w * l * l;
    }
    float scale = sl2 ? slx / sl2 : 0.0f;
    float best = scale * slx;
    for (int is = -9; is <= 9; ++is) {
        if (!is) continue;
        iscale = -(nmax + 0.1f * is) / mx;
        slx = sl2 = 0;
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const int l = imax(-nmax, imin(nmax - 1, nearest_int(iscale * x[i])));
            const float w = kw(qw, x, i);
            slx += w * x[i] * l;
            sl2 += w * l * l;
        }
        if (sl2 > 0 && slx * slx > best * sl2) {
            for (int i = 0; i < N; ++i) L[i] = (uint8_t) (nmax + imax(-nmax, imin(nmax - 1, nearest_int(iscale * x[i]))));
            scale = slx / sl2;
            best = scale * slx;
        }
    }
    return scale;
}

// Q3_K without imatrix (gpuq.hip:1469-1508): 3-bit levels, 5 coordinate-descent passes on x^2-weighted error
__device__ float sym3_levels(const float * x, uint8_t * Lout) {
    constexpr int N = 16, nmax = 4;
    float amax = 0, mx = 0;
    for (int i = 0; i < N; ++i) { const float a = fabsf(x[i]); if (a > amax) { amax = a; mx = x[i]; } }
    if (amax < 1e-15f) { for (int i = 0; i < N; ++i) Lout[i] = 0; return 0.f; }
    const float iscale = -nmax / mx;
    int8_t L[N];
    float slx = 0, sl2 = 0;
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const int l = imax(-nmax, imin(nmax - 1, nearest_int(iscale * x[i])));
        L[i] = (int8_t) l;
        const float w = x[i] * x[i];
        slx += w * x[i] * l;
        sl2 += w * l * l;
    }
    for (int pass = 0; pass < 5; ++pass) {
        int changed = 0;
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const float w = x[i] * x[i];
            float a = slx - w * x[i] * L[i];
            if (!(a > 0)) continue;
            float b = sl2 - w * L[i] * L[i];
            const int nl = imax(-nmax, imin(nmax - 1, nearest_int(x[i] * b / a)));
            if (nl == L[i]) continue;
            a += w * x[i] * nl;
            b += w * nl * nl;
            if (b > 0 && a * a * sl2 > slx * slx * b) { L[i] = (int8_t) nl; slx = a; sl2 = b; ++changed; }
        }
        if (!changed) break;
    }
#pragma unroll
    for (int i = 0; i < N; ++i) Lout[i] = (uint8_t) (L[i] + nmax);
    return sl2 > 0.0f ? slx / sl2 : 0.0f;
}

// make_qp_quants (gpuq.hip:114-176) over n scales, one lane; L out
template <int N>
__device__ float qp_levels(int nmax, const float * x, uint8_t * Lo, const float * w) {
    uint8_t L[N];
    float mx = 0;
    for (int i = 0; i < N; ++i) mx = fmaxr(mx, x[i]);
    if (mx < 1e-15f) { for (int i = 0; i < N; ++i) Lo[i] = 0; return 0.f; }
    float iscale = nmax / mx;
    const float scale0 = 1 / iscale;
    float best_mse = 0;
#pragma unroll
    for (int i = 0; i < N; ++i) {
        L[i] = (uint8_t) nearest_int(iscale * x[i]);
        const float d = x[i] - scale0 * L[i];
        best_mse += w[i] * d * d;
    }
    for (int is = -4; is <= 4; ++is) {
        if (!is) continue;
        const float iscale_is = (0.1f * is + nmax) / mx;
        const float scale_is = 1 / iscale_is;
        float mse = 0;
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const int l = imin(nmax, nearest_int(iscale_is * x[i]));
            const float d = x[i] - scale_is * l;
            mse += w[i] * d * d;
        }
        if (mse < best_mse) { best_mse = mse; iscale = iscale_is; }
    }
    float sumlx = 0, suml2 = 0;
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const int l = imin(nmax, nearest_int(iscale * x[i]));
        L[i] = (uint8_t) l;
        sumlx += w[i] * x[i] * l;
        suml2 += w[i] * l * l;
    }
    for (int pass = 0; pass < 5; ++pass) {
        int changed = 0;
#pragma unroll
        for (int i = 0; i < N; ++i) {
            float slx = sumlx - w[i] * x[i] * L[i];
            float sl2 = suml2 - w[i] * L[i] * L[i];
            if (slx > 0 && sl2 > 0) {
                const int nl = imin(nmax, nearest_int(x[i] * sl2 / slx));
                if (nl != L[i]) {
                    slx += w[i] * x[i] * nl;
                    sl2 += w[i] * nl * nl;
                    if (slx * slx * suml2 > sumlx * sumlx * sl2) { L[i] = (uint8_t) nl; sumlx = slx; suml2 = sl2; ++changed; }
                }
            }
        }
        if (!changed) break;
    }
#pragma unroll
    for (int i = 0; i < N; ++i) Lo[i] = L[i];
    return suml2 > 0.0f ? sumlx / suml2 : 0.0f;
}

// The IQ4 levels as floats and, for every integer k in [-127, 112], mu(k) = #{v <= k}: per CTA in shared memory
// (each lane indexes its own level: shared memory serves 16 distinct words without a conflict, where the constant
// cache would serialise them)
struct IQ4Tab { float v[16]; uint8_t mu[240]; };
__device__ __forceinline__ void iq4_tab_init(IQ4Tab & t) {
    for (int i = threadIdx.x; i < 240; i += blockDim.x) {
        int mu = 0;
        for (int j = 0; j < 16; ++j) mu += (i - 127) >= c_iq4[j];
        t.mu[i] = (uint8_t) mu;
    }
    if (threadIdx.x < 16) t.v[threadIdx.x] = (float) c_iq4[threadIdx.x];
}

// nearest of the 16 IQ4 levels (best_index_int8, gpuq.hip:1286-1295): x strictly inside the range lies in
// [v[mu-1], v[mu]) with mu = #{v <= x}; the levels are integers, so mu = #{v <= floor(x)}
__device__ __forceinline__ int iq4_index(float x, const IQ4Tab & t) {
    if (x <= -127.f) return 0;
    if (x >= 113.f) return 15;
    if (!(x == x)) return 15;   // (NaN: the reference's search ends on the last bracket)
    const int mu = t.mu[__float2int_rd(x) + 127];
    return x - t.v[mu - 1] < t.v[mu] - x ? mu - 1 : mu;
}

// one IQ4 sub-block's scale search (gpuq.hip:1311-1359), one lane: returns d (0 when skipped)
__device__ float iq4_sub(const float * xb, const float * w, const IQ4Tab & tb) {
    float amax = 0, mx = 0;
    for (int j = 0; j < 32; ++j) { const float ax = fabsf(xb[j]); if (ax > amax) { amax = ax; mx = xb[j]; } }
    if (amax < 1e-15f) return 0.f;
    float d = -mx / -127;
    float id = 1 / d;
    float sqx = 0, sq2 = 0;
    for (int j = 0; j < 32; ++j) {
        const float q = tb.v[iq4_index(id * xb[j], tb)];
        sqx += w[j] * q * xb[j];
        sq2 += w[j] * q * q;
    }
    d = sq2 > 0 ? sqx / sq2 : 0.f;
    float best = d * sqx;
    for (int t = -7; t <= 7; ++t) {
        id = (t + -127) / mx;
        sqx = sq2 = 0;
        for (int j = 0; j < 32; ++j) {
            const float q = tb.v[iq4_index(id * xb[j], tb)];
            sqx += w[j] * q * xb[j];
            sq2 += w[j] * q * q;
        }
        if (sq2 > 0 && sqx * sqx > best * sq2) { d = sqx / sq2; best = d * sqx; }
    }
    return d;
}

// ------------------------------------------------------------------------------------------------ the kernel
// CTAs an SM the register allocation is held to (measured: Q6_K runs best at 6, the others at 5, except Q4_K and
// Q5_K without an imatrix, which spill there and run best unbounded)
template <int T, bool IMAT> constexpr int kquant_min_ctas() {
    return T == Q6_K ? 6 : ((T == Q4_K || T == Q5_K) && !IMAT) ? 1 : 5;
}

template <int T, int SRC, bool IMAT>
__global__ void __launch_bounds__(128, kquant_min_ctas<T, IMAT>()) k_kquant(const uint8_t * __restrict__ src, const float * __restrict__ qw,
                                               int64_t qw_mod, int64_t qw_div, int64_t qw_mat,
                                               uint8_t * __restrict__ out, int64_t nblocks) {
    using S = KState<T>;
    constexpr int BL = S::BL, SB = S::SB, NB = S::NB, NSUBB = S::NSUBB, TILE = S::TILE, BB = block_bytes(T);
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ IQ4Tab s_iq4;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    S & st = reinterpret_cast<S *>(smem_raw)[wid];
    if constexpr (T == IQ4_NL || T == IQ4_XS) {    // (before any warp leaves: every thread reaches the barrier)
        iq4_tab_init(s_iq4);
        __syncthreads();
    }
    const int64_t b0 = ((int64_t) blockIdx.x * (blockDim.x >> 5) + wid) * NB;   // first block of this warp's tile
    if (b0 >= nblocks) return;
    const int nb = (int) (nblocks - b0 < NB ? nblocks - b0 : NB);                // blocks in this tile
    // ---- loads: 8 weights a lane a pass; importance weights of each block's row
#pragma unroll
    for (int p = 0; p < TILE / 256; ++p) {
        const int e = p * 256 + lane * 8;
        float v[8];
        if (e / BL < nb) decode8<SRC>(src, b0 * BL + e, v);
        else for (int j = 0; j < 8; ++j) v[j] = 0.f;
        const int xe = S::xi(e);                   // (8 elements from e lie in one sub-block)
#pragma unroll
        for (int j = 0; j < 8; ++j) st.x[xe + j] = v[j];
        if (IMAT) {
            const int blk = e / BL;
            float q[8];
            if (blk < nb) {
                const int64_t b = b0 + blk;
                load8_f32(qw + ((b / qw_mat) * qw_mod + (b % qw_mod) / qw_div) * BL + (e % BL), q);
            } else for (int j = 0; j < 8; ++j) q[j] = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) st.w[xe + j] = q[j];   // (raw importances; the search weights below)
        }
    }
    __syncwarp();
    // ---- per block: sumx2 in index order -> sigma2
    if (lane < NB) {
        float s2 = 0;
        for (int i = 0; i < BL; ++i) { const float v = st.x[S::xi(lane * BL + i)]; s2 += v * v; }
        if constexpr (T == IQ4_NL || T == IQ4_XS) st.sigma2[lane] = s2 * (2.f / BL);
        else if constexpr (T == Q2_K) st.sigma2[lane] = s2 / QK;
        else st.sigma2[lane] = 2 * s2 / QK;
    }
    __syncwarp();
    // ---- search weights, elementwise (imatrix paths; the plain paths build theirs inside the search)
    if (IMAT && T != Q6_K) {
#pragma unroll
        for (int p = 0; p < TILE / 256; ++p) {
            const int e = p * 256 + lane * 8;
            const float sg = st.sigma2[e / BL];
#pragma unroll
            for (int j = 0; j < 8; ++j) st.w[S::xi(e) + j] = st.w[S::xi(e) + j] * sqrtf(sg + st.x[S::xi(e) + j] * st.x[S::xi(e) + j]);
        }
    }
    if (!IMAT && (T == IQ4_NL || T == IQ4_XS)) {
#pragma unroll
        for (int p = 0; p < TILE / 256; ++p) {
            const int e = p * 256 + lane * 8;
#pragma unroll
            for (int j = 0; j < 8; ++j) st.w[S::xi(e) + j] = st.x[S::xi(e) + j] * st.x[S::xi(e) + j];
        }
    }
    __syncwarp();
    // ---- the level search, one sub-block a lane
    {
        const int s = lane;                       // sub-block of the tile
        const bool live = s / NSUBB < nb;
        const float * xb = st.x + s * S::SP;
        float * wb = st.w + s * S::SP;
        uint8_t * Lb = st.L + s * SB;
        float scale = 0, mn = 0, swv = 0;
        if (live) {
            if constexpr (T == Q2_K) {
                if (IMAT) {
                    for (int l = 0; l < 16; ++l) swv += wb[l];
                    scale = affine_levels<16, true>(3, xb, wb, Lb, &mn, -0.9f, 0.05f, 36, false);
                } else {
                    for (int l = 0; l < 16; ++l) wb[l] = fabsf(xb[l]);
                    scale = affine_levels<16, false>(3, xb, wb, Lb, &mn, -0.5f, 0.1f, 15, true);
                }
            } else if constexpr (T == Q3_K) {
                if (IMAT) {
                    for (int l = 0; l < 16; ++l) swv += wb[l];
                    scale = sym_levels<16>(4, xb, Lb, wb);
                } else {
                    scale = sym3_levels(xb, Lb);
                }
            } else if constexpr (T == Q4_K || T == Q5_K) {
                constexpr int NMAX = T == Q4_K ? 15 : 31;
                if (IMAT) {
                    for (int l = 0; l < 32; ++l) swv += wb[l];
                    scale = T == Q4_K ? affine_levels<32, true>(NMAX, xb, wb, Lb, &mn, -0.9f, 0.05f, 36, false)
                                      : affine_levels5<32, true>(NMAX, xb, wb, Lb, &mn, -0.9f, 0.05f, 36);
                } else {
                    float s2 = 0;
                    for (int l = 0; l < 32; ++l) s2 += xb[l] * xb[l];
                    const float av = sqrtf(s2 / 32);
                    for (int l = 0; l < 32; ++l) wb[l] = av + fabsf(xb[l]);
                    scale = T == Q4_K ? affine_levels<32, false>(NMAX, xb, wb, Lb, &mn, -1.f, 0.1f, 20, false)
                                      : affine_levels5<32, false>(NMAX, xb, wb, Lb, &mn, -0.5f, 0.1f, 15);
                }
            } else if constexpr (T == Q6_K) {
                scale = sym_levels<16>(32, xb, Lb, IMAT ? wb : nullptr);
            } else {   // IQ4_NL / IQ4_XS
                scale = iq4_sub(xb, wb, s_iq4);
            }
        }
        st.scales[s] = scale;
        st.mins[s] = mn;
        st.sw[s] = swv;
    }
    __syncwarp();
    // ---- per block: the scale codes and super-block scales (one lane a block)
    if (lane < nb) {
        const int k = lane;
        const float * scl = st.scales + k * NSUBB;
        const float * mns = st.mins + k * NSUBB;
        if constexpr (T == Q2_K) {
            if (!IMAT) {
                float max_scale = 0, max_min = 0;
                for (int j = 0; j < 16; ++j) { if (scl[j] > max_scale) max_scale = scl[j]; if (mns[j] > max_min) max_min = mns[j]; }
                uint8_t bytes[16];
                for (int j = 0; j < 16; ++j) bytes[j] = 0;
                uint16_t d16 = half_bits(0.f), dm16 = half_bits(0.f);
                if (max_scale > 0) {
                    const float is = 15.f / max_scale;
                    for (int j = 0; j < 16; ++j) bytes[j] = (uint8_t) nearest_int(is * scl[j]);
                    d16 = half_bits(max_scale / 15.f);
                }
                if (max_min > 0) {
                    const float im = 15.f / max_min;
                    for (int j = 0; j < 16; ++j) bytes[j] |= (uint8_t) (nearest_int(im * mns[j]) << 4);
                    dm16 = half_bits(max_min / 15.f);
                }
                for (int j = 0; j < 16; ++j) { st.sc[k][j] = bytes[j] & 0xF; st.mn[k][j] = bytes[j] >> 4; }
                st.d16[k] = d16; st.dm16[k] = dm16;
            } else {
                uint8_t Ls[16], Lm[16];
                const float dm = qp_levels<16>(15, scl, Ls, st.sw + k * 16);
                const float mm = qp_levels<16>(15, mns, Lm, st.sw + k * 16);
                st.d16[k] = half_bits(dm); st.dm16[k] = half_bits(mm);
                for (int j = 0; j < 16; ++j) { const uint8_t by = (uint8_t) (Ls[j] | (Lm[j] << 4)); st.sc[k][j] = by & 0xF; st.mn[k][j] = by >> 4; }
            }
        } else if constexpr (T == Q3_K) {
            int8_t Ls[16];
            uint16_t d16;
            if (!IMAT) {
                float amax = 0, max_scale = 0;
                for (int j = 0; j < 16; ++j) { const float a = fabsf(scl[j]); if (a > amax) { amax = a; max_scale = scl[j]; } }
                if (max_scale) {
                    const float iscale = -32.f / max_scale;
                    for (int j = 0; j < 16; ++j) { const int8_t l = (int8_t) nearest_int(iscale * scl[j]); Ls[j] = (int8_t) (imax(-32, imin(31, l)) + 32); }
                    d16 = half_bits(1 / iscale);
                } else {
                    for (int j = 0; j < 16; ++j) Ls[j] = -1;
                    d16 = half_bits(0.f);
                }
            } else {
                uint8_t Lu[16];
                d16 = half_bits(sym_levels<16>(32, scl, Lu, st.sw + k * 16));
                for (int j = 0; j < 16; ++j) Ls[j] = (int8_t) Lu[j];
            }
            uint8_t s12[12];
            for (int j = 0; j < 12; ++j) s12[j] = 0;
            for (int j = 0; j < 16; ++j) {
                if (Ls[j] < 0) break;
                const int l = Ls[j];
                if (j < 8) s12[j] = (uint8_t) (l & 0xF); else s12[j - 8] |= (uint8_t) ((l & 0xF) << 4);
                s12[j % 4 + 8] |= (uint8_t) ((l >> 4) << (2 * (j / 4)));
            }
            for (int j = 0; j < 12; ++j) st.q3s[k][j] = s12[j];
            for (int j = 0; j < 16; ++j) {
                int8_t sc = (int8_t) (j < 8 ? s12[j] & 0xF : s12[j - 8] >> 4);
                sc = (int8_t) ((sc | (((s12[8 + j % 4] >> (2 * (j / 4))) & 3) << 4)) - 32);
                st.s6[k][j] = sc;
            }
            st.d16[k] = d16;
        } else if constexpr (T == Q4_K || T == Q5_K) {
            uint8_t ls[8], lm[8];
            uint16_t d16, dm16;
            if (!IMAT) {
                float max_scale = 0, max_min = 0;
                for (int j = 0; j < 8; ++j) { if (scl[j] > max_scale) max_scale = scl[j]; if (mns[j] > max_min) max_min = mns[j]; }
                const float is = max_scale > 0 ? 63.f / max_scale : 0.f;
                const float im = max_min > 0 ? 63.f / max_min : 0.f;
                for (int j = 0; j < 8; ++j) {
                    const uint8_t a = (uint8_t) nearest_int(is * scl[j]), c = (uint8_t) nearest_int(im * mns[j]);
                    ls[j] = a < 63 ? a : 63;
                    lm[j] = c < 63 ? c : 63;
                }
                d16 = half_bits(max_scale / 63.f);
                dm16 = half_bits(max_min / 63.f);
            } else {
                const float db = qp_levels<8>(63, scl, ls, st.sw + k * 8);
                const float mb = qp_levels<8>(63, mns, lm, st.sw + k * 8);
                if (T == Q5_K) for (int j = 0; j < 8; ++j) { if (ls[j] > 63) ls[j] = 63; if (lm[j] > 63) lm[j] = 63; }
                d16 = half_bits(db);
                dm16 = half_bits(mb);
            }
            // the 12 packed scale bytes (gpuq.hip:1597-1604), then read back as ggml does (:1605-1608)
            uint8_t s12[12];
            for (int j = 0; j < 4; ++j) { s12[j] = ls[j]; s12[j + 4] = lm[j]; }
            for (int j = 4; j < 8; ++j) {
                s12[j + 4] = (uint8_t) ((ls[j] & 0xF) | ((lm[j] & 0xF) << 4));
                s12[j - 4] |= (uint8_t) ((ls[j] >> 4) << 6);
                s12[j] |= (uint8_t) ((lm[j] >> 4) << 6);
            }
            for (int j = 0; j < 12; ++j) st.q3s[k][j] = s12[j];
            for (int j = 0; j < 8; ++j) {
                if (j < 4) { st.sc[k][j] = s12[j] & 63; st.mn[k][j] = s12[j + 4] & 63; }
                else { st.sc[k][j] = (uint8_t) ((s12[j + 4] & 0xF) | ((s12[j - 4] >> 6) << 4)); st.mn[k][j] = (uint8_t) ((s12[j + 4] >> 4) | ((s12[j] >> 6) << 4)); }
            }
            st.d16[k] = d16; st.dm16[k] = dm16;
        } else if constexpr (T == Q6_K) {
            float amax = 0, max_scale = 0;
            for (int j = 0; j < 16; ++j) { const float a = fabsf(scl[j]); if (a > amax) { amax = a; max_scale = scl[j]; } }
            if (amax < 1e-15f) {
                st.valid[k] = 0;
            } else {
                st.valid[k] = 1;
                const float iscale = -128.f / max_scale;
                st.d16[k] = half_bits(1 / iscale);
                for (int j = 0; j < 16; ++j) st.s6[k][j] = (int8_t) imin(127, nearest_int(iscale * scl[j]));
            }
        } else if constexpr (T == IQ4_XS) {
            float max_scale = 0, amax_scale = 0;
            for (int j = 0; j < 8; ++j) { const float a = fabsf(scl[j]); if (a > amax_scale) { amax_scale = a; max_scale = scl[j]; } }
            const float d = -max_scale / 32;
            st.d16[k] = half_bits(d);
            const float id = d ? 1 / d : 0.f;
            uint16_t sh = 0;
            for (int j = 0; j < 8; ++j) {
                int l = imax(-32, imin(31, nearest_int(id * scl[j])));
                st.mins[k * 8 + j] = d * l;          // dl: the rounding scale of sub-block j
                l += 32;
                st.sc[k][j] = (uint8_t) (l & 0xf);
                sh |= (uint16_t) ((l >> 4) << (2 * j));
            }
            st.sh[k] = sh;
        } else {   // IQ4_NL: the block scale is the sub-block's
            st.d16[k] = half_bits(scl[0]);
        }
    }
    __syncwarp();
    // ---- final rounding against the stored scales, elementwise
#pragma unroll
    for (int p = 0; p < TILE / 256; ++p) {
        const int e0 = p * 256 + lane * 8;
        const int k = e0 / BL;
        if (k >= nb) continue;
        const int j = (e0 % BL) / SB;         // sub-block in the block
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            const int e = e0 + t;
            const float xv = st.x[S::xi(e)];
            if constexpr (T == Q2_K || T == Q4_K || T == Q5_K) {
                constexpr int NMAX = T == Q2_K ? 3 : T == Q4_K ? 15 : 31;
                const float dj = half_to_float(st.d16[k]) * st.sc[k][j];
                if (!dj) continue;
                const float mj = half_to_float(st.dm16[k]) * st.mn[k][j];
                st.L[e] = (uint8_t) imax(0, imin(NMAX, nearest_int((xv + mj) / dj)));
            } else if constexpr (T == Q3_K) {
                const float dj = half_to_float(st.d16[k]) * st.s6[k][j];
                if (!dj) continue;
                st.L[e] = (uint8_t) (imax(-4, imin(3, nearest_int(xv / dj))) + 4);
            } else if constexpr (T == Q6_K) {
                if (!st.valid[k]) continue;
                const float dj = half_to_float(st.d16[k]) * st.s6[k][j];
                if (!dj) continue;
                st.L[e] = (uint8_t) (imax(-32, imin(31, nearest_int(xv / dj))) + 32);
            } else if constexpr (T == IQ4_XS) {
                const float dl = st.mins[k * 8 + j];
                const float idl = dl ? 1 / dl : 0.f;
                st.L[e] = (uint8_t) iq4_index(idl * xv, s_iq4);
            } else {
                const float s0 = st.scales[k];
                const float id = s0 ? 1 / s0 : 0;
                st.L[e] = (uint8_t) iq4_index(id * xv, s_iq4);
            }
        }
    }
    __syncwarp();
    // ---- block bytes: one output byte a lane, coalesced
    uint8_t * yo = out + b0 * BB;
    for (int i = lane; i < nb * BB; i += 32) {
        const int k = i / BB, o = i % BB;
        const uint8_t * L = st.L + k * BL;
        uint8_t v = 0;
        if constexpr (T == Q2_K) {
            if (o < 16) v = (uint8_t) (st.sc[k][o] | (st.mn[k][o] << 4));
            else if (o < 80) { const int q = o - 16, base = (q / 32) * 128, l = q % 32;
                               v = (uint8_t) (L[base + l] | (L[base + l + 32] << 2) | (L[base + l + 64] << 4) | (L[base + l + 96] << 6)); }
            else if (o < 82) v = (uint8_t) (st.d16[k] >> (8 * (o - 80)));
            else v = (uint8_t) (st.dm16[k] >> (8 * (o - 82)));
        } else if constexpr (T == Q3_K) {
            if (o < 32) { for (int t = 0; t < 8; ++t) v |= (uint8_t) ((L[o + 32 * t] > 3) << t); }
            else if (o < 96) { const int q = o - 32, base = (q / 32) * 128, l = q % 32;
                               auto lo = [&](int e) { return (L[e] > 3 ? L[e] - 4 : L[e]) & 3; };
                               v = (uint8_t) (lo(base + l) | (lo(base + l + 32) << 2) | (lo(base + l + 64) << 4) | (lo(base + l + 96) << 6)); }
            else if (o < 108) v = st.q3s[k][o - 96];
            else v = (uint8_t) (st.d16[k] >> (8 * (o - 108)));
        } else if constexpr (T == Q4_K) {
            if (o < 2) v = (uint8_t) (st.d16[k] >> (8 * o));
            else if (o < 4) v = (uint8_t) (st.dm16[k] >> (8 * (o - 2)));
            else if (o < 16) v = st.q3s[k][o - 4];
            else { const int q = o - 16, base = (q / 32) * 64, l = q % 32; v = (uint8_t) (L[base + l] | (L[base + l + 32] << 4)); }
        } else if constexpr (T == Q5_K) {
            if (o < 2) v = (uint8_t) (st.d16[k] >> (8 * o));
            else if (o < 4) v = (uint8_t) (st.dm16[k] >> (8 * (o - 2)));
            else if (o < 16) v = st.q3s[k][o - 4];
            else if (o < 48) { const int j = o - 16; for (int t = 0; t < 4; ++t) v |= (uint8_t) (((L[64 * t + j] > 15) | ((L[64 * t + j + 32] > 15) << 1)) << (2 * t)); }
            else { const int q = o - 48, base = (q / 32) * 64, l = q % 32; v = (uint8_t) ((L[base + l] & 15) | ((L[base + l + 32] & 15) << 4)); }
        } else if constexpr (T == Q6_K) {
            if (!st.valid[k]) v = 0;
            else if (o < 128) { const int half = o / 64, q = o % 64, l = q % 32, sh = q / 32; const uint8_t * Lh = L + 128 * half;
                                v = (uint8_t) ((Lh[l + 32 * sh] & 0xF) | ((Lh[l + 32 * sh + 64] & 0xF) << 4)); }
            else if (o < 192) { const int half = (o - 128) / 32, l = (o - 128) % 32; const uint8_t * Lh = L + 128 * half;
                                v = (uint8_t) ((Lh[l] >> 4) | ((Lh[l + 32] >> 4) << 2) | ((Lh[l + 64] >> 4) << 4) | ((Lh[l + 96] >> 4) << 6)); }
            else if (o < 208) v = (uint8_t) st.s6[k][o - 192];
            else v = (uint8_t) (st.d16[k] >> (8 * (o - 208)));
        } else if constexpr (T == IQ4_XS) {
            if (o < 2) v = (uint8_t) (st.d16[k] >> (8 * o));
            else if (o < 4) v = (uint8_t) (st.sh[k] >> (8 * (o - 2)));
            else if (o < 8) v = (uint8_t) (st.sc[k][2 * (o - 4)] | (st.sc[k][2 * (o - 4) + 1] << 4));
            else { const int q = o - 8, i32 = q / 16, j = q % 16; v = (uint8_t) (L[32 * i32 + j] | (L[32 * i32 + 16 + j] << 4)); }
        } else {   // IQ4_NL
            if (o < 2) v = (uint8_t) (st.d16[k] >> (8 * o));
            else { const int j = o - 2; v = (uint8_t) (L[j] | (L[16 + j] << 4)); }
        }
        yo[i] = v;
    }
}

// Q8_0 (gpuq.hip:1831-1838): d = amax / 127, the values roundf(x * (1 / d)) as int8. One thread a 32-weight block.
//
// ggml's roundf (half away from zero) is formed as trunc(x + copysign(0.5 - 2^-25, x)) in float32, which equals it
// for every finite |x| < 2^22 (here |x| <= 127 up to rounding): for x >= 0.5 the sum of x and a number just below 0.5
// crosses the integer above x exactly when x >= k + 0.5 (the sum's rounding error, at most half an ulp of the result,
// cannot reach the next integer from below k + 0.5, and an exact tie k + 0.5 rounds up to k + 1), and for
// x < 0.5 - 2^-25 ... 0.5 it stays below 1 - the case where x + 0.5 would round up to 1.0 (x = 0.5 - 2^-25) is the
// reason for the smaller addend. Non-finite x give what the conversion gives for roundf's result (NaN 0, inf
// saturated). The equality is checked against CUDA's roundf over every float below 2^22 by a GPU test.
__device__ __forceinline__ int round_half_away(float x) {
    return __float2int_rz(x + copysignf(0.49999997f, x));
}

// one block: v[32] -> 34 bytes at y (any address space; 2-byte aligned). ggml's amax is a sequential fold,
// amax = MAX(amax, fabsf(x)) with MAX(a, b) = a > b ? a : b, from 0; for a block without NaN that is the maximum of the
// |x| (an fmax reduction); a NaN changes the fold (a NaN operand makes it NaN, the next value replaces it), so a block
// whose sum of values is NaN (any NaN, or infinities of both signs) folds again in ggml's order.
__device__ __forceinline__ void q8_0_block(const float * v, uint8_t * y) {
    // (both reductions as trees: fmaxf is associative, and the sum is NaN in any order exactly when a NaN, or
    // infinities of both signs, are present)
    float m[16], c[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) { m[j] = fmaxf(fabsf(v[j]), fabsf(v[j + 16])); c[j] = v[j] + v[j + 16]; }
#pragma unroll
    for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
        for (int j = 0; j < w; ++j) { m[j] = fmaxf(m[j], m[j + w]); c[j] = c[j] + c[j + w]; }
    float amax = fmaxf(0.0f, m[0]);
    const float chk = c[0];
    if (chk != chk) {
        amax = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) { const float a = fabsf(v[j]); amax = amax > a ? amax : a; }
    }
    const float d = amax / 127;
    const float id = d ? 1.0f / d : 0.0f;
    uint16_t * y16 = reinterpret_cast<uint16_t *>(y);
    y16[0] = half_bits(d);
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
        const uint32_t lo = (uint8_t) round_half_away(v[j] * id), hi = (uint8_t) round_half_away(v[j + 1] * id);
        y16[1 + j / 2] = (uint16_t) (lo | (hi << 8));
    }
}

// the plain form (global loads and stores): blocks after the last whole tile of the bulk kernel, or every block of a
// buffer that a bulk copy cannot address
template <int SRC>
__global__ void __launch_bounds__(256) k_q8_0(const uint8_t * __restrict__ src, uint8_t * __restrict__ out, int64_t nblocks) {
    const int64_t stride = (int64_t) gridDim.x * blockDim.x;
    for (int64_t b = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; b < nblocks; b += stride) {
        float v[32];
#pragma unroll
        for (int k = 0; k < 4; ++k) decode8<SRC>(src, b * 32 + 8 * k, v + 8 * k);
        q8_0_block(v, out + b * 34);
    }
}

template <int T, int SRC, bool IMAT>
__global__ void __launch_bounds__(128) k_legacy(const uint8_t * __restrict__ src, const float * __restrict__ qw,
                                                int64_t qw_mod, int64_t qw_div, int64_t qw_mat,
                                                uint8_t * __restrict__ out, int64_t n_per_row) {
    __shared__ float s_sigma2;
    const int64_t row = blockIdx.x, nb_row = n_per_row / 32;
    if (IMAT) {
        if (threadIdx.x == 0) {
            float s = 0;
            for (int64_t v = 0; v < n_per_row; v += 8) {
                float x8[8];
                decode8<SRC>(src, row * n_per_row + v, x8);
#pragma unroll
                for (int j = 0; j < 8; ++j) s += x8[j] * x8[j];
            }
            s_sigma2 = s / n_per_row;
        }
        __syncthreads();
    }
    for (int64_t ib = threadIdx.x; ib < nb_row; ib += blockDim.x) {
        const int64_t b = row * nb_row + ib;
        float x[32];
#pragma unroll
        for (int k = 0; k < 4; ++k) decode8<SRC>(src, b * 32 + 8 * k, x + 8 * k);
        uint8_t L[32];
        float d, m = 0.f;
        if constexpr (IMAT) {
            const float * q = qw + ((b / qw_mat) * qw_mod + (b % qw_mod) / qw_div) * 32;
            const float sigma2 = s_sigma2;
            float w[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) w[j] = __ldg(q + j) * sqrtf(sigma2 + x[j] * x[j]);
            if constexpr (T == Q5_1) {
                float the_min;
                d = affine_levels5<32, true>(31, x, w, L, &the_min, -0.9f, 0.05f, 36);
                m = -the_min;
            } else {
                d = sym_levels<32>(T == Q4_0 ? 8 : 16, x, L, w);
            }
        } else if constexpr (T == Q5_1) {
            float mn = FLT_MAX, mx = -FLT_MAX;
#pragma unroll
            for (int j = 0; j < 32; ++j) { if (x[j] < mn) mn = x[j]; if (x[j] > mx) mx = x[j]; }
            d = (mx - mn) / 31;
            const float id = d ? 1.0f / d : 0.0f;
            m = mn;
#pragma unroll
            for (int j = 0; j < 32; ++j) L[j] = (uint8_t) ((x[j] - mn) * id + 0.5f);
        } else {
            constexpr int nl = T == Q4_0 ? 8 : 16;
            float amax = 0.0f, mx = 0.0f;
#pragma unroll
            for (int j = 0; j < 32; ++j) if (amax < fabsf(x[j])) { amax = fabsf(x[j]); mx = x[j]; }
            d = mx / -nl;
            const float id = d ? 1.0f / d : 0.0f;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int v = (int8_t) (int) (x[j] * id + (nl + 0.5f));
                L[j] = (uint8_t) (v < 2 * nl - 1 ? v : 2 * nl - 1);
            }
        }
        uint8_t * y = out + b * block_bytes(T);
        const uint16_t dh = half_bits(d);
        y[0] = (uint8_t) dh; y[1] = (uint8_t) (dh >> 8);
        int o = 2;
        if constexpr (T == Q5_1) { const uint16_t mh = half_bits(m); y[2] = (uint8_t) mh; y[3] = (uint8_t) (mh >> 8); o = 4; }
        if constexpr (T != Q4_0) {
            uint32_t h = 0;
#pragma unroll
            for (int j = 0; j < 16; ++j) h |= ((uint32_t) ((L[j] >> 4) & 1) << j) | ((uint32_t) ((L[j + 16] >> 4) & 1) << (j + 16));
#pragma unroll
            for (int k = 0; k < 4; ++k) y[o + k] = (uint8_t) (h >> (8 * k));
            o += 4;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) y[o + j] = (uint8_t) ((L[j] & 15) | ((L[j + 16] & 15) << 4));
    }
}

template <int T, int SRC>
cudaError_t launch_legacy_t(const LaunchArgs & a) {
    const int64_t nb_row = a.n_per_row / 32;
    if (a.n_per_row <= 0 || a.n_per_row % 32 || a.nblocks % nb_row) return cudaErrorInvalidValue;
    const int64_t rows = a.nblocks / nb_row;
    if (rows > 0x7FFFFFFF) return cudaErrorInvalidValue;
    if (a.qw)
        k_legacy<T, SRC, true><<<(unsigned) rows, 128, 0, a.stream>>>((const uint8_t *) a.src, a.qw, a.qw_mod, a.qw_div,
                                                                      a.qw_mat, (uint8_t *) a.out, a.n_per_row);
    else
        k_legacy<T, SRC, false><<<(unsigned) rows, 128, 0, a.stream>>>((const uint8_t *) a.src, nullptr, 1, 1, 1,
                                                                       (uint8_t *) a.out, a.n_per_row);
    return cudaGetLastError();
}

template <int T>
cudaError_t launch_legacy_src(const LaunchArgs & a) {
    switch (a.src_type) {
        case SRC_F32:   return launch_legacy_t<T, SRC_F32>(a);
        case SRC_F16:   return launch_legacy_t<T, SRC_F16>(a);
        case SRC_BF16:  return launch_legacy_t<T, SRC_BF16>(a);
        case SRC_Q8_0:  return launch_legacy_t<T, SRC_Q8_0>(a);
        case SRC_MXFP4: return launch_legacy_t<T, SRC_MXFP4>(a);
        default: return cudaErrorInvalidValue;
    }
}

// Q8_0 on whole tiles of 256 blocks, the bytes moved by the Blackwell copy engine: a persistent CTA keeps three
// source tiles in flight with 1-D TMA bulk loads (cp.async.bulk, completion counted on an mbarrier a stage), its 256
// threads quantize a tile from shared memory (one thread a block, q8_0_block) into a shared-memory copy of the 8,704
// output bytes, and one thread writes them back with a TMA bulk store. Every wait is bounded: a wait that runs out
// sets ST_TIMEOUT in the status word and the CTA drains its own copies (again with bounds) and returns.
constexpr int Q8T = 256, Q8STAGES = 2, Q8OUT = Q8T * 34;
constexpr unsigned Q8_SPIN = 1u << 22;   // try_wait rounds before a wait is declared lost

__device__ __forceinline__ uint32_t smem_u32(const void * p) { return (uint32_t) __cvta_generic_to_shared(p); }
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t phase) {
    uint32_t done;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(done) : "r"(bar), "r"(phase) : "memory");
    return done != 0;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t phase) {
    for (unsigned it = 0; it < Q8_SPIN; ++it) if (mbar_try(bar, phase)) return true;
    return false;
}

template <int SRC>
__global__ void __launch_bounds__(256) k_q8_0_bulk(const uint8_t * __restrict__ src, uint8_t * __restrict__ out,
                                                   int64_t ntiles, unsigned * status) {
    constexpr int IN = Q8T * src_bytes32(SRC);
    extern __shared__ __align__(128) unsigned char q8s[];
    uint8_t * inb = q8s;                          // Q8STAGES x IN
    uint8_t * ob = q8s + Q8STAGES * IN;           // 2 x Q8OUT
    __shared__ __align__(8) uint64_t full[Q8STAGES];
    __shared__ int s_fail;
    const int tid = threadIdx.x;
    const int64_t first = blockIdx.x, stride = gridDim.x;
    const int64_t count = first < ntiles ? (ntiles - 1 - first) / stride + 1 : 0;
    if (tid == 0) {
        s_fail = 0;
        for (int st = 0; st < Q8STAGES; ++st) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&full[st])) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    auto issue = [&](int st, int64_t tile) {      // (thread 0) the tile's source bytes into stage st
        const uint32_t bar = smem_u32(&full[st]);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(IN) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                     ::"r"(smem_u32(inb + st * IN)), "l"(src + tile * IN), "r"(IN), "r"(bar) : "memory");
    };
    if (tid == 0)
        for (int st = 0; st < Q8STAGES && st < count; ++st) issue(st, first + st * stride);
    int64_t i = 0;
    for (; i < count; ++i) {
        const int st = (int) (i % Q8STAGES);
        const uint32_t phase = (uint32_t) ((i / Q8STAGES) & 1);
        if (tid == 0 && i >= 2) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");   // out buffer i&1 free
        if (!mbar_wait_bounded(smem_u32(&full[st]), phase)) atomicOr(&s_fail, 1);
        __syncthreads();
        if (s_fail) break;
        const uint8_t * tin = inb + st * IN;
        uint8_t * tout = ob + (i & 1) * Q8OUT;
        {
            float v[32];
#pragma unroll
            for (int k = 0; k < 4; ++k) decode8<SRC, false>(tin, (int64_t) tid * 32 + 8 * k, v + 8 * k);
            q8_0_block(v, tout + tid * 34);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the staged bytes visible to the bulk store
        __syncthreads();                                                // stage st read, out buffer written
        if (tid == 0) {
            const int64_t tile = first + i * stride;
            asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                         ::"l"(out + tile * Q8OUT), "r"(smem_u32(tout)), "r"(Q8OUT) : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            if (i + Q8STAGES < count) issue(st, first + (i + Q8STAGES) * stride);
        }
    }
    if (tid == 0) {
        if (s_fail) {   // a wait ran out: report it, let the loads still in flight land (bounded) and return
            atomicOr(status, ST_TIMEOUT);
            for (int64_t k = i; k < count && k < i + Q8STAGES; ++k)
                mbar_wait_bounded(smem_u32(&full[k % Q8STAGES]), (uint32_t) ((k / Q8STAGES) & 1));
        }
        asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");     // every store of this CTA complete
    }
}

template <int SRC>
size_t q8_bulk_smem() { return (size_t) Q8STAGES * Q8T * src_bytes32(SRC) + 2 * Q8OUT; }

template <int T, int SRC>
cudaError_t launch_t(const LaunchArgs & a) {
    if constexpr (T == Q8_0) {
        const int64_t ntiles = a.nblocks / Q8T;
        const bool aligned = ((reinterpret_cast<uintptr_t>(a.src) | reinterpret_cast<uintptr_t>(a.out)) & 15) == 0;
        int64_t done = 0;
        if (aligned && ntiles > 0 && a.status) {
            int dev = 0, sms = 148, per_sm = 0;
            cudaGetDevice(&dev);
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
            const size_t smem = q8_bulk_smem<SRC>();
            cudaError_t e = cudaFuncSetAttribute(k_q8_0_bulk<SRC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
            if (e != cudaSuccess) return e;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_q8_0_bulk<SRC>, 256, smem) != cudaSuccess || per_sm < 1) per_sm = 1;
            const int64_t grid = ntiles < (int64_t) sms * per_sm ? ntiles : (int64_t) sms * per_sm;
            k_q8_0_bulk<SRC><<<(unsigned) grid, 256, smem, a.stream>>>((const uint8_t *) a.src, (uint8_t *) a.out, ntiles,
                                                                       a.status);
            if ((e = cudaGetLastError()) != cudaSuccess) return e;
            done = ntiles * Q8T;
        }
        if (done == a.nblocks) return cudaSuccess;
        // the blocks after the last whole tile (or every block, for buffers a bulk copy cannot address)
        int dev = 0, sms = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const int64_t rest = a.nblocks - done;
        const int64_t need = (rest + 255) / 256;
        const int grid = (int) (need < (int64_t) sms * 8 ? (need > 0 ? need : 1) : (int64_t) sms * 8);
        k_q8_0<SRC><<<grid, 256, 0, a.stream>>>((const uint8_t *) a.src + (size_t) done * src_bytes32(SRC),
                                               (uint8_t *) a.out + (size_t) done * 34, rest);
        return cudaGetLastError();
    } else {
        constexpr int WARPS = 4;
        const size_t smem = sizeof(KState<T>) * WARPS;
        static_assert(sizeof(KState<T>) * WARPS <= 48 * 1024, "static smem budget");
        const int64_t per_cta = (int64_t) WARPS * KState<T>::NB;
        const int64_t grid = (a.nblocks + per_cta - 1) / per_cta;
        if (a.qw)
            k_kquant<T, SRC, true><<<(unsigned) grid, WARPS * 32, smem, a.stream>>>(
                (const uint8_t *) a.src, a.qw, a.qw_mod, a.qw_div, a.qw_mat, (uint8_t *) a.out, a.nblocks);
        else
            k_kquant<T, SRC, false><<<(unsigned) grid, WARPS * 32, smem, a.stream>>>(
                (const uint8_t *) a.src, nullptr, 1, 1, 1, (uint8_t *) a.out, a.nblocks);
        return cudaGetLastError();
    }
}

template <int T>
cudaError_t launch_src(const LaunchArgs & a) {
    switch (a.src_type) {
        case SRC_F32:   return launch_t<T, SRC_F32>(a);
        case SRC_F16:   return launch_t<T, SRC_F16>(a);
        case SRC_BF16:  return launch_t<T, SRC_BF16>(a);
        case SRC_Q8_0:  return launch_t<T, SRC_Q8_0>(a);
        case SRC_MXFP4: return launch_t<T, SRC_MXFP4>(a);
        default: return cudaErrorInvalidValue;
    }
}

// every float x with 0 <= x < 2^22 (bit patterns 0 .. 0x4A7FFFFF), and -x: round_half_away(x) against CUDA's roundf
__global__ void k_check_round(uint32_t n, unsigned long long * bad) {
    const uint32_t stride = gridDim.x * blockDim.x;
    unsigned long long local = 0;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const float x = __uint_as_float(i);
        local += round_half_away(x) != (int) roundf(x);
        local += round_half_away(-x) != (int) roundf(-x);
    }
    if (local) atomicAdd(bad, local);
}

}  // namespace

cudaError_t launch_kquant(int type, const LaunchArgs & a) {
    switch (type) {
        case Q2_K: return launch_src<Q2_K>(a);
        case Q3_K: return launch_src<Q3_K>(a);
        case Q4_K: return launch_src<Q4_K>(a);
        case Q5_K: return launch_src<Q5_K>(a);
        case Q6_K: return launch_src<Q6_K>(a);
        case Q8_0: return launch_src<Q8_0>(a);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_legacy(int type, const LaunchArgs & a) {
    switch (type) {
        case Q4_0: return launch_legacy_src<Q4_0>(a);
        case Q5_0: return launch_legacy_src<Q5_0>(a);
        case Q5_1: return launch_legacy_src<Q5_1>(a);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_iq4(int type, const LaunchArgs & a) {
    switch (type) {
        case IQ4_NL: return launch_src<IQ4_NL>(a);
        case IQ4_XS: return launch_src<IQ4_XS>(a);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace gq

// A diagnostic (no counterpart in the reference): the number of floats below 2^22 in magnitude for which the Q8_0
// kernels' rounding differs from CUDA's roundf (0 expected), -1 when the check could not run. Synchronous, current
// device; allocates 8 bytes of device memory for the count.
extern "C" int64_t gpuq_check_q8_rounding(void) {
    unsigned long long * d = nullptr, h = 0;
    if (cudaMalloc(&d, sizeof(h)) != cudaSuccess) { cudaGetLastError(); return -1; }
    cudaMemset(d, 0, sizeof(h));
    gq::k_check_round<<<148 * 8, 256>>>(0x4A800000u, d);
    const bool ok = cudaGetLastError() == cudaSuccess && cudaMemcpy(&h, d, sizeof(h), cudaMemcpyDeviceToHost) == cudaSuccess;
    cudaFree(d);
    return ok ? (int64_t) h : -1;
}
