// ldlq_sub.cu - the IQ2_XXS sub-block variant of LDLQ (trench-gguf tools/ldlq.py:117-272, which the reference runs on
// the CPU only).
//
// What is computed: ggml's IQ2_XXS pass fixes a super-block's scale d and its eight 4-bit sub-block scales; then,
// every `sub` columns (32: a sub-block, 8: one codebook group), each 8-weight group's point is chosen again over all
// 256 points of the IQ2_XXS grid on the error-updated weights, against the values inference produces
// (grid * d * (0.5 + l) * 0.25), with ggml's sign rule (signs follow x; an odd count of minus signs flips the
// cheapest weight), optionally trying the sub-block scale l-K..l+K as well, and the error is fed forward (ldlq.cu's
// float64 GEMMs with K = 32 or 8). The arithmetic is the reference's numpy arithmetic: the dequant scale and the
// costs in float64 (numpy promotes the float32 d with the int64 levels), 4 w |x| in float32 then times the float64
// point, 8-term sums as numpy's pairwise sum ((e0 + e1) + (e2 + e3)) + ((e4 + e5) + (e6 + e7)), first minima (a NaN
// is the smallest, as numpy's argmin), the super-block's sigma2 as numpy's float32 pairwise row sum.
//
// How: k_sub_weff: one warp a row, the row's 256 squares summed by numpy's schedule (two halves, 8 interleaved
// accumulators each) by 16 lanes, then the weights qw * sqrt(sigma2 + x^2). k_sub_points: one warp a row; for each
// scale tried and each group, the lanes take 8 grid points each and the warp reduces to the first minimum; the chosen
// points' error x - q goes out in float64 for the feedback, the group's grid index, sign bits and scale go straight
// into the block's bytes (ggml's pass wrote d; every group's fields are rewritten by the time the super-block ends).
#include <cstdint>
#include "common.cuh"
#include "kernels.h"

namespace gq {
namespace {

// numpy's argmin order: NaN first, then the smaller value, ties to the smaller index
__device__ __forceinline__ bool before(double a, int ia, double b, int ib) {
    const bool na = a != a, nb = b != b;
    if (na != nb) return na;
    if (na) return ia < ib;
    return a < b || (a == b && ia < ib);
}

__device__ __forceinline__ double sum8(const double (&e)[8]) {
    return ((e[0] + e[1]) + (e[2] + e[3])) + ((e[4] + e[5]) + (e[6] + e[7]));
}

__global__ void __launch_bounds__(128) k_sub_weff(const float * __restrict__ blk, const float * __restrict__ qw,
                                                  int64_t qw_div, float * __restrict__ weff, int64_t rows) {
    __shared__ float sq[4][QK];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t r = (int64_t) blockIdx.x * 4 + wid;
    if (r >= rows) return;
    const float * x = blk + r * QK;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) { v[j] = x[lane * 8 + j]; sq[wid][lane * 8 + j] = v[j] * v[j]; }
    __syncwarp();
    // numpy's pairwise float32 sum of 256: halves of 128, each by accumulators r_j = a_j + a_{j+8} + ... in order
    float acc = 0.f;
    if (lane < 16) {
        const float * a = sq[wid] + (lane >> 3) * 128 + (lane & 7);
        acc = a[0];
#pragma unroll
        for (int i = 1; i < 16; ++i) acc = acc + a[8 * i];
    }
    float rj[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) rj[j] = __shfl_sync(0xFFFFFFFFu, acc, j);
    const float h0 = ((rj[0] + rj[1]) + (rj[2] + rj[3])) + ((rj[4] + rj[5]) + (rj[6] + rj[7]));
    const float h1 = ((rj[8] + rj[9]) + (rj[10] + rj[11])) + ((rj[12] + rj[13]) + (rj[14] + rj[15]));
    const float sigma2 = (h0 + h1) / QK;
    const float * q = qw + (r / qw_div) * QK;
#pragma unroll
    for (int j = 0; j < 8; ++j) weff[r * QK + lane * 8 + j] = q[lane * 8 + j] * sqrtf(sigma2 + v[j] * v[j]);
}

__device__ __forceinline__ uint32_t ld32(const uint8_t * p) {
    return (uint32_t) p[0] | ((uint32_t) p[1] << 8) | ((uint32_t) p[2] << 16) | ((uint32_t) p[3] << 24);
}
__device__ __forceinline__ void st32(uint8_t * p, uint32_t v) {
    p[0] = (uint8_t) v; p[1] = (uint8_t) (v >> 8); p[2] = (uint8_t) (v >> 16); p[3] = (uint8_t) (v >> 24);
}

// NG groups of 8 (4: sub = 32; 1: sub = 8) starting at column c0 of the super-block, one warp a row
template <int NG>
__global__ void __launch_bounds__(128) k_sub_points(const float * __restrict__ blk, const float * __restrict__ weff,
                                                    uint8_t * __restrict__ q, double * __restrict__ err, int64_t rows,
                                                    int c0, int scale_search, const uint64_t * __restrict__ grid) {
    constexpr int SUBW = NG * 8;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t r = (int64_t) blockIdx.x * 4 + wid;
    if (r >= rows) return;
    uint8_t * y = q + r * 66;
    const int ib = c0 / 32, g0 = (c0 % 32) / 8;
    const float d = half_to_float((uint16_t) (y[0] | (y[1] << 8)));
    uint8_t * wp = y + 2 + 8 * ib;
    uint32_t w0 = ld32(wp), w1 = ld32(wp + 4);
    const int ls = (int) (w1 >> 28);
    const float * xr = blk + r * QK + c0;      // every lane reads the same addresses: broadcasts from L1
    const float * wr = weff + r * QK + c0;
    const int nss = NG == 4 ? scale_search : 0;
    double best_total = 0;
    int best_l = ls;
    uint64_t best_sel = 0;                     // per group g: bits 11g..: point (8 bits), flipped weight (3 bits)
    bool have = false;
#pragma unroll 1
    for (int dl = -nss; dl <= nss; ++dl) {
        int lt = ls + dl;
        lt = lt < 0 ? 0 : (lt > 15 ? 15 : lt);
        const double db = (double) d * (0.5 + (double) lt) * 0.25;
        double total = 0.0;
        uint64_t sel = 0;
#pragma unroll 1
        for (int g = 0; g < NG; ++g) {
            double ax[8], w[8];
            float w4ax[8];
            int nneg = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float xf = xr[8 * g + i], wf = wr[8 * g + i];
                const float a32 = fabsf(xf);
                ax[i] = (double) a32;
                w[i] = (double) wf;
                w4ax[i] = (4.0f * wf) * a32;
                nneg += xf < 0;
            }
            const bool odd = nneg & 1;
            double bc = 0.0;
            int bp = -1, bf = 0;
#pragma unroll 1
            for (int m = 0; m < 8; ++m) {                 // this lane's points: lane, lane + 32, ...
                const int p = lane + 32 * m;
                const uint64_t pt = __ldg(grid + p);
                double e[8], fl[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const double v = (double) (int) ((pt >> (8 * i)) & 0xFF) * db;
                    const double t = ax[i] - v;
                    e[i] = w[i] * (t * t);
                    fl[i] = (double) w4ax[i] * v;
                }
                int fi = 0;
#pragma unroll
                for (int i = 1; i < 8; ++i) if (before(fl[i], i, fl[fi], fi)) fi = i;
                double c = sum8(e);
                c = c + (odd ? fl[fi] : 0.0);
                if (bp < 0 || before(c, p, bc, bp)) { bc = c; bp = p; bf = fi; }
            }
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) {           // the warp's first minimum
                const double oc = __shfl_xor_sync(0xFFFFFFFFu, bc, o);
                const int op = __shfl_xor_sync(0xFFFFFFFFu, bp, o), of = __shfl_xor_sync(0xFFFFFFFFu, bf, o);
                if (before(oc, op, bc, bp)) { bc = oc; bp = op; bf = of; }
            }
            sel |= (uint64_t) (bp | (bf << 8)) << (11 * g);
            total = total + bc;
        }
        if (!have || total < best_total) {
            have = true;
            best_total = total;
            best_l = lt;
            best_sel = sel;
        }
    }
    // the chosen points: the error for the feedback (float64) and the block's fields
    const double db = (double) d * (0.5 + (double) best_l) * 0.25;
    const bool zero = d == 0.0f;
    if (lane == 0) {
#pragma unroll 1
        for (int g = 0; g < NG; ++g) {
            const int bp = (int) ((best_sel >> (11 * g)) & 0xFF), bf = (int) ((best_sel >> (11 * g + 8)) & 7);
            const uint64_t pt = __ldg(grid + bp);
            int nneg = 0;
            uint32_t negbits = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) if (xr[8 * g + i] < 0) { negbits |= 1u << i; ++nneg; }
            if (nneg & 1) negbits ^= 1u << bf;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const double v = (double) (int) ((pt >> (8 * i)) & 0xFF) * db;
                const double qv = zero ? 0.0 : ((negbits >> i) & 1 ? -v : v);
                err[r * SUBW + 8 * g + i] = (double) xr[8 * g + i] - qv;
            }
            const uint32_t gi = zero ? 0u : (uint32_t) bp, si = zero ? 0u : (negbits & 127u);
            const int gg = g0 + g;
            w0 = (w0 & ~(0xFFu << (8 * gg))) | (gi << (8 * gg));
            w1 = (w1 & ~(0x7Fu << (7 * gg))) | (si << (7 * gg));
        }
        if (NG == 4) w1 = (w1 & 0x0FFFFFFFu) | ((uint32_t) best_l << 28);
        st32(wp, w0);
        st32(wp + 4, w1);
    }
}

}  // namespace

cudaError_t launch_sub_weff(const float * blk, const float * qw, int64_t qw_div, float * weff, int64_t rows, cudaStream_t st) {
    if (rows <= 0 || qw_div <= 0) return cudaErrorInvalidValue;
    k_sub_weff<<<(unsigned) ((rows + 3) / 4), 128, 0, st>>>(blk, qw, qw_div, weff, rows);
    return cudaGetLastError();
}

cudaError_t launch_sub_points(const float * blk, const float * weff, uint8_t * q, double * err, int64_t rows, int sub,
                              int c0, int scale_search, const uint64_t * grid, cudaStream_t st) {
    if (rows <= 0 || !grid || c0 < 0 || c0 % sub || c0 + sub > QK || scale_search < 0 || scale_search > 15)
        return cudaErrorInvalidValue;
    const unsigned nb = (unsigned) ((rows + 3) / 4);
    if (sub == 32) k_sub_points<4><<<nb, 128, 0, st>>>(blk, weff, q, err, rows, c0, scale_search, grid);
    else if (sub == 8) k_sub_points<1><<<nb, 128, 0, st>>>(blk, weff, q, err, rows, c0, scale_search, grid);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

}  // namespace gq
