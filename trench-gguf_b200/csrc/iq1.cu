// iq1.cu - IQ1_S and IQ1_M: ggml's quantize_row_iq1_s_impl / quantize_row_iq1_m_impl on one super-block
// (trench-gguf gpuq.hip:390-514, :517-688).
//
// Per sub-block (32 weights for IQ1_S, 16 for IQ1_M): the weights sorted (stable), weighted prefix sums, then an
// exhaustive scan over every split (i1 <= i2) of the sorted weights into the three levels {-1, 0, +1} + shift,
// keeping the split with the best least-squares score (a strictly sequential rule: ggml accepts when
// sumqx^2 > best*sumq2, re-rounding best at each acceptance); the levels are then snapped to the 2048-point
// codebook (nearest listed neighbour with the shifted level values), the scale refit, and the scales coded
// (IQ1_M also refits the super-block scale over all 256 weights, skipped sub-blocks included).
//
// sm_100a mapping: one warp a tile of 32 sub-blocks (4 IQ1_S or 2 IQ1_M super-blocks), ONE LANE A SUB-BLOCK for
// ggml's sequential work: the stable sort, the prefix sums (run forward inside the scan, not stored), the split scan and
// the refit run in ggml's order inside the lane, so the decisions are ggml's by construction, 32 sub-blocks side by
// side (the reference runs one super-block a thread). The codebook snap is a warp phase: every off-grid group of
// the tile searched 32 at a time, longest neighbour list first (search.cuh). Per-lane arrays live in shared memory
// lane-minor ([element][lane]): every access of the warp hits 32 different banks. One lane a super-block computes
// sumx2 and the super-block scale in index order; the bytes leave through coalesced stores.
#include <type_traits>
#include "common.cuh"
#include "source.cuh"
#include "kernels.h"
#include "search.cuh"

namespace gq {
namespace {

constexpr float DELTA = 0.125f;

template <int T> struct IQ1;
template <> struct IQ1<IQ1_S> { static constexpr int SB = 32, WARPS = 2; static constexpr float EPS = 1e-12f; };
template <> struct IQ1<IQ1_M> { static constexpr int SB = 16, WARPS = 4; static constexpr float EPS = 1e-7f; };

template <int T> struct alignas(16) IQ1Warp {
    static constexpr int SB = IQ1<T>::SB, NSUB = QK / SB, NSB = 32 / NSUB, NH = T == IQ1_M ? 2 : 1, NG = SB / 8;
    float x[SB][32], w[SB][32];              // the lane's sub-block, element-major / lane-minor
    struct Snap {                            // the snap's search schedule (after the scans)
        int m[NG * 32];                      // a (group, lane)'s code3 entry
        uint16_t perm[NG * 32];              // the searches, longest list first
        uint8_t bkt[NG * 32];                // a (group, lane)'s list-length bucket, 0xFF: no search
        int hist[NBKT];
    };
    union {
        Snap snap;
    } u;
    float msc[NSB];                          // a super-block's max sub-block scale
    uint8_t bk[32];                          // the split scan's shift choice a lane
    uint8_t idx[SB][32];                     // stable ascending order of the sub-block's weights
    float scales[32];
    int8_t shifts[32];
    uint8_t dropped[32];                     // sub-block skipped by ggml: nothing written for it
    uint16_t gidx[SB / 8][32];
    float sigma2[NSB];
    uint8_t out[NSB][56];
};

// the shifted level values of level l: x_p = {-1+d, d, 1+d}, x_m = {-1-d, -d, 1-d} (gpuq.hip:404-405)
__device__ __forceinline__ float lvl(int l, bool minus) {
    return minus ? (l == 0 ? -1 - DELTA : (l == 1 ? -DELTA : 1 - DELTA)) : (l == 0 ? -1 + DELTA : (l == 1 ? DELTA : 1 + DELTA));
}

// the snap's search of group g of lane sl's sub-block (iq1_find_best_neighbour2, gpuq.hip:199-232): ggml's
// distance d2 = 0; d2 += w_i (s q_i - x_i)^2 in order with the shifted levels q (minus: x_m), the first strict
// minimum in list order. Returns the grid index, -1 if no listed candidate is finite (ggml would then scan the whole
// grid reading past the group - reported as a device-status error instead).
template <int T>
__device__ int snap_group(const IQ1Warp<T> & st, int sl, int g, int m, float s, bool minus, const SearchTab & tab) {
    float t0[8], t1[8], t2[8];
    const float q0 = lvl(0, minus), q1 = lvl(1, minus), q2 = lvl(2, minus);
#pragma unroll
    for (int i = 0; i < 8; ++i) level_terms(st.w[8 * g + i][sl], st.x[8 * g + i][sl], s, q0, q1, q2, t0[i], t1[i], t2[i]);
    const uint32_t bl = search_list8<false>(m, t0, t1, t2, tab);
    return bl == NONE ? -1 : (int) (bl >> 16);
}

// IQ1_M's running half sums: element v = (w*x, w) goes to half 1's sums when hbit != 0, else to half 0's; the other
// half's sums stay as they are - which is what ggml's adding +0 to them gives, as these sums start at +0 and a sum
// of rounded additions that starts at +0 is never -0. Two predicated additions a half, no select.
__device__ __forceinline__ void half_acc(unsigned hbit, float2 v, float & x0, float & w0, float & x1, float & w1) {
    asm("{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@p add.rn.f32 %2, %2, %5;\n\t"
        "@p add.rn.f32 %3, %3, %6;\n\t"
        "@!p add.rn.f32 %0, %0, %5;\n\t"
        "@!p add.rn.f32 %1, %1, %6;\n\t}"
        : "+f"(x0), "+f"(w0), "+f"(x1), "+f"(w1) : "r"(hbit), "f"(v.x), "f"(v.y));
}

// sorted element j of lane's sub-block as (w*x, w), formed as ggml forms the prefix sums' addends
template <typename W>
__device__ __forceinline__ float2 sorted_wx(const W & st, int j, int lane) {
    const int i = st.idx[j][lane];
    const float wi = st.w[i][lane];
    return make_float2(wi * st.x[i][lane], wi);
}

// group g's levels take the minus shift (IQ1_S: one shift a sub-block; IQ1_M: one a half, bk's two bits)
template <int T> __device__ __forceinline__ bool minus_of(int bk, int g) {
    return T == IQ1_S ? bk == 1 : (g == 0 ? bk >= 2 : (bk % 2) != 0);
}

template <int T, int SRC>
__global__ void __launch_bounds__(32 * IQ1<T>::WARPS) k_iq1(const uint8_t * __restrict__ src, const float * __restrict__ qw,
                                                            int64_t qw_mod, int64_t qw_div, int64_t qw_mat,
                                                            uint8_t * __restrict__ out, int64_t nblocks, SearchTab tab,
                                                            unsigned * status) {
    using W = IQ1Warp<T>;
    constexpr int SB = W::SB, NSUB = W::NSUB, NSB = W::NSB;
    constexpr int BB = block_bytes(T);
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    W & st = reinterpret_cast<W *>(smem_raw)[wid];
    const int64_t b0 = ((int64_t) blockIdx.x * (blockDim.x >> 5) + wid) * NSB;
    if (b0 >= nblocks) return;
    const int nb = (int) (nblocks - b0 < NSB ? nblocks - b0 : NSB);
    // ---- loads: 8 consecutive weights a lane a pass, scattered into the lane-minor layout
    float qr[NSB][8];
#pragma unroll
    for (int k = 0; k < NSB; ++k) {
        const int e = lane * 8;                        // element of super-block k
        float v[8];
        if (k < nb) {
            const int64_t b = b0 + k;
            decode8<SRC>(src, b * QK + e, v);
            load8_f32(qw + ((b / qw_mat) * qw_mod + (b % qw_mod) / qw_div) * QK + e, qr[k]);
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) { v[j] = 0.f; qr[k][j] = 0.f; }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) st.x[(e + j) % SB][k * NSUB + (e + j) / SB] = v[j];
    }
    __syncwarp();
    // ---- sumx2 in index order, one lane a super-block
    if (lane < NSB) {
        float s2 = 0;
#pragma unroll 16
        for (int e = 0; e < QK; ++e) { const float v = st.x[e % SB][lane * NSUB + e / SB]; s2 += v * v; }
        st.sigma2[lane] = 2 * s2 / QK;
    }
    __syncwarp();
#pragma unroll
    for (int k = 0; k < NSB; ++k) {
        const int e = lane * 8;
        const float sg = st.sigma2[k];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float xv = st.x[(e + j) % SB][k * NSUB + (e + j) / SB];
            st.w[(e + j) % SB][k * NSUB + (e + j) / SB] = qr[k][j] * sqrtf(sg + xv * xv);
        }
    }
    __syncwarp();
    // ---- one lane a sub-block: guard, stable sort, prefix sums, the split scan, the codebook snap, the refit
    const int kb = lane / NSUB;                        // super-block of this lane's sub-block
    const bool live = kb < nb;
    float scale = 0.f;
    int shift = T == IQ1_S ? 1 : 0, bk = -1;
    uint64_t lv = 0;                                   // the sub-block's levels, 2 bits an element
    bool dropped = true;
    if (live) {
        float mx = fabsf(st.x[0][lane]);
#pragma unroll 1
        for (int i = 1; i < SB; ++i) mx = fmaxr(mx, fabsf(st.x[i][lane]));
        if (!(mx < IQ1<T>::EPS)) {
            // the stable ascending order of the weights (the reference's insertion sort, gpuq.hip:236-243: ties keep
            // index order). Without NaN it is a rank: element i goes after every j < i with x_j <= x_i and every
            // j > i with x_j < x_i - independent comparisons instead of the insertion's dependent chain. A NaN
            // compares false everywhere and stalls the insertion in place, so a sub-block holding one is sorted by
            // the insertion itself.
            float xs[SB];
            bool nan = false;
#pragma unroll
            for (int i = 0; i < SB; ++i) { xs[i] = st.x[i][lane]; nan |= !(xs[i] == xs[i]); }
            if (!nan) {
#pragma unroll
                for (int i = 0; i < SB; ++i) {
                    int r = 0;
#pragma unroll
                    for (int j = 0; j < SB; ++j) {
                        if (j < i) r += xs[j] <= xs[i];
                        else if (j > i) r += xs[j] < xs[i];
                    }
                    st.idx[r][lane] = (uint8_t) i;
                }
            } else {
                st.idx[0][lane] = 0;
#pragma unroll 1
                for (int i = 1; i < SB; ++i) {
                    const float k = st.x[i][lane];
                    int j = i - 1;
                    while (j >= 0 && st.x[st.idx[j][lane]][lane] > k) { st.idx[j + 1][lane] = st.idx[j][lane]; --j; }
                    st.idx[j + 1][lane] = (uint8_t) i;
                }
            }
            float best = -FLT_MAX;
            int b1 = -1, b2 = -1;
            scale = mx;
            if constexpr (T == IQ1_S) {
                // the prefix sums (gpuq.hip:429-437) are not stored: the scan runs them forward from the sorted
                // elements - the same additions in the same order, so every prefix is the stored one bit for bit
                float sx = 0.f, sw = 0.f;
#pragma unroll 1
                for (int j = 0; j < SB; ++j) {
                    const int i = st.idx[j][lane];
                    const float wi = st.w[i][lane];
                    sx = sx + wi * st.x[i][lane];
                    sw = sw + wi;
                }
                const float tx = sx, tw = sw;
                const float ap = lvl(0, false), bp = lvl(1, false), cp = lvl(2, false);
                const float am = lvl(0, true), bm = lvl(1, true), cm = lvl(2, true);
                float a = 0.f, c = 0.f;                            // sumx[i1], sumw[i1]
                for (int i1 = 0; i1 <= SB; ++i1) {
                    const float x1 = a - 0.f, w1 = c - 0.f;       // (sumx[i1] - sumx[0])
                    const float sx1 = a, sw1 = c;
                    float r = a, e = c;                            // sumx[i2], sumw[i2]
                    for (int i2 = i1; i2 <= SB; ++i2) {
                        const float sx2 = r, sw2 = e;
                        const float dx = sx2 - sx1, dw = sw2 - sw1, ex = tx - sx2, ew = tw - sw2;
                        float qx = x1 * ap + dx * bp + ex * cp;
                        float q2 = w1 * ap * ap + dw * bp * bp + ew * cp * cp;
                        if (q2 > 0 && qx * qx > best * q2) { scale = qx / q2; best = scale * qx; b1 = i1; b2 = i2; bk = 0; }
                        qx = x1 * am + dx * bm + ex * cm;
                        q2 = w1 * am * am + dw * bm * bm + ew * cm * cm;
                        if (q2 > 0 && qx * qx > best * q2) { scale = qx / q2; best = scale * qx; b1 = i1; b2 = i2; bk = 1; }
                        if (i2 < SB) {                             // on to prefix i2 + 1
                            const int i = st.idx[i2][lane];
                            const float wi = st.w[i][lane];
                            r = r + wi * st.x[i][lane];
                            e = e + wi;
                        }
                    }
                    if (i1 < SB) {                                 // on to prefix i1 + 1
                        const int i = st.idx[i1][lane];
                        const float wi = st.w[i][lane];
                        a = a + wi * st.x[i][lane];
                        c = c + wi;
                    }
                }
            } else {
                // the prefix sums split by half of the sub-block (gpuq.hip:559-571) are not stored: both scan loops
                // run them forward from the sorted elements' (w*x, w), the same additions in the same order (a
                // half's sum only moves at its own elements; adding +0 to the other half changes nothing)
                float ax0 = 0.f, ax1 = 0.f, aw0 = 0.f, aw1 = 0.f;
                unsigned hmask = 0;                    // bit j: sorted element j is in the second half
                for (int j = 0; j < SB; ++j) {
                    const int i = st.idx[j][lane], h = i < SB / 2 ? 0 : 1;
                    const float wi = st.w[i][lane], wx = wi * st.x[i][lane];
                    hmask |= (unsigned) h << j;
                    if (h) { ax1 = ax1 + wx; aw1 = aw1 + wi; } else { ax0 = ax0 + wx; aw0 = aw0 + wi; }
                }
                const float p2 = 1 + DELTA, m2 = 1 - DELTA;
                const float cp1 = (-1 + DELTA) * (-1 + DELTA) - DELTA * DELTA, cp2 = DELTA * DELTA - (1 + DELTA) * (1 + DELTA);
                const float cm1 = (-1 - DELTA) * (-1 - DELTA) - (-DELTA) * (-DELTA), cm2 = (-DELTA) * (-DELTA) - (1 - DELTA) * (1 - DELTA);
                const float tx0 = ax0, tx1 = ax1, tw0 = aw0, tw1 = aw1;
                const float txp0 = tx0 * p2, txp1 = tx1 * p2, txm0 = tx0 * m2, txm1 = tx1 * m2;
                const float twp0 = tw0 * p2 * p2, twp1 = tw1 * p2 * p2, twm0 = tw0 * m2 * m2, twm1 = tw1 * m2 * m2;
                float a0 = 0.f, a1 = 0.f, c0 = 0.f, c1 = 0.f;          // px[h][i1], pw[h][i1]
                for (int i1 = 0; i1 <= SB; ++i1) {
                    const float c0p = c0 * cp1, c1p = c1 * cp1, c0m = c0 * cm1, c1m = c1 * cm1;
                    float r0 = a0, r1 = a1, e0 = c0, e1 = c1;           // px[h][i2], pw[h][i2]
                    for (int i2 = i1; i2 <= SB; ++i2) {
                        const float sx0 = a0 + r0, sx1 = a1 + r1;
                        const float qxp0 = txp0 - sx0, qxm0 = txm0 - sx0, qxp1 = txp1 - sx1, qxm1 = txm1 - sx1;
                        const float q2p0 = twp0 + c0p + e0 * cp2, q2m0 = twm0 + c0m + e0 * cm2;
                        const float q2p1 = twp1 + c1p + e1 * cp2, q2m1 = twm1 + c1m + e1 * cm2;
                        const float sqx[4] = {qxp0 + qxp1, qxp0 + qxm1, qxm0 + qxp1, qxm0 + qxm1};
                        const float sq2[4] = {q2p0 + q2p1, q2p0 + q2m1, q2m0 + q2p1, q2m0 + q2m1};
#pragma unroll
                        for (int c = 0; c < 4; ++c)
                            if (sq2[c] > 0 && sqx[c] * sqx[c] > best * sq2[c]) {
                                scale = sqx[c] / sq2[c]; best = scale * sqx[c]; b1 = i1; b2 = i2; bk = c;
                            }
                        if (i2 < SB) half_acc(hmask & (1u << i2), sorted_wx(st, i2, lane), r0, e0, r1, e1);   // prefix i2 + 1
                    }
                    if (i1 < SB) half_acc(hmask & (1u << i1), sorted_wx(st, i1, lane), a0, c0, a1, c1);       // prefix i1 + 1
                }
            }
            if (b1 >= 0) {
                dropped = false;
#pragma unroll 1
                for (int j = 0; j < SB; ++j) lv |= (uint64_t) (j < b1 ? 0 : j < b2 ? 1 : 2) << (2 * st.idx[j][lane]);
                if (scale < 0) {
                    lv = (0xAAAAAAAAAAAAAAAAull >> (64 - 2 * SB)) - lv;   // every level l -> 2 - l (no borrows)
                    scale = -scale;
                    bk = T == IQ1_S ? 1 - bk : 3 - bk;
                }
            } else {
                scale = 0.f;
            }
        }
    }
    // ---- the codebook snap of every group of the tile's 32 sub-blocks: the groups off the grid searched 32 at a
    //      time, longest neighbour list first (independent exact searches: the order changes no result)
    typename W::Snap & sn = st.u.snap;
    __syncwarp();                                      // (the prefix sums are dead: their space holds the schedule)
    for (int i = lane; i < NBKT; i += 32) sn.hist[i] = 0;
    st.scales[lane] = scale;
    st.bk[lane] = (uint8_t) bk;
    __syncwarp();
    bool all_on = true;
#pragma unroll
    for (int g = 0; g < W::NG; ++g) {
        uint8_t b = 0xFF;
        if (!dropped) {
            int c3 = 0, p3 = 1;
#pragma unroll
            for (int i = 0; i < 8; ++i) { c3 += (int) ((lv >> (2 * (8 * g + i))) & 3u) * p3; p3 *= 3; }
            const int m = __ldg(tab.code3 + c3);
            sn.m[g * 32 + lane] = m;
            if (m >= 0) {
                st.gidx[g][lane] = (uint16_t) m;
            } else {
                all_on = false;
                b = (uint8_t) len_bucket(list_cnt(m));
                atomicAdd(&sn.hist[b], 1);
            }
        }
        sn.bkt[g * 32 + lane] = b;
    }
    __syncwarp();
    const int nreq = bucket_offsets(sn.hist, lane);
    __syncwarp();
#pragma unroll
    for (int g = 0; g < W::NG; ++g) {
        const int b = sn.bkt[g * 32 + lane];
        if (b != 0xFF) sn.perm[atomicAdd(&sn.hist[b], 1)] = (uint16_t) (g * 32 + lane);
    }
    __syncwarp();
    for (int k0 = 0; k0 < nreq; k0 += 32) {
        if (k0 + lane < nreq) {
            const int item = sn.perm[k0 + lane], g = item >> 5, sl = item & 31;
            int gi = snap_group<T>(st, sl, g, sn.m[item], st.scales[sl], minus_of<T>(st.bk[sl], g), tab);
            if (gi < 0) { atomicOr(status, ST_NO_NEIGHBOUR); gi = 0; }
            st.gidx[g][sl] = (uint16_t) gi;
        }
    }
    __syncwarp();
    // ---- the refit over the snapped levels (when a group left the grid), the shift code
    if (!dropped) {
        if (!all_on) {
            float sqx = 0, sq2 = 0;
#pragma unroll 1
            for (int g = 0; g < W::NG; ++g) {
                const bool minus = minus_of<T>(bk, g);
                const uint32_t lev = __ldg(tab.glev + st.gidx[g][lane]);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float ww = st.w[8 * g + j][lane], q = lvl((lev >> (2 * j)) & 3u, minus);
                    sqx += ww * q * st.x[8 * g + j][lane];
                    sq2 += ww * q * q;
                }
            }
            if (sqx > 0 && sq2 > 0) scale = sqx / sq2;
        }
        shift = T == IQ1_S ? (bk == 1 ? -1 : 1) : bk;
    }
    st.scales[lane] = dropped ? 0.f : scale;
    st.shifts[lane] = (int8_t) shift;
    st.dropped[lane] = (uint8_t) dropped;
    __syncwarp();
    // ---- the block bytes: each lane writes its sub-block's fields, one lane a super-block the scales
    if (live) {
        uint8_t * y = st.out[kb];
        const int ib = lane % NSUB;
        if constexpr (T == IQ1_S) {
            uint16_t h = 0;
            for (int k = 0; k < 4; ++k) {
                const int gi = st.dropped[lane] ? 0 : st.gidx[k][lane];
                y[2 + 4 * ib + k] = (uint8_t) (gi & 255);
                h |= (uint16_t) ((gi >> 8) << (3 * k));
            }
            y[34 + 2 * ib] = (uint8_t) (h & 255);
            y[35 + 2 * ib] = (uint8_t) (h >> 8);
        } else {
            const int g0 = st.dropped[lane] ? 0 : st.gidx[0][lane], g1 = st.dropped[lane] ? 0 : st.gidx[1][lane];
            y[2 * ib] = (uint8_t) (g0 & 255);
            y[2 * ib + 1] = (uint8_t) (g1 & 255);
            y[32 + ib] = (uint8_t) ((g0 >> 8) | ((g1 >> 8) << 4));
        }
    }
    __syncwarp();
    if (lane < nb) {
        const float * scl = st.scales + lane * NSUB;
        float max_scale = 0;
#pragma unroll 1
        for (int ib = 0; ib < NSUB; ++ib) if (!st.dropped[lane * NSUB + ib]) max_scale = fmaxr(max_scale, scl[ib]);
        st.msc[lane] = max_scale;
    }
    __syncwarp();
    if constexpr (T == IQ1_M) {
        // the super-block refit's products, one lane a sub-block: q = x_shift(level) * (2 l + 1) with l the
        // sub-block's 3-bit scale code; a dropped sub-block counts with grid point 0 and scale code 0, as ggml's
        // zeroed block bytes make it (gpuq.hip:657-687)
        const float ms = live ? st.msc[kb] : 0.f;
        if (ms) {
            const float id = 1 / (ms / 15);
            const int l = imax(0, imin(7, nearest_int(0.5f * (id * st.scales[lane] - 1))));
            const int sh = st.shifts[lane];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const bool minus = k == 0 ? sh >= 2 : (sh % 2) != 0;
                const uint32_t lev = __ldg(tab.glev + (st.dropped[lane] ? 0 : st.gidx[k][lane]));
#pragma unroll
                for (int j = 0; j < 8; ++j) {   // (x and w are dead after this: the products take their slots)
                    const float ww = st.w[8 * k + j][lane], q = lvl((lev >> (2 * j)) & 3u, minus) * (2 * l + 1);
                    const float px = ww * q * st.x[8 * k + j][lane], pq = ww * q * q;
                    st.x[8 * k + j][lane] = px;
                    st.w[8 * k + j][lane] = pq;
                }
            }
        }
        __syncwarp();
    }
    if (lane < nb) {
        uint8_t * y = st.out[lane];
        const float * scl = st.scales + lane * NSUB;
        const float max_scale = st.msc[lane];
        if constexpr (T == IQ1_S) {
            y[0] = y[1] = 0;
            if (max_scale) {
                const float d = max_scale / 15;
                const uint16_t hd = half_bits(d * 1.125f);
                y[0] = hd & 255; y[1] = hd >> 8;
                const float id = 1 / d;
#pragma unroll 1
                for (int ib = 0; ib < 8; ++ib) {
                    int l = imax(0, imin(7, nearest_int(0.5f * (id * scl[ib] - 1))));
                    if (st.shifts[lane * NSUB + ib] == -1) l |= 8;
                    y[35 + 2 * ib] |= (uint8_t) ((l << 12) >> 8);
                }
            }
        } else {
            for (int i = 48; i < 56; ++i) y[i] = 0;
            if (max_scale) {
                uint64_t sc = 0;                       // the four 16-bit scale words, word i in bits 16i..16i+15
                float d = max_scale / 15;
                const float id = 1 / d;
                float sqx = 0, sq2 = 0;
                for (int ib = 0; ib < 16; ++ib) {
                    const int sl = lane * NSUB + ib;
                    const int l = imax(0, imin(7, nearest_int(0.5f * (id * scl[ib] - 1))));
                    sc |= (uint64_t) l << (16 * (ib / 4) + 3 * (ib % 4));
                    const int m = st.shifts[sl];       // shift code: bit 0 -> 0x80, bit 1 -> 0x08
                    y[32 + ib] |= (uint8_t) ((m & 1) * 0x80 | (m & 2) * 4);
                    for (int e = 0; e < 16; ++e) { sqx += st.x[e][sl]; sq2 += st.w[e][sl]; }
                }
                if (sq2 > 0) d = sqx / sq2;
                const uint64_t s = half_bits(d * 1.1125f);
                sc |= ((s & 0x000f) << 12) | ((s & 0x00f0) << 24) | ((s & 0x0f00) << 36) | ((s & 0xf000) << 48);
                for (int i = 0; i < 8; ++i) y[48 + i] = (uint8_t) (sc >> (8 * i));
            }
        }
    }
    __syncwarp();
    uint8_t * yo = out + b0 * BB;
    for (int i = lane; i < nb * BB; i += 32) yo[i] = st.out[i / BB][i % BB];
}

template <int T, int SRC>
cudaError_t launch_t(const LaunchArgs & a) {
    using W = IQ1Warp<T>;
    constexpr int WARPS = IQ1<T>::WARPS;
    const size_t smem = sizeof(W) * WARPS;
    const cudaError_t e = cudaFuncSetAttribute(k_iq1<T, SRC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (e != cudaSuccess) return e;
    const int64_t per_cta = (int64_t) WARPS * W::NSB;
    const int64_t grid = (a.nblocks + per_cta - 1) / per_cta;
    k_iq1<T, SRC><<<(unsigned) grid, WARPS * 32, smem, a.stream>>>((const uint8_t *) a.src, a.qw, a.qw_mod, a.qw_div,
                                                                   a.qw_mat, (uint8_t *) a.out, a.nblocks, a.tab, a.status);
    return cudaGetLastError();
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

}  // namespace

cudaError_t launch_iq1(int type, const LaunchArgs & a) {
    switch (type) {
        case IQ1_S: return launch_src<IQ1_S>(a);
        case IQ1_M: return launch_src<IQ1_M>(a);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace gq
