// iq_grid.cu - the grid-trial i-quants: IQ2_XXS, IQ2_XS, IQ2_S, IQ3_XXS, IQ3_S.
//
// What is computed: ggml's quantize_row_{iq2_xxs,iq2_xs,iq2_s,iq3_xxs,iq3_s}_impl on one 256-weight super-block
// (trench-gguf gpuq.hip:246-387, :825-969, :691-822, :995-1143, :1146-1283): per sub-block, signs split off (with
// the even-parity fix for the 7-bit sign fields), 13..31 trial inverse scales, each rounding the magnitudes to the
// 2l+1 lattice, snapping every off-grid group to its nearest listed codebook neighbour, and scoring the trial by
// its least-squares scale; the best trial is refined, the groups left off the grid are snapped again with the
// final scale, and the sub-block scales are coded against the super-block scale.
//
// How it runs on sm_100a: one warp a super-block, FP32-ALU bound. Lanes own independent work only:
//   * elementwise weights and sign groups (8 weights a lane),
//   * make_qp_quants (IQ2_XXS): its trial scales one a lane, its coordinate descent with the lanes over the 32
//     elements (the first lane whose test passes is ggml's next change),
//   * the trials: every (sub-block, trial) task's groups rounded, then the batch's neighbour searches sorted by
//     list length and run 32 at a time, one whole list a lane (search.cuh), then each task's sums in index order,
//   * the (sub-block, group) pairs of the re-gridding.
// The neighbour searches dominate (3k..22k candidate points a super-block). ggml's sequential decisions (which
// trial wins: a strict `>` scan in trial order) are replayed in trial order by one lane per sub-block from the stored
// per-trial sums, so the choice is bit-identical. Sums that ggml runs in index order (sumx2 over 256, the
// 16/32-weight sums) run in index order inside one lane.
#include <type_traits>
#include "common.cuh"
#include "search.cuh"
#include "source.cuh"
#include "kernels.h"

namespace gq {
namespace {

template <int T> struct GT;
template <> struct GT<IQ2_XXS> {   // gpuq.hip:246-387
    static constexpr int SB = 32, GD = 8, KMAXQ = 3, NTR = 6, SIGMA_X2 = 0, PARITY = 1, QP_FIRST = 1, REGRID_ALL = 1,
                         REGRID_ANY = 0, INIT_ON = 1, EPS_ZERO = 0;
    static constexpr float STEP = 0.1f, EPS = 1e-15f;
};
template <> struct GT<IQ2_XS> {    // gpuq.hip:825-969
    static constexpr int SB = 16, GD = 8, KMAXQ = 3, NTR = 9, SIGMA_X2 = 0, PARITY = 1, QP_FIRST = 0, REGRID_ALL = 0,
                         REGRID_ANY = 1, INIT_ON = 1, EPS_ZERO = 0;
    static constexpr float STEP = 0.1f, EPS = 1e-15f;
};
template <> struct GT<IQ2_S> {     // gpuq.hip:691-822
    static constexpr int SB = 16, GD = 8, KMAXQ = 3, NTR = 9, SIGMA_X2 = 1, PARITY = 0, QP_FIRST = 0, REGRID_ALL = 0,
                         REGRID_ANY = 1, INIT_ON = 1, EPS_ZERO = 0;
    static constexpr float STEP = 0.1f, EPS = 1e-8f;
};
template <> struct GT<IQ3_XXS> {   // gpuq.hip:995-1143
    static constexpr int SB = 32, GD = 4, KMAXQ = 8, NTR = 15, SIGMA_X2 = 1, PARITY = 1, QP_FIRST = 0, REGRID_ALL = 0,
                         REGRID_ANY = 1, INIT_ON = 1, EPS_ZERO = 0;
    static constexpr float STEP = 0.2f, EPS = 1e-8f;
};
template <> struct GT<IQ3_S> {     // gpuq.hip:1146-1283
    static constexpr int SB = 32, GD = 4, KMAXQ = 8, NTR = 9, SIGMA_X2 = 1, PARITY = 0, QP_FIRST = 0, REGRID_ALL = 1,
                         REGRID_ANY = 1, INIT_ON = 0, EPS_ZERO = 1;
    static constexpr float STEP = 0.2f, EPS = 0.f;
};

template <int T> struct Shape {
    using P = GT<T>;
    static constexpr int NSUB = QK / P::SB;           // sub-blocks a super-block
    static constexpr int NG = P::SB / P::GD;          // codebook groups a sub-block
    static constexpr int NT = 2 * P::NTR + 1;         // trials a sub-block
    static constexpr int NTASK = NSUB * NT;
    static constexpr int PAD = P::SB + 1;             // padded sub-block stride (conflict-free across sub-blocks)
    static constexpr int BITS = P::GD == 8 ? 2 : 3;   // packed level bits a dimension
    static constexpr int NSG = P::SB / 8;             // 8-weight sign bytes a sub-block
    static constexpr int NROUND = (NTASK + 31) / 32;  // rounds of 32 trials
    static constexpr int NRG = NSUB * NG;             // re-grid searches a super-block
    // trial rounds scheduled together (their searches sorted by list length): at most 640 searches a batch
    static constexpr int RB = NROUND < 640 / (32 * NG) ? NROUND : (640 / (32 * NG) > 0 ? 640 / (32 * NG) : 1);
    static constexpr int BT = RB * 32 < NTASK ? RB * 32 : NTASK;   // tasks a batch holds
};

// per-warp shared state of one super-block
template <int T> struct alignas(16) WarpState {
    using S = Shape<T>;
    struct QP {                                       // make_qp_quants (IQ2_XXS)
        float mse[S::NSUB][9];                        // trial errors
        float sums[S::NSUB][2];                       // sumlx, suml2 at the chosen trial scale
        float isc[S::NSUB];                           // the chosen inverse scale
        float res[S::NSUB];                           // the descent's scale, where it ran
    };
    struct Regrid {                                   // the re-grid's searches, split into runs
        int m[32];                                    // a search's code3 entry (its lane)
        uint16_t owner[32];                           // a run's search lane | run index << 5
        float bd[32];                                 // a run's best distance and entry
        uint32_t be[32];
    };
    struct Sched {                                    // one batch of trial rounds
        uint16_t perm[S::BT * S::NG];                 // the batch's searches, longest first
        uint8_t bkt[S::RB * 32 * S::NG];              // a (task, group)'s list-length bucket, 0xFF: on the grid
        int hist[NBKT];                               // bucket counts, then cursors
    };
    struct Sums { float sqx[S::BT], sq2[S::BT]; };     // the batch's tasks' index-order sums
    // With the trials in one batch, the sums are written after the batch's schedule is dead and read before the
    // next use of the union: they share it (the smaller warp state lets more warps share an SM).
    static constexpr bool SUMS_IN_U = S::RB >= S::NROUND;
    union {                                           // (phase-disjoint uses of one buffer)
        float x2[QK];                                 // x*x, for sumx2
        QP qp;
        Sched sch;
        Regrid rg;
        std::conditional_t<SUMS_IN_U, Sums, char> sums;
        uint8_t out[112];                             // the block's bytes (after the trials)
    } u;
    float w[S::NSUB * S::PAD], wa[S::NSUB * S::PAD], xv[S::NSUB * S::PAD];
    float qmax[S::NSUB];                              // make_qp_quants' max (from 0)
    std::conditional_t<SUMS_IN_U, char, Sums> own_sums;
    __device__ Sums & sums() {
        if constexpr (SUMS_IN_U) return u.sums; else return own_sums;
    }
    uint16_t t_lev[S::BT][S::NG];                     // the batch's tasks' levels and on-grid groups
    uint8_t t_on[S::BT];
    float p6_best[S::NSUB];                           // ggml's trial choice so far: its best (the scale is scale[])
    uint8_t p6_on[S::NSUB];                           // its on-grid groups
    float denom[S::NSUB], scale[S::NSUB];
    uint16_t lev[S::NSUB][S::NG];
    int32_t gidx[S::NSUB][S::NG];
    uint8_t signs[S::NSUB][S::NSG];
    uint8_t skip[S::NSUB], regrid[S::NSUB];
    float sigma2;
};

__device__ __forceinline__ int eidx(int sb, int pad, int e) { return (e / sb) * pad + (e % sb); }

// make_qp_quants (gpuq.hip:114-176), split in two. Trial k's weighted error over one sub-block: k = 0 the
// initial inverse scale nmax/max (levels stored unclamped, as ggml), k = 1..8 the trial scales is = -4..-1, 1..4.
// (one code path for all k, so the trial lanes do not diverge: k = 0 keeps ggml's uint8_t levels, the others
// its MIN(nmax, l))
template <int N>
__device__ float qp_trial_mse(int k, int nmax, float mx, const float * x, const float * w) {
    const int is = k <= 4 ? k - 5 : k - 4;
    const float iscale = (k == 0 ? (float) nmax : 0.1f * is + nmax) / mx;
    const float scale = 1 / iscale;
    float mse = 0;
#pragma unroll 1
    for (int i = 0; i < N; ++i) {
        const int r = nearest_int(iscale * x[i]);
        const int l = k == 0 ? (r & 255) : imin(nmax, r);
        const float d = x[i] - scale * l;
        mse += w[i] * d * d;
    }
    return mse;
}

// ... then ggml's choice among the trials (first strict minimum in trial order) and its coordinate descent, with
// the lanes over the 32 elements of one sub-block (warp-collective; every lane calls it with the same sub-block).
// A pass of the descent visits the elements in order and changes element i only when its new level improves
// sumlx^2/suml2; an element that does not change leaves the sums as they were, so all lanes test their element
// against the current sums at once and the first lane whose test passes is the next change - ggml's sequential
// pass exactly, in (changes + 1) rounds. sumlx and suml2 enter from the index-order sums of the signed levels,
// while L holds them as ggml's uint8_t array does (a negative level, from the one sign-flipped weight of an odd
// group, wraps), exactly as the reference's pass reads them.
//
// One element's test (gpuq.hip:156-170): its level against the current sums with itself taken out, and whether
// ggml takes the new level (the sums with it put back in are returned for that case).
__device__ __forceinline__ bool qp_try(int nmax, float x, float w, int L, float sumlx, float suml2, bool on, int & nl,
                                       float & slx, float & sl2) {
    slx = sumlx - w * x * L;
    sl2 = suml2 - w * L * L;
    nl = L;
    bool acc = false;
    if (on && slx > 0 && sl2 > 0) {
        nl = imin(nmax, nearest_int(x * sl2 / slx));
        if (nl != L) {
            slx += w * x * nl;
            sl2 += w * nl * nl;
            acc = slx * slx * suml2 > sumlx * sumlx * sl2;
        }
    }
    return acc;
}

// The whole descent of one sub-block; returns the scale.
__device__ float qp_descent_warp(int lane, int nmax, float x, float w, float sumlx, float suml2, int L) {
    for (int pass = 0; pass < 5; ++pass) {
        int changed = 0, from = 0;
        for (;;) {
            float slx, sl2;
            int nl;
            const bool acc = qp_try(nmax, x, w, L, sumlx, suml2, lane >= from, nl, slx, sl2);
            const unsigned hit = __ballot_sync(0xFFFFFFFFu, acc);
            if (!hit) break;
            const int f = __ffs(hit) - 1;
            sumlx = __shfl_sync(0xFFFFFFFFu, slx, f);
            suml2 = __shfl_sync(0xFFFFFFFFu, sl2, f);
            if (lane == f) L = nl & 255;                // (ggml keeps the levels in uint8_t)
            ++changed;
            from = f + 1;
        }
        if (!changed) break;
    }
    return suml2 > 0.0f ? sumlx / suml2 : 0.0f;
}

// ggml's choice of make_qp_quants' inverse scale: the initial nmax/max, replaced by a later trial only on a strictly
// smaller error
__device__ __forceinline__ float qp_iscale(int nmax, float mx, const float * mse) {
    float iscale = nmax / mx, best_mse = mse[0];
    for (int k = 1; k <= 8; ++k) {
        const int is = k <= 4 ? k - 5 : k - 4;
        if (mse[k] < best_mse) { best_mse = mse[k]; iscale = (0.1f * is + nmax) / mx; }
    }
    return iscale;
}

// the lattice value 2l+1 of a 3-bit level, as a float, by the 2^23 bias (exact, full-rate FADD)
__device__ __forceinline__ float odd_level(uint32_t l) { return u2f(0x4B000000u + 2 * l + 1) - 8388608.f; }

template <int GD>
__device__ __forceinline__ int level_of(uint32_t lev, int i) { return GD == 8 ? (lev >> (2 * i)) & 3 : (lev >> (3 * i)) & 7; }

template <int GD>
__device__ __forceinline__ int code3_of(uint32_t lev) {
    if constexpr (GD == 4) return (int) lev;   // base 8 = the packed 3-bit levels
    int c = 0, p = 1;
#pragma unroll
    for (int i = 0; i < 8; ++i) { c += (int) ((lev >> (2 * i)) & 3u) * p; p *= 3; }
    return c;
}

// a trial's inverse scale: (2 kmaxq - 1 + is * step) / denom, is = t - ntrial (ggml's expression)
template <int T>
__device__ __forceinline__ float trial_id(int t, float denom) {
    return ((float) (2 * GT<T>::KMAXQ - 1) + (float) (t - GT<T>::NTR) * GT<T>::STEP) / denom;
}

// ggml's rounding of one group at inverse scale id: l = clamp(nearest_int(0.5*(id*x - 1)), 0, kmaxq-1); returns
// the packed levels and the grid-table entry of the code (>= 0 grid index, < 0 the neighbour list)
template <int GD, int KMAXQ>
__device__ __forceinline__ uint32_t round_levels(const float * xv, float id, int * c3) {
    constexpr int BITS = GD == 8 ? 2 : 3;
    uint32_t lev = 0;
    int c = 0, p3 = 1;
#pragma unroll
    for (int i = 0; i < GD; ++i) {
        const int l = imax(0, imin(KMAXQ - 1, nearest_int(0.5f * (id * xv[i] - 1))));
        lev |= (uint32_t) l << (BITS * i);
        c += l * p3;
        p3 *= (GD == 8 ? 3 : 8);
    }
    *c3 = c;
    return lev;
}
template <int GD, int KMAXQ>
__device__ __forceinline__ uint32_t round_group(const float * xv, float id, const SearchTab & tab, int * m) {
    int c3;
    const uint32_t lev = round_levels<GD, KMAXQ>(xv, id, &c3);
    *m = __ldg(tab.code3 + c3);
    return lev;
}

// the 8-d grids: one lane's own search (iq2_find_best_neighbour, gpuq.hip:178-197): the 24 per-dimension terms
// formed once, then per candidate 8 selects and ggml's 8 additions; the next entry loaded one step ahead
__device__ __forceinline__ uint32_t search_lane8(int m, const float * xv, const float * wa, float s, const SearchTab & tab) {
    float t0[8], t1[8], t2[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) level_terms(wa[i], xv[i], s, 1.f, 3.f, 5.f, t0[i], t1[i], t2[i]);
    const uint32_t bl = search_list8(m, t0, t1, t2, tab);
    return bl == NONE ? NONE : (bl & 0xFFFFu);
}

// the 4-d grids: cnt consecutive entries of a list (lists of 2..38 points), ggml's distance and first-minimum rule
// (iq3_find_best_neighbour, gpuq.hip:972-992). Returns the winning entry (NONE if none is below FLT_MAX), its
// distance in best.
__device__ uint32_t search_run4(const uint32_t * lst, int cnt, const float * xv, const float * wa, float s, float & best) {
    best = FLT_MAX;
    uint32_t bl = NONE;
    for (int j = 0; j < cnt; ++j) {
        const uint32_t e = __ldg(lst + j);
        float d2 = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float d = s * odd_level((e >> (3 * i)) & 7u) - xv[i];
            d2 += wa[i] * d * d;
        }
        if (d2 < best) { best = d2; bl = e; }
    }
    return bl;
}
__device__ uint32_t search_lane4(int m, const float * xv, const float * wa, float s, const SearchTab & tab) {
    float best;
    const uint32_t bl = search_run4(tab.neigh + list_off(m) + 1, list_cnt(m), xv, wa, s, best);
    return bl == NONE ? NONE : (bl & 0xFFFFu);
}

// cnt entries of a list from lst, either grid; the terms of the 8-d grids formed here
template <int GD>
__device__ __forceinline__ uint32_t search_run(const uint32_t * lst, int cnt, const float * xv, const float * wa, float s,
                                               float & best) {
    if constexpr (GD == 8) {
        float t0[8], t1[8], t2[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) level_terms(wa[i], xv[i], s, 1.f, 3.f, 5.f, t0[i], t1[i], t2[i]);
        return search_run8(lst, cnt, t0, t1, t2, best);
    } else {
        return search_run4(lst, cnt, xv, wa, s, best);
    }
}

// ------------------------------------------------------------------------------------------------ the kernel
template <int T, int SRC>
__global__ void __launch_bounds__(128) k_iq_grid(const uint8_t * __restrict__ src, const float * __restrict__ qw,
                                                 int64_t qw_mod, int64_t qw_div, int64_t qw_mat,
                                                 uint8_t * __restrict__ out, int64_t nblocks, SearchTab tab,
                                                 unsigned * status) {
    using P = GT<T>;
    using S = Shape<T>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    WarpState<T> & st = reinterpret_cast<WarpState<T> *>(smem_raw)[wid];
    const int64_t b = (int64_t) blockIdx.x * (blockDim.x >> 5) + wid;
    if (b >= nblocks) return;

    // ---- P0: this lane's 8 weights and importances (weights lane*8 .. lane*8+7)
    float xr[8], qr[8];
    decode8<SRC>(src, b * QK + lane * 8, xr);
    load8_f32(qw + ((b / qw_mat) * qw_mod + (b % qw_mod) / qw_div) * QK + lane * 8, qr);
    {
        float4 * x2 = reinterpret_cast<float4 *>(st.u.x2 + lane * 8);
        x2[0] = make_float4(xr[0] * xr[0], xr[1] * xr[1], xr[2] * xr[2], xr[3] * xr[3]);
        x2[1] = make_float4(xr[4] * xr[4], xr[5] * xr[5], xr[6] * xr[6], xr[7] * xr[7]);
    }
    __syncwarp();
    // ---- P1: sumx2 in index order (one lane; the products were formed by their lanes)
    if (lane == 0) {
        float s2 = 0;
        const float4 * x2 = reinterpret_cast<const float4 *>(st.u.x2);
#pragma unroll 8
        for (int e = 0; e < QK / 4; ++e) { const float4 v = x2[e]; s2 += v.x; s2 += v.y; s2 += v.z; s2 += v.w; }
        st.sigma2 = P::SIGMA_X2 ? 2 * s2 / QK : s2 / QK;
    }
    __syncwarp();
    const float sigma2 = st.sigma2;
    // ---- P2 + P3: weights, sqrt weights, signs of this lane's 8-weight group
    {
        float wr[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            wr[j] = qr[j] * sqrtf(sigma2 + xr[j] * xr[j]);
            const int ei = eidx(P::SB, S::PAD, lane * 8 + j);
            st.w[ei] = wr[j];
            st.wa[ei] = sqrtf(wr[j]);
        }
        int nflip = 0;
        unsigned sg = 0;
        float xv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (xr[j] >= 0) xv[j] = xr[j]; else { xv[j] = -xr[j]; ++nflip; sg |= 1u << j; }
        }
        if (P::PARITY && (nflip % 2)) {
            int im = 0;
            float mn = wr[0] * xr[0] * xr[0];
#pragma unroll
            for (int j = 1; j < 8; ++j) { const float a = wr[j] * xr[j] * xr[j]; if (a < mn) { mn = a; im = j; } }
#pragma unroll
            for (int j = 0; j < 8; ++j) if (j == im) xv[j] = -xv[j];
            sg ^= 1u << im;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int ei = eidx(P::SB, S::PAD, lane * 8 + j);
            st.xv[ei] = xv[j];
        }
        const int e0 = lane * 8;
        st.signs[e0 / P::SB][(e0 % P::SB) / 8] = (uint8_t) (P::PARITY ? (sg & 127u) : sg);
    }
    __syncwarp();
    // ---- P4: sub-block guard and the trial range (IQ2_XXS: make_qp_quants, its 9 trials one a lane)
    if (lane < S::NSUB) {
        const float * xv = st.xv + lane * S::PAD;
        float mx = xv[0], qm = fmaxr(0.f, xv[0]);   // (make_qp_quants' own max starts at 0)
#pragma unroll 1
        for (int i = 1; i < P::SB; ++i) { mx = fmaxr(mx, xv[i]); qm = fmaxr(qm, xv[i]); }
        st.qmax[lane] = qm;
        const int skip = P::EPS_ZERO ? !mx : mx < P::EPS;
        st.skip[lane] = (uint8_t) skip;
        st.denom[lane] = mx;
        st.scale[lane] = skip ? 0.f : mx / (2 * P::KMAXQ - 1);
    }
    __syncwarp();
    if constexpr (P::QP_FIRST) {
        constexpr int NMAX = P::KMAXQ + 1;
        for (int task = lane; task < S::NSUB * 9; task += 32) {
            const int s = task / 9, k = task - s * 9;
            if (st.skip[s]) continue;
            st.u.qp.mse[s][k] = qp_trial_mse<P::SB>(k, NMAX, st.qmax[s], st.xv + s * S::PAD, st.w + s * S::PAD);
        }
        __syncwarp();
        // the chosen inverse scale and the two sums at it in index order (sumlx on lanes 0..7, suml2 on lanes
        // 8..15, one sub-block a lane): both are (w * y) * l, y = x or l
        static_assert(P::SB == 32 && S::NSUB == 8, "one lane an element, 16 sum lanes");
        if (lane < 2 * S::NSUB) {
            const int s = lane & 7, which = lane >> 3;
            if (!st.skip[s] && !(st.qmax[s] < 1e-15f)) {
                const float * xs = st.xv + s * S::PAD;
                const float * ws = st.w + s * S::PAD;
                const float iscale = qp_iscale(NMAX, st.qmax[s], st.u.qp.mse[s]);
                if (!which) st.u.qp.isc[s] = iscale;
                float sum = 0;
#pragma unroll 4
                for (int i = 0; i < 32; ++i) {
                    const float l = (float) imin(NMAX, nearest_int(iscale * xs[i]));
                    sum += ws[i] * (which ? l : xs[i]) * l;
                }
                st.u.qp.sums[s][which] = sum;
            }
        }
        __syncwarp();
        // the descent, lanes over the 32 elements: the first pass's first test of every sub-block at once; a
        // sub-block where no element changes is done (almost all of them), the others run the whole descent
        unsigned moved = 0;
#pragma unroll 1
        for (int s = 0; s < S::NSUB; ++s) {
            if (st.skip[s] || st.qmax[s] < 1e-15f) continue;
            const float x = st.xv[s * S::PAD + lane], w = st.w[s * S::PAD + lane];
            const int L = imin(NMAX, nearest_int(st.u.qp.isc[s] * x)) & 255;
            float slx, sl2;
            int nl;
            if (__ballot_sync(0xFFFFFFFFu, qp_try(NMAX, x, w, L, st.u.qp.sums[s][0], st.u.qp.sums[s][1], true, nl, slx, sl2)))
                moved |= 1u << s;
        }
#pragma unroll 1
        for (int s = 0; s < S::NSUB; ++s) {
            if (!(moved & (1u << s))) continue;
            const float x = st.xv[s * S::PAD + lane], w = st.w[s * S::PAD + lane];
            const int L = imin(NMAX, nearest_int(st.u.qp.isc[s] * x)) & 255;
            const float scale = qp_descent_warp(lane, NMAX, x, w, st.u.qp.sums[s][0], st.u.qp.sums[s][1], L);
            if (lane == 0) st.u.qp.res[s] = scale;
        }
        __syncwarp();
        if (lane < S::NSUB && !st.skip[lane]) {
            const int s = lane;
            float scale = 0.f;
            if (moved & (1u << s)) {
                scale = st.u.qp.res[s];
            } else if (!(st.qmax[s] < 1e-15f)) {
                const float sumlx = st.u.qp.sums[s][0], suml2 = st.u.qp.sums[s][1];
                scale = suml2 > 0.0f ? sumlx / suml2 : 0.0f;
            }
            st.scale[s] = scale;
            st.denom[s] = scale * P::KMAXQ;
            if (!(scale * P::KMAXQ > 0)) st.skip[s] = 1;
        }
        __syncwarp();
    }
    constexpr unsigned ALL = (1u << S::NG) - 1;
    if (lane < S::NSUB) {                                   // the trial choice's starting state
        st.p6_best[lane] = 0.f;
        st.p6_on[lane] = (uint8_t) (P::INIT_ON ? ALL : 0u);
        for (int g = 0; g < S::NG; ++g) st.lev[lane][g] = 0;
    }
    __syncwarp();
    // ---- P5: the trials, (sub-block, trial) tasks 32 a round, in batches of RB rounds:
    //   R  every task's groups rounded at the task's inverse scale (levels and on-grid flags kept); the groups
    //      off the grid counted by the length of their neighbour list;
    //   S  those searches ordered longest list first (a counting sort over list-length buckets);
    //   Q  the searches 32 at a time in that order, one a lane, so the lanes of a step run lists of about the same
    //      length (the order changes nothing in a result: every search is independent and exact);
    //   M  each task's sums over its groups in index order;
    //   then ggml's trial choice over the batch's trials, one lane a sub-block (its state carried to the next batch).
    for (int rb = 0; rb < S::NROUND; rb += S::RB) {
        const int nr = S::NROUND - rb < S::RB ? S::NROUND - rb : S::RB;
        auto & sch = st.u.sch;
        for (int i = lane; i < NBKT; i += 32) sch.hist[i] = 0;
        __syncwarp();
        for (int r = 0; r < nr; ++r) {                                          // R
            const int task = (rb + r) * 32 + lane;
            const int s = task < S::NTASK ? task / S::NT : 0, t = task - s * S::NT;
            const bool live = task < S::NTASK && !st.skip[s];
            const float id = live ? trial_id<T>(t, st.denom[s]) : 1.f;
            const float * xv = st.xv + s * S::PAD;
            // all the task's codes first, then their table loads together (in flight at once), then the bookkeeping
            int c3[S::NG], m[S::NG];
#pragma unroll
            for (int g = 0; g < S::NG; ++g) {
                const uint32_t lev = round_levels<P::GD, P::KMAXQ>(xv + g * P::GD, id, &c3[g]);
                if (live) st.t_lev[r * 32 + lane][g] = (uint16_t) lev;
            }
#pragma unroll
            for (int g = 0; g < S::NG; ++g) m[g] = live ? __ldg(tab.code3 + c3[g]) : 0;
            unsigned onb = 0;
#pragma unroll
            for (int g = 0; g < S::NG; ++g) {
                uint8_t bk = 0xFF;
                if (live) {
                    if (m[g] >= 0) {
                        onb |= 1u << g;
                    } else {
                        bk = (uint8_t) len_bucket(list_cnt(m[g]));
                        atomicAdd(&sch.hist[bk], 1);
                    }
                }
                sch.bkt[(r * 32 + lane) * S::NG + g] = bk;
            }
            if (task < S::NTASK) st.t_on[r * 32 + lane] = (uint8_t) onb;
        }
        __syncwarp();
        const int nreq = bucket_offsets(sch.hist, lane);                        // S
        __syncwarp();
        for (int i = lane; i < nr * 32 * S::NG; i += 32) {
            const int bk = sch.bkt[i];
            if (bk != 0xFF) sch.perm[atomicAdd(&sch.hist[bk], 1)] = (uint16_t) i;
        }
        __syncwarp();
        for (int k0 = 0; k0 < nreq; k0 += 32) {                                 // Q
            if (k0 + lane < nreq) {
                const int item = sch.perm[k0 + lane];
                const int slot = item / S::NG, g = item - slot * S::NG;
                const int task = rb * 32 + slot;
                const int s = task / S::NT;
                const float ts = 1 / trial_id<T>(task - s * S::NT, st.denom[s]);
                const float * xv = st.xv + s * S::PAD + g * P::GD;
                const float * wa = st.wa + s * S::PAD + g * P::GD;
                const int m = __ldg(tab.code3 + code3_of<P::GD>(st.t_lev[slot][g]));
                uint32_t lev = P::GD == 8 ? search_lane8(m, xv, wa, ts, tab) : search_lane4(m, xv, wa, ts, tab);
                if (lev == NONE) { atomicOr(status, ST_NO_NEIGHBOUR); lev = 0; }
                st.t_lev[slot][g] = (uint16_t) lev;
            }
        }
        __syncwarp();
#pragma unroll 1
        for (int r = 0; r < nr; ++r) {                                          // M
            const int task = (rb + r) * 32 + lane;
            if (task >= S::NTASK) continue;
            const int s = task / S::NT;
            float sqx = 0, sq2 = 0;
            if (!st.skip[s]) {
                const float * xs = st.xv + s * S::PAD;
                const float * w = st.w + s * S::PAD;
#pragma unroll 1
                for (int g = 0; g < S::NG; ++g) {
                    const uint32_t lev = st.t_lev[r * 32 + lane][g];
#pragma unroll
                    for (int i = 0; i < P::GD; ++i) {
                        const float q = odd_level(level_of<P::GD>(lev, i));
                        const int e = g * P::GD + i;
                        sqx += w[e] * xs[e] * q;   // (ggml's w*x*q, in that order)
                        sq2 += w[e] * q * q;
                    }
                }
            }
            st.sums().sqx[r * 32 + lane] = sqx;
            st.sums().sq2[r * 32 + lane] = sq2;
        }
        __syncwarp();
        // ggml's trial choice (gpuq.hip:305-332) replayed in trial order over this batch's trials of each sub-block,
        // one lane a sub-block, carrying its state from batch to batch: the same comparisons in the same order as one
        // pass over all the trials; the winner's levels are copied while the batch still holds them
        if (lane < S::NSUB && !st.skip[lane]) {
            const int s = lane, b0 = rb * 32;
            const int t0 = imax(0, b0 - s * S::NT), t1 = imin(S::NT, imin(S::NTASK, b0 + nr * 32) - s * S::NT);
            float scale = st.scale[s], best = st.p6_best[s];
            int take = -1;
#pragma unroll 1
            for (int t = t0; t < t1; ++t) {
                const int slot = s * S::NT + t - b0;
                const float sqx = st.sums().sqx[slot], sq2 = st.sums().sq2[slot];
                if (sq2 > 0 && sqx * sqx > best * sq2) { scale = sqx / sq2; best = scale * sqx; take = slot; }
            }
            if (take >= 0) {
#pragma unroll 1
                for (int g = 0; g < S::NG; ++g) st.lev[s][g] = st.t_lev[take][g];
                st.p6_on[s] = st.t_on[take];
            }
            st.scale[s] = scale;
            st.p6_best[s] = best;
        }
        __syncwarp();
    }
    // ---- P6: which groups to snap again, from ggml's trial choice (replayed batch by batch above)
    if (lane < S::NSUB) {
        const int s = lane;
        uint8_t rg = 0;
        if (!st.skip[s]) {
            const unsigned on = st.p6_on[s];
            const int n_off = __popc(~on & ALL);
            if ((P::REGRID_ANY ? n_off > 0 : true) && st.scale[s] > 0) rg = (uint8_t) (P::REGRID_ALL ? ALL : (~on & ALL));
        }
        st.regrid[s] = rg;
    }
    __syncwarp();
    // ---- P7: snap the chosen groups again with the final scale, one (sub-block, group) a lane. The 8-d searches of
    //      a round are split into at most 32 runs of about equal length, one a lane, and each search takes the first
    //      strict minimum over its runs in list order (the same candidates and distances as one lane's whole list)
    auto & rg = st.u.rg;
    for (int r0 = 0; r0 < S::NRG; r0 += 32) {
        const int r = r0 + lane;
        const int s = r < S::NRG ? r / S::NG : 0, g = r - s * S::NG;
        const bool act = r < S::NRG && (st.regrid[s] & (1u << g));
        const float scale = act ? st.scale[s] : 1.f;
        int m = 0;
        uint32_t lev = 0;
        if (act) lev = round_group<P::GD, P::KMAXQ>(st.xv + s * S::PAD + g * P::GD, 1 / scale, tab, &m);
        const int n = act && m < 0 ? list_cnt(m) : 0;
        if constexpr (P::GD == 4) {   // (the 4-d lists are short: one lane a list)
            if (n) lev = search_lane4(m, st.xv + s * S::PAD + g * P::GD, st.wa + s * S::PAD + g * P::GD, scale, tab);
        }
        int run = 0, first = 0, nrun = 0;
        const int nruns = P::GD == 8 ? split_runs(n, lane, &run, &first, &nrun) : 0;
        if (nruns) {
            rg.m[lane] = m;
            for (int c = 0; c < nrun; ++c) rg.owner[first + c] = (uint16_t) (lane | (c << 5));
            __syncwarp();
            if (lane < nruns) {
                const int o = rg.owner[lane], ol = o & 31, c = o >> 5;
                const int orr = r0 + ol, os = orr / S::NG, og = orr - os * S::NG;
                const int om = rg.m[ol], j0 = c * run, cnt = imin(list_cnt(om), j0 + run) - j0;
                float bd;
                rg.be[lane] = search_run<P::GD>(tab.neigh + list_off(om) + 1 + j0, cnt, st.xv + os * S::PAD + og * P::GD,
                                                st.wa + os * S::PAD + og * P::GD, st.scale[os], bd);
                rg.bd[lane] = bd;
            }
            __syncwarp();
            if (n) {
                float best = FLT_MAX;
                uint32_t bl = NONE;
                for (int c = 0; c < nrun; ++c)
                    if (rg.bd[first + c] < best) { best = rg.bd[first + c]; bl = rg.be[first + c]; }
                lev = bl == NONE ? NONE : (bl & 0xFFFFu);
            }
            __syncwarp();
        }
        if (act) {
            if (lev == NONE) { atomicOr(status, ST_NO_NEIGHBOUR); lev = 0; }
            st.lev[s][g] = (uint16_t) lev;
        }
    }
    __syncwarp();
    // ---- P8: refit, signs, grid indices (one sub-block a lane)
    if (lane < S::NSUB) {
        const int s = lane;
        if (!st.skip[s]) {
            float scale = st.scale[s];
            if (st.regrid[s]) {
                const float * xs = st.xv + s * S::PAD;
                const float * w = st.w + s * S::PAD;
                float sqx = 0, sq2 = 0;
#pragma unroll 4
                for (int e = 0; e < P::SB; ++e) {
                    const float q = odd_level(level_of<P::GD>(st.lev[s][e / P::GD], e % P::GD));
                    sqx += w[e] * xs[e] * q;
                    sq2 += w[e] * q * q;
                }
                if (sq2 > 0) scale = sqx / sq2;
            }
            if (scale < 0) {
                scale = -scale;
                for (int k = 0; k < S::NSG; ++k)
                    st.signs[s][k] = (uint8_t) (P::PARITY ? (~st.signs[s][k]) & 127 : (uint8_t) ~st.signs[s][k]);
            }
#pragma unroll 1
            for (int g = 0; g < S::NG; ++g) {
                const int gi = __ldg(tab.code3 + code3_of<P::GD>(st.lev[s][g]));
                if (gi < 0) atomicOr(status, ST_OFF_GRID);
                st.gidx[s][g] = gi < 0 ? 0 : gi;
            }
            st.scale[s] = scale;
        } else {
            st.scale[s] = 0.f;
        }
    }
    __syncwarp();
    // ---- P9: super-block scale and the block bytes, then a coalesced store. IQ2_XXS: lane 0 the super-block scale
    //      (ggml's max in sub-block order), one lane a sub-block its 8 bytes; the other types: lane 0 all of it
    if constexpr (T == IQ2_XXS) {
        if (lane == 0) {
            float max_scale = 0;
#pragma unroll 1
            for (int s = 0; s < S::NSUB; ++s) if (!st.skip[s]) max_scale = fmaxr(max_scale, st.scale[s]);
            st.sigma2 = max_scale;   // (sigma2 is dead: it carries the max to the other lanes)
        }
        __syncwarp();
        const float max_scale = st.sigma2;
        uint8_t * y = st.u.out;
        if (lane < S::NSUB) {
            const int s = lane;
            uint32_t q0 = 0, q1 = 0;
            if (max_scale) {
                const float d = max_scale / 31;
                const float idd = 1 / d;
                if (!st.skip[s]) {
#pragma unroll 1
                    for (int k = 0; k < 4; ++k) { q0 |= (uint32_t) st.gidx[s][k] << (8 * k); q1 |= (uint32_t) st.signs[s][k] << (7 * k); }
                }
                q1 |= (uint32_t) imax(0, imin(15, nearest_int(0.5f * (idd * st.scale[s] - 1)))) << 28;
                if (s == 0) { const uint16_t h = half_bits(d); y[0] = h & 255; y[1] = h >> 8; }
            } else if (s == 0) {
                y[0] = y[1] = 0;
            }
#pragma unroll 1
            for (int j = 0; j < 4; ++j) { y[2 + 8 * s + j] = (q0 >> (8 * j)) & 255; y[6 + 8 * s + j] = (q1 >> (8 * j)) & 255; }
        }
    } else if (lane == 0) {
        uint8_t * y = st.u.out;
        for (int i = 0; i < block_bytes(T); ++i) y[i] = 0;
        float max_scale = 0;
#pragma unroll 1
        for (int s = 0; s < S::NSUB; ++s) if (!st.skip[s]) max_scale = fmaxr(max_scale, st.scale[s]);
        const float d = max_scale / 31;
        const float idd = 1 / d;
        auto scale4 = [&](int s) { return imax(0, imin(15, nearest_int(0.5f * (idd * st.scale[s] - 1)))); };
        if constexpr (T == IQ2_XS) {
            if (max_scale) {
                const uint16_t h = half_bits(d);
                y[0] = h & 255; y[1] = h >> 8;
                for (int s = 0; s < 16; ++s) {
                    if (!st.skip[s])
                        for (int k = 0; k < 2; ++k) {
                            const uint16_t v = (uint16_t) (st.gidx[s][k] | (st.signs[s][k] << 9));
                            y[2 + 2 * (2 * s + k)] = v & 255; y[3 + 2 * (2 * s + k)] = v >> 8;
                        }
                    y[66 + s / 2] |= (uint8_t) (scale4(s) << (4 * (s % 2)));
                }
            }
        } else if constexpr (T == IQ2_S) {
            for (int s = 0; s < 16; ++s) {
                if (st.skip[s]) continue;
                for (int k = 0; k < 2; ++k) {
                    const int i8 = 2 * s + k;
                    y[2 + i8] = (uint8_t) (st.gidx[s][k] & 255);
                    y[66 + i8 / 4] |= (uint8_t) ((st.gidx[s][k] >> 8) << (2 * (i8 % 4)));
                    y[34 + i8] = st.signs[s][k];
                }
            }
            if (max_scale) {
                const uint16_t h = half_bits(d * 0.9875f);
                y[0] = h & 255; y[1] = h >> 8;
                for (int s = 0; s < 16; ++s) y[74 + s / 2] |= (uint8_t) (scale4(s) << (4 * (s % 2)));
            }
        } else if constexpr (T == IQ3_XXS) {
            if (max_scale) {
                const uint16_t h = half_bits(d * 1.0125f);
                y[0] = h & 255; y[1] = h >> 8;
                for (int s = 0; s < 8; ++s) {
                    uint32_t ss = 0;
                    if (!st.skip[s]) {
                        for (int k = 0; k < 8; ++k) y[2 + 8 * s + k] = (uint8_t) st.gidx[s][k];
                        ss = st.signs[s][0] | (st.signs[s][1] << 7) | (st.signs[s][2] << 14) | ((uint32_t) st.signs[s][3] << 21);
                    }
                    ss |= (uint32_t) scale4(s) << 28;
                    for (int j = 0; j < 4; ++j) y[66 + 4 * s + j] = (ss >> (8 * j)) & 255;
                }
            }
        } else {   // IQ3_S: qs / signs advance only past sub-blocks that were not skipped (gpuq.hip:1188-1190, :1266-1268)
            int qo = 0, so = 0;
            for (int s = 0; s < 8; ++s) {
                if (st.skip[s]) continue;
                for (int k = 0; k < 8; ++k) {
                    y[2 + qo + k] = (uint8_t) (st.gidx[s][k] & 255);
                    y[66 + s] |= (uint8_t) ((st.gidx[s][k] >> 8) << k);
                }
                qo += 8;
                for (int k = 0; k < 4; ++k) y[74 + so + k] = st.signs[s][k];
                so += 4;
            }
            if (max_scale) {
                const uint16_t h = half_bits(d * 1.033f);
                y[0] = h & 255; y[1] = h >> 8;
                for (int s = 0; s < 8; s += 2) y[106 + s / 2] = (uint8_t) (scale4(s) | (scale4(s + 1) << 4));
            }
        }
    }
    __syncwarp();
    uint8_t * yo = out + b * block_bytes(T);
    for (int i = lane; i < block_bytes(T); i += 32) yo[i] = st.u.out[i];
}

template <int T, int SRC>
cudaError_t launch_t(const LaunchArgs & a) {
    constexpr int WARPS = 4;
    const size_t smem = sizeof(WarpState<T>) * WARPS;
    const cudaError_t e = cudaFuncSetAttribute(k_iq_grid<T, SRC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (e != cudaSuccess) return e;

    const int64_t grid = (a.nblocks + WARPS - 1) / WARPS;
    k_iq_grid<T, SRC><<<(unsigned) grid, WARPS * 32, smem, a.stream>>>(
        (const uint8_t *) a.src, a.qw, a.qw_mod, a.qw_div, a.qw_mat, (uint8_t *) a.out, a.nblocks, a.tab, a.status);
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

cudaError_t launch_iq_grid(int type, const LaunchArgs & a) {
    switch (type) {
        case IQ2_XXS: return launch_src<IQ2_XXS>(a);
        case IQ2_XS:  return launch_src<IQ2_XS>(a);
        case IQ2_S:   return launch_src<IQ2_S>(a);
        case IQ3_XXS: return launch_src<IQ3_XXS>(a);
        case IQ3_S:   return launch_src<IQ3_S>(a);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace gq
