// search.cuh - the warp-balanced nearest-neighbour search of the 8-d codebooks (IQ1_S/IQ1_M, IQ2_XXS/XS/S).
//
// What is computed: for each of up to 32 searches (one a lane) ggml's listed-neighbour rule
// (iq2_find_best_neighbour gpuq.hip:178-197, iq1_find_best_neighbour2 :199-232): over the candidate points of
// the search's list, d2 = 0; d2 += w_i (s q_i - x_i)^2 for i = 0..7 in order; the first strict minimum in list
// order wins, and a distance that is NaN or not below FLT_MAX never wins.
//
// How: a lane holds its search's 24 per-dimension terms w_i (s q_l - x_i)^2 (three levels l) in registers, so a
// candidate costs 8 two-way selects and ggml's 8 additions in ggml's order. The lists differ in length (1..292
// points), so one lane a list leaves most lanes idle while the longest list runs. The warp therefore splits the
// work in two phases: with K = ceil(total candidates / 32), every lane first runs the first K candidates of its own
// list; the candidates beyond K are then laid end to end (a prefix sum of the leftovers) and every lane takes an
// equal contiguous share, loading the terms of whichever search its share crosses into from shared memory. A lane
// keeps one running minimum a search and merges it into the search's slot as (d2 bits << 32 | list position):
// d2 >= +0, so the float bits order like the values, and on equal distances the smaller list position - ggml's
// first minimum - wins (64-bit atomicMin in shared memory where several lanes share a search).
#pragma once
#include "common.cuh"

namespace gq {

constexpr uint32_t NONE = 0xFFFFFFFFu;

// per-warp shared scratch of one batch of up to 32 searches
struct alignas(16) Search8Scratch {
    float4 terms[32][6];             // a search's terms: levels 0, 1, 2 of dimensions 0..7 (8 floats a level)
    unsigned long long key[32];      // a search's best (d2 bits << 32 | list position), ~0 while none
    int cstart[33];                  // the searches with leftovers, compacted: first flattened position; [n] = total
    int cslot[32];                   // ... their lane (slot of key/terms)
    int clofs[32];                   // ... their list offset in tab.neigh
};

// the three level terms of one dimension, ggml's expression w * diff * diff with diff = s * q - x
__device__ __forceinline__ void level_terms(float w, float x, float s, float q0, float q1, float q2,
                                            float & t0, float & t1, float & t2) {
    const float d0 = s * q0 - x, d1 = s * q1 - x, d2 = s * q2 - x;
    t0 = w * d0 * d0;
    t1 = w * d1 * d1;
    t2 = w * d2 * d2;
}

// ggml's distance of one candidate (entry: packed 2-bit levels in bits 0..15), additions in dimension order.
// Level 2 has bit 1 set, level 1 bit 0 (level 3 does not occur). Per dimension: a select between the level-0 and
// level-1 terms, then two additions predicated on bit 1 - exactly one of them executes, so d2 gets ggml's single
// rounded addition of the chosen term - which puts two of the five instructions on the FMA pipe instead of the
// integer pipe that a second select would use.
// (PRED = false: two selects, for kernels where the predicated form costs registers)
template <bool PRED = true>
__device__ __forceinline__ float cand_dist(uint32_t e, const float (&t0)[8], const float (&t1)[8], const float (&t2)[8]) {
    float d2 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if (!PRED) {
            const bool hi = e & (2u << (2 * i)), lo = e & (1u << (2 * i));
            d2 += hi ? t2[i] : (lo ? t1[i] : t0[i]);
            continue;
        }
        const float t01 = (e & (1u << (2 * i))) ? t1[i] : t0[i];
        asm("{\n\t.reg .pred ph;\n\t.reg .b32 m;\n\t"
            "and.b32 m, %1, %4;\n\t"
            "setp.ne.b32 ph, m, 0;\n\t"
            "@ph add.rn.f32 %0, %0, %3;\n\t"
            "@!ph add.rn.f32 %0, %0, %2;\n\t}"
            : "+f"(d2) : "r"(e), "f"(t01), "f"(t2[i]), "r"(2u << (2 * i)));
    }
    return d2;
}

// one lane's whole list (code3 entry m < 0): the first strict minimum of ggml's distance in list order, the next
// entry loaded one step ahead. Returns the winning entry, NONE if no distance is finite.
template <bool PRED = true>
__device__ __forceinline__ uint32_t search_list8(int m, const float (&t0)[8], const float (&t1)[8], const float (&t2)[8],
                                                 const SearchTab & tab) {
    const uint32_t * lst = tab.neigh + list_off(m) + 1;
    const int n = list_cnt(m);
    float best = FLT_MAX;
    uint32_t bl = NONE;
    uint32_t e = __ldg(lst);
#pragma unroll 2
    for (int j = 0; j < n; ++j) {
        const uint32_t en = __ldg(lst + j + 1);   // (one past a list: the next count word or the pad word)
        const float d2 = cand_dist<PRED>(e, t0, t1, t2);
        if (d2 < best) { best = d2; bl = e; }
        e = en;
    }
    return bl;
}

// list-length bucket of a search schedule (longest first): exact below 48, then 8 lengths a bucket (lists of 176
// points and more share the last one)
constexpr int NBKT = 64, BKT_PER_LANE = NBKT / 32;
__device__ __forceinline__ int len_bucket(int n) { return n < 48 ? n : min(NBKT - 1, 48 + ((n - 48) >> 3)); }

// Warp-collective: the exclusive start of every bucket when the buckets are laid out longest first, written back
// over the counts in hist[NBKT]; returns the number of items counted.
__device__ __forceinline__ int bucket_offsets(int * hist, int lane) {
    int c[BKT_PER_LANE], local = 0;
#pragma unroll
    for (int k = 0; k < BKT_PER_LANE; ++k) { c[k] = hist[NBKT - 1 - (BKT_PER_LANE * lane + k)]; local += c[k]; }
    int incl = local;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int v = __shfl_up_sync(0xFFFFFFFFu, incl, d);
        if (lane >= d) incl += v;
    }
    const int total = __shfl_sync(0xFFFFFFFFu, incl, 31);
    int run = incl - local;
#pragma unroll
    for (int k = 0; k < BKT_PER_LANE; ++k) { hist[NBKT - 1 - (BKT_PER_LANE * lane + k)] = run; run += c[k]; }
    return total;
}

__device__ __forceinline__ unsigned long long best_key(float d2, int j) {
    return ((unsigned long long) f2u(d2) << 32) | (unsigned) j;
}

// Warp-collective: every lane of the warp calls it, with or without a search of its own. req: this lane searches;
// lofs: the offset of its list in tab.neigh (the count word); t0/t1/t2: its terms for levels 0, 1, 2.
// Returns this lane's winning list entry (grid index << 16 | packed levels), NONE when it has no search or no
// listed distance is finite.
__device__ __forceinline__ uint32_t search8_warp(Search8Scratch & sc, int lane, bool req, int lofs,
                                              const float (&t0)[8], const float (&t1)[8], const float (&t2)[8],
                                              const SearchTab & tab) {
    const int n = req ? (int) __ldg(tab.neigh + lofs) : 0;
    int total = n;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) total += __shfl_xor_sync(0xFFFFFFFFu, total, d);
    if (total == 0) return NONE;                       // (warp-uniform)
    const int K = (total + 31) >> 5;
    __syncwarp();                                      // the previous batch's readers are done with the scratch
    // ---- phase 1: the first K candidates of the lane's own list
    {
        unsigned long long k = ~0ull;
        const int na = min(n, K);
        if (na > 0) {
            const uint32_t * lst = tab.neigh + lofs + 1;
            float bestd = FLT_MAX;
            int bestj = -1;
            uint32_t e = __ldg(lst);
            for (int j = 0; j < na; ++j) {
                const uint32_t en = __ldg(lst + j + 1);   // (one past a list: the next count word or the pad word)
                const float d2 = cand_dist(e, t0, t1, t2);
                if (d2 < bestd) { bestd = d2; bestj = j; }
                e = en;
            }
            if (bestj >= 0) k = best_key(bestd, bestj);
        }
        sc.key[lane] = k;
    }
    // ---- phase 2: the leftovers beyond K, flattened and shared out evenly
    const int m = n > K ? n - K : 0;
    const unsigned mask = __ballot_sync(0xFFFFFFFFu, m > 0);
    if (mask) {
        int incl = m;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int v = __shfl_up_sync(0xFFFFFFFFu, incl, d);
            if (lane >= d) incl += v;
        }
        const int left = __shfl_sync(0xFFFFFFFFu, incl, 31);
        const int nc = __popc(mask);
        if (m > 0) {
            const int ci = __popc(mask & ((1u << lane) - 1u));
            sc.cstart[ci] = incl - m;
            sc.cslot[ci] = lane;
            sc.clofs[ci] = lofs;
            float4 * tt = sc.terms[lane];
            tt[0] = make_float4(t0[0], t0[1], t0[2], t0[3]); tt[1] = make_float4(t0[4], t0[5], t0[6], t0[7]);
            tt[2] = make_float4(t1[0], t1[1], t1[2], t1[3]); tt[3] = make_float4(t1[4], t1[5], t1[6], t1[7]);
            tt[4] = make_float4(t2[0], t2[1], t2[2], t2[3]); tt[5] = make_float4(t2[4], t2[5], t2[6], t2[7]);
        }
        if (lane == 0) sc.cstart[nc] = left;
        __syncwarp();
        const int per = (left + 31) >> 5;
        int p = lane * per;
        const int p1 = min(p + per, left);
        if (p < p1) {
            int r = 0;                                 // the last compacted search starting at or before p
#pragma unroll
            for (int h = 16; h; h >>= 1) if (r + h < nc && sc.cstart[r + h] <= p) r += h;
            int rend = sc.cstart[r + 1];
            int j = p - sc.cstart[r];
            int slot = sc.cslot[r];
            const uint32_t * lst = tab.neigh + sc.clofs[r] + 1 + K;
            float a[8], b[8], c[8];
            auto load = [&](int sl) {
                const float4 * tt = sc.terms[sl];
                const float4 v0 = tt[0], v1 = tt[1], v2 = tt[2], v3 = tt[3], v4 = tt[4], v5 = tt[5];
                a[0] = v0.x; a[1] = v0.y; a[2] = v0.z; a[3] = v0.w; a[4] = v1.x; a[5] = v1.y; a[6] = v1.z; a[7] = v1.w;
                b[0] = v2.x; b[1] = v2.y; b[2] = v2.z; b[3] = v2.w; b[4] = v3.x; b[5] = v3.y; b[6] = v3.z; b[7] = v3.w;
                c[0] = v4.x; c[1] = v4.y; c[2] = v4.z; c[3] = v4.w; c[4] = v5.x; c[5] = v5.y; c[6] = v5.z; c[7] = v5.w;
            };
            load(slot);
            float bestd = FLT_MAX;
            int bestj = -1;
            uint32_t e = __ldg(lst + j);
            for (;;) {
                const uint32_t en = __ldg(lst + j + 1);
                const float d2 = cand_dist(e, a, b, c);
                if (d2 < bestd) { bestd = d2; bestj = j; }
                ++p; ++j;
                if (p == p1) break;
                if (p == rend) {                       // into the next search's leftover
                    if (bestj >= 0) atomicMin(&sc.key[slot], best_key(bestd, bestj + K));
                    ++r;
                    rend = sc.cstart[r + 1];
                    slot = sc.cslot[r];
                    lst = tab.neigh + sc.clofs[r] + 1 + K;
                    j = 0;
                    load(slot);
                    bestd = FLT_MAX;
                    bestj = -1;
                    e = __ldg(lst);
                } else {
                    e = en;
                }
            }
            if (bestj >= 0) atomicMin(&sc.key[slot], best_key(bestd, bestj + K));
        }
    }
    __syncwarp();
    if (!req) return NONE;
    const unsigned long long k = sc.key[lane];
    return k == ~0ull ? NONE : __ldg(tab.neigh + lofs + 1 + (uint32_t) k);
}

}  // namespace gq
