// search.cuh - the 8-d codebooks' neighbour search (IQ1_S/IQ1_M, IQ2_XXS/XS/S) and the length-sorted schedule
// that runs many of them on one warp.
//
// What is computed: ggml's listed-neighbour rule (iq2_find_best_neighbour gpuq.hip:178-197,
// iq1_find_best_neighbour2 :199-232): over the candidate points of a code's list, d2 = 0; d2 += w_i (s q_i - x_i)^2
// for i = 0..7 in order; the first strict minimum in list order wins, and a distance that is NaN or not below
// FLT_MAX never wins.
//
// How: one lane runs one whole list. Its 24 per-dimension terms w_i (s q_l - x_i)^2 (three levels l) are formed
// once, so a candidate costs a select and two predicated additions a dimension, in ggml's order, with the next list
// entry loaded one step ahead. The lists differ in length (1..292 points), so a kernel collects a batch of
// searches, counts them into list-length buckets and runs them longest first, 32 at a time: the lanes of a step
// then run lists of about the same length. A search depends only on its own inputs, so the order changes no result.
#pragma once
#include "common.cuh"

namespace gq {

constexpr uint32_t NONE = 0xFFFFFFFFu;

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

// one lane's run over cnt consecutive entries of a list (lst: the first of them): the first strict minimum of
// ggml's distance in list order, the next entry loaded one step ahead. Returns the winning entry (NONE if no
// distance is below FLT_MAX) and its distance in best.
template <bool PRED = true>
__device__ __forceinline__ uint32_t search_run8(const uint32_t * lst, int cnt, const float (&t0)[8], const float (&t1)[8],
                                                const float (&t2)[8], float & best) {
    best = FLT_MAX;
    uint32_t bl = NONE;
    uint32_t e = __ldg(lst);
#pragma unroll 2
    for (int j = 0; j < cnt; ++j) {
        const uint32_t en = __ldg(lst + j + 1);   // (one past a run: the list's next entry, its count word or the pad word)
        const float d2 = cand_dist<PRED>(e, t0, t1, t2);
        if (d2 < best) { best = d2; bl = e; }
        e = en;
    }
    return bl;
}

// one lane's whole list (code3 entry m < 0). Returns the winning entry, NONE if no distance is finite.
template <bool PRED = true>
__device__ __forceinline__ uint32_t search_list8(int m, const float (&t0)[8], const float (&t1)[8], const float (&t2)[8],
                                                 const SearchTab & tab) {
    float best;
    return search_run8<PRED>(tab.neigh + list_off(m) + 1, list_cnt(m), t0, t1, t2, best);
}

// Warp-collective sums and exclusive prefix sums of one int a lane
__device__ __forceinline__ int warp_sum(int v) { return (int) __reduce_add_sync(0xFFFFFFFFu, (unsigned) v); }
__device__ __forceinline__ int warp_excl_prefix(int v, int lane) {
    int incl = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int u = __shfl_up_sync(0xFFFFFFFFu, incl, d);
        if (lane >= d) incl += u;
    }
    return incl - v;
}

// Warp-collective split of up to 32 searches (lane i: a list of n >= 0 entries) into at most 32 runs of at most
// *run entries, a search's runs on consecutive lanes from *first: the smallest run length tried (from the even
// split up, by quarters) that needs no more than 32 runs. Returns the number of runs; 0 when there is no search.
__device__ __forceinline__ int split_runs(int n, int lane, int * run, int * first, int * nruns) {
    const int total = warp_sum(n);
    if (!total) return 0;
    int len = (total + 31) / 32, cnt;
    for (;;) {
        cnt = warp_sum(n ? (n + len - 1) / len : 0);
        if (cnt <= 32) break;
        len += (len + 3) / 4;
    }
    const int k = n ? (n + len - 1) / len : 0;
    *run = len;
    *nruns = k;
    *first = warp_excl_prefix(k, lane);
    return cnt;
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

}  // namespace gq
