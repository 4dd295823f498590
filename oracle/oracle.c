/* oracle/oracle.c - TEST INFRASTRUCTURE ONLY. Never linked into, loaded by or called from the product library.
 *
 * A plain, sequential CPU restatement of the quantizer hot path of trench-gguf (gpuq/gpuq.hip, v0.5.0), which in
 * turn states ggml's quantize_row_*_impl / *_ref / dequantize_row_* (llama.cpp ac8e1694d). One block at a time, one
 * thread, every float expression in the reference's operand order, every sum in its index order. Built with
 * -ffp-contract=off -fno-fast-math (no FMA, IEEE division and square root), as ggml-base and the reference are.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this file, and only as the checker.
 *
 * Parity pin: the tests compare this restatement with (a) the reference's own block functions compiled on the
 * host from the reference sources (oracle/_ref, built by oracle/Makefile), block for block, on the reference
 * self-test's input recipe and the benchmark configurations' distributions; (b) gguf-py's ggml-exact Q8_0 quantizer and its
 * dequantizers of every type; (c) the golden fixtures in tests/golden/ written from (a).
 *
 * Citations: "gpuq.hip:N" is trench-gguf gpuq/gpuq.hip line N.
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>

#define QK 256
enum { O_IQ2_XXS = 16, O_IQ2_XS = 17, O_IQ3_XXS = 18, O_IQ1_S = 19, O_IQ4_NL = 20, O_IQ3_S = 21, O_IQ2_S = 22,
       O_IQ4_XS = 23, O_IQ1_M = 29, O_Q8_0 = 8, O_Q2_K = 10, O_Q3_K = 11, O_Q4_K = 12, O_Q5_K = 13, O_Q6_K = 14 };
enum { O_SRC_F32 = 0, O_SRC_F16 = 1, O_SRC_Q8_0 = 8, O_SRC_BF16 = 30, O_SRC_MXFP4 = 39 };

/* ------------------------------------------------------------------------------------------------ scalar helpers */
static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ggml's float -> half (ggml_compute_fp32_to_fp16; gpuq.hip:91-106) */
static uint16_t o_half(float f) {
    float base = (fabsf(f) * 0x1.0p+112f) * 0x1.0p-110f;
    const uint32_t w = f2u(f), shl1 = w + w, sign = w & 0x80000000u;
    uint32_t bias = shl1 & 0xFF000000u;
    if (bias < 0x71000000u) bias = 0x71000000u;
    base = u2f((bias >> 1) + 0x07800000u) + base;
    const uint32_t bits = f2u(base);
    const uint32_t nonsign = ((bits >> 13) & 0x7C00u) + (bits & 0x0FFFu);
    return (uint16_t) ((sign >> 16) | (shl1 > 0xFF000000u ? 0x7E00u : nonsign));
}

/* half -> float, exact (gpuq.hip:2108-2120) */
static float o_unhalf(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1F, m = h & 0x3FF;
    if (e == 0) {
        if (!m) return u2f(sign);
        e = 113;
        while (!(m & 0x400)) { m <<= 1; --e; }
        return u2f(sign | (e << 23) | ((m & 0x3FF) << 13));
    }
    if (e == 31) return u2f(sign | 0x7F800000u | (m << 13));
    return u2f(sign | ((e + 112) << 23) | (m << 13));
}

/* round to nearest, ties to even, by the 1.5*2^23 bias (nearest_int; gpuq.hip:108-112) */
static int o_rint(float v) { return (int) (f2u(v + 12582912.f) & 0x007FFFFF) - 0x00400000; }

static int imin(int a, int b) { return a < b ? a : b; }
static int imax(int a, int b) { return a > b ? a : b; }
static float fmaxr(float a, float b) { return a > b ? a : b; }   /* the reference's MAX(a, b) */

/* ------------------------------------------------------------------------------------------------ tables */
typedef struct { int type; int ngrid, nmap, nneigh; uint64_t * grid; int32_t * map; uint16_t * neigh; } otab_t;
static otab_t g_tab[16];
static int g_ntab = 0;

static const otab_t * find_tab(int type) {
    for (int i = 0; i < g_ntab; ++i) if (g_tab[i].type == type) return &g_tab[i];
    return NULL;
}
static const otab_t * search_tab(int type) { return find_tab(type == O_IQ1_M ? O_IQ1_S : type); }
static const otab_t * dequant_tab(int type) { return find_tab(1000 + (type == O_IQ1_M ? O_IQ1_S : type)); }

/* ------------------------------------------------------------------------------------------------ shared searches */
/* make_qp_quants (gpuq.hip:114-176): positive levels 0..nmax of x with weights w, 8 trial scales then coordinate
 * descent; returns the least-squares scale */
static float o_qp_levels(int n, int nmax, const float * x, uint8_t * L, const float * w) {
    float mx = 0;
    for (int i = 0; i < n; ++i) mx = fmaxr(mx, x[i]);
    if (mx < 1e-15f) { memset(L, 0, n); return 0.f; }
    float iscale = nmax / mx;
    for (int i = 0; i < n; ++i) L[i] = (uint8_t) o_rint(iscale * x[i]);
    const float scale0 = 1 / iscale;
    float best_mse = 0;
    for (int i = 0; i < n; ++i) { const float d = x[i] - scale0 * L[i]; best_mse += w[i] * d * d; }
    for (int is = -4; is <= 4; ++is) {
        if (!is) continue;
        const float iscale_is = (0.1f * is + nmax) / mx;
        const float scale_is = 1 / iscale_is;
        float mse = 0;
        for (int i = 0; i < n; ++i) {
            const int l = imin(nmax, o_rint(iscale_is * x[i]));
            const float d = x[i] - scale_is * l;
            mse += w[i] * d * d;
        }
        if (mse < best_mse) { best_mse = mse; iscale = iscale_is; }
    }
    float sumlx = 0, suml2 = 0;
    for (int i = 0; i < n; ++i) {
        const int l = imin(nmax, o_rint(iscale * x[i]));
        L[i] = (uint8_t) l;
        sumlx += w[i] * x[i] * l;
        suml2 += w[i] * l * l;
    }
    for (int pass = 0; pass < 5; ++pass) {
        int changed = 0;
        for (int i = 0; i < n; ++i) {
            float slx = sumlx - w[i] * x[i] * L[i];
            float sl2 = suml2 - w[i] * L[i] * L[i];
            if (slx > 0 && sl2 > 0) {
                const int nl = imin(nmax, o_rint(x[i] * sl2 / slx));
                if (nl != L[i]) {
                    slx += w[i] * x[i] * nl;
                    sl2 += w[i] * nl * nl;
                    if (slx * slx * suml2 > sumlx * sumlx * sl2) { L[i] = (uint8_t) nl; sumlx = slx; suml2 = sl2; ++changed; }
                }
            }
        }
        if (!changed) break;
    }
    return suml2 > 0.0f ? sumlx / suml2 : 0.0f;
}

/* nearest listed codebook point to x (weights w, scale s) in the 2l+1 lattice; the first minimum wins
 * (iq2_find_best_neighbour gpuq.hip:178-197, iq3_find_best_neighbour :972-992); -1 if no candidate is finite */
static int o_listed_nearest(const uint16_t * list, const uint64_t * grid, int dims, const float * x, const float * w,
                            float s, int8_t * L) {
    const int n = list[0];
    float best = FLT_MAX;
    int gi = -1;
    for (int j = 1; j <= n; ++j) {
        const int8_t * p = (const int8_t *) (grid + list[j]);
        float d2 = 0;
        for (int i = 0; i < dims; ++i) { const float q = p[i]; const float d = s * q - x[i]; d2 += w[i] * d * d; }
        if (d2 < best) { best = d2; gi = list[j]; }
    }
    if (gi < 0) return -1;
    const int8_t * p = (const int8_t *) (grid + gi);
    for (int i = 0; i < dims; ++i) L[i] = (int8_t) ((p[i] - 1) / 2);
    return gi;
}

/* ------------------------------------------------------------------------------------------------ grid-trial i-quants
 * IQ2_XXS (gpuq.hip:246-387), IQ2_XS (:825-969), IQ2_S (:691-822), IQ3_XXS (:995-1143), IQ3_S (:1146-1283) share
 * one search: per sub-block, sign split, trial inverse scales, grid rounding with neighbour fallback, least-squares
 * scale, re-gridding of the groups that fell off the grid. The variants differ only in the parameters below. */
typedef struct {
    int sb, gd, bits, kmaxq, ntrial;  /* sub-block length, group dims, map bits a level, levels, trials +-ntrial */
    float step;                       /* trial step of the inverse scale */
    int sigma_x2;                     /* sigma2 = (sigma_x2 ? 2 : 1) * sumx2 / 256 */
    int parity;                       /* even-parity signs (7-bit fields) */
    float eps;                        /* sub-block skipped when max < eps; eps < 0: when max == 0 */
    int qp_first;                     /* IQ2_XXS: trial range from make_qp_quants' scale */
    int regrid_all;                   /* re-grid every group (else only the groups found off the grid) */
    int regrid_any;                   /* re-grid only if some group was off the grid (all but IQ2_XXS) */
    int init_on_grid;                 /* the groups' initial on-grid flags (IQ3_S starts with false) */
} ofam_t;

static const ofam_t FAM_IQ2_XXS = {32, 8, 2, 3, 6, 0.1f, 0, 1, 1e-15f, 1, 1, 0, 1};
static const ofam_t FAM_IQ2_XS  = {16, 8, 2, 3, 9, 0.1f, 0, 1, 1e-15f, 0, 0, 1, 1};
static const ofam_t FAM_IQ2_S   = {16, 8, 2, 3, 9, 0.1f, 1, 0, 1e-8f,  0, 0, 1, 1};
static const ofam_t FAM_IQ3_XXS = {32, 4, 3, 8, 15, 0.2f, 1, 1, 1e-8f, 0, 0, 1, 1};
static const ofam_t FAM_IQ3_S   = {32, 4, 3, 8, 9, 0.2f, 1, 0, -1.f,   0, 1, 1, 0};

typedef struct {                    /* one sub-block's outcome */
    int skipped;                    /* max below the guard: nothing written for it */
    float scale;
    int8_t L[32];
    uint8_t signs[4];               /* 8-weight sign bytes (7 bits with the parity fix) */
    int gidx[8];                    /* grid index a group */
} osub_t;

static int o_code(const int8_t * L, int gd, int bits) {
    int u = 0;
    for (int i = 0; i < gd; ++i) u |= L[i] << (bits * i);
    return u;
}

/* round x*id to levels of one group; returns the grid index (neighbour search when off the grid), -1 on failure */
static int o_group_to_grid(const ofam_t * F, const otab_t * T, const float * xv, const float * wa, float id, float s,
                           int8_t * L, int * on_grid) {
    for (int i = 0; i < F->gd; ++i) L[i] = (int8_t) imax(0, imin(F->kmaxq - 1, o_rint(0.5f * (id * xv[i] - 1))));
    const int u = o_code(L, F->gd, F->bits);
    int gi = T->map[u];
    *on_grid = gi >= 0;
    if (gi < 0) gi = o_listed_nearest(T->neigh - T->map[u] - 1, T->grid, F->gd, xv, wa, s, L);
    return gi;
}

static int o_fam_sub(const ofam_t * F, const otab_t * T, const float * xb, const float * qw, float sigma2, osub_t * o) {
    const int n = F->sb, ng = n / F->gd, nsg = n / 8;
    float w[32], wa[32], xv[32];
    int8_t Laux[32];
    int on[8], on_aux[8];
    memset(o, 0, sizeof(*o));
    for (int i = 0; i < n; ++i) w[i] = qw[i] * sqrtf(sigma2 + xb[i] * xb[i]);
    for (int i = 0; i < n; ++i) wa[i] = sqrtf(w[i]);
    for (int k = 0; k < nsg; ++k) {   /* signs of 8 weights, the parity fix flips the cheapest one (gpuq.hip:272-289) */
        int nflip = 0;
        unsigned s = 0;
        for (int i = 0; i < 8; ++i) {
            const float v = xb[8 * k + i];
            if (v >= 0) xv[8 * k + i] = v; else { xv[8 * k + i] = -v; ++nflip; s |= 1u << i; }
        }
        if (F->parity && (nflip % 2)) {
            int im = 0;
            float mn = w[8 * k] * xb[8 * k] * xb[8 * k];
            for (int i = 1; i < 8; ++i) {
                const float a = w[8 * k + i] * xb[8 * k + i] * xb[8 * k + i];
                if (a < mn) { mn = a; im = i; }
            }
            xv[8 * k + im] = -xv[8 * k + im];
            s ^= 1u << im;
        }
        o->signs[k] = (uint8_t) (F->parity ? (s & 127) : s);
    }
    float mx = xv[0];
    for (int i = 1; i < n; ++i) mx = fmaxr(mx, xv[i]);
    if (F->eps < 0 ? !mx : mx < F->eps) { o->skipped = 1; return 0; }
    float scale, denom;
    if (F->qp_first) {
        uint8_t Lq[32];
        scale = o_qp_levels(n, F->kmaxq + 1, xv, Lq, w);
        denom = scale * F->kmaxq;
        if (denom <= 0) { o->skipped = 1; return 0; }
        for (int i = 0; i < n; ++i) o->L[i] = (int8_t) Lq[i];
    } else {
        scale = mx / (2 * F->kmaxq - 1);
        denom = mx;
    }
    for (int k = 0; k < ng; ++k) on[k] = F->init_on_grid;
    float best = 0;
    for (int is = -F->ntrial; is <= F->ntrial; ++is) {
        const float id = (2 * F->kmaxq - 1 + is * F->step) / denom;
        const float ts = 1 / id;
        for (int k = 0; k < ng; ++k)
            if (o_group_to_grid(F, T, xv + F->gd * k, wa + F->gd * k, id, ts, Laux + F->gd * k, &on_aux[k]) < 0) return -1;
        float sqx = 0, sq2 = 0;
        for (int i = 0; i < n; ++i) { const float q = 2 * Laux[i] + 1; sqx += w[i] * xv[i] * q; sq2 += w[i] * q * q; }
        if (sq2 > 0 && sqx * sqx > best * sq2) {
            scale = sqx / sq2;
            best = scale * sqx;
            memcpy(o->L, Laux, n);
            memcpy(on, on_aux, sizeof(on));
        }
    }
    int n_off = 0;
    for (int k = 0; k < ng; ++k) n_off += !on[k];
    if ((F->regrid_any ? n_off > 0 : 1) && scale > 0) {
        const float id = 1 / scale;
        for (int k = 0; k < ng; ++k) {
            if (!F->regrid_all && on[k]) continue;
            int dummy;
            if (o_group_to_grid(F, T, xv + F->gd * k, wa + F->gd * k, id, scale, o->L + F->gd * k, &dummy) < 0) return -1;
        }
        float sqx = 0, sq2 = 0;
        for (int i = 0; i < n; ++i) { const float q = 2 * o->L[i] + 1; sqx += w[i] * xv[i] * q; sq2 += w[i] * q * q; }
        if (sq2 > 0) scale = sqx / sq2;
    }
    if (scale < 0) {
        scale = -scale;
        for (int k = 0; k < nsg; ++k) o->signs[k] = (uint8_t) (F->parity ? (~o->signs[k]) & 127 : ~o->signs[k]);
    }
    for (int k = 0; k < ng; ++k) {
        const int gi = T->map[o_code(o->L + F->gd * k, F->gd, F->bits)];
        if (gi < 0) return -1;
        o->gidx[k] = gi;
    }
    o->scale = scale;
    return 0;
}

static float o_sumx2(const float * x) { float s = 0; for (int i = 0; i < QK; ++i) s += x[i] * x[i]; return s; }

/* the 4-bit sub-block scale code (gpuq.hip:382-383 and its siblings) */
static int o_scale4(float id, float s) { return imax(0, imin(15, o_rint(0.5f * (id * s - 1)))); }

static int o_iq2_xxs(const float * x, const float * qw, uint8_t * y, const otab_t * T) {   /* gpuq.hip:246-387 */
    uint32_t q2[16] = {0};
    float scales[8];
    float max_scale = 0;
    const float sigma2 = o_sumx2(x) / QK;
    memset(y, 0, 66);
    for (int ib = 0; ib < 8; ++ib) {
        osub_t o;
        if (o_fam_sub(&FAM_IQ2_XXS, T, x + 32 * ib, qw + 32 * ib, sigma2, &o)) return -1;
        if (o.skipped) { scales[ib] = 0; continue; }
        for (int k = 0; k < 4; ++k) {
            q2[2 * ib] |= (uint32_t) o.gidx[k] << (8 * k);
            q2[2 * ib + 1] |= (uint32_t) o.signs[k] << (7 * k);
        }
        scales[ib] = o.scale;
        max_scale = fmaxr(max_scale, o.scale);
    }
    if (!max_scale) return 0;
    const float d = max_scale / 31;
    const uint16_t h = o_half(d);
    memcpy(y, &h, 2);
    const float id = 1 / d;
    for (int ib = 0; ib < 8; ++ib) q2[2 * ib + 1] |= (uint32_t) o_scale4(id, scales[ib]) << 28;
    memcpy(y + 2, q2, 64);
    return 0;
}

static int o_iq2_xs(const float * x, const float * qw, uint8_t * y, const otab_t * T) {    /* gpuq.hip:825-969 */
    uint16_t q2[32] = {0};
    float scales[16];
    float max_scale = 0;
    const float sigma2 = o_sumx2(x) / QK;
    memset(y, 0, 74);
    for (int ib = 0; ib < 16; ++ib) {
        osub_t o;
        if (o_fam_sub(&FAM_IQ2_XS, T, x + 16 * ib, qw + 16 * ib, sigma2, &o)) return -1;
        if (o.skipped) { scales[ib] = 0; continue; }
        for (int k = 0; k < 2; ++k) q2[2 * ib + k] = (uint16_t) (o.gidx[k] | (o.signs[k] << 9));
        scales[ib] = o.scale;
        max_scale = fmaxr(max_scale, o.scale);
    }
    if (!max_scale) return 0;
    const float d = max_scale / 31;
    const uint16_t h = o_half(d);
    memcpy(y, &h, 2);
    const float id = 1 / d;
    for (int ib = 0; ib < 16; ++ib) y[66 + ib / 2] |= (uint8_t) (o_scale4(id, scales[ib]) << (4 * (ib % 2)));
    memcpy(y + 2, q2, 64);
    return 0;
}

static int o_iq2_s(const float * x, const float * qw, uint8_t * y, const otab_t * T) {     /* gpuq.hip:691-822 */
    float scales[16];
    float max_scale = 0;
    const float sigma2 = 2 * o_sumx2(x) / QK;
    uint8_t * qs = y + 2, * qh = y + 66, * sc = y + 74;
    memset(y, 0, 82);
    for (int ib = 0; ib < 16; ++ib) {
        osub_t o;
        if (o_fam_sub(&FAM_IQ2_S, T, x + 16 * ib, qw + 16 * ib, sigma2, &o)) return -1;
        if (o.skipped) { scales[ib] = 0; continue; }
        for (int k = 0; k < 2; ++k) {
            const int i8 = 2 * ib + k;
            qs[i8] = (uint8_t) (o.gidx[k] & 255);
            qh[i8 / 4] |= (uint8_t) ((o.gidx[k] >> 8) << (2 * (i8 % 4)));
            qs[32 + i8] = o.signs[k];
        }
        scales[ib] = o.scale;
        max_scale = fmaxr(max_scale, o.scale);
    }
    if (!max_scale) return 0;
    const float d = max_scale / 31;
    const uint16_t h = o_half(d * 0.9875f);
    memcpy(y, &h, 2);
    const float id = 1 / d;
    for (int ib = 0; ib < 16; ++ib) sc[ib / 2] |= (uint8_t) (o_scale4(id, scales[ib]) << (4 * (ib % 2)));
    return 0;
}

static int o_iq3_xxs(const float * x, const float * qw, uint8_t * y, const otab_t * T) {   /* gpuq.hip:995-1143 */
    uint8_t q3[64] = {0};
    uint32_t ss[8] = {0};
    float scales[8];
    float max_scale = 0;
    const float sigma2 = 2 * o_sumx2(x) / QK;
    memset(y, 0, 98);
    for (int ib = 0; ib < 8; ++ib) {
        osub_t o;
        if (o_fam_sub(&FAM_IQ3_XXS, T, x + 32 * ib, qw + 32 * ib, sigma2, &o)) return -1;
        if (o.skipped) { scales[ib] = 0; continue; }
        for (int k = 0; k < 8; ++k) q3[8 * ib + k] = (uint8_t) o.gidx[k];
        ss[ib] = o.signs[0] | (o.signs[1] << 7) | (o.signs[2] << 14) | ((uint32_t) o.signs[3] << 21);
        scales[ib] = o.scale;
        max_scale = fmaxr(max_scale, o.scale);
    }
    if (!max_scale) return 0;
    const float d = max_scale / 31;
    const uint16_t h = o_half(d * 1.0125f);
    memcpy(y, &h, 2);
    const float id = 1 / d;
    for (int ib = 0; ib < 8; ++ib) ss[ib] |= (uint32_t) o_scale4(id, scales[ib]) << 28;
    memcpy(y + 2, q3, 64);
    memcpy(y + 66, ss, 32);
    return 0;
}

static int o_iq3_s(const float * x, const float * qw, uint8_t * y, const otab_t * T) {     /* gpuq.hip:1146-1283 */
    float scales[8];
    float max_scale = 0;
    const float sigma2 = 2 * o_sumx2(x) / QK;
    uint8_t * qs = y + 2, * qh = y + 66, * signs = y + 74, * sc = y + 106;
    memset(y, 0, 110);
    for (int ib = 0; ib < 8; ++ib) {
        osub_t o;
        if (o_fam_sub(&FAM_IQ3_S, T, x + 32 * ib, qw + 32 * ib, sigma2, &o)) return -1;
        if (o.skipped) { scales[ib] = 0; continue; }   /* qs / signs do not advance for a skipped sub-block */
        for (int k = 0; k < 8; ++k) {
            qs[k] = (uint8_t) (o.gidx[k] & 255);
            qh[(8 * ib + k) / 8] |= (uint8_t) ((o.gidx[k] >> 8) << ((8 * ib + k) % 8));
        }
        qs += 8;
        for (int k = 0; k < 4; ++k) signs[k] = o.signs[k];
        signs += 4;
        scales[ib] = o.scale;
        max_scale = fmaxr(max_scale, o.scale);
    }
    if (!max_scale) return 0;
    const float d = max_scale / 31;
    const uint16_t h = o_half(d * 1.033f);
    memcpy(y, &h, 2);
    const float id = 1 / d;
    for (int ib = 0; ib < 8; ib += 2) sc[ib / 2] = (uint8_t) (o_scale4(id, scales[ib]) | (o_scale4(id, scales[ib + 1]) << 4));
    return 0;
}

/* ------------------------------------------------------------------------------------------------ IQ1_S / IQ1_M */
/* stable ascending order of n keys (glibc qsort is a stable merge sort at these sizes; gpuq.hip:234-243) */
static void o_stable_order(const float * key, int * idx, int n) {
    float k[32];
    memcpy(k, key, n * sizeof(float));
    for (int j = 0; j < n; ++j) idx[j] = j;
    for (int i = 1; i < n; ++i) {
        const float kv = k[i];
        const int v = idx[i];
        int j = i - 1;
        while (j >= 0 && k[j] > kv) { k[j + 1] = k[j]; idx[j + 1] = idx[j]; --j; }
        k[j + 1] = kv;
        idx[j + 1] = v;
    }
}

/* nearest listed point with the shifted level values xg (iq1_find_best_neighbour2, gpuq.hip:199-232). When no
 * listed distance is finite the reference scans the whole grid reading x[i] for grid index i (ggml's own
 * indexing): that fallback reads past the 8 weights, so it is treated here as a failure (-1). */
static int o_iq1_nearest(const uint16_t * list, const uint64_t * grid, const float * x, const float * w, float s,
                         const float * xg, int8_t * L) {
    const int n = list[0];
    float best = FLT_MAX;
    int gi = -1;
    for (int j = 1; j <= n; ++j) {
        const int8_t * p = (const int8_t *) (grid + list[j]);
        float d2 = 0;
        for (int i = 0; i < 8; ++i) { const float q = xg[(p[i] - 1) / 2]; const float d = s * q - x[i]; d2 += w[i] * d * d; }
        if (d2 < best) { best = d2; gi = list[j]; }
    }
    if (gi < 0) return -1;
    const int8_t * p = (const int8_t *) (grid + gi);
    for (int i = 0; i < 8; ++i) L[i] = (int8_t) ((p[i] - 1) / 2);
    return gi;
}

static const float IQ1_XP[3] = {-1 + 0.125f, 0.125f, 1 + 0.125f};
static const float IQ1_XM[3] = {-1 - 0.125f, -0.125f, 1 - 0.125f};

static int o_iq1_s(const float * x, const float * qw, uint8_t * y, const otab_t * T) {     /* gpuq.hip:390-514 */
    float scales[8], w[32], sumx[33], sumw[33];
    int8_t L[32], shifts[8];
    int idx[32];
    uint16_t qh[8] = {0};
    uint8_t * qs = y + 2;
    float max_scale = 0;
    memset(y, 0, 50);
    const float sigma2 = 2 * o_sumx2(x) / QK;
    for (int ib = 0; ib < 8; ++ib) {
        const float * xb = x + 32 * ib;
        const float * qb = qw + 32 * ib;
        for (int i = 0; i < 32; ++i) w[i] = qb[i] * sqrtf(sigma2 + xb[i] * xb[i]);
        float mx = fabsf(xb[0]);
        for (int i = 1; i < 32; ++i) mx = fmaxr(mx, fabsf(xb[i]));
        if (mx < 1e-12f) { scales[ib] = 0; shifts[ib] = 1; continue; }
        o_stable_order(xb, idx, 32);
        sumx[0] = sumw[0] = 0;
        for (int j = 0; j < 32; ++j) { sumx[j + 1] = sumx[j] + w[idx[j]] * xb[idx[j]]; sumw[j + 1] = sumw[j] + w[idx[j]]; }
        float best = -FLT_MAX, scale = mx;
        int b1 = -1, b2 = -1, bshift = 0;
        for (int i1 = 0; i1 <= 32; ++i1) {
            for (int i2 = i1; i2 <= 32; ++i2) {
                for (int sh = 0; sh < 2; ++sh) {
                    const float * xs = sh ? IQ1_XM : IQ1_XP;
                    const float sqx = (sumx[i1] - sumx[0]) * xs[0] + (sumx[i2] - sumx[i1]) * xs[1] + (sumx[32] - sumx[i2]) * xs[2];
                    const float sq2 = (sumw[i1] - sumw[0]) * xs[0] * xs[0] + (sumw[i2] - sumw[i1]) * xs[1] * xs[1] +
                                      (sumw[32] - sumw[i2]) * xs[2] * xs[2];
                    if (sq2 > 0 && sqx * sqx > best * sq2) {
                        scale = sqx / sq2; best = scale * sqx;
                        b1 = i1; b2 = i2; bshift = sh ? -1 : 1;
                    }
                }
            }
        }
        if (b1 < 0 || b2 < 0 || !bshift) { scales[ib] = 0; shifts[ib] = 1; continue; }
        for (int j = 0; j < 32; ++j) L[idx[j]] = (int8_t) (j < b1 ? 0 : j < b2 ? 1 : 2);
        if (scale < 0) {
            for (int j = 0; j < 32; ++j) L[j] = (int8_t) (2 - L[j]);
            scale = -scale; bshift = -bshift;
        }
        const float * xx = bshift == 1 ? IQ1_XP : IQ1_XM;
        int gidx[4], all_on = 1;
        for (int k = 0; k < 4; ++k) {
            int gi = T->map[o_code(L + 8 * k, 8, 2)];
            if (gi < 0) {
                all_on = 0;
                gi = o_iq1_nearest(T->neigh - T->map[o_code(L + 8 * k, 8, 2)] - 1, T->grid, xb + 8 * k, w + 8 * k, scale, xx, L + 8 * k);
                if (gi < 0) return -1;
            }
            gidx[k] = gi;
        }
        if (!all_on) {
            float sqx = 0, sq2 = 0;
            for (int k = 0; k < 4; ++k) {
                const int8_t * p = (const int8_t *) (T->grid + gidx[k]);
                for (int j = 0; j < 8; ++j) {
                    const float ww = w[8 * k + j], q = xx[(p[j] - 1) / 2];
                    sqx += ww * q * xb[8 * k + j];
                    sq2 += ww * q * q;
                }
            }
            if (sqx > 0 && sq2 > 0) scale = sqx / sq2;
        }
        uint16_t h = 0;
        for (int k = 0; k < 4; ++k) { qs[4 * ib + k] = (uint8_t) (gidx[k] & 255); h |= (uint16_t) ((gidx[k] >> 8) << (3 * k)); }
        qh[ib] = h;
        scales[ib] = scale;
        shifts[ib] = (int8_t) bshift;
        max_scale = fmaxr(max_scale, scale);
    }
    if (max_scale) {
        const float d = max_scale / 15;
        const uint16_t hd = o_half(d * 1.125f);
        memcpy(y, &hd, 2);
        const float id = 1 / d;
        for (int ib = 0; ib < 8; ++ib) {
            int l = imax(0, imin(7, o_rint(0.5f * (id * scales[ib] - 1))));
            if (shifts[ib] == -1) l |= 8;
            qh[ib] |= (uint16_t) (l << 12);
        }
    }
    memcpy(y + 34, qh, 16);
    return 0;
}

static int o_iq1_m(const float * x, const float * qw, uint8_t * y, const otab_t * T) {     /* gpuq.hip:517-688 */
    float scales[16], w[16];
    int8_t L[16], shifts[16];
    int idx[16];
    uint8_t * qs = y, * qh = y + 32, * scb = y + 48;
    float max_scale = 0;
    memset(y, 0, 56);
    const float sigma2 = 2 * o_sumx2(x) / QK;
    for (int ib = 0; ib < 16; ++ib) {
        const float * xb = x + 16 * ib;
        const float * qb = qw + 16 * ib;
        for (int i = 0; i < 16; ++i) w[i] = qb[i] * sqrtf(sigma2 + xb[i] * xb[i]);
        float mx = fabsf(xb[0]);
        for (int i = 1; i < 16; ++i) mx = fmaxr(mx, fabsf(xb[i]));
        if (mx < 1e-7f) { scales[ib] = 0; shifts[ib] = 0; continue; }
        o_stable_order(xb, idx, 16);
        float px[2][17], pw[2][17];
        px[0][0] = px[1][0] = pw[0][0] = pw[1][0] = 0;
        for (int j = 0; j < 16; ++j) {   /* prefix sums split by half of the sub-block (gpuq.hip:559-571) */
            const int i = idx[j], h = i < 8 ? 0 : 1;
            px[h][j + 1] = px[h][j] + w[i] * xb[i];
            px[1 - h][j + 1] = px[1 - h][j];
            pw[h][j + 1] = pw[h][j] + w[i];
            pw[1 - h][j + 1] = pw[1 - h][j];
        }
        const float txs[2] = {px[0][16], px[1][16]}, tws[2] = {pw[0][16], pw[1][16]};
        const float p2 = IQ1_XP[2], m2 = IQ1_XM[2];
        const float cp1 = IQ1_XP[0] * IQ1_XP[0] - IQ1_XP[1] * IQ1_XP[1], cp2 = IQ1_XP[1] * IQ1_XP[1] - IQ1_XP[2] * IQ1_XP[2];
        const float cm1 = IQ1_XM[0] * IQ1_XM[0] - IQ1_XM[1] * IQ1_XM[1], cm2 = IQ1_XM[1] * IQ1_XM[1] - IQ1_XM[2] * IQ1_XM[2];
        float best = -FLT_MAX, scale = mx;
        int b1 = -1, b2 = -1, bk = -1;
        for (int i1 = 0; i1 <= 16; ++i1) {
            for (int i2 = i1; i2 <= 16; ++i2) {
                float qxp[2], qxm[2], q2p[2], q2m[2], sqx[4], sq2[4];
                for (int h = 0; h < 2; ++h) {
                    const float sx = px[h][i1] + px[h][i2];
                    qxp[h] = txs[h] * p2 - sx;
                    qxm[h] = txs[h] * m2 - sx;
                    q2p[h] = tws[h] * p2 * p2 + pw[h][i1] * cp1 + pw[h][i2] * cp2;
                    q2m[h] = tws[h] * m2 * m2 + pw[h][i1] * cm1 + pw[h][i2] * cm2;
                }
                sqx[0] = qxp[0] + qxp[1]; sqx[1] = qxp[0] + qxm[1]; sqx[2] = qxm[0] + qxp[1]; sqx[3] = qxm[0] + qxm[1];
                sq2[0] = q2p[0] + q2p[1]; sq2[1] = q2p[0] + q2m[1]; sq2[2] = q2m[0] + q2p[1]; sq2[3] = q2m[0] + q2m[1];
                for (int k = 0; k < 4; ++k) {
                    if (sq2[k] > 0 && sqx[k] * sqx[k] > best * sq2[k]) {
                        scale = sqx[k] / sq2[k]; best = scale * sqx[k];
                        b1 = i1; b2 = i2; bk = k;
                    }
                }
            }
        }
        if (b1 < 0 || b2 < 0 || bk < 0) { scales[ib] = 0; shifts[ib] = 0; continue; }
        for (int j = 0; j < 16; ++j) L[idx[j]] = (int8_t) (j < b1 ? 0 : j < b2 ? 1 : 2);
        if (scale < 0) {
            for (int j = 0; j < 16; ++j) L[j] = (int8_t) (2 - L[j]);
            scale = -scale;
            bk = 3 - bk;
        }
        int gidx[2], all_on = 1;
        for (int k = 0; k < 2; ++k) {
            const float * xx = k == 0 ? (bk < 2 ? IQ1_XP : IQ1_XM) : (bk % 2 == 0 ? IQ1_XP : IQ1_XM);
            const int u = o_code(L + 8 * k, 8, 2);
            int gi = T->map[u];
            if (gi < 0) {
                all_on = 0;
                gi = o_iq1_nearest(T->neigh - T->map[u] - 1, T->grid, xb + 8 * k, w + 8 * k, scale, xx, L + 8 * k);
                if (gi < 0) return -1;
            }
            gidx[k] = gi;
        }
        if (!all_on) {
            float sqx = 0, sq2 = 0;
            for (int k = 0; k < 2; ++k) {
                const float * xx = k == 0 ? (bk < 2 ? IQ1_XP : IQ1_XM) : (bk % 2 == 0 ? IQ1_XP : IQ1_XM);
                const int8_t * p = (const int8_t *) (T->grid + gidx[k]);
                for (int j = 0; j < 8; ++j) {
                    const float ww = w[8 * k + j], q = xx[(p[j] - 1) / 2];
                    sqx += ww * q * xb[8 * k + j];
                    sq2 += ww * q * q;
                }
            }
            if (sqx > 0 && sq2 > 0) scale = sqx / sq2;
        }
        qs[2 * ib] = (uint8_t) (gidx[0] & 255);
        qs[2 * ib + 1] = (uint8_t) (gidx[1] & 255);
        qh[ib] = (uint8_t) ((gidx[0] >> 8) | ((gidx[1] >> 8) << 4));
        scales[ib] = scale;
        shifts[ib] = (int8_t) bk;
        max_scale = fmaxr(max_scale, scale);
    }
    if (!max_scale) return 0;
    /* 3-bit scales, the shift bits, then the super-block scale refit over the whole block (gpuq.hip:657-687) */
    static const uint8_t masks[4] = {0x00, 0x80, 0x08, 0x88};
    uint16_t sc[4] = {0, 0, 0, 0};
    float d = max_scale / 15;
    const float id = 1 / d;
    float sqx = 0, sq2 = 0;
    for (int ib = 0; ib < 16; ++ib) {
        const int l = imax(0, imin(7, o_rint(0.5f * (id * scales[ib] - 1))));
        sc[ib / 4] |= (uint16_t) (l << (3 * (ib % 4)));
        qh[ib] |= masks[shifts[ib]];
        const float * xb = x + 16 * ib;
        const float * qb = qw + 16 * ib;
        for (int i = 0; i < 16; ++i) w[i] = qb[i] * sqrtf(sigma2 + xb[i] * xb[i]);
        for (int k = 0; k < 2; ++k) {
            const float * xx = k == 0 ? (shifts[ib] < 2 ? IQ1_XP : IQ1_XM) : (shifts[ib] % 2 == 0 ? IQ1_XP : IQ1_XM);
            const int gi = qs[2 * ib + k] + ((qh[ib] << (8 - 4 * k)) & 0x700);
            const int8_t * p = (const int8_t *) (T->grid + gi);
            for (int j = 0; j < 8; ++j) {
                const float ww = w[8 * k + j], q = xx[(p[j] - 1) / 2] * (2 * l + 1);
                sqx += ww * q * xb[8 * k + j];
                sq2 += ww * q * q;
            }
        }
    }
    if (sq2 > 0) d = sqx / sq2;
    const uint16_t s = o_half(d * 1.1125f);
    sc[0] |= (uint16_t) ((s & 0x000f) << 12);
    sc[1] |= (uint16_t) ((s & 0x00f0) << 8);
    sc[2] |= (uint16_t) ((s & 0x0f00) << 4);
    sc[3] |= (uint16_t) (s & 0xf000);
    memcpy(scb, sc, 8);
    return 0;
}

/* ------------------------------------------------------------------------------------------------ IQ4_NL / IQ4_XS */
static const int8_t IQ4_VALUES[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

/* nearest of the 16 non-linear levels (best_index_int8, gpuq.hip:1286-1295) */
static int o_iq4_index(float x) {
    if (x <= IQ4_VALUES[0]) return 0;
    if (x >= IQ4_VALUES[15]) return 15;
    int lo = 0, hi = 15;
    while (hi - lo > 1) { const int mid = (lo + hi) / 2; if (x < IQ4_VALUES[mid]) hi = mid; else lo = mid; }
    return x - IQ4_VALUES[hi - 1] < IQ4_VALUES[hi] - x ? hi - 1 : hi;
}

/* iq4_nl_impl with ntry 7 (gpuq.hip:1297-1388); sb = 32 (IQ4_NL) or 256 (IQ4_XS) */
static void o_iq4(int sb, const float * x, const float * qw, uint16_t * dh, uint8_t * q4, uint16_t * sh, uint8_t * sl) {
    float scales[8], w[32];
    uint8_t L[256];
    float sigma2 = 0;
    for (int j = 0; j < sb; ++j) sigma2 += x[j] * x[j];
    sigma2 *= 2.f / sb;
    memset(q4, 0, sb / 2);
    *dh = o_half(0.f);
    float max_scale = 0, amax_scale = 0;
    for (int ib = 0; ib < sb / 32; ++ib) {
        const float * xb = x + 32 * ib;
        uint8_t * Lb = L + 32 * ib;
        if (qw) for (int j = 0; j < 32; ++j) w[j] = qw[32 * ib + j] * sqrtf(sigma2 + xb[j] * xb[j]);
        else for (int j = 0; j < 32; ++j) w[j] = xb[j] * xb[j];
        float amax = 0, mx = 0;
        for (int j = 0; j < 32; ++j) { const float a = fabsf(xb[j]); if (a > amax) { amax = a; mx = xb[j]; } }
        if (amax < 1e-15f) { scales[ib] = 0; continue; }
        float d = -mx / IQ4_VALUES[0];
        float id = 1 / d;
        float sqx = 0, sq2 = 0;
        for (int j = 0; j < 32; ++j) {
            const int l = o_iq4_index(id * xb[j]);
            Lb[j] = (uint8_t) l;
            const float q = IQ4_VALUES[l];
            sqx += w[j] * q * xb[j];
            sq2 += w[j] * q * q;
        }
        d = sq2 > 0 ? sqx / sq2 : 0.f;
        float best = d * sqx;
        for (int t = -7; t <= 7; ++t) {
            id = (t + IQ4_VALUES[0]) / mx;
            sqx = sq2 = 0;
            for (int j = 0; j < 32; ++j) {
                const float q = IQ4_VALUES[o_iq4_index(id * xb[j])];
                sqx += w[j] * q * xb[j];
                sq2 += w[j] * q * q;
            }
            if (sq2 > 0 && sqx * sqx > best * sq2) { d = sqx / sq2; best = d * sqx; }
        }
        scales[ib] = d;
        const float ad = fabsf(d);
        if (ad > amax_scale) { amax_scale = ad; max_scale = d; }
    }
    if (sb > 32) {
        *sh = 0;
        const float d = -max_scale / 32;
        *dh = o_half(d);
        const float id = d ? 1 / d : 0.f;
        for (int ib = 0; ib < sb / 32; ++ib) {
            int l = imax(-32, imin(31, o_rint(id * scales[ib])));
            const float dl = d * l;
            const float idl = dl ? 1 / dl : 0.f;
            for (int j = 0; j < 32; ++j) L[32 * ib + j] = (uint8_t) o_iq4_index(idl * x[32 * ib + j]);
            l += 32;
            if (ib % 2 == 0) sl[ib / 2] = (uint8_t) (l & 0xf); else sl[ib / 2] |= (uint8_t) ((l & 0xf) << 4);
            *sh |= (uint16_t) ((l >> 4) << (2 * (ib % 8)));
        }
    } else {
        *dh = o_half(scales[0]);
        const float id = scales[0] ? 1 / scales[0] : 0;
        for (int j = 0; j < sb; ++j) L[j] = (uint8_t) o_iq4_index(id * x[j]);
    }
    for (int i = 0; i < sb / 32; ++i)
        for (int j = 0; j < 16; ++j) q4[16 * i + j] = (uint8_t) (L[32 * i + j] | (L[32 * i + 16 + j] << 4));
}

static int o_iq4_xs(const float * x, const float * qw, uint8_t * y) {      /* gpuq.hip:1390-1394 */
    uint16_t dh, sh = 0;
    o_iq4(256, x, qw, &dh, y + 8, &sh, y + 4);
    memcpy(y, &dh, 2);
    memcpy(y + 2, &sh, 2);
    return 0;
}
static int o_iq4_nl(const float * x, const float * qw, uint8_t * y) {      /* gpuq.hip:1395-1398 */
    uint16_t dh, sh;
    o_iq4(32, x, qw, &dh, y + 2, &sh, NULL);
    memcpy(y, &dh, 2);
    return 0;
}

/* ------------------------------------------------------------------------------------------------ k-quants, Q8_0 */
static float o_kw(const float * qw, const float * x, int i) { return qw ? qw[i] : x[i] * x[i]; }

/* signed levels -nmax..nmax-1 over 19 trial scales (sym_levels, gpuq.hip:1428-1466); L stores l + nmax */
static float o_sym(int n, int nmax, const float * x, int8_t * L, const float * qw) {
    float amax = 0, mx = 0;
    for (int i = 0; i < n; ++i) { const float a = fabsf(x[i]); if (a > amax) { amax = a; mx = x[i]; } }
    if (amax < 1e-15f) { memset(L, 0, n); return 0.f; }
    float iscale = -nmax / mx;
    float slx = 0, sl2 = 0;
    for (int i = 0; i < n; ++i) {
        const int l = imax(-nmax, imin(nmax - 1, o_rint(iscale * x[i])));
        L[i] = (int8_t) (l + nmax);
        const float w = o_kw(qw, x, i);
        slx += w * x[i] * l;
        sl2 += w * l * l;
    }
    float scale = sl2 ? slx / sl2 : 0.0f;
    float best = scale * slx;
    for (int is = -9; is <= 9; ++is) {
        if (!is) continue;
        iscale = -(nmax + 0.1f * is) / mx;
        slx = sl2 = 0;
        for (int i = 0; i < n; ++i) {
            const int l = imax(-nmax, imin(nmax - 1, o_rint(iscale * x[i])));
            const float w = o_kw(qw, x, i);
            slx += w * x[i] * l;
            sl2 += w * l * l;
        }
        if (sl2 > 0 && slx * slx > best * sl2) {
            for (int i = 0; i < n; ++i) L[i] = (int8_t) (nmax + imax(-nmax, imin(nmax - 1, o_rint(iscale * x[i]))));
            scale = slx / sl2;
            best = scale * slx;
        }
    }
    return scale;
}

/* Q3_K without imatrix: 3-bit signed levels with 5 coordinate-descent passes (sym3_levels, gpuq.hip:1469-1508) */
static float o_sym3(int n, int nmax, const float * x, int8_t * L) {
    float amax = 0, mx = 0;
    for (int i = 0; i < n; ++i) { const float a = fabsf(x[i]); if (a > amax) { amax = a; mx = x[i]; } }
    if (amax < 1e-15f) { memset(L, 0, n); return 0.f; }
    const float iscale = -nmax / mx;
    float slx = 0, sl2 = 0;
    for (int i = 0; i < n; ++i) {
        const int l = imax(-nmax, imin(nmax - 1, o_rint(iscale * x[i])));
        L[i] = (int8_t) l;
        const float w = x[i] * x[i];
        slx += w * x[i] * l;
        sl2 += w * l * l;
    }
    for (int pass = 0; pass < 5; ++pass) {
        int changed = 0;
        for (int i = 0; i < n; ++i) {
            const float w = x[i] * x[i];
            float a = slx - w * x[i] * L[i];
            if (!(a > 0)) continue;
            float b = sl2 - w * L[i] * L[i];
            const int nl = imax(-nmax, imin(nmax - 1, o_rint(x[i] * b / a)));
            if (nl == L[i]) continue;
            a += w * x[i] * nl;
            b += w * nl * nl;
            if (b > 0 && a * a * sl2 > slx * slx * b) { L[i] = (int8_t) nl; slx = a; sl2 = b; ++changed; }
        }
        if (!changed) break;
    }
    for (int i = 0; i < n; ++i) L[i] = (int8_t) (L[i] + nmax);
    return sl2 > 0.0f ? slx / sl2 : 0.0f;
}

/* affine levels 0..nmax with a min (affine_levels<with_imatrix>, gpuq.hip:1513-1587): imatrix = ggml's make_qkx3,
 * plain = make_qkx2 */
static float o_affine(int imat, int n, int nmax, const float * x, const float * wts, uint8_t * L, float * the_min,
                      uint8_t * Laux, float rmin, float rdelta, int nstep, int use_mad) {
    float mn = x[0], mx = x[0];
    float sum_w = imat ? o_kw(wts, x, 0) : wts[0];
    float sum_x = sum_w * x[0];
    for (int i = 1; i < n; ++i) {
        if (x[i] < mn) mn = x[i];
        if (x[i] > mx) mx = x[i];
        const float w = imat ? o_kw(wts, x, i) : wts[i];
        sum_w += w;
        sum_x += w * x[i];
    }
    if (mn > 0) mn = 0;
    if (imat ? mx <= mn : mx == mn) { memset(L, 0, n); *the_min = -mn; return 0.f; }
    float iscale = nmax / (mx - mn);
    float scale = 1 / iscale;
    float best = 0;
    for (int i = 0; i < n; ++i) {
        L[i] = (uint8_t) imax(0, imin(nmax, o_rint(iscale * (x[i] - mn))));
        float d = scale * L[i] + mn - x[i];
        d = use_mad ? fabsf(d) : d * d;
        best += (imat ? o_kw(wts, x, i) : wts[i]) * d;
    }
    if (nstep < 1) { *the_min = -mn; return scale; }
    for (int is = 0; is <= nstep; ++is) {
        iscale = (rmin + rdelta * is + nmax) / (mx - mn);
        float sl = 0, sl2 = 0, sxl = 0;
        for (int i = 0; i < n; ++i) {
            int l;
            if (imat) { const float v = iscale * (x[i] - mn); l = v > 0 ? o_rint(v < nmax ? v : (float) nmax) : 0; }
            else l = imax(0, imin(nmax, o_rint(iscale * (x[i] - mn))));
            Laux[i] = (uint8_t) l;
            const float w = imat ? o_kw(wts, x, i) : wts[i];
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
        for (int i = 0; i < n; ++i) {
            float d = ts * Laux[i] + tm - x[i];
            d = use_mad ? fabsf(d) : d * d;
            err += (imat ? o_kw(wts, x, i) : wts[i]) * d;
        }
        if (err < best) { memcpy(L, Laux, n); best = err; scale = ts; mn = tm; }
    }
    *the_min = -mn;
    return scale;
}

static void o_pack2(const uint8_t * L, uint8_t * qs) {   /* gpuq.hip:1590-1594 */
    for (int base = 0; base < QK; base += 128)
        for (int l = 0; l < 32; ++l)
            qs[base / 4 + l] = (uint8_t) (L[base + l] | (L[base + l + 32] << 2) | (L[base + l + 64] << 4) | (L[base + l + 96] << 6));
}

static void o_affine_round(const float * x, uint8_t * L, int g, int ng, int nmax, float d, float dmin,
                           const uint8_t * sc, const uint8_t * mn) {   /* gpuq.hip:1611-1619 */
    for (int j = 0; j < ng; ++j) {
        const float dj = d * sc[j];
        if (!dj) continue;
        const float mj = dmin * mn[j];
        for (int i = 0; i < g; ++i) L[g * j + i] = (uint8_t) imax(0, imin(nmax, o_rint((x[g * j + i] + mj) / dj)));
    }
}

static int o_q2_k(const float * x, const float * qw, uint8_t * y) {   /* gpuq.hip:1621-1668; y: scales qs d dmin */
    uint8_t L[QK], Laux[16], Ls[16], Lm[16];
    float scales[16], mins[16], w[16];
    uint8_t * ysc = y, * yqs = y + 16;
    uint16_t d16, dm16;
    if (!qw) {
        float max_scale = 0, max_min = 0;
        for (int j = 0; j < 16; ++j) {
            for (int l = 0; l < 16; ++l) w[l] = fabsf(x[16 * j + l]);
            scales[j] = o_affine(0, 16, 3, x + 16 * j, w, L + 16 * j, &mins[j], Laux, -0.5f, 0.1f, 15, 1);
            if (scales[j] > max_scale) max_scale = scales[j];
            if (mins[j] > max_min) max_min = mins[j];
        }
        memset(ysc, 0, 16);
        if (max_scale > 0) {
            const float is = 15.f / max_scale;
            for (int j = 0; j < 16; ++j) ysc[j] = (uint8_t) o_rint(is * scales[j]);
            d16 = o_half(max_scale / 15.f);
        } else d16 = o_half(0.f);
        if (max_min > 0) {
            const float im = 15.f / max_min;
            for (int j = 0; j < 16; ++j) ysc[j] |= (uint8_t) (o_rint(im * mins[j]) << 4);
            dm16 = o_half(max_min / 15.f);
        } else dm16 = o_half(0.f);
    } else {
        const float sigma2 = o_sumx2(x) / QK;
        float sw[16];
        for (int j = 0; j < 16; ++j) {
            for (int l = 0; l < 16; ++l) w[l] = qw[16 * j + l] * sqrtf(sigma2 + x[16 * j + l] * x[16 * j + l]);
            sw[j] = 0;
            for (int l = 0; l < 16; ++l) sw[j] += w[l];
            scales[j] = o_affine(1, 16, 3, x + 16 * j, w, L + 16 * j, &mins[j], Laux, -0.9f, 0.05f, 36, 0);
        }
        const float dm = o_qp_levels(16, 15, scales, Ls, sw);
        const float mm = o_qp_levels(16, 15, mins, Lm, sw);
        d16 = o_half(dm);
        dm16 = o_half(mm);
        for (int j = 0; j < 16; ++j) ysc[j] = (uint8_t) (Ls[j] | (Lm[j] << 4));
    }
    memcpy(y + 80, &d16, 2);
    memcpy(y + 82, &dm16, 2);
    uint8_t sc[16], mn[16];
    for (int j = 0; j < 16; ++j) { sc[j] = ysc[j] & 0xF; mn[j] = ysc[j] >> 4; }
    o_affine_round(x, L, 16, 16, 3, o_unhalf(d16), o_unhalf(dm16), sc, mn);
    o_pack2(L, yqs);
    return 0;
}

static int o_q3_k(const float * x, const float * qw, uint8_t * y) {   /* gpuq.hip:1670-1724; y: hmask qs scales d */
    int8_t L[QK], Ls[16];
    float scales[16];
    uint8_t * hm = y, * yqs = y + 32, * ysc = y + 96;
    uint16_t d16;
    memset(ysc, 0, 12);
    if (!qw) {
        float amax = 0, max_scale = 0;
        for (int j = 0; j < 16; ++j) {
            scales[j] = o_sym3(16, 4, x + 16 * j, L + 16 * j);
            const float a = fabsf(scales[j]);
            if (a > amax) { amax = a; max_scale = scales[j]; }
        }
        if (max_scale) {
            const float iscale = -32.f / max_scale;
            for (int j = 0; j < 16; ++j) {
                const int8_t l = (int8_t) o_rint(iscale * scales[j]);   /* narrowed to int8 before the clamp */
                Ls[j] = (int8_t) (imax(-32, imin(31, l)) + 32);
            }
            d16 = o_half(1 / iscale);
        } else {
            for (int j = 0; j < 16; ++j) Ls[j] = -1;
            d16 = o_half(0.f);
        }
    } else {
        const float sigma2 = 2 * o_sumx2(x) / QK;
        float w[16], sw[16];
        for (int j = 0; j < 16; ++j) {
            for (int l = 0; l < 16; ++l) w[l] = qw[16 * j + l] * sqrtf(sigma2 + x[16 * j + l] * x[16 * j + l]);
            float s = 0;
            for (int l = 0; l < 16; ++l) s += w[l];
            sw[j] = s;
            scales[j] = o_sym(16, 4, x + 16 * j, L + 16 * j, w);
        }
        d16 = o_half(o_sym(16, 32, scales, Ls, sw));
    }
    for (int j = 0; j < 16; ++j) {
        if (Ls[j] < 0) break;
        const int l = Ls[j];
        if (j < 8) ysc[j] = (uint8_t) (l & 0xF); else ysc[j - 8] |= (uint8_t) ((l & 0xF) << 4);
        ysc[j % 4 + 8] |= (uint8_t) ((l >> 4) << (2 * (j / 4)));
    }
    memcpy(y + 108, &d16, 2);
    const float d = o_unhalf(d16);
    for (int j = 0; j < 16; ++j) {
        int8_t sc = (int8_t) (j < 8 ? ysc[j] & 0xF : ysc[j - 8] >> 4);
        sc = (int8_t) ((sc | (((ysc[8 + j % 4] >> (2 * (j / 4))) & 3) << 4)) - 32);
        const float dj = d * sc;
        if (!dj) continue;
        for (int i = 0; i < 16; ++i) L[16 * j + i] = (int8_t) (imax(-4, imin(3, o_rint(x[16 * j + i] / dj))) + 4);
    }
    memset(hm, 0, 32);
    for (int j = 0; j < QK; ++j)
        if (L[j] > 3) { hm[j % 32] |= (uint8_t) (1 << (j / 32)); L[j] = (int8_t) (L[j] - 4); }
    o_pack2((const uint8_t *) L, yqs);
    return 0;
}

static void o_pack_k4(const uint8_t * ls, const uint8_t * lm, uint8_t * s) {   /* gpuq.hip:1597-1604 */
    for (int j = 0; j < 4; ++j) { s[j] = ls[j]; s[j + 4] = lm[j]; }
    for (int j = 4; j < 8; ++j) {
        s[j + 4] = (uint8_t) ((ls[j] & 0xF) | ((lm[j] & 0xF) << 4));
        s[j - 4] |= (uint8_t) ((ls[j] >> 4) << 6);
        s[j] |= (uint8_t) ((lm[j] >> 4) << 6);
    }
}
static void o_unpack_k4(int j, const uint8_t * s, uint8_t * sc, uint8_t * m) {   /* gpuq.hip:1605-1608 */
    if (j < 4) { *sc = s[j] & 63; *m = s[j + 4] & 63; }
    else { *sc = (uint8_t) ((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4)); *m = (uint8_t) ((s[j + 4] >> 4) | ((s[j] >> 6) << 4)); }
}

/* Q4_K / Q5_K common part (q_affine32, gpuq.hip:1727-1774); y: d dmin scales[12] ... */
static void o_affine32(int nmax, const float * x, const float * qw, uint8_t * y, uint8_t * L, float rmin_plain,
                       int nstep_plain) {
    uint8_t Laux[32], ls[8], lm[8];
    float scales[8], mins[8], w[32];
    uint16_t d16, dm16;
    if (!qw) {
        float max_scale = 0, max_min = 0;
        for (int j = 0; j < 8; ++j) {
            float s2 = 0;
            for (int l = 0; l < 32; ++l) s2 += x[32 * j + l] * x[32 * j + l];
            const float av = sqrtf(s2 / 32);
            for (int l = 0; l < 32; ++l) w[l] = av + fabsf(x[32 * j + l]);
            scales[j] = o_affine(0, 32, nmax, x + 32 * j, w, L + 32 * j, &mins[j], Laux, rmin_plain, 0.1f, nstep_plain, 0);
            if (scales[j] > max_scale) max_scale = scales[j];
            if (mins[j] > max_min) max_min = mins[j];
        }
        const float is = max_scale > 0 ? 63.f / max_scale : 0.f;
        const float im = max_min > 0 ? 63.f / max_min : 0.f;
        for (int j = 0; j < 8; ++j) {
            const uint8_t a = (uint8_t) o_rint(is * scales[j]), b = (uint8_t) o_rint(im * mins[j]);
            ls[j] = a < 63 ? a : 63;
            lm[j] = b < 63 ? b : 63;
        }
        d16 = o_half(max_scale / 63.f);
        dm16 = o_half(max_min / 63.f);
    } else {
        float s2 = 0;
        for (int l = 0; l < QK; ++l) s2 += x[l] * x[l];
        const float sigma2 = 2 * s2 / QK;
        float sw[8];
        for (int j = 0; j < 8; ++j) {
            for (int l = 0; l < 32; ++l) w[l] = qw[32 * j + l] * sqrtf(sigma2 + x[32 * j + l] * x[32 * j + l]);
            float s = 0;
            for (int l = 0; l < 32; ++l) s += w[l];
            sw[j] = s;
            scales[j] = o_affine(1, 32, nmax, x + 32 * j, w, L + 32 * j, &mins[j], Laux, -0.9f, 0.05f, 36, 0);
        }
        const float db = o_qp_levels(8, 63, scales, ls, sw);
        const float mb = o_qp_levels(8, 63, mins, lm, sw);
        if (nmax == 31) for (int j = 0; j < 8; ++j) { if (ls[j] > 63) ls[j] = 63; if (lm[j] > 63) lm[j] = 63; }
        d16 = o_half(db);
        dm16 = o_half(mb);
    }
    memcpy(y, &d16, 2);
    memcpy(y + 2, &dm16, 2);
    o_pack_k4(ls, lm, y + 4);
    uint8_t sc[8], mn[8];
    for (int j = 0; j < 8; ++j) o_unpack_k4(j, y + 4, &sc[j], &mn[j]);
    o_affine_round(x, L, 32, 8, nmax, o_unhalf(d16), o_unhalf(dm16), sc, mn);
}

static int o_q4_k(const float * x, const float * qw, uint8_t * y) {   /* gpuq.hip:1776-1781 */
    uint8_t L[QK];
    o_affine32(15, x, qw, y, L, -1.f, 20);
    for (int base = 0, o = 0; base < QK; base += 64, o += 32)
        for (int l = 0; l < 32; ++l) y[16 + o + l] = (uint8_t) (L[base + l] | (L[base + l + 32] << 4));
    return 0;
}

static int o_q5_k(const float * x, const float * qw, uint8_t * y) {   /* gpuq.hip:1783-1794; qh at 16, qs at 48 */
    uint8_t L[QK];
    o_affine32(31, x, qw, y, L, -0.5f, 15);
    uint8_t * qh = y + 16, * qs = y + 48;
    memset(qh, 0, 32);
    for (int base = 0, o = 0, bit = 0; base < QK; base += 64, o += 32, bit += 2)
        for (int j = 0; j < 32; ++j) {
            int a = L[base + j], b = L[base + j + 32];
            if (a > 15) { a -= 16; qh[j] |= (uint8_t) (1 << bit); }
            if (b > 15) { b -= 16; qh[j] |= (uint8_t) (2 << bit); }
            qs[o + j] = (uint8_t) (a | (b << 4));
        }
    return 0;
}

static int o_q6_k(const float * x, const float * qw, uint8_t * y) {   /* gpuq.hip:1796-1829; ql qh scales d */
    int8_t L[QK];
    float scales[16];
    uint8_t * ql = y, * qh = y + 128;
    int8_t * ysc = (int8_t *) (y + 192);
    float amax = 0, max_scale = 0;
    for (int b = 0; b < 16; ++b) {
        scales[b] = o_sym(16, 32, x + 16 * b, L + 16 * b, qw ? qw + 16 * b : NULL);
        const float a = fabsf(scales[b]);
        if (a > amax) { amax = a; max_scale = scales[b]; }
    }
    if (amax < 1e-15f) { memset(y, 0, 210); return 0; }
    const float iscale = -128.f / max_scale;
    const uint16_t d16 = o_half(1 / iscale);
    memcpy(y + 208, &d16, 2);
    for (int b = 0; b < 16; ++b) ysc[b] = (int8_t) imin(127, o_rint(iscale * scales[b]));
    const float d = o_unhalf(d16);
    for (int j = 0; j < 16; ++j) {
        const float dj = d * ysc[j];
        if (!dj) continue;
        for (int i = 0; i < 16; ++i) L[16 * j + i] = (int8_t) (imax(-32, imin(31, o_rint(x[16 * j + i] / dj))) + 32);
    }
    for (int half = 0; half < 2; ++half) {
        const int8_t * Lh = L + 128 * half;
        uint8_t * qlh = ql + 64 * half, * qhh = qh + 32 * half;
        for (int l = 0; l < 32; ++l) {
            qlh[l] = (uint8_t) ((Lh[l] & 0xF) | ((Lh[l + 64] & 0xF) << 4));
            qlh[l + 32] = (uint8_t) ((Lh[l + 32] & 0xF) | ((Lh[l + 96] & 0xF) << 4));
            qhh[l] = (uint8_t) ((Lh[l] >> 4) | ((Lh[l + 32] >> 4) << 2) | ((Lh[l + 64] >> 4) << 4) | ((Lh[l + 96] >> 4) << 6));
        }
    }
    return 0;
}

static int o_q8_0(const float * x, uint8_t * y) {   /* gpuq.hip:1831-1838 */
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) amax = fmaxr(amax, fabsf(x[j]));
    const float d = amax / 127;
    const float id = d ? 1.0f / d : 0.0f;
    const uint16_t h = o_half(d);
    memcpy(y, &h, 2);
    for (int j = 0; j < 32; ++j) y[2 + j] = (uint8_t) (int8_t) roundf(x[j] * id);
    return 0;
}

/* ------------------------------------------------------------------------------------------------ dispatch */
enum { O_F16 = 1, O_Q4_0 = 2, O_Q5_0 = 6, O_Q5_1 = 7 };
static int o_is_legacy(int t) { return t == O_Q4_0 || t == O_Q5_0 || t == O_Q5_1; }

static size_t o_bytes(int type) {
    switch (type) {
        case O_F16: return 2; case O_Q4_0: return 18; case O_Q5_0: return 22; case O_Q5_1: return 24;
        case O_IQ2_XXS: return 66; case O_IQ2_XS: return 74; case O_IQ2_S: return 82; case O_IQ3_XXS: return 98;
        case O_IQ3_S: return 110; case O_IQ1_S: return 50; case O_IQ1_M: return 56; case O_IQ4_NL: return 18;
        case O_IQ4_XS: return 136; case O_Q2_K: return 84; case O_Q3_K: return 110; case O_Q4_K: return 144;
        case O_Q5_K: return 176; case O_Q6_K: return 210; case O_Q8_0: return 34; default: return 0;
    }
}
static int o_len(int type) { return type == O_F16 ? 1 : type == O_IQ4_NL || type == O_Q8_0 || o_is_legacy(type) ? 32 : QK; }

/* ------------------------------------------------------------------------------------------------ Q4_0, Q5_0, Q5_1
 * llama-quantize's fallbacks for rows a k-quant or i-quant cannot hold (tools/requant_experts.py:181-183; the
 * reference runs them through ggml on the CPU). Without an imatrix ggml's quantize_row_q4_0_ref / q5_0_ref / q5_1_ref
 * (32-weight blocks; d = max/-8 or max/-16 from the value of largest magnitude, or (max - min)/31 and the min);
 * with one ggml's quantize_row_*_impl: sigma2 = the mean of x^2 over the WHOLE ROW, weights qw * sqrt(sigma2 + x^2),
 * then make_qx_quants (Q4_0: 8 levels a side, Q5_0: 16; o_sym) or make_qkx3_quants (Q5_1: 31 levels, trials
 * -0.9 + 0.05 k for k = 0..36; o_affine). Blocks: Q4_0 d qs[16]; Q5_0 d qh[4] qs[16]; Q5_1 d m qh[4] qs[16]. */
static float o_sym(int n, int nmax, const float * x, int8_t * L, const float * qw);
static float o_affine(int imat, int n, int nmax, const float * x, const float * wts, uint8_t * L, float * the_min,
                      uint8_t * Laux, float rmin, float rdelta, int nstep, int use_mad);

static void o_put_half(uint8_t * y, float f) { const uint16_t h = o_half(f); memcpy(y, &h, 2); }
static void o_pack_nibbles(const int * L, uint8_t * qs) { for (int j = 0; j < 16; ++j) qs[j] = (uint8_t) ((L[j] & 15) | ((L[j + 16] & 15) << 4)); }
static void o_pack_fifth(const int * L, uint8_t * qh) {
    uint32_t h = 0;
    for (int j = 0; j < 16; ++j) { h |= (uint32_t) ((L[j] >> 4) & 1) << j; h |= (uint32_t) ((L[j + 16] >> 4) & 1) << (j + 16); }
    memcpy(qh, &h, 4);
}

/* one 32-weight block; w = NULL: the *_ref path */
static void o_legacy_block(int type, const float * x, const float * w, uint8_t * y) {
    int L[32];
    if (type == O_Q5_1) {
        float d, m;
        if (!w) {
            float mn = FLT_MAX, mx = -FLT_MAX;
            for (int j = 0; j < 32; ++j) { if (x[j] < mn) mn = x[j]; if (x[j] > mx) mx = x[j]; }
            d = (mx - mn) / 31;
            const float id = d ? 1.0f / d : 0.0f;
            m = mn;
            for (int j = 0; j < 32; ++j) L[j] = (uint8_t) ((x[j] - mn) * id + 0.5f);
        } else {
            uint8_t Lu[32], aux[32];
            float the_min;
            d = o_affine(1, 32, 31, x, w, Lu, &the_min, aux, -0.9f, 0.05f, 36, 0);
            m = -the_min;
            for (int j = 0; j < 32; ++j) L[j] = Lu[j];
        }
        o_put_half(y, d);
        o_put_half(y + 2, m);
        o_pack_fifth(L, y + 4);
        o_pack_nibbles(L, y + 8);
        return;
    }
    const int nl = type == O_Q4_0 ? 8 : 16;
    float d;
    if (!w) {
        float amax = 0, mx = 0;
        for (int j = 0; j < 32; ++j) if (amax < fabsf(x[j])) { amax = fabsf(x[j]); mx = x[j]; }
        d = mx / -nl;
        const float id = d ? 1.0f / d : 0.0f;
        for (int j = 0; j < 32; ++j) { const int v = (int8_t) (x[j] * id + (nl + 0.5f)); L[j] = v < 2 * nl - 1 ? v : 2 * nl - 1; }
    } else {
        int8_t Ls[32];
        d = o_sym(32, nl, x, Ls, w);
        for (int j = 0; j < 32; ++j) L[j] = Ls[j];
    }
    o_put_half(y, d);
    if (type == O_Q4_0) o_pack_nibbles(L, y + 2);
    else { o_pack_fifth(L, y + 2); o_pack_nibbles(L, y + 6); }
}

/* one row of n weights (ggml's quantize_q*_0 / q5_1 call quantize_row_*_impl a row at a time) */
static void o_legacy_row(int type, const float * x, int64_t n, const float * qw, uint8_t * y) {
    float sigma2 = 0, w[32];
    if (qw) {
        float s = 0;
        for (int64_t j = 0; j < n; ++j) s += x[j] * x[j];
        sigma2 = s / n;
    }
    for (int64_t ib = 0; ib < n / 32; ++ib) {
        const float * xb = x + 32 * ib;
        if (qw) for (int j = 0; j < 32; ++j) w[j] = qw[32 * ib + j] * sqrtf(sigma2 + xb[j] * xb[j]);
        o_legacy_block(type, xb, qw ? w : NULL, y + ib * o_bytes(type));
    }
}
static int o_needs_tab(int type) {
    return type == O_IQ2_XXS || type == O_IQ2_XS || type == O_IQ2_S || type == O_IQ3_XXS || type == O_IQ3_S ||
           type == O_IQ1_S || type == O_IQ1_M;
}

static int o_block(int type, const float * x, const float * qw, uint8_t * y, const otab_t * T) {
    switch (type) {
        case O_IQ2_XXS: return o_iq2_xxs(x, qw, y, T);
        case O_IQ2_XS:  return o_iq2_xs(x, qw, y, T);
        case O_IQ2_S:   return o_iq2_s(x, qw, y, T);
        case O_IQ3_XXS: return o_iq3_xxs(x, qw, y, T);
        case O_IQ3_S:   return o_iq3_s(x, qw, y, T);
        case O_IQ1_S:   return o_iq1_s(x, qw, y, T);
        case O_IQ1_M:   return o_iq1_m(x, qw, y, T);
        case O_IQ4_XS:  return o_iq4_xs(x, qw, y);
        case O_IQ4_NL:  return o_iq4_nl(x, qw, y);
        case O_Q2_K:    return o_q2_k(x, qw, y);
        case O_Q3_K:    return o_q3_k(x, qw, y);
        case O_Q4_K:    return o_q4_k(x, qw, y);
        case O_Q5_K:    return o_q5_k(x, qw, y);
        case O_Q6_K:    return o_q6_k(x, qw, y);
        case O_Q8_0:    return o_q8_0(x, y);
        default: return -1;
    }
}

typedef struct {
    int type; const float * x; const float * qw; uint8_t * y; int64_t b0, b1, qw_mod, qw_div, qw_mat;
    const otab_t * T; int failed;
} ojob_t;

static void * o_run(void * arg) {
    ojob_t * j = (ojob_t *) arg;
    const int bs = o_len(j->type);
    const size_t bb = o_bytes(j->type);
    for (int64_t b = j->b0; b < j->b1; ++b) {
        const float * qb = j->qw ? j->qw + ((b / j->qw_mat) * j->qw_mod + (b % j->qw_mod) / j->qw_div) * bs : NULL;
        if (o_block(j->type, j->x + b * bs, qb, j->y + b * bb, j->T)) { j->failed = 1; return NULL; }
    }
    return NULL;
}

static size_t o_blocks(int type, const float * x, const float * qw, void * y, int64_t nblocks, int64_t qw_mod,
                       int64_t qw_div, int64_t qw_mat, int nthreads) {
    const otab_t * T = o_needs_tab(type) ? search_tab(type) : NULL;
    if (!o_bytes(type) || (o_needs_tab(type) && !T)) return 0;
    if (o_needs_tab(type) && !qw) return 0;   /* the search i-quants need importance weights */
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    ojob_t jobs[256];
    pthread_t th[256];
    const int64_t per = (nblocks + nthreads - 1) / nthreads;
    int nj = 0;
    for (int i = 0; i < nthreads; ++i) {
        const int64_t b0 = i * per, b1 = b0 + per < nblocks ? b0 + per : nblocks;
        if (b0 >= b1) break;
        jobs[nj] = (ojob_t){type, x, qw, (uint8_t *) y, b0, b1, qw_mod, qw_div, qw_mat, T, 0};
        ++nj;
    }
    if (nj == 1) o_run(&jobs[0]);
    else {
        for (int i = 0; i < nj; ++i) pthread_create(&th[i], NULL, o_run, &jobs[i]);
        for (int i = 0; i < nj; ++i) pthread_join(th[i], NULL);
    }
    for (int i = 0; i < nj; ++i) if (jobs[i].failed) return 0;
    return (size_t) nblocks * o_bytes(type);
}

/* ------------------------------------------------------------------------------------------------ dequantizers */
static float o_sign(uint8_t s, int j) { return (s >> j) & 1 ? -1.f : 1.f; }
static uint8_t o_ksigns(unsigned k) { return (uint8_t) (k | ((__builtin_popcount(k) & 1) << 7)); }

/* ggml's to_float of the i-quant types (gpuq.hip:1858-2021) */
static int o_dequant_block(int type, const uint8_t * q, float * y, const uint64_t * G) {
    uint16_t h;
    memcpy(&h, q, 2);
    const float d = o_unhalf(h);
    switch (type) {
    case O_IQ2_XXS:
        for (int ib = 0; ib < 8; ++ib) {
            uint32_t a[2];
            memcpy(a, q + 2 + 8 * ib, 8);
            const float db = d * (0.5f + (a[1] >> 28)) * 0.25f;
            for (int l = 0; l < 4; ++l) {
                const uint8_t * g = (const uint8_t *) (G + ((a[0] >> (8 * l)) & 255));
                const uint8_t s = o_ksigns((a[1] >> (7 * l)) & 127);
                for (int j = 0; j < 8; ++j) y[32 * ib + 8 * l + j] = db * g[j] * o_sign(s, j);
            }
        }
        return 0;
    case O_IQ2_XS:
        for (int ib = 0; ib < 8; ++ib) {
            const uint8_t sc = q[66 + ib];
            const float db[2] = {d * (0.5f + (sc & 0xf)) * 0.25f, d * (0.5f + (sc >> 4)) * 0.25f};
            for (int l = 0; l < 4; ++l) {
                uint16_t v;
                memcpy(&v, q + 2 + 2 * (4 * ib + l), 2);
                const uint8_t * g = (const uint8_t *) (G + (v & 511));
                const uint8_t s = o_ksigns(v >> 9);
                for (int j = 0; j < 8; ++j) y[32 * ib + 8 * l + j] = db[l / 2] * g[j] * o_sign(s, j);
            }
        }
        return 0;
    case O_IQ2_S:
        for (int ib = 0; ib < 8; ++ib) {
            const uint8_t sc = q[74 + ib];
            const float db[2] = {d * (0.5f + (sc & 0xf)) * 0.25f, d * (0.5f + (sc >> 4)) * 0.25f};
            for (int l = 0; l < 4; ++l) {
                const int gi = q[2 + 4 * ib + l] | ((q[66 + ib] << (8 - 2 * l)) & 0x300);
                const uint8_t * g = (const uint8_t *) (G + gi);
                const uint8_t s = q[2 + 32 + 4 * ib + l];
                for (int j = 0; j < 8; ++j) y[32 * ib + 8 * l + j] = db[l / 2] * g[j] * o_sign(s, j);
            }
        }
        return 0;
    case O_IQ3_XXS:
        for (int ib = 0; ib < 8; ++ib) {
            uint32_t a;
            memcpy(&a, q + 66 + 4 * ib, 4);
            const float db = d * (0.5f + (a >> 28)) * 0.5f;
            for (int l = 0; l < 4; ++l) {
                const uint8_t s = o_ksigns((a >> (7 * l)) & 127);
                const uint8_t * g1 = (const uint8_t *) (G + q[2 + 8 * ib + 2 * l]);
                const uint8_t * g2 = (const uint8_t *) (G + q[2 + 8 * ib + 2 * l + 1]);
                for (int j = 0; j < 4; ++j) {
                    y[32 * ib + 8 * l + j] = db * g1[j] * o_sign(s, j);
                    y[32 * ib + 8 * l + j + 4] = db * g2[j] * o_sign(s, j + 4);
                }
            }
        }
        return 0;
    case O_IQ3_S:
        for (int ib = 0; ib < 8; ++ib) {
            const uint8_t sc = q[106 + ib / 2];
            const float db = d * (1 + 2 * ((ib % 2) ? (sc >> 4) : (sc & 0xf)));
            const uint8_t hb = q[66 + ib];
            for (int l = 0; l < 4; ++l) {
                const int g1i = q[2 + 8 * ib + 2 * l] | ((hb << (8 - 2 * l)) & 256);
                const int g2i = q[2 + 8 * ib + 2 * l + 1] | ((hb << (7 - 2 * l)) & 256);
                const uint8_t * g1 = (const uint8_t *) (G + g1i), * g2 = (const uint8_t *) (G + g2i);
                const uint8_t s = q[74 + 4 * ib + l];
                for (int j = 0; j < 4; ++j) {
                    y[32 * ib + 8 * l + j] = db * g1[j] * o_sign(s, j);
                    y[32 * ib + 8 * l + j + 4] = db * g2[j] * o_sign(s, j + 4);
                }
            }
        }
        return 0;
    case O_IQ1_S:
        for (int ib = 0; ib < 8; ++ib) {
            uint16_t qh;
            memcpy(&qh, q + 34 + 2 * ib, 2);
            const float dl = d * (2 * ((qh >> 12) & 7) + 1);
            const float delta = qh & 0x8000 ? -0.125f : 0.125f;
            for (int l = 0; l < 4; ++l) {
                const int8_t * g = (const int8_t *) (G + (q[2 + 4 * ib + l] | (((qh >> (3 * l)) & 7) << 8)));
                for (int j = 0; j < 8; ++j) y[32 * ib + 8 * l + j] = dl * (g[j] + delta);
            }
        }
        return 0;
    case O_IQ1_M: {
        uint16_t sc[4];
        memcpy(sc, q + 48, 8);
        const uint16_t s16 = (uint16_t) ((sc[0] >> 12) | ((sc[1] >> 8) & 0x00f0) | ((sc[2] >> 4) & 0x0f00) | (sc[3] & 0xf000));
        const float dd = o_unhalf(s16);
        for (int ib = 0; ib < 8; ++ib) {
            const float dl1 = dd * (2 * ((sc[ib / 2] >> (6 * (ib % 2))) & 7) + 1);
            const float dl2 = dd * (2 * ((sc[ib / 2] >> (6 * (ib % 2) + 3)) & 7) + 1);
            const uint8_t * qs = q + 4 * ib, * qh = q + 32 + 2 * ib;
            const int gi[4] = {qs[0] | ((qh[0] << 8) & 0x700), qs[1] | ((qh[0] << 4) & 0x700),
                               qs[2] | ((qh[1] << 8) & 0x700), qs[3] | ((qh[1] << 4) & 0x700)};
            const float delta[4] = {qh[0] & 0x08 ? -0.125f : 0.125f, qh[0] & 0x80 ? -0.125f : 0.125f,
                                    qh[1] & 0x08 ? -0.125f : 0.125f, qh[1] & 0x80 ? -0.125f : 0.125f};
            for (int l = 0; l < 4; ++l) {
                const int8_t * g = (const int8_t *) (G + gi[l]);
                const float dl = l < 2 ? dl1 : dl2;
                for (int j = 0; j < 8; ++j) y[32 * ib + 8 * l + j] = dl * (g[j] + delta[l]);
            }
        }
        return 0;
    }
    case O_IQ4_XS: {
        uint16_t sh;
        memcpy(&sh, q + 2, 2);
        for (int ib = 0; ib < 8; ++ib) {
            const int ls = ((q[4 + ib / 2] >> (4 * (ib % 2))) & 0xf) | (((sh >> (2 * ib)) & 3) << 4);
            const float dl = d * (ls - 32);
            for (int j = 0; j < 16; ++j) {
                const uint8_t v = q[8 + 16 * ib + j];
                y[32 * ib + j] = dl * IQ4_VALUES[v & 0xf];
                y[32 * ib + j + 16] = dl * IQ4_VALUES[v >> 4];
            }
        }
        return 0;
    }
    default: return -1;
    }
}

/* ------------------------------------------------------------------------------------------------ C API */
#ifdef __cplusplus
extern "C" {
#endif
int orc_init(const char * path) {
    FILE * f = fopen(path, "rb");
    if (!f) return 2;
    for (int i = 0; i < g_ntab; ++i) { free(g_tab[i].grid); free(g_tab[i].map); free(g_tab[i].neigh); }
    g_ntab = 0;
    int32_t hdr[4];
    while (g_ntab < 16 && fread(hdr, sizeof(hdr), 1, f) == 1) {
        otab_t t = {hdr[0], hdr[1], hdr[2], hdr[3], (uint64_t *) malloc(8 * (size_t) hdr[1] + 8),
                    (int32_t *) malloc(4 * (size_t) hdr[2] + 4), (uint16_t *) malloc(2 * (size_t) hdr[3] + 2)};
        if (fread(t.grid, 8, hdr[1], f) != (size_t) hdr[1] || fread(t.map, 4, hdr[2], f) != (size_t) hdr[2] ||
            fread(t.neigh, 2, hdr[3], f) != (size_t) hdr[3]) { fclose(f); return 3; }
        g_tab[g_ntab++] = t;
    }
    fclose(f);
    return g_ntab ? 0 : 5;
}

size_t orc_block_bytes(int type) { return o_bytes(type); }
int orc_block_len(int type) { return o_len(type); }

/* nmat matrices [nrow x n_per_row]; matrix m takes imatrix row m (ggml_quantize_chunk per matrix) */
size_t orc_quantize_batch(int type, const float * x, void * y, int64_t nmat, int64_t nrow, int64_t n_per_row,
                          const float * imatrix, int nthreads) {
    const int bs = o_len(type);
    if (!o_bytes(type) || nmat <= 0 || nrow <= 0 || n_per_row % bs) return 0;
    const int64_t nb_row = n_per_row / bs, nb_mat = nrow * nb_row;
    if (type == O_F16) {   /* ggml_quantize_chunk's F16: ggml_fp32_to_fp16_row, value by value (the imatrix unused) */
        (void) nthreads;
        uint16_t * h = (uint16_t *) y;
        for (int64_t i = 0; i < nmat * nb_mat; ++i) h[i] = o_half(x[i]);
        return (size_t) nmat * nb_mat * 2;
    }
    if (o_is_legacy(type)) {   /* (row by row: the imatrix path's sigma2 is a row's) */
        (void) nthreads;
        for (int64_t r = 0; r < nmat * nrow; ++r)
            o_legacy_row(type, x + r * n_per_row, n_per_row, imatrix ? imatrix + (r / nrow) * n_per_row : NULL,
                         (uint8_t *) y + (size_t) r * nb_row * o_bytes(type));
        return (size_t) nmat * nb_mat * o_bytes(type);
    }
    const float * qw = (imatrix && type != O_Q8_0) ? imatrix : NULL;
    return o_blocks(type, x, qw, y, nmat * nb_mat, nb_row, 1, nb_mat, nthreads);
}

/* block b weighted by qw + ((b % qw_mod) / qw_div) * 256 (the device API's addressing) */
size_t orc_quantize_blocks(int type, const float * x, void * y, int64_t nblocks, const float * qw, int64_t qw_mod,
                           int64_t qw_div, int nthreads) {
    if (nblocks <= 0 || qw_mod <= 0 || qw_div <= 0) return 0;
    return o_blocks(type, x, qw, y, nblocks, qw_mod, qw_div, INT64_MAX, nthreads);
}

/* ggml's dequantize_row_q2_K .. q6_K (ggml-quants.c; the reference leaves them to ggml on the CPU): one super-block,
 * in ggml's output order and operand order. */
static void o_scale_min_k4(int j, const uint8_t * q, int * sc, int * m) {
    if (j < 4) { *sc = q[j] & 63; *m = q[j + 4] & 63; }
    else { *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4); *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4); }
}

static int o_dequant_kquant(int type, const uint8_t * x, float * y) {
    uint16_t h0, h1;
    if (type == O_Q2_K) {                       /* scales[16] qs[64] d dmin */
        memcpy(&h0, x + 80, 2); memcpy(&h1, x + 82, 2);
        const float d = o_unhalf(h0), dmin = o_unhalf(h1);
        for (int half = 0; half < 2; ++half) {
            const uint8_t * qs = x + 16 + 32 * half;
            for (int j = 0; j < 4; ++j)
                for (int part = 0; part < 2; ++part) {
                    const uint8_t sc = x[8 * half + 2 * j + part];
                    const float dl = d * (sc & 0xF), ml = dmin * (sc >> 4);
                    for (int l = 0; l < 16; ++l) *y++ = dl * ((int8_t) ((qs[16 * part + l] >> (2 * j)) & 3)) - ml;
                }
        }
        return 0;
    }
    if (type == O_Q3_K) {                       /* hmask[32] qs[64] scales[12] d */
        memcpy(&h0, x + 108, 2);
        const float d_all = o_unhalf(h0);
        int8_t scales[16];
        for (int i = 0; i < 16; ++i) {
            const uint8_t lo = x[96 + (i & 7)];
            scales[i] = (int8_t) ((i < 8 ? lo & 0xF : lo >> 4) | (((x[104 + (i & 3)] >> (2 * (i >> 2))) & 3) << 4));
        }
        for (int half = 0; half < 2; ++half) {
            const uint8_t * qs = x + 32 + 32 * half;
            for (int j = 0; j < 4; ++j) {
                const uint8_t m = (uint8_t) (1u << (4 * half + j));
                for (int part = 0; part < 2; ++part) {
                    const float dl = d_all * (scales[8 * half + 2 * j + part] - 32);
                    for (int l = 0; l < 16; ++l)
                        *y++ = dl * ((int8_t) ((qs[16 * part + l] >> (2 * j)) & 3) - ((x[16 * part + l] & m) ? 0 : 4));
                }
            }
        }
        return 0;
    }
    if (type == O_Q4_K || type == O_Q5_K) {     /* d dmin scales[12] (qh[32]) qs[128] */
        memcpy(&h0, x, 2); memcpy(&h1, x + 2, 2);
        const float d = o_unhalf(h0), dmin = o_unhalf(h1);
        const uint8_t * qs = x + (type == O_Q4_K ? 16 : 48);
        for (int c = 0; c < 4; ++c)
            for (int hi = 0; hi < 2; ++hi) {
                int sc, m;
                o_scale_min_k4(2 * c + hi, x + 4, &sc, &m);
                const float d1 = d * sc, m1 = dmin * m;
                for (int l = 0; l < 32; ++l) {
                    const int v = hi ? qs[32 * c + l] >> 4 : qs[32 * c + l] & 0xF;
                    *y++ = type == O_Q4_K ? d1 * v - m1 : d1 * (v + ((x[16 + l] >> (2 * c + hi)) & 1 ? 16 : 0)) - m1;
                }
            }
        return 0;
    }
    if (type == O_Q6_K) {                       /* ql[128] qh[64] scales[16] d */
        memcpy(&h0, x + 208, 2);
        const float d = o_unhalf(h0);
        for (int half = 0; half < 2; ++half)
            for (int qq = 0; qq < 4; ++qq)
                for (int l = 0; l < 32; ++l) {
                    const uint8_t ql = x[64 * half + 32 * (qq & 1) + l], qh = x[128 + 32 * half + l];
                    const int v = ((qq < 2 ? ql & 0xF : ql >> 4) | (((qh >> (2 * qq)) & 3) << 4)) - 32;
                    const int8_t sc = (int8_t) x[192 + 8 * half + l / 16 + 2 * qq];
                    *y++ = d * sc * (int8_t) v;
                }
        return 0;
    }
    return 1;
}

static int o_is_kquant256(int t) { return t == O_Q2_K || t == O_Q3_K || t == O_Q4_K || t == O_Q5_K || t == O_Q6_K; }

size_t orc_dequantize(int type, const void * q, float * out, int64_t nblocks) {
    if (o_is_kquant256(type)) {
        const size_t bb = o_bytes(type);
        for (int64_t b = 0; b < nblocks; ++b)
            if (o_dequant_kquant(type, (const uint8_t *) q + b * bb, out + b * QK)) return 0;
        return (size_t) nblocks * QK * 4;
    }
    const otab_t * T = dequant_tab(type);
    if (type != O_IQ4_XS && !T) return 0;
    const size_t bb = o_bytes(type);
    for (int64_t b = 0; b < nblocks; ++b)
        if (o_dequant_block(type, (const uint8_t *) q + b * bb, out + b * QK, T ? T->grid : NULL)) return 0;
    return (size_t) nblocks * QK * 4;
}

/* source bytes -> floats (kdq, gpuq.hip:2123-2141) */
/* NVFP4's scale byte (unsigned E4M3, times 0.5 - gguf-py's ue4m3_to_fp32) and an E4M3 value (the FN variant, NaN
 * read as 0 - tools/requant_table.py's e4m3_lut), from their definitions, in double then float (exact) */
static float o_ue4m3_half(uint8_t x) {
    if (x == 0 || x == 0x7F) return 0.0f;
    const int e = (x >> 3) & 0xF, m = x & 7;
    return (float) (0.5 * (e == 0 ? m * ldexp(1.0, -9) : (1.0 + m / 8.0) * ldexp(1.0, e - 7)));
}
static float o_e4m3(uint8_t x) {
    const int e = (x >> 3) & 0xF, m = x & 7;
    const double s = x & 0x80 ? -1.0 : 1.0;
    if (e == 15 && m == 7) return 0.0f;
    return (float) (e == 0 ? s * (m / 8.0) * ldexp(1.0, -6) : s * (1.0 + m / 8.0) * ldexp(1.0, e - 7));
}

static int o_is_block_src(int s) {
    return s == O_IQ2_XXS || s == O_IQ2_XS || s == O_IQ2_S || s == O_IQ3_XXS || s == O_IQ3_S || s == O_IQ1_S ||
           s == O_IQ1_M || s == O_IQ4_XS || o_is_kquant256(s);
}

size_t orc_dequantize(int type, const void * q, float * out, int64_t nblocks);

size_t orc_decode(int src, const void * raw, float * out, int64_t n) {
    static const int8_t kv[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};
    if (n <= 0 || n % 32) return 0;
    const uint8_t * r = (const uint8_t *) raw;
    if (o_is_block_src(src)) {   /* the k-quants and i-quants as sources: ggml's to_float */
        if (n % QK) return 0;
        return orc_dequantize(src, raw, out, n / QK);
    }
    if (src == 40) {             /* NVFP4: 64 values, 4 scales then 4 x 8 bytes (group j: low nibbles, then high) */
        if (n % 64) return 0;
        for (int64_t b = 0; b < n / 64; ++b) {
            const uint8_t * q = r + 36 * b;
            for (int j = 0; j < 4; ++j) {
                const float d = o_ue4m3_half(q[j]);
                for (int i = 0; i < 8; ++i) {
                    out[64 * b + 16 * j + i] = d * kv[q[4 + 8 * j + i] & 15];
                    out[64 * b + 16 * j + 8 + i] = d * kv[q[4 + 8 * j + i] >> 4];
                }
            }
        }
        return (size_t) n * 4;
    }
    if (src == 43) {             /* unsloth's MXFP8 rows: E8M0 scale 2^(e-127) (255: 0), 32 E4M3 values */
        for (int64_t b = 0; b < n / 32; ++b) {
            const uint8_t * q = r + 33 * b;
            const float sc = q[0] == 255 ? 0.0f : (float) ldexp(1.0, q[0] - 127);
            for (int j = 0; j < 32; ++j) out[32 * b + j] = o_e4m3(q[1 + j]) * sc;
        }
        return (size_t) n * 4;
    }
    for (int64_t b = 0; b < n / 32; ++b) {
        float * y = out + 32 * b;
        switch (src) {
        case O_SRC_F32: memcpy(y, r + 128 * b, 128); break;
        case O_SRC_F16: for (int j = 0; j < 32; ++j) { uint16_t h; memcpy(&h, r + 64 * b + 2 * j, 2); y[j] = o_unhalf(h); } break;
        case O_SRC_BF16: for (int j = 0; j < 32; ++j) { uint16_t h; memcpy(&h, r + 64 * b + 2 * j, 2); y[j] = u2f((uint32_t) h << 16); } break;
        case O_SRC_Q8_0: {
            const uint8_t * q = r + 34 * b;
            const float d = o_unhalf((uint16_t) (q[0] | (q[1] << 8)));
            for (int j = 0; j < 32; ++j) y[j] = (int8_t) q[2 + j] * d;
            break;
        }
        case O_SRC_MXFP4: {
            const uint8_t * q = r + 17 * b;
            const float d = u2f(q[0] < 2 ? 0x00200000u << q[0] : (uint32_t) (q[0] - 1) << 23);
            for (int j = 0; j < 16; ++j) { y[j] = kv[q[1 + j] & 15] * d; y[j + 16] = kv[q[1 + j] >> 4] * d; }
            break;
        }
        default: return 0;
        }
    }
    return (size_t) n * 4;
}
#ifdef __cplusplus
}
#endif

#ifdef ORACLE_COUNT_OPS
thread_local unsigned long long g_fops = 0, g_fcmp = 0;
extern "C" unsigned long long orc_fops(int reset) { const unsigned long long v = g_fops; if (reset) g_fops = 0; return v; }
extern "C" unsigned long long orc_fcmps(int reset) { const unsigned long long v = g_fcmp; if (reset) g_fcmp = 0; return v; }
#endif
