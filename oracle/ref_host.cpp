// oracle/ref_host.cpp - TEST INFRASTRUCTURE ONLY (never linked into the product library).
//
// Builds trench-gguf's own per-block quantizers, dequantizers and source decoder (gpuq/gpuq.hip, extracted into
// oracle/_ref/gpuq_ref_body.inc by extract_ref.sh) as host C++, so the reference's arithmetic runs on the CPU:
// it pins the C restatement in oracle/oracle.c and serves as the timed CPU baseline of bench.py ("kind":
// "reference"). Compiled with -ffp-contract=off -fno-fast-math like ggml-base (no FMA), so the float results equal
// what the reference's GPU build (-fmad=false -prec-div=true -prec-sqrt=true) and ggml compute.
//
// The device-only spellings are mapped to host code by the shim below; the kernels kq / kdqq / kdq (gpuq.hip:1840,
// 2023, 2123) are called once per block with blockIdx.x = block, so the reference's own imatrix addressing runs.
// The reference's __trap() on impossible states (GPUQ_TRAP, gpuq.hip:82-86) becomes a C++ exception: the call
// returns 0 and ref_last_trap() names the block.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <thread>
#include <vector>
#include <atomic>

namespace refshim {
struct Dim3 { unsigned x = 0, y = 0, z = 0; };
struct Trap : std::exception {};
}
static thread_local refshim::Dim3 blockIdx, blockDim, threadIdx;
static inline uint32_t __float_as_uint(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
static inline float __uint_as_float(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
static inline int __float_as_int(float f) { int i; std::memcpy(&i, &f, 4); return i; }
static inline int __popc(uint32_t v) { return __builtin_popcount(v); }
[[noreturn]] static void ref_trap() { throw refshim::Trap(); }
#define __device__
#define __host__
#define __global__ static inline
#define __constant__ static const
#define __builtin_trap() ref_trap()

#include "_ref/gpuq_ref_body.inc"

#undef __builtin_trap

namespace {
struct HostTab { int type; std::vector<uint64_t> grid; std::vector<int32_t> map; std::vector<uint16_t> neigh; };
std::vector<HostTab> g_tabs;
std::atomic<long long> g_trap_block{-1};

const HostTab * find_tab(int want) {
    for (auto & t : g_tabs) if (t.type == want) return &t;
    return nullptr;
}
Tab tab_for_type(int type) {           // as gpuq.hip:2051-2056
    if (type == T_IQ4_NL || type == T_IQ4_XS) return Tab{nullptr, nullptr, nullptr};
    const HostTab * t = find_tab(type == T_IQ1_M ? T_IQ1_S : type);
    return t ? Tab{t->grid.data(), t->map.data(), t->neigh.data()} : Tab{nullptr, nullptr, nullptr};
}
DqTab dq_for_type(int type) {          // as gpuq.hip:2045-2049
    const HostTab * t = find_tab(1000 + (type == T_IQ1_M ? T_IQ1_S : type));
    return DqTab{t ? t->grid.data() : nullptr};
}
size_t bbytes(int type) {
    switch (type) {
        case T_IQ2_XXS: return sizeof(block_iq2_xxs); case T_IQ2_S: return sizeof(block_iq2_s);
        case T_IQ1_S: return sizeof(block_iq1_s); case T_IQ1_M: return sizeof(block_iq1_m);
        case T_IQ2_XS: return sizeof(block_iq2_xs); case T_IQ3_XXS: return sizeof(block_iq3_xxs);
        case T_IQ3_S: return sizeof(block_iq3_s); case T_IQ4_NL: return sizeof(block_iq4_nl);
        case T_IQ4_XS: return sizeof(block_iq4_xs); case T_Q2_K: return sizeof(block_q2_K);
        case T_Q3_K: return sizeof(block_q3_K); case T_Q4_K: return sizeof(block_q4_K);
        case T_Q5_K: return sizeof(block_q5_K); case T_Q6_K: return sizeof(block_q6_K);
        case T_Q8_0: return sizeof(block_q8_0); default: return 0;
    }
}
int blen(int type) { return type == T_IQ4_NL || type == T_Q8_0 ? 32 : QK_K; }

// one block b through the reference kernel kq<> (gpuq.hip:1840-1848)
template <typename B, void (*Q)(const float *, const float *, B *, Tab), int BS = QK_K>
void run_kq(const float * x, const float * qw, void * y, int64_t b0, int64_t b1, int64_t nblocks, int64_t qw_mod,
            int64_t qw_div, Tab t, int64_t qw_mat) {
    blockDim.x = 1; threadIdx.x = 0;
    for (int64_t b = b0; b < b1; ++b) {
        blockIdx.x = (unsigned) b;
        if ((int64_t) blockIdx.x != b) {   // (kq's blockIdx is 32-bit: shift the pointers instead)
            blockIdx.x = 0;
            const float * xb = x + b * BS;
            B * yb = (B *) y + b;
            const float * qb = qw ? qw + ((b / qw_mat) * qw_mod + (b % qw_mod) / qw_div) * BS : nullptr;
            Q(xb, qb, yb, t);
            continue;
        }
        try {
            kq<B, Q, BS>(x, qw, (B *) y, nblocks, qw_mod, qw_div, t, qw_mat);
        } catch (const refshim::Trap &) {
            long long e = -1;
            g_trap_block.compare_exchange_strong(e, (long long) b);
            return;
        }
    }
}

bool dispatch(int type, const float * x, const float * qw, void * y, int64_t b0, int64_t b1, int64_t nblocks,
              int64_t qw_mod, int64_t qw_div, int64_t qw_mat) {
    const Tab t = tab_for_type(type);
#define RQ(B, F, ...) run_kq<B, F, ##__VA_ARGS__>(x, qw, y, b0, b1, nblocks, qw_mod, qw_div, t, qw_mat)
    switch (type) {
        case T_IQ2_XXS: RQ(block_iq2_xxs, q_iq2_xxs); break;
        case T_IQ2_S:   RQ(block_iq2_s,   q_iq2_s  ); break;
        case T_IQ1_S:   RQ(block_iq1_s,   q_iq1_s  ); break;
        case T_IQ1_M:   RQ(block_iq1_m,   q_iq1_m  ); break;
        case T_IQ2_XS:  RQ(block_iq2_xs,  q_iq2_xs ); break;
        case T_IQ3_XXS: RQ(block_iq3_xxs, q_iq3_xxs); break;
        case T_IQ3_S:   RQ(block_iq3_s,   q_iq3_s  ); break;
        case T_IQ4_XS:  RQ(block_iq4_xs,  q_iq4_xs ); break;
        case T_IQ4_NL:  RQ(block_iq4_nl,  q_iq4_nl, QK4_NL); break;
        case T_Q2_K:    RQ(block_q2_K,    q_q2_k   ); break;
        case T_Q3_K:    RQ(block_q3_K,    q_q3_k   ); break;
        case T_Q4_K:    RQ(block_q4_K,    q_q4_k   ); break;
        case T_Q5_K:    RQ(block_q5_K,    q_q5_k   ); break;
        case T_Q6_K:    RQ(block_q6_K,    q_q6_k   ); break;
        case T_Q8_0:    RQ(block_q8_0,    q_q8_0, 32); break;
        default: return false;
    }
#undef RQ
    return true;
}

size_t run_blocks(int type, const float * x, const float * qw, void * y, int64_t nblocks, int64_t qw_mod,
                  int64_t qw_div, int64_t qw_mat, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    g_trap_block = -1;
    if (nthreads == 1 || nblocks < 64) {
        if (!dispatch(type, x, qw, y, 0, nblocks, nblocks, qw_mod, qw_div, qw_mat)) return 0;
    } else {
        std::vector<std::thread> th;
        const int64_t per = (nblocks + nthreads - 1) / nthreads;
        for (int i = 0; i < nthreads; ++i) {
            const int64_t b0 = i * per, b1 = std::min<int64_t>(nblocks, b0 + per);
            if (b0 >= b1) break;
            th.emplace_back([=] { dispatch(type, x, qw, y, b0, b1, nblocks, qw_mod, qw_div, qw_mat); });
        }
        for (auto & t : th) t.join();
    }
    return g_trap_block >= 0 ? 0 : (size_t) nblocks * bbytes(type);
}
}  // namespace

extern "C" {

// the tables file (gpuq_tables.bin record format, gpuq_tables.c:5-8); 0 on success
int ref_init(const char * path) {
    FILE * f = std::fopen(path, "rb");
    if (!f) return 2;
    g_tabs.clear();
    int32_t hdr[4];
    while (std::fread(hdr, sizeof(hdr), 1, f) == 1) {
        HostTab t{hdr[0], std::vector<uint64_t>(hdr[1]), std::vector<int32_t>(hdr[2]), std::vector<uint16_t>(hdr[3])};
        if (std::fread(t.grid.data(), 8, hdr[1], f) != (size_t) hdr[1] ||
            std::fread(t.map.data(), 4, hdr[2], f) != (size_t) hdr[2] ||
            std::fread(t.neigh.data(), 2, hdr[3], f) != (size_t) hdr[3]) { std::fclose(f); return 3; }
        g_tabs.push_back(std::move(t));
    }
    std::fclose(f);
    return g_tabs.empty() ? 5 : 0;
}

size_t ref_block_bytes(int type) { return bbytes(type); }
int ref_block_len(int type) { return blen(type); }
long long ref_last_trap(void) { return g_trap_block.load(); }

// nmat matrices [nrow x n_per_row] -> dst; matrix m weighted by imatrix row m (or no imatrix): the addressing of
// quantize_gx (gpuq.hip:2166-2180)
size_t ref_quantize_batch(int type, const float * x, void * y, int64_t nmat, int64_t nrow, int64_t n_per_row,
                          const float * imatrix, int nthreads) {
    const size_t bb = bbytes(type);
    const int bs = blen(type);
    if (!bb || nmat <= 0 || nrow <= 0 || n_per_row % bs) return 0;
    const int64_t nb_row = n_per_row / bs, nb_mat = nrow * nb_row;
    const float * qw = (imatrix && type != T_Q8_0) ? imatrix : nullptr;
    return run_blocks(type, x, qw, y, nmat * nb_mat, nb_row, 1, nb_mat, nthreads);
}

// block b weighted by qw + ((b % qw_mod) / qw_div) * 256: the addressing of gpuq_quantize_dev (gpuq.hip:2283-2289)
size_t ref_quantize_blocks(int type, const float * x, void * y, int64_t nblocks, const float * qw, int64_t qw_mod,
                           int64_t qw_div, int nthreads) {
    if (!bbytes(type) || nblocks <= 0 || qw_mod <= 0 || qw_div <= 0) return 0;
    return run_blocks(type, x, qw, y, nblocks, qw_mod, qw_div, INT64_MAX, nthreads);
}

// ggml's to_float of the i-quant types (gpuq.hip:1850-2028)
size_t ref_dequantize(int type, const void * q, float * out, int64_t nblocks) {
    const DqTab t = dq_for_type(type);
    if (type != T_IQ4_XS && !t.grid) return 0;
    blockDim.x = 1; threadIdx.x = 0;
    for (int64_t b = 0; b < nblocks; ++b) {
        const uint8_t * qb = (const uint8_t *) q + b * bbytes(type);
        float * ob = out + b * QK_K;
        switch (type) {
            case T_IQ2_XXS: dq_iq2_xxs((const block_iq2_xxs *) qb, ob, t); break;
            case T_IQ2_XS:  dq_iq2_xs((const block_iq2_xs *) qb, ob, t); break;
            case T_IQ2_S:   dq_iq2_s((const block_iq2_s *) qb, ob, t); break;
            case T_IQ3_XXS: dq_iq3_xxs((const block_iq3_xxs *) qb, ob, t); break;
            case T_IQ3_S:   dq_iq3_s((const block_iq3_s *) qb, ob, t); break;
            case T_IQ1_S:   dq_iq1_s((const block_iq1_s *) qb, ob, t); break;
            case T_IQ1_M:   dq_iq1_m((const block_iq1_m *) qb, ob, t); break;
            case T_IQ4_XS:  dq_iq4_xs((const block_iq4_xs *) qb, ob, t); break;
            default: return 0;
        }
    }
    return (size_t) nblocks * QK_K * 4;
}

// source bytes (F32/F16/BF16/Q8_0/MXFP4) -> floats through kdq (gpuq.hip:2123-2141)
size_t ref_decode(int src, const void * raw, float * out, int64_t n) {
    if (n <= 0 || n % 32) return 0;
    if (src != S_F32 && src != S_F16 && src != S_BF16 && src != S_Q8_0 && src != S_MXFP4) return 0;
    blockDim.x = 1; threadIdx.x = 0;
    for (int64_t b = 0; b < n / 32; ++b) {
        if ((int64_t) (unsigned) b != b) return 0;
        blockIdx.x = (unsigned) b;
        kdq(src, (const uint8_t *) raw, out, n);
    }
    return (size_t) n * 4;
}
}
