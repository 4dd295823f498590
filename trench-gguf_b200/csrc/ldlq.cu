// ldlq.cu - the error-feedback steps of LDLQ / GPTQ re-quantization (trench-gguf tools/ldlq.py:391-431) on sm_100a.
//
// What is computed, for step k of the 256-column block loop and every group g (the matrices that share one Hessian
// factor: an expert's gate and up, or one matrix), in the reference's arithmetic (tools/ldlq.py:427-429):
//     Es = E U_kk^-1                                                        (float64; "scale")
//     W~[:, c] = f32( W~[:, c] - f32( sum_i Es[:, i] * U[k*256 + i, c] ) )   for every column c >= (k+1)*256 ("update")
// where E = f32(W~_k - to_float(Q_k)) widened to float64 is the block's rounding error and U the upper Cholesky factor
// of the damped Hessian's inverse. U_kk^-1 is the diagonal block R_kk of the Hessian's own factor R (Hp = R R^T, U =
// R^-1), so the first product is a plain multiplication, as the second. Sums in float64, the cast and the subtraction
// in float32, as the reference's `Wp[:, :, c1:] -= (Es @ U[c0:c1, c1:]).to(float32)`.
//
// How: one float64 GEMM kernel on the tensor cores (mma.sync m8n8k4 f64: sm_100a's FP64 matrix path - tcgen05 has no
// float64 kind) with two epilogues: float64 stores (scale), or the float32 read-modify-write of W~ (update). CTA tile
// 128 rows x 64 columns, 8 warps of 32 x 32, K = 256 in chunks of 32 staged by cp.async into a two-stage ring; row
// strides padded by 4 doubles so the fragment loads of a half-warp hit 16 distinct bank pairs. One launch covers every
// group (grid z).
//
// Layouts (all device memory, row-major):
//   W~  float32 [nblk][ngroups][rows][256]  (column block major: block k of every group is one contiguous
//       [ngroups * rows, 256] slab, the quantize kernel's input)
//   E, Es  float64 [ngroups][rows][256]
//   U   float64 [ngroups][ne0][ne0] (update: the rows of block k and the columns after it are read)
//   Rd  float64 [ngroups][nblk][256][256] (scale: the diagonal blocks U_kk^-1)
#include <cstdint>
#include "common.cuh"
#include "kernels.h"

namespace gq {
namespace {

constexpr int UBM = 128, UBN = 64, UBK = 32, UTHREADS = 256, USTAGES = 2;
constexpr int BPAD = UBN + 4;   // doubles a row of the B (U) tile

// K = KD (256: a super-block; 32 or 8: the IQ2_XXS sub-block variant), staged UBK (or all of a shorter K) at a time;
// A rows padded by 4 doubles (conflict-free fragment loads for both strides)
template <int KD> struct UpdSmem {
    static constexpr int KC = KD < UBK ? KD : UBK, APAD = KC + 4;
    double a[USTAGES][UBM * APAD];
    double b[USTAGES][KC * BPAD];
};

__device__ __forceinline__ void cp_async16(void * smem, const void * gmem) {
    const unsigned s = (unsigned) __cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// D = A (8x4) * B (4x8) + D, float64; lane l holds A[l/4][l%4], B[l%4][l/4], D[l/4][2*(l%4) + {0, 1}]
__device__ __forceinline__ void dmma_8x8x4(double (&d)[2], double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};\n"
                 : "+d"(d[0]), "+d"(d[1])
                 : "d"(a), "d"(b));
}

// One tile of A [rows][KD] (group g) times B [KD][ldb] (columns n0 .. n0+63, those below ncol), float64. SUB:
// W~ -= f32(product) at columns n0.. of the column-block-major W~; else the product is stored to Out
// [ngroups][rows][KD] at columns n0..
template <bool SUB, int KD>
__global__ void __launch_bounds__(UTHREADS, 2) k_ldlq_gemm(const double * __restrict__ A, const double * __restrict__ B,
                                                           int64_t b_group_stride, int64_t ldb, int64_t n_first,
                                                           int64_t ncol, void * __restrict__ out, int64_t ngroups,
                                                           int64_t rows) {
    using SM = UpdSmem<KD>;
    constexpr int KC = SM::KC, APAD = SM::APAD;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    SM & sm = *reinterpret_cast<SM *>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int wm = warp >> 1, wn = warp & 1;             // 4 x 2 warps
    const int64_t g = blockIdx.z;
    const int64_t m0 = (int64_t) blockIdx.y * UBM;
    const int64_t n0 = n_first + (int64_t) blockIdx.x * UBN;   // first column of the tile (in B's columns)
    const double * Eg = A + g * rows * KD;
    const double * Gk = B + g * b_group_stride;

    auto load = [&](int stage, int kk) {
        // A: 128 rows x KC doubles; B: KC rows x 64 doubles (columns at or past ncol read as 0), 16-byte pieces
#pragma unroll
        for (int i = tid; i < UBM * (KC / 2); i += UTHREADS) {
            const int r = i / (KC / 2), ch = i % (KC / 2);
            double * dst = &sm.a[stage][r * APAD + ch * 2];
            if (m0 + r < rows) cp_async16(dst, Eg + (m0 + r) * KD + kk + ch * 2);
            else { dst[0] = 0.0; dst[1] = 0.0; }
        }
#pragma unroll
        for (int i = tid; i < KC * (UBN / 2); i += UTHREADS) {
            const int r = i / (UBN / 2), ch = i % (UBN / 2);
            double * dst = &sm.b[stage][r * BPAD + ch * 2];
            if (n0 + ch * 2 < ncol) cp_async16(dst, Gk + (int64_t) (kk + r) * ldb + n0 + ch * 2);
            else { dst[0] = 0.0; dst[1] = 0.0; }
        }
    };

    double acc[4][4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = 0.0;

    constexpr int NKT = KD / KC;
    load(0, 0);
    cp_commit();
#pragma unroll 1
    for (int kt = 0; kt < NKT; ++kt) {
        if (kt + 1 < NKT) {
            load((kt + 1) & 1, (kt + 1) * KC);
            cp_commit();
            cp_wait<1>();
        } else {
            cp_wait<0>();
        }
        __syncthreads();
        const double * As = sm.a[kt & 1] + (wm * 32 + (lane >> 2)) * APAD + (lane & 3);
        const double * Bs = sm.b[kt & 1] + (lane & 3) * BPAD + wn * 32 + (lane >> 2);
#pragma unroll
        for (int kq = 0; kq < KC / 4; ++kq) {
            double a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[i * 8 * APAD + kq * 4];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kq * 4 * BPAD + j * 8];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) dmma_8x8x4(acc[i][j], a[i], b[j]);
        }
        __syncthreads();
    }
    // epilogue, two adjacent columns a lane: W~ = f32(W~ - f32(acc)) (one 8-byte access), or the float64 product
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t row = m0 + wm * 32 + i * 8 + (lane >> 2);
        if (row >= rows) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t col = n0 + wn * 32 + j * 8 + (lane & 3) * 2;
            if (col >= ncol) continue;
            if constexpr (SUB) {
                const int64_t blk = col / QK, cc = col % QK;
                float2 * p = reinterpret_cast<float2 *>(static_cast<float *>(out) + ((blk * ngroups + g) * rows + row) * QK + cc);
                float2 w = *p;
                w.x = w.x - (float) acc[i][j][0];
                w.y = w.y - (float) acc[i][j][1];
                *p = w;
            } else {
                *reinterpret_cast<double2 *>(static_cast<double *>(out) + (g * rows + row) * KD + col) =
                    make_double2(acc[i][j][0], acc[i][j][1]);
            }
        }
    }
}

// C = alpha A B (+ beta C), float64 row-major (A [M][lda], B [K][ldb], C [M][ldc]), on the same tiles as
// k_ldlq_gemm with a K range per tile: TRI_NONE every k; TRI_B_LOWER B lower-triangular (B[k][n] = 0 for k < n: an
// N-tile starting at n0 needs k >= n0); TRI_A_LOWER A lower-triangular (A[m][k] = 0 for k > m: an M-tile ending at
// m1 needs k < m1). The triangular factor's own triangle is read as stored (its zeros included), so the sums are
// a full product's, in the same order, skipping only the blocks that are zero.
template <int TRI>
__global__ void __launch_bounds__(UTHREADS, 2) k_dgemm(const double * __restrict__ A, int64_t lda,
                                                       const double * __restrict__ B, int64_t ldb, double * C, int64_t ldc,
                                                       int64_t M, int64_t N, int64_t K, double alpha, double beta,
                                                       int64_t sa, int64_t sb, int64_t sc) {
    A += blockIdx.z * sa;                                 // (grid z: products of one shape at fixed strides)
    B += blockIdx.z * sb;
    C += blockIdx.z * sc;
    using SM = UpdSmem<UBK>;
    constexpr int KC = UBK, APAD = SM::APAD;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    SM & sm = *reinterpret_cast<SM *>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int wm = warp >> 1, wn = warp & 1;
    const int64_t m0 = (int64_t) blockIdx.y * UBM, n0 = (int64_t) blockIdx.x * UBN;
    int64_t k_lo = 0, k_hi = K;
    if (TRI == 1) k_lo = n0 / KC * KC;
    if (TRI == 2) k_hi = m0 + UBM < K ? m0 + UBM : K;
    const int64_t nkt = k_hi > k_lo ? (k_hi - k_lo + KC - 1) / KC : 0;

    auto load = [&](int stage, int64_t kk) {
#pragma unroll
        for (int i = tid; i < UBM * (KC / 2); i += UTHREADS) {
            const int r = i / (KC / 2), ch = i % (KC / 2);
            double * dst = &sm.a[stage][r * APAD + ch * 2];
            if (m0 + r < M && kk + ch * 2 < K) cp_async16(dst, A + (m0 + r) * lda + kk + ch * 2);
            else { dst[0] = 0.0; dst[1] = 0.0; }
        }
#pragma unroll
        for (int i = tid; i < KC * (UBN / 2); i += UTHREADS) {
            const int r = i / (UBN / 2), ch = i % (UBN / 2);
            double * dst = &sm.b[stage][r * BPAD + ch * 2];
            if (kk + r < K && n0 + ch * 2 < N) cp_async16(dst, B + (kk + r) * ldb + n0 + ch * 2);
            else { dst[0] = 0.0; dst[1] = 0.0; }
        }
    };

    double acc[4][4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = 0.0;
    if (nkt > 0) {
        load(0, k_lo);
        cp_commit();
    }
#pragma unroll 1
    for (int64_t kt = 0; kt < nkt; ++kt) {
        if (kt + 1 < nkt) {
            load((int) ((kt + 1) & 1), k_lo + (kt + 1) * KC);
            cp_commit();
            cp_wait<1>();
        } else {
            cp_wait<0>();
        }
        __syncthreads();
        const double * As = sm.a[kt & 1] + (wm * 32 + (lane >> 2)) * APAD + (lane & 3);
        const double * Bs = sm.b[kt & 1] + (lane & 3) * BPAD + wn * 32 + (lane >> 2);
#pragma unroll
        for (int kq = 0; kq < KC / 4; ++kq) {
            double a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[i * 8 * APAD + kq * 4];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kq * 4 * BPAD + j * 8];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) dmma_8x8x4(acc[i][j], a[i], b[j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t row = m0 + wm * 32 + i * 8 + (lane >> 2);
        if (row >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t col = n0 + wn * 32 + j * 8 + (lane & 3) * 2;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                if (col + h >= N) continue;
                double * c = C + row * ldc + col + h;
                *c = beta != 0.0 ? alpha * acc[i][j][h] + beta * *c : alpha * acc[i][j][h];
            }
        }
    }
}

}  // namespace

template <bool SUB, int KD>
cudaError_t launch_gemm(const double * A, const double * B, int64_t b_group_stride, int64_t ldb, int64_t n_first,
                        int64_t ncol, void * out, int64_t ngroups, int64_t rows, cudaStream_t st) {
    const size_t smem = sizeof(UpdSmem<KD>);
    const cudaError_t e = cudaFuncSetAttribute(k_ldlq_gemm<SUB, KD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (e != cudaSuccess) return e;
    const dim3 grid((unsigned) ((ncol - n_first + UBN - 1) / UBN), (unsigned) ((rows + UBM - 1) / UBM), (unsigned) ngroups);
    if (grid.y > 65535 || ngroups > 65535) return cudaErrorInvalidValue;
    k_ldlq_gemm<SUB, KD><<<grid, UTHREADS, smem, st>>>(A, B, b_group_stride, ldb, n_first, ncol, out, ngroups, rows);
    return cudaGetLastError();
}

// Es = E Rd[step] for the step-th KD x KD diagonal block (Rd: [ngroups][nsteps][KD][KD])
cudaError_t launch_ldlq_scale(const double * E, const double * Rd, double * Es, int64_t ngroups, int64_t rows,
                              int64_t nsteps, int kd, int64_t step, cudaStream_t st) {
    if (ngroups <= 0 || rows <= 0 || step < 0 || step >= nsteps) return cudaErrorInvalidValue;
    const double * B = Rd + step * (int64_t) kd * kd;
    const int64_t gs = nsteps * (int64_t) kd * kd;
    switch (kd) {
        case 256: return launch_gemm<false, 256>(E, B, gs, kd, 0, kd, Es, ngroups, rows, st);
        case 32:  return launch_gemm<false, 32>(E, B, gs, kd, 0, kd, Es, ngroups, rows, st);
        case 8:   return launch_gemm<false, 8>(E, B, gs, kd, 0, kd, Es, ngroups, rows, st);
        default: return cudaErrorInvalidValue;
    }
}

// W~[:, c] -= f32(Es U[a.., c]) for every column c >= a + kd, a = step * kd (U: [ngroups][ne0][ne0])
cudaError_t launch_ldlq_update(const double * Es, const double * U, float * W, int64_t ngroups, int64_t rows, int64_t ne0,
                               int kd, int64_t step, cudaStream_t st) {
    const int64_t a = step * kd, c1 = a + kd;
    if (ngroups <= 0 || rows <= 0 || ne0 % QK || step < 0 || c1 >= ne0) return cudaErrorInvalidValue;
    const double * B = U + a * ne0;
    switch (kd) {
        case 256: return launch_gemm<true, 256>(Es, B, ne0 * ne0, ne0, c1, ne0, W, ngroups, rows, st);
        case 32:  return launch_gemm<true, 32>(Es, B, ne0 * ne0, ne0, c1, ne0, W, ngroups, rows, st);
        case 8:   return launch_gemm<true, 8>(Es, B, ne0 * ne0, ne0, c1, ne0, W, ngroups, rows, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace gq

namespace gq {

cudaError_t launch_dgemm(int tri, const double * A, int64_t lda, const double * B, int64_t ldb, double * C, int64_t ldc,
                         int64_t M, int64_t N, int64_t K, double alpha, double beta, int64_t batch, int64_t sa,
                         int64_t sb, int64_t sc, cudaStream_t st) {
    if (M <= 0 || N <= 0 || K <= 0 || tri < 0 || tri > 2 || batch <= 0 || batch > 65535) return cudaErrorInvalidValue;
    const size_t smem = sizeof(UpdSmem<UBK>);
    const dim3 grid((unsigned) ((N + UBN - 1) / UBN), (unsigned) ((M + UBM - 1) / UBM), (unsigned) batch);
    if (grid.y > 65535) return cudaErrorInvalidValue;
    cudaError_t e = cudaSuccess;
    switch (tri) {
        case 0: e = cudaFuncSetAttribute(k_dgemm<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
                if (e == cudaSuccess)
                    k_dgemm<0><<<grid, UTHREADS, smem, st>>>(A, lda, B, ldb, C, ldc, M, N, K, alpha, beta, sa, sb, sc);
                break;
        case 1: e = cudaFuncSetAttribute(k_dgemm<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
                if (e == cudaSuccess)
                    k_dgemm<1><<<grid, UTHREADS, smem, st>>>(A, lda, B, ldb, C, ldc, M, N, K, alpha, beta, sa, sb, sc);
                break;
        default: e = cudaFuncSetAttribute(k_dgemm<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
                 if (e == cudaSuccess)
                     k_dgemm<2><<<grid, UTHREADS, smem, st>>>(A, lda, B, ldb, C, ldc, M, N, K, alpha, beta, sa, sb, sc);
                 break;
    }
    return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace gq
