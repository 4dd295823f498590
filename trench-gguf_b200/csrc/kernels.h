// kernels.h - the library's internal launch interface (host side; no torch types anywhere).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include "common.cuh"

namespace gq {

// One quantize launch: nblocks blocks of the target type from the source bytes `src` (ggml source type
// src_type: F32 / F16 / BF16 / Q8_0 / MXFP4, decoded in the kernel's loads). Block b takes the importance weights
// qw + ((b / qw_mat) * qw_mod + (b % qw_mod) / qw_div) * block_len (trench-gguf's kq addressing, gpuq.hip:1841-1847),
// or none when qw is null (k-quants, Q8_0 and IQ4_*: ggml's no-imatrix paths).
struct LaunchArgs {
    int src_type;
    const void * src;
    const float * qw;
    int64_t qw_mod, qw_div, qw_mat;
    void * out;
    int64_t nblocks;
    SearchTab tab;
    unsigned * status;
    cudaStream_t stream;
    int64_t n_per_row;   // the row length (Q4_0 / Q5_0 / Q5_1 with an imatrix scale by a whole row's mean square)
};

cudaError_t launch_iq_grid(int type, const LaunchArgs & a);   // IQ2_XXS IQ2_XS IQ2_S IQ3_XXS IQ3_S
cudaError_t launch_iq1(int type, const LaunchArgs & a);       // IQ1_S IQ1_M
cudaError_t launch_iq4(int type, const LaunchArgs & a);       // IQ4_NL IQ4_XS
cudaError_t launch_kquant(int type, const LaunchArgs & a);    // Q2_K .. Q6_K, Q8_0
cudaError_t launch_legacy(int type, const LaunchArgs & a);    // Q4_0 Q5_0 Q5_1 (whole rows: a.n_per_row)

// ggml's to_float of the i-quant types with grids and IQ4_XS: nblocks super-blocks -> nblocks*256 floats
cudaError_t launch_dequant(int type, const void * q, float * out, int64_t nblocks, DequantTab tab, cudaStream_t st);
// LDLQ block error E = blk - to_float(q), float32 maths, stored as float64 (f64) or float32
cudaError_t launch_dequant_error(int type, const void * q, const float * blk, void * err, bool f64, int64_t nblocks,
                                 DequantTab tab, cudaStream_t st);
// LDLQ's error-feedback steps (ldlq.cu), every group (matrices sharing one factor) in one launch, for feedback blocks
// of kd columns (256: super-blocks; 32 or 8: the IQ2_XXS sub-block variant), step = the block's index:
// scale Es = E Rd[step] (Rd [ngroups][ne0/kd][kd][kd] f64: U's diagonal blocks inverted), E and Es [ngroups][rows][kd];
// update W~[:, c] = f32(W~[:, c] - f32(Es U[step*kd.., c])) for c >= (step+1)*kd, W~ column-block major
// [ne0/256][ngroups][rows][256] f32, U [ngroups][ne0][ne0] f64
cudaError_t launch_ldlq_scale(const double * E, const double * Rd, double * Es, int64_t ngroups, int64_t rows,
                              int64_t nsteps, int kd, int64_t step, cudaStream_t st);
cudaError_t launch_ldlq_update(const double * Es, const double * U, float * W, int64_t ngroups, int64_t rows, int64_t ne0,
                               int kd, int64_t step, cudaStream_t st);
// the IQ2_XXS sub-block variant of LDLQ (ldlq_sub.cu): the weights qw * sqrt(sigma2 + x^2) of a super-block's rows
// (sigma2: numpy's float32 row sum of x^2 / 256; row r takes importance row r / qw_div), and the points of the groups
// in columns [c0, c0 + sub) chosen again over the whole grid (sub 32: with scale search; 8), err = x - q (float64)
cudaError_t launch_sub_weff(const float * blk, const float * qw, int64_t qw_div, float * weff, int64_t rows, cudaStream_t st);
cudaError_t launch_sub_points(const float * blk, const float * weff, uint8_t * q, double * err, int64_t rows, int sub,
                              int c0, int scale_search, const uint64_t * grid, cudaStream_t st);
// C = alpha A B (+ beta C), float64 row-major, with a triangular factor's zero blocks skipped (tri 1: B lower, 2: A
// lower), on the float64 tensor-core path (ldlq.cu)
// (batch products of the same shape, operand i at A + i sa, B + i sb, C + i sc)
cudaError_t launch_dgemm(int tri, const double * A, int64_t lda, const double * B, int64_t ldb, double * C, int64_t ldc,
                         int64_t M, int64_t N, int64_t K, double alpha, double beta, int64_t batch, int64_t sa,
                         int64_t sb, int64_t sc, cudaStream_t st);
// H += X^T X on the tensor cores (xtx.cu): X [rows][ld] float32 or bf16, optional row scale, float32-accurate sums
// added in float64 to H [dim][dim]; scratch: the bf16 parts of X laid out as tensor-core operands
int xtx_parts(int src, bool scaled);
size_t xtx_scratch_bytes(int src, int64_t rows, int64_t dim, bool scaled);
cudaError_t launch_xtx(int src, const void * x, int64_t ldx, const float * scale, int64_t rows, int64_t dim, double * H,
                       int accumulate, void * scratch, size_t scratch_bytes, unsigned * status, cudaStream_t st);
// n values of any readable source (common.cuh src_block_len) -> n floats; tab: the dequant grid of an i-quant source
cudaError_t launch_decode(int src, const void * raw, float * out, int64_t n, DequantTab tab, cudaStream_t st);
// the same, value i (of this pass; value v0 + i of the tensor) multiplied by scale[(v0 + i) / per_mat] when scale
// is not null (a per-matrix second scale, as NVFP4 experts carry)
cudaError_t launch_stage(int src, const void * raw, float * out, int64_t n, DequantTab tab, const float * scale,
                         int64_t per_mat, int64_t v0, cudaStream_t st);

// The current device's search table of `type` (from gpuq_init), or null when the device is not initialized or the
// type has no table. Implemented in api.cu.
const SearchTab * current_search_tab(int type, bool * device_ready);
// Records the reason of a failed call for gpuq_last_error(). Implemented in api.cu.
void set_last_error(const char * msg);
// Looks up gpuq_requantize_noalloc's static scratch array on device `dev` (current), loading its module at set-up.
// Implemented in noalloc.cu; gpuq_init calls it for every device it prepares.
void noalloc_prepare(int dev);

inline bool is_iq_grid(int t) { return t == IQ2_XXS || t == IQ2_XS || t == IQ2_S || t == IQ3_XXS || t == IQ3_S; }
inline bool is_iq1(int t) { return t == IQ1_S || t == IQ1_M; }
inline bool is_iq4(int t) { return t == IQ4_NL || t == IQ4_XS; }
inline bool is_kquant(int t) { return t == Q2_K || t == Q3_K || t == Q4_K || t == Q5_K || t == Q6_K || t == Q8_0; }
inline bool is_legacy(int t) { return t == Q4_0 || t == Q5_0 || t == Q5_1; }
// the types ggml also quantizes without an imatrix (k-quants' and the legacy types' *_ref paths, IQ4 with x^2 weights)
inline bool takes_no_imatrix(int t) { return is_kquant(t) || is_iq4(t) || is_legacy(t) || t == F16; }
// F16 (f16.cu): ggml's float -> half of every value (a.nblocks values; any count for F32/F16/BF16 sources)
cudaError_t launch_f16(const LaunchArgs & a);
inline bool needs_search_tab(int t) { return is_iq_grid(t) || is_iq1(t); }

inline cudaError_t launch_quantize(int type, const LaunchArgs & a) {
    if (is_iq_grid(type)) return launch_iq_grid(type, a);
    if (is_iq1(type)) return launch_iq1(type, a);
    if (is_iq4(type)) return launch_iq4(type, a);
    if (is_kquant(type)) return launch_kquant(type, a);
    if (is_legacy(type)) return launch_legacy(type, a);
    if (type == F16) return launch_f16(a);
    return cudaErrorInvalidValue;
}

}  // namespace gq
