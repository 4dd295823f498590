/* include/gpuq.h - C ABI of libgpuq_cuda.so, the B200 (sm_100a) quantizer library.
 *
 * A drop-in replacement for trench-gguf's gpuq library: the first twelve entry points have the signatures, argument
 * meaning and return conventions of trench-gguf gpuq/gpuq.hip (cited per entry), so its ctypes callers
 * (tools/requant_experts.py, tools/convert_hf.py, tools/requant_table.py, tools/ldlq.py, gpuq/test_gpuq.py) load it
 * unchanged through GPUQ_LIB / GPUQ_DIR. Outputs are byte-identical to ggml_quantize_chunk / ggml's to_float.
 *
 * Types (ggml type ids): IQ2_XXS 16, IQ2_XS 17, IQ3_XXS 18, IQ1_S 19, IQ4_NL 20, IQ3_S 21, IQ2_S 22, IQ4_XS 23,
 * IQ1_M 29, Q8_0 8, Q2_K 10, Q3_K 11, Q4_K 12, Q5_K 13, Q6_K 14. Sources: F32 0, F16 1, Q8_0 8, BF16 30, MXFP4 39.
 *
 * Errors: the init functions return a non-zero code, every other entry returns 0 bytes; gpuq_last_error() then
 * says why (an extension). Nothing traps the GPU: impossible search states are reported through gpuq_status().
 */
#ifndef GPUQ_H
#define GPUQ_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Reads the tables file (trench-gguf gpuq_tables.bin format) and prepares device `device`, which becomes the
 * current device and the one the host API uses. 0 ok; 1 no such device, 2 cannot open, 3 short or corrupt file,
 * 4 allocation failed, 5 no tables. The device state it builds lasts until exit; a device reset (cudaDeviceReset)
 * invalidates it. Replaces gpuq_init, gpuq/gpuq.hip:2059-2080. */
int gpuq_init(const char * tables, int device);

/* Bytes of one block of `type`, 0 for a type this library does not produce. Replaces gpuq.hip:2082-2101. Beyond the
 * reference's types: Q4_0, Q5_0, Q5_1 (32-value blocks) and F16 (type 1, "blocks" of one value, 2 bytes: ggml's
 * float -> half of every value, the fallback trench-gguf writes for rows that are not a multiple of 32). */
size_t gpuq_block_bytes(int type);

/* 1 when gpuq_quantize* takes `type` with (with_imatrix = 1) or without (0) an importance matrix.
 * Replaces gpuq.hip:2213-2215. */
int gpuq_can_quantize(int type, int with_imatrix);

/* nrow x n_per_row float32 host weights -> host bytes; imatrix: n_per_row weights or NULL (k-quants, Q8_0, IQ4_*).
 * Returns the bytes written, 0 on error. Replaces gpuq.hip:2228-2232. */
size_t gpuq_quantize(int type, const float * src, void * dst, int64_t nrow, int64_t n_per_row, const float * imatrix);

/* nmat matrices of nrow x n_per_row; matrix m weighted by imatrix row m (imatrix: nmat x n_per_row or NULL).
 * Replaces gpuq.hip:2217-2226. */
size_t gpuq_quantize_batch(int type, const float * src, void * dst, int64_t nmat, int64_t nrow, int64_t n_per_row,
                           const float * imatrix);

/* 1 when the source type can be decoded on the GPU. Replaces gpuq.hip:2235, which reads F32, F16, BF16, Q8_0 and
 * MXFP4; this library also reads NVFP4 (40), the MXFP8 row layout of unsloth's type 43 (33-byte blocks: an E8M0
 * scale byte and 32 E4M3 values, tools/requant_table.py:8-9), and the k-quant and i-quant types that
 * gpuq_can_dequantize_type reports (the reference's callers then leave their "(gpu quant, cpu dequant)" path).
 * The first five are decoded inside the quantize kernels; the others by a decode pass of their own. */
int gpuq_can_dequantize(int src);

/* Source tensor bytes of ggml type `src` (host) -> quantized `type` (host), decoded on the GPU.
 * Replaces gpuq.hip:2252-2255. */
size_t gpuq_requantize(int src, const void * raw, int type, void * dst, int64_t nrow, int64_t n_per_row,
                       const float * imatrix);

/* The batched form: nmat matrices, matrix m weighted by imatrix row m; n_per_row a multiple of the source's block
 * (32 values; NVFP4 64; k-/i-quant sources 256) - any length for the F16 target from F32, F16 or BF16 sources.
 * Replaces gpuq.hip:2237-2250. */
size_t gpuq_requantize_batch(int src, const void * raw, int type, void * dst, int64_t nmat, int64_t nrow,
                             int64_t n_per_row, const float * imatrix);

/* gpuq_requantize_batch with a second scale a matrix: matrix m's decoded values are multiplied by mat_scale[m] in
 * float32 before quantizing (no counterpart in the reference's library: its callers fold NVFP4 experts' per-expert
 * scale into CPU-decoded floats, `f32 *= esc[e]`, tools/requant_experts.py:240-248, 704-706; this is the same product
 * after the GPU's decode). mat_scale: nmat floats (host). */
size_t gpuq_requantize_scaled_batch(int src, const void * raw, int type, void * dst, int64_t nmat, int64_t nrow,
                                    int64_t n_per_row, const float * imatrix, const float * mat_scale);

/* Device API: nblocks contiguous 256-weight super-blocks of d_x (float32, device) -> d_dst (device); block b takes
 * the 256 importance weights d_qw + ((b % qw_mod) / qw_div) * 256. The 256-block i-quants, as the reference, and
 * the k-quants Q2_K..Q6_K (an extension: d_qw may then be NULL for ggml's no-imatrix path); not IQ4_NL or Q8_0.
 * On `stream` (a cudaStream_t), no synchronisation. Returns nblocks * block bytes, 0 on a bad argument or launch
 * error. Replaces gpuq_quantize_dev, gpuq.hip:2279-2289. */
size_t gpuq_quantize_dev(int type, const float * d_x, void * d_dst, int64_t nblocks, const float * d_qw,
                         int64_t qw_mod, int64_t qw_div, void * stream);

/* 1 when gpuq_dequantize_dev decodes `type`: the seven grid i-quants and IQ4_XS (as the reference), and the k-quants
 * Q2_K..Q6_K (an extension: the reference's LDLQ callers then keep those types on the GPU too, GpuQuant.supported,
 * tools/ldlq.py:352-354). Replaces gpuq.hip:2291-2299. */
int gpuq_can_dequantize_type(int type);

/* ggml's to_float on the device: nblocks super-blocks -> nblocks * 256 floats, bit for bit.
 * Replaces gpuq.hip:2301-2320. */
size_t gpuq_dequantize_dev(int type, const void * d_q, float * d_out, int64_t nblocks, void * stream);

/* n values of source type `src` (device bytes) -> n floats (device); n a multiple of 32 and of the source's block
 * (every source gpuq_can_dequantize reports). Replaces gpuq.hip:2322-2328. */
size_t gpuq_dequantize_src_dev(int src, const void * d_raw, float * d_out, int64_t n, void * stream);

/* ---- extensions (no counterpart in the reference; callers find them with hasattr) ---- */

/* Why the last call on this thread failed (empty if it did not). */
const char * gpuq_last_error(void);

/* The current device's status word: bit 0 a neighbour search found no finite candidate, bit 1 a final code fell
 * off the grid (ggml would trap; both mean non-finite input), bit 2 an input the kernel refused, bit 3 a bounded wait
 * inside a kernel (TMA copies, tensor-core products) ran out. reset != 0 clears it. Synchronises the device. */
unsigned gpuq_status(int reset);

/* gpuq_init on several devices: the host API then shards every call over them (whole matrices - experts - or row
 * ranges of one matrix, contiguous slices of the output, no collective), one host thread a device.
 * Same return codes as gpuq_init; devices[0] becomes the current device. */
int gpuq_init_devices(const char * tables, const int * devices, int ndev);

/* How many devices the host API shards over (0 before gpuq_init). */
int gpuq_device_count(void);

/* The device-pointer form of gpuq_requantize_batch: source bytes of type `src` already on the current device ->
 * d_dst, matrix m weighted by d_imatrix row m (nmat x n_per_row floats, device; NULL for the no-imatrix types).
 * Decodes inside the quantize kernel, so the sources are the five it reads (F32, F16, BF16, Q8_0, MXFP4; others:
 * gpuq_dequantize_src_dev first); on `stream`, no synchronisation, no library scratch. d_dst must hold
 * nmat * nrow * n_per_row / block_len * gpuq_block_bytes(type) bytes, block_len being 1 for F16, 32 for Q8_0,
 * IQ4_NL, Q4_0, Q5_0 and Q5_1, and 256 for every other type: the kernel writes them all and cannot see the
 * allocation. The value count is a multiple of 32, except for the F16 target from an F32, F16 or BF16 source. */
size_t gpuq_requantize_dev(int src, const void * d_raw, int type, void * d_dst, int64_t nmat, int64_t nrow,
                           int64_t n_per_row, const float * d_imatrix, void * stream);

/* LDLQ's block error on the device: E = blk - to_float(d_q) for nblocks super-blocks of `type`, computed in float32
 * (ggml's to_float, bit for bit) and stored as float64 (f64 != 0) or float32, as tools/ldlq.py:427 forms it from
 * gpuq_dequantize_dev. d_blk: nblocks x 256 floats. Returns the bytes written to d_err, 0 on error. */
size_t gpuq_dequantize_error_dev(int type, const void * d_q, const float * d_blk, void * d_err, int f64, int64_t nblocks,
                                 void * stream);

/* LDLQ's error feedback on the device, in two calls (no counterpart as calls in the reference: they are
 * tools/ldlq.py:428-429, `Es = E U_BB^-1; Wp[:, :, c1:] -= (Es @ U[c0:c1, c1:]).to(float32)`, as this library's own
 * float64 tensor-core kernels, every group in one launch), for a feedback block of kdim columns (256: a super-block;
 * 32 or 8: the IQ2_XXS sub-block variant, tools/ldlq.py:262-266), block `step` = columns [step*kdim, (step+1)*kdim).
 * A group is the matrices that share one Hessian factor (an expert's gate and up, or one matrix), `rows` their rows.
 * gpuq_ldlq_scale_dev:  Es = E Rd[step], float64 (Rd: the inverses of U's kdim x kdim diagonal blocks)
 *   d_err, d_es: float64 [ngroups][rows][kdim]; d_rd: float64 [ngroups][nsteps][kdim][kdim]. Returns bytes of d_es.
 * gpuq_ldlq_update_dev: for every column c >= (step+1)*kdim: W[c] = f32(W[c] - f32(sum_i Es[i] * U[step*kdim+i][c]))
 *   (float64 sum, float32 cast and subtraction); d_w: float32 [ne0/256][ngroups][rows][256] (column-block major),
 *   d_u: float64 [ngroups][ne0][ne0]. Returns the bytes of d_w updated.
 * Float64 arrays 16-byte aligned; on `stream`, no synchronisation; 0 on a bad argument. */
size_t gpuq_ldlq_scale_dev(const double * d_err, const double * d_rd, double * d_es, int64_t ngroups, int64_t rows,
                           int64_t nsteps, int64_t kdim, int64_t step, void * stream);
size_t gpuq_ldlq_update_dev(const double * d_es, const double * d_u, float * d_w, int64_t ngroups, int64_t rows,
                            int64_t ne0, int64_t kdim, int64_t step, void * stream);

/* The IQ2_XXS sub-block variant's two kernels (tools/ldlq.py:117-272, which the reference runs on the CPU; no
 * counterpart in its library). gpuq_ldlq_sub_weff_dev: for a super-block's rows d_blk [rows][256] (float32), the
 * weights d_weff = qw * sqrt(sigma2 + x^2), sigma2 = (numpy's float32 sum of x^2 over the row) / 256, row r taking the
 * 256 importance values of row r / qw_div of d_qw. gpuq_ldlq_sub_points_dev: with d (and, for sub 8, the sub-block
 * scales) from ggml's IQ2_XXS bytes d_q [rows][66], the groups of columns [c0, c0 + sub) choose their points again
 * over the whole grid (sub 32 also tries the sub-block scale +-scale_search); the group fields of d_q are rewritten
 * and d_err [rows][sub] (float64) receives x - q for the feedback. On `stream`, no synchronisation; 0 on a bad
 * argument. */
size_t gpuq_ldlq_sub_weff_dev(const float * d_blk, const float * d_qw, int64_t qw_div, float * d_weff, int64_t rows,
                              void * stream);
size_t gpuq_ldlq_sub_points_dev(const float * d_blk, const float * d_weff, void * d_q, double * d_err, int64_t rows, int sub,
                                int c0, int scale_search, void * stream);

/* LDLQ's triangular inverse as products on the float64 tensor-core path: C = alpha A B (+ beta C, beta != 0),
 * row-major float64 A [M][lda], B [K][ldb], C [M][ldc]; tri 1: B is lower-triangular (K == N) and tri 2: A is
 * lower-triangular (K == M) - the blocks of the product the triangle makes zero are skipped; tri 0: a full product.
 * K, N, lda, ldb even; A and B 16-byte aligned. On `stream`, no synchronisation; returns the bytes of C written, 0 on
 * a bad argument. No counterpart in the reference (its factorisation is torch's cholesky_inverse). */
size_t gpuq_dgemm_dev(int tri, int64_t M, int64_t N, int64_t K, double alpha, const double * d_a, int64_t lda,
                      const double * d_b, int64_t ldb, double beta, double * d_c, int64_t ldc, void * stream);
/* `batch` such products of one shape in one launch, product i on d_a + i stride_a, d_b + i stride_b, d_c + i stride_c
 * (strides in doubles; even for A and B); returns the bytes of every C written. */
size_t gpuq_dgemm_batched_dev(int tri, int64_t M, int64_t N, int64_t K, double alpha, const double * d_a, int64_t lda,
                              const double * d_b, int64_t ldb, double beta, double * d_c, int64_t ldc, int64_t batch,
                              int64_t stride_a, int64_t stride_b, int64_t stride_c, void * stream);

/* The Hessian of a layer's inputs on the tensor cores: H = (S X)^T (S X) (accumulate 0) or H += (S X)^T (S X)
 * (accumulate 1), the float32 GEMM a row chunk of
 * tools/hessian_from_dump.py:73-79 (`_xtx`: `H += (xc.T @ xc).double()`) for one chunk as one call.
 * d_x: [rows][ld_x] values of type src (0: F32, 30: BF16 - the activation dumps' type), the first dim of a row used;
 * d_scale: NULL, or a float32 per row (a gated Hessian's routing weight: x * s in float32); d_h: float64 [dim][dim]
 * row-major, written or added to (exactly symmetric if it was). The sums over the rows are float32-accurate (bf16
 * tensor-core products of an exact three-part split of each float32 value, float32 accumulation over at most 1,024
 * rows; a BF16 source without a scale needs one product), then added in float64. d_scratch: gpuq_xtx_scratch_bytes(src, rows, dim, d_scale != NULL)
 * bytes, 16-byte aligned, owned by the caller (the parts of X laid out as tensor-core operands). On `stream`, no
 * synchronisation. Returns the bytes of X read, 0 on a bad argument (see gpuq_last_error). A wait inside the kernel
 * that runs out sets bit 3 of gpuq_status. No counterpart in the reference's library (it runs torch's GEMM). */
size_t gpuq_xtx_scratch_bytes(int src, int64_t rows, int64_t dim, int scaled);
size_t gpuq_xtx_dev(int src, const void * d_x, int64_t ld_x, const float * d_scale, int64_t rows, int64_t dim, double * d_h,
                    int accumulate, void * d_scratch, size_t scratch_bytes, void * stream);

/* A diagnostic with no counterpart in the reference: how many floats x with |x| < 2^22 round differently in the Q8_0
 * kernels (which form ggml's roundf as trunc(x + copysign(0.5 - 2^-25, x))) than in CUDA's roundf: 0 expected; -1 if
 * the check could not run. Synchronous, on the current device. */
int64_t gpuq_check_q8_rounding(void);

/* Scratch size of gpuq_requantize_noalloc, held on every GPU that gpuq_init prepares, from gpuq_init to exit. */
#define GPUQ_NOALLOC_SCRATCH_BYTES ((size_t) 64 << 20)

/* No counterpart in the reference: gpuq_requantize_batch for callers that must not allocate device memory while
 * they run (a process sharing the GPU under a fixed memory budget, or whose allocator owns all device memory).
 * Same arguments, same bytes out, but the imatrix, the source bytes and the output are staged in a static device
 * array of GPUQ_NOALLOC_SCRATCH_BYTES instead of buffers grown with cudaMalloc; it calls no cudaMalloc/cudaFree.
 * A call whose staged bytes exceed the array returns 0 and says how much it needed (gpuq_last_error).
 * gpuq_init must have run for the current device: it looks up the array's address there, which loads the array at
 * set-up (if that lookup failed, the first call retries it: make that call before any stream capture). Under lazy
 * module loading, the first launch of each quantize kernel loads its code (a driver allocation): warm each type up
 * once during set-up, or run with CUDA_MODULE_LOADING=EAGER. Sizes are checked before any product is formed.
 * All calls on a device share the array, so calls that overlap on one GPU race; each call clears the status word it
 * uses. Calls across a device reset (cudaDeviceReset) are not supported. Synchronous, on the default stream. */
size_t gpuq_requantize_noalloc(int src, const void * raw, int type, void * dst, int64_t nmat, int64_t nrow,
                               int64_t n_per_row, const float * imatrix);

#ifdef __cplusplus
}
#endif
#endif
