// noalloc.cu - gpuq_requantize_noalloc: the host API's requantize without any device allocation.
//
// Who needs it: callers that must not allocate device memory while they run - code that shares a GPU under a fixed
// memory budget or a caching allocator that owns every byte (an inference server quantizing on the side), or a
// host process that has to keep its footprint constant after start-up. gpuq_requantize_batch grows its staging
// buffers with cudaMalloc on demand; this entry point instead stages the source bytes, the importance matrix and
// the output in one file-scope scratch array that every GPU loading the library holds from load to exit.
//
// Contract:
//   * the scratch holds GPUQ_NOALLOC_SCRATCH_BYTES (64 MiB): a status word, then the imatrix, the source bytes and
//     the output, each 256-byte aligned; a call that does not fit returns 0 with the needed size in
//     gpuq_last_error() - split the tensor (whole rows) into smaller calls;
//   * gpuq_init must have run for the current device (it uploads the search tables: that allocation happens once,
//     at set-up). gpuq_init also looks up the scratch array's device address (cudaGetSymbolAddress, with that device
//     current), which loads this file's device module - and so the 64 MiB array - at set-up even under CUDA's lazy
//     module loading; should that lookup fail there, the first call on the device retries it, so make that first
//     call before any stream capture;
//   * under lazy module loading (CUDA_MODULE_LOADING=LAZY, the default) the first launch of a quantize kernel loads
//     that kernel's code into device memory (the driver's allocation, once a kernel and device): callers that must
//     see no change in device memory after set-up make one warm-up call of each type they use during set-up, or run
//     with CUDA_MODULE_LOADING=EAGER;
//   * the cached address is the array's address in the device's primary context: resetting the device
//     (cudaDeviceReset) invalidates it, as it invalidates every other piece of the library's device state (the
//     tables, the staging buffers) - the library does not support calls across a device reset;
//   * every call on a device shares the one array, which keeps the last call's bytes: the status word is cleared
//     at the start of each call, and calls that overlap on the same GPU (other host threads) race on it.
// Nothing here calls cudaMalloc, cudaFree or an allocating library routine: copies are cudaMemcpy, the kernel is the
// library's own quantize kernel, on the default stream.
#include <cstdio>
#include <mutex>
#include "common.cuh"
#include "kernels.h"
#include "../../include/gpuq.h"

namespace gq {
namespace {

constexpr size_t SCRATCH = GPUQ_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[SCRATCH];

constexpr int MAXDEV = 64;
std::mutex g_mu;
unsigned char * g_addr[MAXDEV] = {};   // the array's device address on each device (set-up, once a device)

size_t up256(size_t n) { return (n + 255) & ~(size_t) 255; }

// the device address of the scratch array on the current device; nullptr (and an error) when it cannot be had
unsigned char * scratch_address(int dev) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (dev < 0 || dev >= MAXDEV) return nullptr;
    if (!g_addr[dev]) {
        void * p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            cudaGetLastError();   // (not left behind for the caller's next CUDA call)
            char msg[256];
            snprintf(msg, sizeof(msg), "gpuq_requantize_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                     cudaGetErrorString(e));
            set_last_error(msg);
            return nullptr;
        }
        g_addr[dev] = (unsigned char *) p;
    }
    return g_addr[dev];
}

}  // namespace

// called by gpuq_init for each device it prepares (that device current): loads the array at set-up
void noalloc_prepare(int dev) {
    if (!scratch_address(dev)) set_last_error("");   // (a failure here is retried, and reported, by the first call)
}

}  // namespace gq

using namespace gq;

extern "C" size_t gpuq_requantize_noalloc(int src, const void * raw, int type, void * dst, int64_t nmat, int64_t nrow,
                                          int64_t n_per_row, const float * imatrix) {
    char msg[256];
    const int sb = src_bytes32(src), bb = block_bytes(type), bl = block_len(type);
    if (!sb || !bb || nmat <= 0 || nrow <= 0 || n_per_row <= 0 || n_per_row % bl || !raw || !dst) {
        set_last_error("gpuq_requantize_noalloc: bad arguments (source or target type, shape, or null pointer)");
        return 0;
    }
    if (!imatrix && !takes_no_imatrix(type)) {
        set_last_error("gpuq_requantize_noalloc: this type needs an importance matrix");
        return 0;
    }
    // every size below is bounded by the scratch before it is multiplied out, so no product can wrap: each of the
    // imatrix, the source and the output must fit the array on its own
    const int64_t lim = (int64_t) SCRATCH;
    if (n_per_row > lim / 4 || nmat > lim / 4 / n_per_row || nrow > lim / 4 / n_per_row ||
        nmat > lim / nrow / n_per_row) {
        snprintf(msg, sizeof(msg), "gpuq_requantize_noalloc: %lld x %lld x %lld values exceed the %zu-byte scratch "
                 "limit: quantize fewer rows a call", (long long) nmat, (long long) nrow, (long long) n_per_row, SCRATCH);
        set_last_error(msg);
        return 0;
    }
    const int64_t n = nmat * nrow * n_per_row;   // < 64 Mi: no overflow in the byte counts below
    const bool any_len = type == F16 && elementwise_src(src);   // (F16 takes rows of any length from these)
    if (n % 32 && !any_len) { set_last_error("gpuq_requantize_noalloc: the value count must be a multiple of 32"); return 0; }
    const bool want_qw = imatrix && type != Q8_0 && type != F16;   // (both ignore it, as ggml_quantize_chunk)
    const size_t qw_bytes = want_qw ? (size_t) nmat * n_per_row * 4 : 0;
    const size_t in_bytes = any_len ? (size_t) n * (src == SRC_F32 ? 4 : 2) : (size_t) (n / 32) * sb;
    const int64_t nblocks = n / bl;
    const size_t out_bytes = (size_t) nblocks * bb;
    const size_t need = 256 + up256(qw_bytes) + up256(in_bytes) + up256(out_bytes);
    if (need > SCRATCH) {
        snprintf(msg, sizeof(msg), "gpuq_requantize_noalloc: needs %zu bytes of scratch, the limit is %zu bytes (%d MiB): "
                 "quantize fewer rows a call", need, SCRATCH, (int) (SCRATCH >> 20));
        set_last_error(msg);
        return 0;
    }
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) { set_last_error("gpuq_requantize_noalloc: no current device"); return 0; }
    bool ready = false;
    const SearchTab * tab = current_search_tab(type, &ready);
    if (!ready) { set_last_error("gpuq_requantize_noalloc: gpuq_init has not run for the current device"); return 0; }
    if (needs_search_tab(type) && !tab) { set_last_error("gpuq_requantize_noalloc: no search tables for this type"); return 0; }
    unsigned char * base = scratch_address(dev);
    if (!base) return 0;
    unsigned * status = reinterpret_cast<unsigned *>(base);
    float * d_qw = reinterpret_cast<float *>(base + 256);
    unsigned char * d_in = base + 256 + up256(qw_bytes);
    unsigned char * d_out = d_in + up256(in_bytes);
    if (cudaMemset(status, 0, sizeof(unsigned)) != cudaSuccess ||
        (want_qw && cudaMemcpy(d_qw, imatrix, qw_bytes, cudaMemcpyHostToDevice) != cudaSuccess) ||
        cudaMemcpy(d_in, raw, in_bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
        set_last_error("gpuq_requantize_noalloc: host-to-device copy failed");
        return 0;
    }
    LaunchArgs a{};
    a.src_type = src;
    a.src = d_in;
    a.qw = want_qw ? d_qw : nullptr;
    a.qw_mod = n_per_row / bl; a.qw_div = 1; a.qw_mat = nrow * (n_per_row / bl);
    a.out = d_out;
    a.nblocks = nblocks;
    a.tab = tab ? *tab : SearchTab{};
    a.status = status;
    a.stream = 0;
    a.n_per_row = n_per_row;
    if (launch_quantize(type, a) != cudaSuccess) { set_last_error("gpuq_requantize_noalloc: kernel launch failed"); return 0; }
    unsigned st = 0;
    if (cudaMemcpy(dst, d_out, out_bytes, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(&st, status, sizeof(st), cudaMemcpyDeviceToHost) != cudaSuccess) {
        set_last_error("gpuq_requantize_noalloc: device-to-host copy failed");
        return 0;
    }
    if (st) {
        snprintf(msg, sizeof(msg), "gpuq_requantize_noalloc: device status 0x%x (non-finite input?)", st);
        set_last_error(msg);
        return 0;
    }
    set_last_error("");
    return out_bytes;
}
