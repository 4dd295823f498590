// peak.cu - measures this GPU's FP32 issue rate for separate FADD / FMUL (no FMA: the quantizers are built with
// -fmad=false, so every floating-point operation they execute is one of these). The roofline denominator of the
// search kernels. Built into libgpuq_peak.so (bench tooling; not part of libgpuq_cuda.so).
#include <cuda_runtime.h>

__global__ void k_fp32_peak(float * out, int iters, float a, float b) {
    float x[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = (float) (threadIdx.x + j);
    for (int i = 0; i < iters; ++i) {
#pragma unroll
        for (int u = 0; u < 16; ++u) {
#pragma unroll
            for (int j = 0; j < 8; j += 2) { x[j] = x[j] * a; x[j + 1] = x[j + 1] + b; }
        }
    }
    float s = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) s += x[j];
    if (s == 1234.5f) out[threadIdx.x] = s;   // (keeps the chains alive)
}

extern "C" double peak_fp32_ops_per_s(int dev) {
    if (cudaSetDevice(dev) != cudaSuccess) return 0;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    float * out = nullptr;
    cudaMalloc(&out, 1024 * sizeof(float));
    const int blocks = sms * 8, threads = 256, iters = 4096;
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    k_fp32_peak<<<blocks, threads>>>(out, iters, 0.99999f, 1e-7f);
    cudaEventRecord(e0);
    const int reps = 5;
    for (int r = 0; r < reps; ++r) k_fp32_peak<<<blocks, threads>>>(out, iters, 0.99999f, 1e-7f);
    cudaEventRecord(e1);
    cudaEventSynchronize(e1);
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaFree(out);
    const double ops = (double) reps * blocks * threads * iters * 16 * 8;
    return ms > 0 ? ops / (ms * 1e-3) : 0;
}

// FP64 FMA rate (2 flop each): the roofline denominator of LDLQ's float64 factorisation and error-feedback update
__global__ void k_fp64_peak(double * out, int iters, double a, double b) {
    double x[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = (double) (threadIdx.x + j);
    for (int i = 0; i < iters; ++i) {
#pragma unroll
        for (int u = 0; u < 16; ++u) {
#pragma unroll
            for (int j = 0; j < 8; ++j) x[j] = fma(x[j], a, b);
        }
    }
    double s = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) s += x[j];
    if (s == 1234.5) out[threadIdx.x] = s;
}

extern "C" double peak_fp64_flop_per_s(int dev) {
    if (cudaSetDevice(dev) != cudaSuccess) return 0;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    double * out = nullptr;
    cudaMalloc(&out, 1024 * sizeof(double));
    const int blocks = sms * 8, threads = 256, iters = 1024;
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    k_fp64_peak<<<blocks, threads>>>(out, iters, 0.9999999, 1e-9);
    cudaEventRecord(e0);
    const int reps = 5;
    for (int r = 0; r < reps; ++r) k_fp64_peak<<<blocks, threads>>>(out, iters, 0.9999999, 1e-9);
    cudaEventRecord(e1);
    cudaEventSynchronize(e1);
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaFree(out);
    const double flop = 2.0 * reps * blocks * threads * iters * 16 * 8;
    return ms > 0 ? flop / (ms * 1e-3) : 0;
}
