// FP32 / FP64 FMA-pipe peak of the current device, measured: the roofline
// denominator of the stepper, whose hot loop is scalar FMA work and not a
// tensor-core contraction. Every thread runs 8 independent FMA chains (enough
// to cover the pipe latency) for `iters` iterations over a grid that fills
// every SM; flops = 2 x chains x iters x threads.
#include <cuda_runtime.h>

#include "../../include/phyzb.h"

namespace {

template <class T>
__global__ void __launch_bounds__(256) fma_chains(T* out, int iters, T a, T b) {
    T x0 = T(threadIdx.x), x1 = x0 + T(1), x2 = x0 + T(2), x3 = x0 + T(3);
    T x4 = x0 + T(4), x5 = x0 + T(5), x6 = x0 + T(6), x7 = x0 + T(7);
#pragma unroll 4
    for (int i = 0; i < iters; i++) {
        x0 = fma(x0, a, b);
        x1 = fma(x1, a, b);
        x2 = fma(x2, a, b);
        x3 = fma(x3, a, b);
        x4 = fma(x4, a, b);
        x5 = fma(x5, a, b);
        x6 = fma(x6, a, b);
        x7 = fma(x7, a, b);
    }
    const T s = x0 + x1 + x2 + x3 + x4 + x5 + x6 + x7;
    if (s == T(-1.2345)) out[threadIdx.x] = s;  // keeps the chains live
}

template <class T>
int measure(double* tflops) {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return PHYZB_ERR_CUDA;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return PHYZB_ERR_CUDA;
    T* out = nullptr;
    if (cudaMalloc(&out, 256 * sizeof(T)) != cudaSuccess) return PHYZB_ERR_CUDA;
    const int threads = 256, blocks = sms * 8, iters = sizeof(T) == 8 ? 8192 : 16384;
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    float best = 1e30f;
    for (int r = 0; r < 5; r++) {
        cudaEventRecord(e0);
        fma_chains<T><<<blocks, threads>>>(out, iters, T(0.999999), T(1e-7));
        cudaEventRecord(e1);
        cudaEventSynchronize(e1);
        float ms = 0.f;
        cudaEventElapsedTime(&ms, e0, e1);
        if (r > 0 && ms < best) best = ms;  // first launch is the warm-up
    }
    const cudaError_t err = cudaGetLastError();
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaFree(out);
    if (err != cudaSuccess) return PHYZB_ERR_CUDA;
    const double flops = 2.0 * 8.0 * iters * (double)threads * blocks;
    *tflops = flops / (best * 1e-3) / 1e12;
    return PHYZB_OK;
}

}  // namespace

extern "C" int phyzb_measure_fma_peak(int precision, double* tflops) {
    if (!tflops) return PHYZB_ERR_INVALID;
    return precision == PHYZB_F64 ? measure<double>(tflops) : measure<float>(tflops);
}
